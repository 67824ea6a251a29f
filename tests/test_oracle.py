"""CPU: the oracle is pinned to the reference's own outputs before it is
trusted as the checker of the CUDA path."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN_CASES, bf16_ulp, fp32_floor
from oracle import qsa_oracle as O
from oracle.eager_port import torch_eager_port


def _args(z):
    return (z["q"], z["k"], z["v"], float(z["k_scale"]), float(z["v_scale"]), z["btable"], z["t2r"],
            z["indices"], z["gate"])


def test_e4m3_table_matches_torch():
    b = torch.arange(256, dtype=torch.uint8)
    ref = b.view(torch.float8_e4m3fn).to(torch.float64).numpy()
    tab = O.e4m3fn_table()
    assert np.array_equal(np.isnan(ref), np.isnan(tab))
    fin = ~np.isnan(ref)
    assert np.array_equal(ref[fin], tab[fin])
    assert np.nanmax(tab) == 448.0


def test_bf16_rounding_matches_torch():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(100_000, generator=g) * torch.exp(torch.randn(100_000, generator=g) * 4)
    ref = x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(O.f32_to_bf16(x.numpy()), ref)


def test_e4m3_quantiser_matches_torch_on_clamped_inputs():
    g = torch.Generator().manual_seed(2)
    x = (torch.randn(50_000, generator=g) * torch.exp(torch.randn(50_000, generator=g) * 3)).clamp(-448, 448)
    ref = x.to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(O.f32_to_e4m3fn_sat(x.numpy()), ref)


def test_decode_slots_hand_example():
    # P=4, 2 requests x 3 pages, 6 physical pages
    btable = np.array([[5, 0, 2], [1, -1, 4]], dtype=np.int32)
    indices = np.array([[0, 5, 11, 12, -1], [3, 4, 9, 8, 2]], dtype=np.int32)
    s = O.decode_slots(indices, btable, None, page_size=4, num_pages=6)
    # row 0: t=0 -> page 5 off 0 -> 20; t=5 -> page 0 off 1 -> 1; t=11 -> page 2 off 3 -> 11;
    #        t=12 -> logical page 3 >= 3 -> masked; -1 masked
    # row 1: t=3 -> page 1 off 3 -> 7; t=4 -> btable -1 -> masked; t=9 -> page 4 off 1 -> 17;
    #        t=8 -> page 4 off 0 -> 16; t=2 -> page 1 off 2 -> 6
    assert s.tolist() == [[20, 1, 11, -1, -1], [7, -1, 17, 16, 6]]
    s2 = O.decode_slots(indices, btable, None, 4, 6, counts=np.array([2, 0]))
    assert s2.tolist() == [[20, 1, -1, -1, -1], [-1] * 5]
    # row 0 reads block-table row 1 through t2r; row 1's request id 7 is out of range
    s3 = O.decode_slots(indices, btable, np.array([1, 7]), 4, 6)
    assert s3[0].tolist() == [4, -1, 19, -1, -1] and s3[1].tolist() == [-1] * 5


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_oracle_matches_reference_eager(golden, name):
    """numpy oracle (eager rules: NaN empty rows, clamped t2r, no counts) vs
    the reference's torch_eager output, within one bf16 ulp (plus the fp32
    accumulation floor of the case)."""
    z = golden[name]
    ref = O.bf16_to_f32(z["out_eager"]).astype(np.float64)
    o = O.attention(*_args(z), empty_row="nan", t2r_policy="clamp")
    assert np.array_equal(np.isnan(ref), np.isnan(o))
    fin = ~np.isnan(ref)
    err = np.abs(o[fin] - ref[fin])
    assert np.all(err <= bf16_ulp(ref[fin]) + fp32_floor(z)), float(err.max())


@pytest.mark.parametrize("name", [n for n in GOLDEN_CASES if n != "edge_range"])
def test_oracle_matches_reference_loop(golden, name):
    """numpy oracle with the count rule vs the reference's loop ``reference()``."""
    z = golden[name]
    assert "out_loop" in z
    ref = O.bf16_to_f32(z["out_loop"]).astype(np.float64)
    o = O.attention(*_args(z), counts=z["counts"])
    err = np.abs(o - ref)
    assert np.all(err <= bf16_ulp(ref) + fp32_floor(z)), float(err.max())


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_eager_port_is_bit_exact_to_reference(golden, name):
    """The CPU port times the same ATen sequence as torch_eager: bit-exact."""
    z = golden[name]
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    q = t(z["q"].view(np.int16)).view(torch.bfloat16)
    gate = t(z["gate"].view(np.int16)).view(torch.bfloat16)
    k = t(z["k"]).view(torch.float8_e4m3fn)
    v = t(z["v"]).view(torch.float8_e4m3fn)
    out = torch_eager_port(q, k, v, float(z["k_scale"]), float(z["v_scale"]), t(z["btable"]), t(z["t2r"]),
                           t(z["indices"]), gate)
    got = out.view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(got, z["out_eager"])


def test_kat_closed_form(golden):
    z = golden["kat"]
    o = O.attention_bf16(*_args(z), counts=z["counts"])
    assert np.all(o == O.kat_expected_bf16())
    assert np.all(z["out_loop"] == O.kat_expected_bf16())
    assert np.all(z["out_eager"] == O.kat_expected_bf16())


def test_edge_semantics(golden):
    """Empty rows: zeros under the count rule, NaN in the eager rule; the
    early-stopping count changes only its own row."""
    z = golden["edge"]
    o = O.attention(*_args(z), counts=z["counts"])
    assert np.all(o[4] == 0) and np.all(o[5] == 0)
    e = O.attention(*_args(z), empty_row="nan")
    assert np.all(np.isnan(e[4])) and not np.any(np.isnan(e[5]))
    s = O.decode_slots(z["indices"], z["btable"], z["t2r"], 16, z["k"].shape[0], counts=z["counts"])
    assert np.all(s[3, 17:] == -1) and np.all(s[3, :17] >= 0)
    assert s[0, 3] == -1  # negative logical token
    assert len(set(s[1].tolist())) == 1  # duplicates decode to the same slot
