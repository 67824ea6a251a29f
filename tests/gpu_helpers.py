"""Helpers shared by the GPU tests: moving fixtures to the device, the oracle
on a compact subset of a large workload, tolerance checks."""

from __future__ import annotations

import numpy as np
import torch

from conftest import bf16_ulp
from oracle import qsa_oracle as O

# north_star: BF16 outputs within atol 2e-2 / rtol 2e-2 of the FP32 reference
ATOL = 2e-2
RTOL = 2e-2


def np_to_dev(z: dict, device="cuda") -> dict:
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)
    return dict(
        q=t(z["q"].view(np.int16)).view(torch.bfloat16),
        gate=t(z["gate"].view(np.int16)).view(torch.bfloat16),
        k=t(z["k"]).view(torch.float8_e4m3fn),
        v=t(z["v"]).view(torch.float8_e4m3fn),
        btable=t(z["btable"]), t2r=t(z["t2r"]), indices=t(z["indices"]), counts=t(z["counts"]),
        k_scale=float(z["k_scale"]), v_scale=float(z["v_scale"]),
    )


def bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> uint16 bit patterns on the host."""
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def u8(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.uint8).cpu().numpy()


def check_close(out_bits: np.ndarray, ref: np.ndarray, atol=ATOL, rtol=RTOL, what=""):
    """The parity gate: |out - ref| <= atol + rtol * |ref| everywhere (NaN
    positions must agree). Returns the max abs error."""
    out = O.bf16_to_f32(out_bits).astype(np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert out.shape == ref.shape, (out.shape, ref.shape)
    nan_o, nan_r = np.isnan(out), np.isnan(ref)
    assert np.array_equal(nan_o, nan_r), f"{what}: NaN positions differ"
    fin = ~nan_r
    err = np.abs(out[fin] - ref[fin])
    bad = err > atol + rtol * np.abs(ref[fin])
    assert not bad.any(), f"{what}: {int(bad.sum())} elements out of tolerance, max err {err.max():.3e}"
    return float(err.max()) if err.size else 0.0


# Tight check, beyond the gate: within one bf16 spacing of the float64
# oracle, plus an absolute floor for outputs near zero (weighted averages of
# +-values cancel, and a 1e-6 fp32 accumulation difference is many ulps of a
# 1e-5 result).
TIGHT_ABS = 2e-5


def max_ulps(out_bits: np.ndarray, ref: np.ndarray, abs_floor: float = TIGHT_ABS) -> float:
    """Largest error, after the absolute floor, in units of the bf16 spacing
    at the reference value (<= 1 means correctly rounded up to one step)."""
    out = O.bf16_to_f32(out_bits).astype(np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    fin = ~np.isnan(ref)
    if not fin.any():
        return 0.0
    err = np.maximum(np.abs(out[fin] - ref[fin]) - abs_floor, 0.0)
    return float((err / bf16_ulp(ref[fin])).max())


def compact_subset(w, rows):
    """The oracle's view of ``rows`` of a (large) device workload: the pages
    those rows' block-table entries name, copied into a compact host cache,
    and their block-table rows remapped to it. Returns numpy inputs for
    ``qsa_oracle.attention`` with identity t2r."""
    rows = torch.as_tensor(rows, dtype=torch.long, device=w.btable.device)
    req = w.t2r.to(torch.long)[rows]
    bt = w.btable[req].to(torch.long)  # [n, ppr]
    num_pages = w.k.shape[0]
    ok = (bt >= 0) & (bt < num_pages)
    pages = torch.unique(bt[ok])
    remap = torch.full((num_pages,), -1, dtype=torch.long, device=bt.device)
    remap[pages] = torch.arange(pages.numel(), device=bt.device)
    bt_c = torch.where(ok, remap[bt.clamp(0, num_pages - 1)], torch.full_like(bt, -1))
    k_c = w.k.view(torch.uint8)[pages]
    v_c = w.v.view(torch.uint8)[pages]
    counts = None if w.counts is None else w.counts[rows].cpu().numpy()
    return dict(
        q=bits(w.q[rows]), gate=bits(w.gate[rows]), k=k_c.cpu().numpy(), v=v_c.cpu().numpy(),
        btable=bt_c.to(torch.int32).cpu().numpy(), t2r=np.arange(rows.numel(), dtype=np.int32),
        indices=w.indices[rows].cpu().numpy(), counts=counts,
    )


def oracle_subset(w, rows, **kw):
    c = compact_subset(w, rows)
    return O.attention(c["q"], c["k"], c["v"], w.k_scale, w.v_scale, c["btable"], c["t2r"], c["indices"],
                       c["gate"], counts=c["counts"], softmax_scale=w.softmax_scale, **kw)
