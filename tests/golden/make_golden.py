"""Generate the golden vectors that pin the oracle to the reference.

Run once in a container that has the reference checkout (given as
``--reference-dir`` or ``$QSA_REFERENCE_DIR``) and the ``cutlass`` DSL
package, which ``sm89_cutedsl`` imports at module level:

    python tests/golden/make_golden.py --reference-dir DIR [--only CASE ...]

It imports the reference's own ``sm89_torch.torch_eager`` (sm89_torch.py:27-54)
and ``sm89_cutedsl.reference`` (sm89_cutedsl.py:83-116), sets the module globals
those functions read to each case's shape, runs them on CPU on seeded inputs and
writes ``<case>.npz`` next to this script: the inputs as raw bit patterns (bf16
as uint16, FP8 E4M3FN as uint8) and both reference outputs as bf16 bits.

``torch_eager`` reads ``TOPK`` as both the slice width of ``indices`` and the
logical-token bound (sm89_torch.py:30-31) and ``NUM_REQUESTS * MAX_PAGES`` as
the physical-page bound (:38-39), so each case sets ``TOPK`` to the context
length ``pages_per_req * P`` and uses ``num_pages == B * pages_per_req``.
``reference`` reads the valid count from an extra last column of ``indices``
(sm89_cutedsl.py:87, :92); the fixtures store indices ``[B, K]`` and counts
``[B]`` separately and append the column only for that call.

Two cases come from the reference's own generator, ``make_tensors``
(sm89_cutedsl.py:43-79), called with its shape globals shrunk: seed 42, K/V
``bf16 randn * 0.1`` cast to E4M3FN (most bytes in the smallest exponents and
the subnormals), an identity block table, sequential indices with the count
in the last column, and ``k_scale = v_scale = 0.1``. ``range`` stresses the
dynamic range of the FP8 term splits: one query element per head far above
the others and K/V spread out to +-448, so that the probabilities span many
decades.
"""

from __future__ import annotations

import argparse

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _bits16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def _bits8(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.uint8).numpy().copy()


def _fp8(x: torch.Tensor) -> torch.Tensor:
    return x.clamp(-448.0, 448.0).to(torch.float8_e4m3fn)


def _load_reference(ref_dir: str):
    sys.path.insert(0, ref_dir)
    import sm89_cutedsl  # noqa: F401  (imports cutlass; never calls it here)
    import sm89_torch

    return sm89_torch, sys.modules["sm89_cutedsl"]


def _run_reference(mods, case):
    """Call the two reference oracles with their globals set to the case."""
    sm89_torch, sm89_cutedsl = mods
    b, hq, d = case["q"].shape
    num_pages, p, hkv, _ = case["k"].shape
    nreq, ppr = case["btable"].shape
    g = dict(
        NUM_REQUESTS=nreq, NUM_Q_HEADS=hq, NUM_KV_HEADS=hkv, GROUP_SIZE=hq // hkv,
        HEAD_DIM=d, PAGE_SIZE=p, MAX_PAGES=ppr, TOPK=ppr * p,
    )
    for mod in (sm89_torch, sm89_cutedsl):
        for name, val in g.items():
            setattr(mod, name, val)
    ks, vs = case["k_scale"], case["v_scale"]
    args = (case["q"], case["k"], case["v"], ks, vs, case["btable"], case["t2r"])
    # torch_eager ignores any count column and slices the first TOPK columns.
    eager = sm89_torch.torch_eager(*args, case["indices"], case["gate"])
    if not case.get("loop", True):
        # reference() indexes btable[req, t // P] without a range check
        # (sm89_cutedsl.py:99-101), so it cannot take a logical page past the
        # block table; such cases pin torch_eager only.
        return eager, None
    # reference() wants [rows, K+1] with the valid count in the last column.
    idx_cnt = torch.cat([case["indices"], case["counts"][:, None]], dim=1)
    loop = sm89_cutedsl.reference(*args, idx_cnt, case["gate"])
    return eager, loop


def _paged_case(seed, b, hq, hkv, d, p, ppr, topk, kv_std=1.0, sample=False,
                ragged=None, k_scale=1.0, v_scale=1.0):
    """Seeded inputs in the layout of the build's benchmark configurations."""
    gen = torch.Generator().manual_seed(seed)
    num_pages = b * ppr
    q = torch.randn(b, hq, d, generator=gen).to(torch.bfloat16)
    gate = torch.randn(b, hq, d, generator=gen).to(torch.bfloat16)
    k = _fp8(torch.randn(num_pages, p, hkv, d, generator=gen) * kv_std)
    v = _fp8(torch.randn(num_pages, p, hkv, d, generator=gen) * kv_std)
    btable = torch.randperm(num_pages, generator=gen).to(torch.int32).view(b, ppr)
    ctx = ppr * p
    indices = torch.full((b, topk), -1, dtype=torch.int32)
    counts = torch.zeros(b, dtype=torch.int32)
    for r in range(b):
        n = topk if ragged is None else int(ragged[r])
        if sample:
            sel = torch.randperm(ctx, generator=gen)[:n]
        else:
            sel = torch.randperm(n, generator=gen)
        indices[r, :n] = sel.to(torch.int32)
        counts[r] = n
    return dict(q=q, k=k, v=v, gate=gate, btable=btable, t2r=torch.arange(b, dtype=torch.int32),
                indices=indices, counts=counts, k_scale=k_scale, v_scale=v_scale)


def _make_tensors_case(mods, rows, topk):
    """The reference's own fixture generator with shrunk globals."""
    sm89_cutedsl = mods[1]
    g = dict(NUM_REQUESTS=rows, NUM_Q_HEADS=32, NUM_KV_HEADS=8, GROUP_SIZE=4, HEAD_DIM=128, PAGE_SIZE=16,
             TOPK=topk, MAX_PAGES=topk // 16)
    for name, val in g.items():
        setattr(sm89_cutedsl, name, val)
    q, k, v, ks, vs, btable, t2r, idx, gate = sm89_cutedsl.make_tensors("cpu")
    return dict(q=q, k=k, v=v, gate=gate, btable=btable, t2r=t2r, indices=idx[:, :topk].contiguous(),
                counts=idx[:, topk].contiguous(), k_scale=float(ks), v_scale=float(vs))


def _range_case(seed):
    """FP8 dynamic-range stress: per head, one query element 2^14 (about
    1.6e4) times the others' scale; K/V ~ N(0, 150) clamped to +-448 (a
    quarter of the bytes at the top exponents); k_scale 0.05, so that a
    head's scores spread over about +-16 and its probabilities over about 14
    decades; one row with V at +-448 everywhere."""
    c = _paged_case(seed, b=3, hq=32, hkv=8, d=128, p=16, ppr=4, topk=64, kv_std=150.0, k_scale=0.05,
                    v_scale=0.5)
    gen = torch.Generator().manual_seed(seed + 1)
    b, hq, d = c["q"].shape
    q = torch.randn(b, hq, d, generator=gen) * 5e-4
    big = torch.randint(0, d, (b, hq), generator=gen)
    q[torch.arange(b)[:, None], torch.arange(hq)[None, :], big] = 8.0 * torch.sign(torch.randn(b, hq, generator=gen))
    c["q"] = q.to(torch.bfloat16)
    v = c["v"].view(torch.uint8).clone()
    pages = c["btable"][2].long()
    sign = (torch.rand(pages.numel(), 16, 8, d, generator=gen) < 0.5).to(torch.uint8) << 7
    v[pages] = 0x7E | sign  # +-448
    c["v"] = v.view(torch.float8_e4m3fn)
    return c


def cases(mods=None):
    out = {}
    # the reference's CPU-runnable case, B=4, 4 pages/request,
    # Top-K 64 = every token in random order, 16 shuffled pages.
    out["cfg0"] = _paged_case(0, b=4, hq=32, hkv=8, d=128, p=16, ppr=4, topk=64)
    # configs[2] in miniature: sparse sampling without replacement, unsorted.
    out["sparse"] = _paged_case(2, b=3, hq=32, hkv=8, d=128, p=16, ppr=8, topk=48, sample=True)
    # configs[4] in miniature: GQA group 8, ragged lengths padded with -1, K/V std 0.5.
    out["gqa8_ragged"] = _paged_case(4, b=4, hq=64, hkv=8, d=128, p=16, ppr=6, topk=96,
                                     kv_std=0.5, sample=True, ragged=[96, 1, 37, 80])
    # The reference fixture's own scales (k_scale = v_scale = 0.1,
    # sm89_cutedsl.py:79) on a longer selection than one 128-token tile.
    out["scales"] = _paged_case(5, b=2, hq=32, hkv=8, d=128, p=16, ppr=10, topk=150,
                                sample=True, k_scale=0.1, v_scale=0.1)

    # Edge cases: masked entries of every kind, duplicates, a count column that
    # stops early, an empty row and an all-masked row.
    e = _paged_case(7, b=6, hq=32, hkv=8, d=128, p=16, ppr=4, topk=40, sample=True)
    idx = e["indices"]
    bt = e["btable"]
    num_pages = e["k"].shape[0]
    idx[0, 3] = -5                      # negative logical token
    idx[1, :] = idx[1, 0]               # all duplicates of one token
    bt[2, 1] = -1                       # unmapped page in the block table
    bt[2, 2] = num_pages                # page id past the cache
    e["counts"][3] = 17                 # count column stops early (CUDA/CuTe rule)
    idx[4, :] = -1                      # every entry masked -> empty row
    e["counts"][5] = 0                  # count 0 -> empty row for the count rule only
    out["edge"] = e
    # Logical tokens past the context (page index >= pages_per_req).
    r = _paged_case(8, b=2, hq=32, hkv=8, d=128, p=16, ppr=4, topk=40, sample=True)
    r["indices"][0, 7] = 4 * 16         # first token past the context
    r["indices"][0, 9] = 10_000         # far past it
    r["indices"][1, 0] = 2**31 - 1      # largest int32
    r["loop"] = False
    out["edge_range"] = r

    # The closed-form known answer of sm89_cuda.cu:347-399: q = gate = 0,
    # K = V = 1.0 (byte 0x38), scales 0.1 -> every output is bf16(0.05).
    kat = _paged_case(9, b=2, hq=32, hkv=8, d=128, p=16, ppr=4, topk=64, k_scale=0.1, v_scale=0.1)
    kat["q"].zero_()
    kat["gate"].zero_()
    kat["k"] = torch.full_like(kat["k"].view(torch.uint8), 0x38).view(torch.float8_e4m3fn)
    kat["v"] = kat["k"].clone()
    out["kat"] = kat

    if mods is not None:
        # the reference's own generator (sm89_cutedsl.py:43-79)
        out["mt_small"] = _make_tensors_case(mods, rows=4, topk=64)
        out["mt_tile"] = _make_tensors_case(mods, rows=2, topk=256)
    out["range"] = _range_case(11)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-dir", default=os.environ.get("QSA_REFERENCE_DIR"))
    ap.add_argument("--only", nargs="*", help="write only these cases (default: all)")
    args = ap.parse_args()
    if not args.reference_dir:
        ap.error("give the reference checkout as --reference-dir or $QSA_REFERENCE_DIR")
    mods = _load_reference(args.reference_dir)
    for name, c in cases(mods).items():
        if args.only and name not in args.only:
            continue
        eager, loop = _run_reference(mods, c)
        np.savez_compressed(
            HERE / f"{name}.npz",
            q=_bits16(c["q"]), gate=_bits16(c["gate"]), k=_bits8(c["k"]), v=_bits8(c["v"]),
            btable=c["btable"].numpy(), t2r=c["t2r"].numpy(), indices=c["indices"].numpy(),
            counts=c["counts"].numpy(), k_scale=np.float64(c["k_scale"]),
            v_scale=np.float64(c["v_scale"]),
            out_eager=_bits16(eager),
            **({} if loop is None else {"out_loop": _bits16(loop)}),
        )
        print(f"{name}: q{tuple(c['q'].shape)} k{tuple(c['k'].shape)} "
              f"idx{tuple(c['indices'].shape)} -> {HERE / (name + '.npz')}")



if __name__ == "__main__":
    main()
