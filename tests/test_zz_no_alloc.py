"""qsa_b200_decode_noalloc, the allocation-free C entry point (split scratch in
a fixed device array of the library), checked through the C ABI against
qsa_b200_decode with a caller-supplied workspace.

The file name sorts last, so pytest collects it after every other test; it
passes alone and after them.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from gpu_helpers import bits, check_close
from oracle import qsa_oracle as O

# (workload config, overrides, rows): split-K with G 4 (3 chunks of 512),
# ragged G 8 with per-row counts (4 chunks), split-K with G 17 (two virtual
# KV heads per cache head, partials for every query head), and a
# single-chunk shape that uses no scratch at all
SHAPES = {
    "split_g4": (0, dict(ppr=100, topk=1500, mode="sample"), 64),
    "ragged_g8": (4, dict(ppr=160, topk=2048, len_lo=64, len_hi=2048), 32),
    "split_g17": (0, dict(hq=136, hkv=8, ppr=100, topk=1500, mode="sample"), 16),
    "one_chunk": (1, {}, 32),
}


def _make_args(capi, w, out):
    return capi.make_args(w.q, w.k, w.v, w.btable, w.t2r, w.indices, w.gate, out, counts=w.counts,
                          k_scale=w.k_scale, v_scale=w.v_scale, softmax_scale=w.softmax_scale)


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(SHAPES))
def test_noalloc_matches_decode_on_two_consecutive_calls(name):
    from qsa_b200 import capi
    from qsa_b200.inputs import make_workload

    cfg, over, rows = SHAPES[name]
    stream = torch.cuda.current_stream().cuda_stream
    works = [make_workload(cfg, "cuda", seed=seed, rows=rows, **over) for seed in (41, 42)]
    outs_na = [torch.full_like(w.q, float("nan")) for w in works]
    args_na = [_make_args(capi, w, o) for w, o in zip(works, outs_na)]
    assert capi.workspace_bytes(args_na[0]) <= capi.NOALLOC_SCRATCH_BYTES
    # two consecutive allocation-free calls on one stream: the second reuses
    # the scratch the first wrote
    for a in args_na:
        assert capi.decode_noalloc(a, stream) == capi.OK
    torch.cuda.synchronize()
    for i, w in enumerate(works):
        out_ref = torch.empty_like(w.q)
        a = _make_args(capi, w, out_ref)
        need = capi.workspace_bytes(a)
        ws = torch.empty(max(need, 256), dtype=torch.uint8, device="cuda") if need > 0 else None
        assert capi.decode(a, ws, need, stream) == capi.OK
        torch.cuda.synchronize()
        check_close(bits(outs_na[i]), O.bf16_to_f32(bits(out_ref)), what=f"{name} call {i}")
    assert capi.device_error() == 0


def test_noalloc_rejects_a_split_above_its_fixed_scratch():
    """Refused before any device call, so this runs without a GPU: 1024 rows x
    128 query heads (group 16, whose chunks are never merged inside the decode
    kernel) x 4 chunks need about 270 MB of split partials."""
    from qsa_b200 import capi

    a = capi.DecodeArgs()
    fake = 1 << 20  # aligned stand-in pointers: nothing is dereferenced
    for f in ("q", "k_cache", "v_cache", "indices", "btable", "gate", "out"):
        setattr(a, f, ctypes.c_void_p(fake))
    a.softmax_scale, a.k_scale, a.v_scale = 128 ** -0.5, 1.0, 1.0
    a.rows, a.num_q_heads, a.num_kv_heads, a.head_dim = 1024, 128, 8, 128
    a.page_size, a.pages_per_req, a.num_reqs, a.num_pages = 16, 128, 1024, 1024 * 128
    a.topk, a.indices_stride, a.count_column, a.btable_stride = 2048, 2048, 0, 128
    a.kernel = capi.KERNEL_AUTO
    assert capi.workspace_bytes(a) > capi.NOALLOC_SCRATCH_BYTES
    assert capi.decode_noalloc(a) == capi.ERR_TOO_LARGE
    assert "QSA_B200_NOALLOC_SCRATCH_BYTES" in capi.status_string(capi.ERR_TOO_LARGE)
    a.rows = 0  # an empty batch is still a no-op
    assert capi.decode_noalloc(a) == capi.OK
