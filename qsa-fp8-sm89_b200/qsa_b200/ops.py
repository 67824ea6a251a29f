"""The torch-callable operator contract of the reference's decode path.

Three call shapes, matching the reference's own entry points:

* ``run(q, k_fp8, v_fp8, k_scale, v_scale, btable, t2r, indices, gate)`` --
  same positional order, argument meaning and result as the reference's
  ``run`` (sm89_cutedsl.py:311-351): ``indices`` is ``[rows, topk + 1]`` with
  the valid count in its last column, a new bf16 ``[rows, Hq, D]`` tensor is
  returned and the call synchronises the device, as the reference does
  (sm89_cutedsl.py:350).
* ``launch(q, k, v, indices, btable, t2r, gate, out, k_scale, v_scale)`` --
  the reference's Triton launcher (sm89_triton.py:118-142): same count-column
  layout, caller-provided ``out``, asynchronous.
* ``qsa_decode(...)`` -- the general form: ``indices`` ``[rows, K]`` padded
  with -1 (the layout of the reference's eager path, sm89_torch.py:30), optional per-row
  ``counts``, optional explicit ``softmax_scale`` and ``out``; asynchronous on
  the current stream.

Every call goes through ``torch.ops.qsa_b200.decode`` into the C ABI of
``libqsa_b200.so``; CUDA tensors only, no CPU path.

Semantics (identical for the three shapes). For row r, query head h and KV
head g = h // (Hq // Hkv)::

    out[r,h] = softmax_t(q[r,h] . K[slot_t, g] * k_scale * softmax_scale)
               . V[slot_t, g] * v_scale  *  sigmoid(gate[r,h])

with ``softmax_scale = D ** -0.5`` by default (sm89_torch.py:47) and
``slot_t = btable[t2r[r], t // P] * P + t % P``. Entries with ``t < 0``,
``t // P >= pages_per_req``, a block-table entry outside ``[0, num_pages)``
or a column at or past the row's count are masked. A row whose ``t2r`` entry
is out of range, or that has no valid entry, gives zeros (as the reference's
``reference()`` does, sm89_cutedsl.py:93-106; the eager path would give NaN).
"""

from __future__ import annotations

import math

import torch

from . import capi
from ._lib import load_torch_ops

_KERNELS = {"auto": capi.KERNEL_AUTO, "tc": capi.KERNEL_TC, "simt": capi.KERNEL_SIMT}


def _kernel_code(kernel) -> int:
    if isinstance(kernel, int):
        return kernel
    try:
        return _KERNELS[kernel]
    except KeyError:
        raise ValueError(f"kernel must be one of {sorted(_KERNELS)}, got {kernel!r}") from None


def qsa_decode(q, k, v, k_scale, v_scale, btable, t2r, indices, gate, out=None, counts=None, *,
               softmax_scale=None, count_column=False, topk=None, kernel="auto"):
    """Sparse paged GQA FP8 decode attention with a sigmoid gate.

    Args:
        q, gate: bf16 ``[rows, Hq, 128]`` (contiguous).
        k, v: FP8 E4M3FN ``[num_pages, P, Hkv, 128]`` (contiguous).
        k_scale, v_scale: float dequantisation scales of the caches.
        btable: int32 ``[num_reqs, pages_per_req]`` physical page ids.
        t2r: int32 ``[rows]`` Top-K row -> block-table row, or None (identity).
        indices: int32 ``[rows, K]`` logical token ids (negative = masked);
            with ``count_column=True`` the last column holds the valid count.
        out: optional bf16 output, shaped like ``q``.
        counts: optional int32 ``[rows]`` valid-prefix lengths.
        softmax_scale: score scale (default ``D ** -0.5``).
        topk: number of index columns to read (default: all but the count
            column).
        kernel: "auto" (default), "tc" (tensor-core kernel) or "simt"
            (CUDA-core kernel, any group size).

    Returns ``out``. Runs asynchronously on the current CUDA stream.
    """
    ops = load_torch_ops()
    if out is None:
        out = torch.empty_like(q)
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(q.shape[-1])
    if topk is None:
        topk = indices.shape[1] - (1 if count_column else 0)
    ops.decode(q, k, v, btable, t2r, indices, gate, counts, float(softmax_scale), float(k_scale),
               float(v_scale), bool(count_column), int(topk), _kernel_code(kernel), out)
    return out


def run(q, k_fp8, v_fp8, k_scale, v_scale, btable, t2r, indices, gate):
    """Drop-in for the reference's ``run`` (sm89_cutedsl.py:311-351)."""
    out = torch.zeros_like(q)
    qsa_decode(q, k_fp8, v_fp8, k_scale, v_scale, btable, t2r, indices, gate, out=out, count_column=True)
    torch.cuda.synchronize(q.device)
    return out


def launch(q, k, v, indices, btable, t2r, gate, out, k_scale, v_scale):
    """Drop-in for the reference's Triton ``launch`` (sm89_triton.py:118-142)."""
    return qsa_decode(q, k, v, k_scale, v_scale, btable, t2r, indices, gate, out=out, count_column=True)


def slots(indices, btable, t2r, page_size, num_pages, counts=None, *, count_column=False, topk=None):
    """Physical token slot of every Top-K entry (int64 ``[rows, topk]``, -1
    where masked) -- the index decode every kernel runs, exposed for the
    bit-exact check (sm89_torch.py:30-39)."""
    ops = load_torch_ops()
    if topk is None:
        topk = indices.shape[1] - (1 if count_column else 0)
    out = torch.empty((indices.shape[0], topk), dtype=torch.int64, device=indices.device)
    ops.slots(btable, t2r, indices, counts, bool(count_column), int(topk), int(page_size), int(num_pages), out)
    return out


def qsa_cache_write(k_new, v_new, slots, k_scale, v_scale, k_cache, v_cache):
    """Writes new keys and values into the paged FP8 caches the decode reads:
    ``cache[slot, g, :] = e4m3fn(x[t, g, :] * (1 / scale))`` for ``slot =
    slots[t]`` (``phys_page * P + offset``), in place, asynchronous on the
    current stream.

    The layout and the scale convention are the reference's cache producer
    (sm89_cutedsl.py:48-62: ``[num_pages, P, Hkv, 128]`` E4M3FN, dequantised
    as ``value * scale``). ``1 / scale`` is rounded to fp32 once and each
    product is an fp32 product, rounded to the nearest E4M3FN value (ties
    to even) and saturated at +-448: a finite
    value beyond the range or an infinity becomes +-448 and NaN stays NaN,
    where ``torch``'s cast gives NaN for ``|x| >= 464``. Negative slots and
    slots past the cache are skipped.

    Args:
        k_new, v_new: bf16, fp16 or fp32 ``[tokens, Hkv, 128]``, heads
            contiguous (a token stride is allowed).
        slots: int64 ``[tokens]``.
        k_scale, v_scale: positive dequantisation scales.
        k_cache, v_cache: float8_e4m3fn (or uint8) ``[num_pages, P, Hkv, 128]``.
    """
    load_torch_ops().cache_write(k_new, v_new, slots, float(k_scale), float(v_scale), k_cache, v_cache)
    return k_cache, v_cache


def qsa_topk_select(scores, k, lengths=None, out=None):
    """Top-K indices for the decode from per-position scores: for each row of
    fp32 ``scores[rows, ctx]``, the positions of the ``k`` highest scores in
    ascending position order, int32 ``[rows, k]``, asynchronous on the
    current stream.

    A position is a candidate when it is below the row's ``lengths`` entry
    (all ``ctx`` positions without ``lengths``) and its score is neither NaN
    nor -inf. At the k-th score lower positions win; a row with fewer than
    ``k`` candidates is padded with -1. The result is the ``indices`` argument
    of ``qsa_decode`` (a position is a logical token index).
    """
    from . import capi

    if scores.dtype != torch.float32 or scores.dim() != 2 or scores.stride(1) != 1 or not scores.is_cuda:
        raise ValueError("scores must be a CUDA float32 [rows, ctx] tensor with unit inner stride")
    if lengths is not None:
        if lengths.dtype != torch.int32 or not lengths.is_contiguous() or lengths.numel() != scores.shape[0]:
            raise ValueError("lengths must be a contiguous int32 [rows] tensor")
        if lengths.device != scores.device:
            raise ValueError(f"lengths is on {lengths.device} but scores is on {scores.device}")
    if out is None:
        out = torch.empty(scores.shape[0], int(k), dtype=torch.int32, device=scores.device)
    else:
        if out.dtype != torch.int32 or out.dim() != 2 or out.stride(1) != 1 or out.shape != (scores.shape[0], int(k)):
            raise ValueError("out must be an int32 [rows, k] tensor with unit inner stride")
        if out.device != scores.device:
            raise ValueError(f"out is on {out.device} but scores is on {scores.device}")
    # the launch goes to the scores' device and its current stream
    with torch.cuda.device(scores.device):
        st = capi.topk_select(capi.make_topk_args(scores, k, out, lengths),
                              torch.cuda.current_stream(scores.device).cuda_stream)
    if st != 0:
        raise RuntimeError(f"qsa_b200_topk_select failed: {capi.lib().qsa_b200_status_string(st).decode()}")
    return out


def token_slots(btable, reqs, positions, page_size):
    """Physical slot ``btable[req, pos // P] * P + pos % P`` of each (request,
    position) pair, as int64 -- the ``slots`` argument of
    ``qsa_cache_write`` for tokens appended at logical positions (the rule the
    decode reads them back with, sm89_torch.py:31-44)."""
    reqs = reqs.to(torch.long)
    positions = positions.to(torch.long)
    return btable.to(torch.long)[reqs, positions // page_size] * page_size + positions % page_size


def tc_supports_group(group: int) -> bool:
    """Group sizes (Hq / Hkv) of the tensor-core kernel: 1 to 32 (above 16 as
    two halves per KV head), every size the library takes."""
    return 1 <= group <= 32


def tc_merges_chunks(rows: int, num_q_heads: int, num_kv_heads: int, topk: int, sm_count: int) -> bool:
    """Whether the tensor-core decode merges the chunks of split rows itself
    (the rule of tc_merges_chunks in csrc/qsa_decode_tc.cu): more than one
    chunk but at most 32, a group of at most 8, at least two (row, KV head)
    pairs per SM. Otherwise split rows go through the combine kernel."""
    chunks = -(-topk // chunk_tokens(num_q_heads, num_kv_heads))
    return (1 < chunks <= 32 and num_q_heads // num_kv_heads <= 8 and rows * num_kv_heads >= 2 * sm_count
            and rows * num_kv_heads * chunks < (1 << 30))


def chunk_tokens(num_q_heads, num_kv_heads) -> int:
    """Top-K entries one work item covers: 512 for every group size."""
    return 512


def workspace_bytes(rows, num_q_heads, num_kv_heads, topk, kernel="auto", sm_count=None) -> int:
    """Device workspace one call needs, each part 256-byte aligned: the row
    map of the tensor-core kernel (one int32 token slot per Top-K entry,
    rows x chunks x chunk entries), its tile flags (16 bytes per row and
    chunk) and its item claim counter, then, when a Top-K row spans more than
    one chunk and the chunks are not merged inside the decode kernel
    (``tc_merges_chunks``), the per-chunk partial outputs and log-sum-exps.
    ``sm_count`` defaults to the current CUDA device's (148 without one)."""
    a256 = lambda x: -(-x // 256) * 256
    c = chunk_tokens(num_q_heads, num_kv_heads)
    chunks = 1 if topk <= c else -(-topk // c)
    group = num_q_heads // num_kv_heads
    tc = kernel == "tc" or (kernel == "auto" and tc_supports_group(group))
    total = a256(rows * chunks * c * 4) + a256(rows * chunks * 16) + 256 if (tc and rows > 0) else 0
    if sm_count is None:
        sm_count = (torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
                    if torch.cuda.is_available() else 148)
    if chunks > 1 and not (tc and tc_merges_chunks(rows, num_q_heads, num_kv_heads, topk, sm_count)):
        n = rows * num_q_heads * chunks
        total += a256(n * 128 * 4) + a256(n * 4)
    return total