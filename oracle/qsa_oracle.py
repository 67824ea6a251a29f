"""Numpy restatement of the reference's sparse paged GQA FP8 decode attention.

TEST INFRASTRUCTURE ONLY -- the checker for the CUDA path, never part of it.

The reference (Ammar-Alnagar/QSA-FP8-SM89) defines the operation twice:

* ``torch_eager`` (sm89_torch.py:27-54): vectorised ATen ops, the parity
  oracle named by the build's north star;
* ``reference`` (sm89_cutedsl.py:83-116): a per-row Python loop that reads
  the valid-token count from an extra last column of ``indices``.

This module restates both in numpy, in float64, on raw bit patterns (bf16 as
uint16, FP8 E4M3FN as uint8) so that no library conversion routine stands
between the oracle and the data. It is pinned against outputs of the
reference itself (``tests/golden/``, made by ``tests/golden/make_golden.py``).

Conventions shared with the CUDA path (each one cites the reference line it
follows):

* slot addressing: ``slot = btable[req, t // P] * P + t % P`` and the K/V row
  of KV head ``g`` is ``(slot * Hkv + g) * D`` bytes into the cache
  (sm89_torch.py:33-37, :43; sm89_cuda.cu:149-165);
* a token is valid when ``t >= 0``, ``t // P < pages_per_req`` (torch_eager's
  ``t < TOPK`` with ``TOPK = pages_per_req * P``), ``0 <= phys < num_pages``
  (sm89_torch.py:31, :38; sm89_cuda.cu:160-164) and, when per-row counts are
  given, ``column < count`` (sm89_cuda.cu:113-115, :146);
* a row whose request id is out of range, or that has no valid token,
  produces zeros -- as ``reference`` does (sm89_cutedsl.py:93-106) and as the
  CUDA kernel does for the empty row (sm89_cuda.cu:201-207). ``torch_eager``
  instead yields NaN for an empty row (softmax over all -inf) and clamps the
  request id (sm89_torch.py:36, :48-49); ``empty_row="nan"`` and
  ``t2r_policy="clamp"`` reproduce those two behaviours for pinning.
"""

from __future__ import annotations

import math

import numpy as np

__all__ = [
    "e4m3fn_table",
    "bf16_to_f32",
    "f32_to_bf16",
    "f32_to_e4m3fn_sat",
    "cache_write",
    "decode_slots",
    "attention",
    "attention_bf16",
    "unique_kv_rows",
]


def e4m3fn_table() -> np.ndarray:
    """Value of every FP8 E4M3FN byte as float64 (OCP FP8 spec, bias 7).

    ``s eeee mmm``: e == 0 is subnormal ``m/8 * 2^-6``; ``0x7F``/``0xFF`` are
    NaN; there are no infinities; the largest finite magnitude is 448.
    Used where the reference casts FP8 to float32 (sm89_torch.py:43-44),
    which is exact.
    """
    tab = np.empty(256, dtype=np.float64)
    for b in range(256):
        s = -1.0 if b & 0x80 else 1.0
        e = (b >> 3) & 0xF
        m = b & 0x7
        if e == 0xF and m == 0x7:
            tab[b] = np.nan
        elif e == 0:
            tab[b] = s * (m / 8.0) * 2.0 ** -6
        else:
            tab[b] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return tab


_E4M3 = e4m3fn_table()


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> float32 (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns with round-to-nearest-even (as
    ``Tensor.to(torch.bfloat16)`` at sm89_torch.py:54). NaN stays NaN."""
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = x.view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    out = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    out[nan] = 0x7FC0
    return out


def f32_to_e4m3fn_sat(x: np.ndarray) -> np.ndarray:
    """float -> FP8 E4M3FN bytes, round-to-nearest-even, saturating at +-448.

    The reference's generator casts ``randn * 0.1`` with ``.to(float8_e4m3fn)``
    (sm89_cutedsl.py:51-64); the build's generators clamp to +-448 first, so
    saturation and round-to-nearest agree with torch on every finite input.
    Brute force over the 256-entry table: exact, test-only.
    """
    x = np.asarray(x, dtype=np.float64)
    # positive codes 0x00..0x7E in increasing value order
    pos_codes = np.arange(0x7F, dtype=np.uint8)
    pos_vals = _E4M3[pos_codes]
    a = np.minimum(np.abs(x), 448.0)
    idx = np.searchsorted(pos_vals, a)  # first value >= a
    idx = np.clip(idx, 1, len(pos_vals) - 1)
    lo = pos_vals[idx - 1]
    hi = pos_vals[idx]
    pick_hi = (hi - a < a - lo) | ((hi - a == a - lo) & ((pos_codes[idx] & 1) == 0))
    code = np.where(pick_hi, pos_codes[idx], pos_codes[idx - 1]).astype(np.uint8)
    code = np.where(a == 0.0, np.uint8(0), code)
    neg = np.signbit(x)
    code = np.where(neg, code | np.uint8(0x80), code).astype(np.uint8)
    code = np.where(np.isnan(x), np.uint8(0x7F), code).astype(np.uint8)
    return code


def topk_select(scores, k, lengths=None):
    """The Top-K index producer's rule, the checker of qsa_topk_kernel. The
    reference has no producer (it consumes indices; sm89_cutedsl.py:72-76
    builds sequential ones), so this is the rule the library states: per row,
    the positions of the k highest scores in ascending position order. A
    position is a candidate when it is below the row's length (clamped to
    [0, ctx]) and its score is neither NaN nor -inf; at the k-th score lower
    positions win; fewer than k candidates are padded with -1."""
    s = np.asarray(scores, dtype=np.float32)
    rows, ctx = s.shape
    out = np.full((rows, k), -1, dtype=np.int32)
    for r in range(rows):
        n = ctx if lengths is None else min(max(int(lengths[r]), 0), ctx)
        v = s[r, :n]
        cand = np.nonzero(~np.isnan(v) & (v != -np.inf))[0]
        # highest score first, then the lower position (np.lexsort: last key first)
        order = cand[np.lexsort((cand, -v[cand].astype(np.float64)))]
        pick = np.sort(order[:k])
        out[r, :len(pick)] = pick
    return out


def cache_write(k_cache, v_cache, k_new, v_new, slots, k_scale, v_scale):
    """The paged cache producer: new keys / values quantised into the FP8
    caches at physical token slots; returns updated copies of the caches.

    The reference fills its caches with ``(randn * 0.1).to(float8_e4m3fn)``
    in the ``[num_pages, P, Hkv, 128]`` layout and dequantises them as
    ``value * scale`` (sm89_cutedsl.py:48-62, :79; sm89_torch.py:43-44). The
    writer stores ``e4m3fn(x * inv)`` with ``inv = float32(1 / scale)`` (an
    IEEE float32 division, once) and a float32 product, then
    :func:`f32_to_e4m3fn_sat` (nearest, ties to even, saturating at +-448,
    NaN kept). ``k_cache``/``v_cache`` are uint8 byte arrays, ``k_new``/
    ``v_new`` float32 ``[tokens, Hkv, 128]`` (bf16 / fp16 inputs converted
    exactly beforehand), ``slots`` int ``[tokens]``: ``phys_page * P +
    offset``; a negative slot or one past the cache is skipped.
    """
    kc = np.array(k_cache, dtype=np.uint8, copy=True)
    vc = np.array(v_cache, dtype=np.uint8, copy=True)
    npages, page, hkv, d = kc.shape
    s = np.asarray(slots, dtype=np.int64)
    ok = (s >= 0) & (s < npages * page)
    k_inv = np.float32(1.0) / np.float32(k_scale)
    v_inv = np.float32(1.0) / np.float32(v_scale)
    kq = f32_to_e4m3fn_sat(np.asarray(k_new, dtype=np.float32)[ok] * k_inv)
    vq = f32_to_e4m3fn_sat(np.asarray(v_new, dtype=np.float32)[ok] * v_inv)
    kc.reshape(npages * page, hkv, d)[s[ok]] = kq
    vc.reshape(npages * page, hkv, d)[s[ok]] = vq
    return kc, vc


def decode_slots(
    indices: np.ndarray,
    btable: np.ndarray,
    t2r: np.ndarray | None,
    page_size: int,
    num_pages: int,
    counts: np.ndarray | None = None,
    t2r_policy: str = "zero",
) -> np.ndarray:
    """Index decode + block-table gather + slot addressing (bit-exact target).

    Returns int64 ``[B, K]``: the physical token slot ``phys * P + t % P`` of
    every selected entry, or -1 where the entry is masked. Follows
    sm89_torch.py:30-39 (``logical // PAGE_SIZE``, ``logical % PAGE_SIZE``,
    ``btable[request_ids, logical_page]`` with the validity masks) and the
    count-column rule of sm89_cuda.cu:113-115, :146-164.

    ``t2r_policy``: ``"zero"`` masks every entry of a row whose request id is
    outside ``[0, B_req)``; ``"clamp"`` clamps it like sm89_torch.py:36.
    """
    idx = np.asarray(indices, dtype=np.int64)
    bt = np.asarray(btable, dtype=np.int64)
    rows, k = idx.shape
    nreq, pages_per_req = bt.shape
    if t2r is None:
        req = np.arange(rows, dtype=np.int64)
    else:
        req = np.asarray(t2r, dtype=np.int64).reshape(rows)
    if t2r_policy == "clamp":
        row_ok = np.ones(rows, dtype=bool)
        req = np.clip(req, 0, nreq - 1)
    else:
        row_ok = (req >= 0) & (req < nreq)
        req = np.where(row_ok, req, 0)
    valid = idx >= 0
    t = np.where(valid, idx, 0)
    lp = t // page_size
    po = t % page_size
    valid &= lp < pages_per_req
    lp = np.where(valid, lp, 0)
    phys = bt[req[:, None], lp]
    valid &= (phys >= 0) & (phys < num_pages)
    valid &= row_ok[:, None]
    if counts is not None:
        c = np.clip(np.asarray(counts, dtype=np.int64).reshape(rows), 0, k)
        valid &= np.arange(k)[None, :] < c[:, None]
    return np.where(valid, phys * page_size + po, -1).astype(np.int64)


def attention(
    q_bits: np.ndarray,
    k_bytes: np.ndarray,
    v_bytes: np.ndarray,
    k_scale: float,
    v_scale: float,
    btable: np.ndarray,
    t2r: np.ndarray | None,
    indices: np.ndarray,
    gate_bits: np.ndarray,
    counts: np.ndarray | None = None,
    softmax_scale: float | None = None,
    empty_row: str = "zero",
    t2r_policy: str = "zero",
) -> np.ndarray:
    """Gated sparse paged GQA attention in float64 (before the bf16 store).

    ``out[r,h] = softmax_t(q[r,h]·K[slot_t,g]·k_scale·scale)·V[slot_t,g]·v_scale
    ⊙ sigmoid(gate[r,h])`` with ``g = h // (Hq/Hkv)`` and
    ``scale = D**-0.5`` unless ``softmax_scale`` is given (sm89_torch.py:43-53).

    Shapes: q/gate ``[B,Hq,D]`` (uint16 bf16 bits), K/V ``[num_pages,P,Hkv,D]``
    (uint8 E4M3FN bytes), btable ``[B_req, pages_per_req]``, indices ``[B,K]``.
    """
    q = bf16_to_f32(q_bits).astype(np.float64)
    gate = bf16_to_f32(gate_bits).astype(np.float64)
    rows, hq, d = q.shape
    num_pages, page_size, hkv, d2 = k_bytes.shape
    assert d2 == d and hq % hkv == 0
    grp = hq // hkv
    scale = (d ** -0.5) if softmax_scale is None else float(softmax_scale)
    slots = decode_slots(indices, btable, t2r, page_size, num_pages, counts, t2r_policy)
    kr = np.asarray(k_bytes, dtype=np.uint8).reshape(num_pages * page_size, hkv, d)
    vr = np.asarray(v_bytes, dtype=np.uint8).reshape(num_pages * page_size, hkv, d)
    out = np.zeros((rows, hq, d), dtype=np.float64)
    for r in range(rows):
        sl = slots[r]
        sel = sl[sl >= 0]
        if sel.size == 0:
            if empty_row == "nan":
                out[r] = np.nan
            continue
        keys = _E4M3[kr[sel]]  # [n, Hkv, D]
        vals = _E4M3[vr[sel]]
        qg = q[r].reshape(hkv, grp, d)
        s = np.einsum("hgd,nhd->hgn", qg, keys) * (k_scale * scale)
        m = s.max(axis=-1, keepdims=True)
        p = np.exp(s - m)
        p /= p.sum(axis=-1, keepdims=True)
        ctx = np.einsum("hgn,nhd->hgd", p, vals) * v_scale
        out[r] = ctx.reshape(hq, d)
    sig = 1.0 / (1.0 + np.exp(-gate))
    return out * sig


def attention_bf16(*args, **kwargs) -> np.ndarray:
    """``attention`` rounded to bf16 bit patterns, like the reference's store
    (sm89_torch.py:54)."""
    return f32_to_bf16(attention(*args, **kwargs).astype(np.float32))


def unique_kv_rows(slots: np.ndarray, hkv: int) -> tuple[int, int]:
    """(logical, unique) count of (slot, kv_head) rows touched by ``slots``.

    The measurement's byte accounting: logical rows count duplicates, unique
    rows count each distinct slot once per KV head.
    """
    valid = slots[slots >= 0]
    return int(valid.size) * hkv, int(np.unique(valid).size) * hkv


def kat_expected_bf16() -> int:
    """bf16 bit pattern of the reference's closed-form known answer: q=gate=0,
    K=V=1.0 (byte 0x38), k_scale=v_scale=0.1 -> every output is bf16(0.05)
    (sm89_cuda.cu:347-352, :391)."""
    return int(f32_to_bf16(np.array([0.1 * 1.0 * 0.5], dtype=np.float32))[0])


def softmax_scale_default(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
