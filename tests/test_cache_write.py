"""The paged FP8 cache writer (qsa_b200_cache_write / qsa_cache_write).

CPU: the oracle's quantiser against torch's cast and the saturation rule,
and the C ABI's argument checks (they run before any device is touched).
GPU: bit-exact against the oracle on every input type, with saturating,
NaN, infinite, signed-zero and subnormal values and skipped slots; a
write-then-decode round trip; the write bandwidth on a large batch.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from gpu_helpers import bits, check_close
from oracle import qsa_oracle as O

D = 128


# ------------------------------------------------------------------ CPU ----
def test_quantiser_saturates_where_torch_gives_nan():
    x = np.array([447.0, 448.0, 449.0, 463.0, 464.0, 465.0, 480.0, 1e30, np.inf, -np.inf, -500.0],
                 dtype=np.float32)
    got = O.f32_to_e4m3fn_sat(x)
    assert got.tolist() == [0x7E] * 9 + [0xFE, 0xFE]
    torch_bits = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert torch_bits[5] == 0x7F and torch_bits[8] == 0x7F  # torch: NaN from 465 and inf
    assert O.f32_to_e4m3fn_sat(np.array([np.nan], np.float32))[0] & 0x7F == 0x7F


def test_quantiser_round_trips_every_finite_code_and_ties_to_even():
    tab = O.e4m3fn_table()
    codes = np.array([c for c in range(256) if not np.isnan(tab[c])], dtype=np.uint8)
    assert np.array_equal(O.f32_to_e4m3fn_sat(tab[codes].astype(np.float32)), codes)
    # midpoints between neighbouring positive codes go to the even code
    pos = np.arange(0x7E, dtype=np.uint8)
    mid = ((tab[pos] + tab[pos + 1]) / 2).astype(np.float32)
    assert np.all(O.f32_to_e4m3fn_sat(mid) % 2 == 0)


def test_oracle_writer_places_rows_and_skips_bad_slots():
    npages, page, hkv = 3, 4, 2
    kc = np.full((npages, page, hkv, D), 0x11, np.uint8)
    vc = np.full((npages, page, hkv, D), 0x22, np.uint8)
    k_new = np.ones((4, hkv, D), np.float32)
    v_new = -np.ones((4, hkv, D), np.float32)
    slots = np.array([5, -1, 12, 0])  # 12 = num_pages * page: past the cache
    k2, v2 = O.cache_write(kc, vc, k_new, v_new, slots, 0.5, 2.0)
    flat_k, flat_v = k2.reshape(-1, hkv, D), v2.reshape(-1, hkv, D)
    assert np.all(flat_k[5] == 0x40) and np.all(flat_k[0] == 0x40)  # 1 / 0.5 = 2.0
    assert np.all(flat_v[5] == 0xB0) and np.all(flat_v[0] == 0xB0)  # -1 / 2 = -0.5
    untouched = [i for i in range(npages * page) if i not in (0, 5)]
    assert np.all(flat_k[untouched] == 0x11) and np.all(flat_v[untouched] == 0x22)


def _args(**over):
    from qsa_b200 import capi

    a = capi.CacheWriteArgs()
    a.k, a.v, a.slots, a.k_cache, a.v_cache = (ctypes.c_void_p(0x10000 * (i + 1)) for i in range(5))
    a.k_scale, a.v_scale = 1.0, 1.0
    a.tokens, a.num_kv_heads, a.head_dim, a.page_size, a.num_pages = 4, 8, 128, 16, 64
    a.token_stride = 8 * 128
    a.input_dtype = capi.DTYPE_BF16
    for k, v in over.items():
        setattr(a, k, v)
    return a


def test_cache_write_rejects_bad_arguments_before_the_device():
    from qsa_b200 import capi

    L = capi.lib()
    assert L.qsa_b200_cache_write(None, None) == capi.ERR_NULL_POINTER
    cases = [
        (dict(head_dim=64), capi.ERR_UNSUPPORTED),
        (dict(input_dtype=7), capi.ERR_UNSUPPORTED),
        (dict(k_scale=0.0), capi.ERR_BAD_VALUE),
        (dict(v_scale=float("inf")), capi.ERR_BAD_VALUE),
        (dict(v_scale=float("nan")), capi.ERR_BAD_VALUE),
        (dict(tokens=-1), capi.ERR_BAD_SHAPE),
        (dict(num_pages=0), capi.ERR_BAD_SHAPE),
        (dict(token_stride=8 * 128 - 1), capi.ERR_BAD_SHAPE),
        (dict(k=None), capi.ERR_NULL_POINTER),
        (dict(slots=None), capi.ERR_NULL_POINTER),
        (dict(k=ctypes.c_void_p(0x10008)), capi.ERR_MISALIGNED),
        (dict(k_cache=ctypes.c_void_p(0x20004)), capi.ERR_MISALIGNED),
        (dict(slots=ctypes.c_void_p(0x30004)), capi.ERR_MISALIGNED),
        (dict(token_stride=8 * 128 + 4), capi.ERR_MISALIGNED),  # 8-byte rows of bf16 break 16-byte alignment
    ]
    for over, want in cases:
        assert capi.cache_write(_args(**over)) == want, over
    assert capi.cache_write(_args(tokens=0)) == capi.OK  # nothing to do, no device needed
    assert capi.status_string(capi.ERR_BAD_VALUE) == "a scale is not a positive finite number"


# ------------------------------------------------------------------ GPU ----
def _special_values(n, gen):
    """Random values over the whole E4M3 range and beyond, with the edge
    cases: saturation, NaN, infinities, signed zeros, subnormals, ties."""
    x = torch.randn(n, generator=gen) * torch.exp(torch.randn(n, generator=gen) * 3)
    tab = torch.from_numpy(O.e4m3fn_table()).float()
    fin = tab[~torch.isnan(tab)]
    edge = torch.cat([
        torch.tensor([0.0, -0.0, 447.0, 448.0, 449.0, 463.0, 464.0, 465.0, 1e30, -1e30, float("inf"),
                      -float("inf"), float("nan"), 2.0 ** -10, 3 * 2.0 ** -10, 2.0 ** -12]),
        fin,
        (fin[:-1] + fin[1:]) / 2,  # midpoints: ties to even
    ])
    x[: edge.numel()] = edge
    return x


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_cache_write_bit_exact_against_oracle(dtype):
    from qsa_b200 import qsa_cache_write

    gen = torch.Generator().manual_seed(7)
    npages, page, hkv, tokens = 64, 16, 8, 700
    k_scale, v_scale = 0.37, 1.0 / 3.0
    k_new = _special_values(tokens * hkv * D, gen).view(tokens, hkv, D).to(dtype)
    v_new = _special_values(tokens * hkv * D, gen).flip(0).view(tokens, hkv, D).to(dtype)
    slots = torch.randperm(npages * page, generator=gen)[:tokens].to(torch.int64)
    slots[::50] = -1
    slots[7] = npages * page  # past the cache: skipped
    slots[8] = 1 << 40
    kc0 = torch.randint(0, 256, (npages, page, hkv, D), generator=gen, dtype=torch.uint8)
    vc0 = torch.randint(0, 256, (npages, page, hkv, D), generator=gen, dtype=torch.uint8)
    kc, vc = kc0.cuda().view(torch.float8_e4m3fn), vc0.cuda().view(torch.float8_e4m3fn)
    qsa_cache_write(k_new.cuda(), v_new.cuda(), slots.cuda(), k_scale, v_scale, kc, vc)
    torch.cuda.synchronize()
    ref_k, ref_v = O.cache_write(kc0.numpy(), vc0.numpy(), k_new.float().numpy(), v_new.float().numpy(),
                                 slots.numpy(), k_scale, v_scale)
    for got, ref in ((kc, ref_k), (vc, ref_v)):
        g = got.view(torch.uint8).cpu().numpy()
        nan_ref = (ref & 0x7F) == 0x7F
        assert np.array_equal((g & 0x7F) == 0x7F, nan_ref), "NaN positions differ"
        assert np.array_equal(g[~nan_ref], ref[~nan_ref])


@pytest.mark.gpu
def test_write_then_decode_round_trip():
    """Tokens appended at logical positions through token_slots +
    qsa_cache_write are read back by the decode exactly as the oracle reads
    the quantised cache."""
    from qsa_b200 import qsa_cache_write, qsa_decode, token_slots

    gen = torch.Generator().manual_seed(11)
    rows, hq, hkv, page, ppr = 6, 16, 4, 16, 8
    npages = rows * ppr
    ctx = ppr * page
    btable = torch.randperm(npages, generator=gen).view(rows, ppr).to(torch.int32)
    kc = torch.zeros(npages, page, hkv, D, dtype=torch.uint8)
    vc = torch.zeros_like(kc)
    reqs = torch.arange(rows).repeat_interleave(ctx)
    pos = torch.arange(ctx).repeat(rows)
    k_new = torch.randn(rows * ctx, hkv, D, generator=gen).to(torch.bfloat16)
    v_new = torch.randn(rows * ctx, hkv, D, generator=gen).to(torch.bfloat16)
    k_scale, v_scale = 0.05, 0.02
    slots = token_slots(btable, reqs, pos, page)
    kc_d, vc_d = kc.cuda().view(torch.float8_e4m3fn), vc.cuda().view(torch.float8_e4m3fn)
    qsa_cache_write(k_new.cuda(), v_new.cuda(), slots.cuda(), k_scale, v_scale, kc_d, vc_d)
    ref_k, ref_v = O.cache_write(kc.numpy(), vc.numpy(), k_new.float().numpy(), v_new.float().numpy(),
                                 slots.numpy(), k_scale, v_scale)
    assert np.array_equal(kc_d.view(torch.uint8).cpu().numpy(), ref_k)
    assert np.array_equal(vc_d.view(torch.uint8).cpu().numpy(), ref_v)
    q = torch.randn(rows, hq, D, generator=gen).to(torch.bfloat16)
    gate = torch.randn(rows, hq, D, generator=gen).to(torch.bfloat16)
    indices = torch.stack([torch.randperm(ctx, generator=gen)[:100] for _ in range(rows)]).to(torch.int32)
    t2r = torch.arange(rows, dtype=torch.int32)
    out = qsa_decode(q.cuda(), kc_d, vc_d, k_scale, v_scale, btable.cuda(), t2r.cuda(), indices.cuda(), gate.cuda())
    torch.cuda.synchronize()
    ref = O.attention(O.f32_to_bf16(q.float().numpy()), ref_k, ref_v, k_scale, v_scale, btable.numpy(), t2r.numpy(),
                      indices.numpy(), O.f32_to_bf16(gate.float().numpy()))
    check_close(bits(out), ref, what="decode of the written cache")


@pytest.mark.gpu
def test_cache_write_bandwidth():
    """A prefill-sized write: 65536 tokens x 8 KV heads of bf16 K and V (268 MB
    read, 134 MB written), timed with CUDA events after warm-up."""
    from qsa_b200 import qsa_cache_write

    tokens, hkv, page = 65536, 8, 16
    npages = tokens // page
    k_new = torch.randn(tokens, hkv, D, device="cuda", dtype=torch.bfloat16)
    v_new = torch.randn(tokens, hkv, D, device="cuda", dtype=torch.bfloat16)
    slots = torch.randperm(tokens, device="cuda")
    kc = torch.empty(npages, page, hkv, D, device="cuda", dtype=torch.float8_e4m3fn)
    vc = torch.empty_like(kc)
    for _ in range(3):
        qsa_cache_write(k_new, v_new, slots, 0.1, 0.1, kc, vc)
    torch.cuda.synchronize()
    n = 20
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(n):
        qsa_cache_write(k_new, v_new, slots, 0.1, 0.1, kc, vc)
    e.record()
    torch.cuda.synchronize()
    us = s.elapsed_time(e) * 1e3 / n
    moved = tokens * hkv * D * (2 * 2 + 2 * 1) + tokens * 8
    print(f"cache write: {tokens} tokens x {hkv} heads, {us:.1f} us per call, {moved / us / 1e3:.0f} GB/s")
    assert moved / us / 1e3 > 1000  # far from HBM-bound would mean a broken access pattern
