"""Top-K index producer: the oracle's rule on hand-made rows (CPU) and the
CUDA kernel bit-exact against the oracle (GPU), including ties, -inf, NaN,
row lengths and a decode fed with the produced indices."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import qsa_oracle as O


def test_oracle_rule_by_hand():
    inf, nan = np.inf, np.nan
    s = np.array([[3, 1, 3, 2, -inf, nan]], dtype=np.float32)
    assert O.topk_select(s, 3).tolist() == [[0, 2, 3]]
    assert O.topk_select(s, 5).tolist() == [[0, 1, 2, 3, -1]]
    assert O.topk_select(s, 3, lengths=[2]).tolist() == [[0, 1, -1]]
    assert O.topk_select(s, 2, lengths=[0]).tolist() == [[-1, -1]]
    ties = np.array([[1, 1, 1, 1], [0.0, -0.0, 0.0, -1]], dtype=np.float32)
    assert O.topk_select(ties, 2).tolist() == [[0, 1], [0, 1]]
    assert O.topk_select(np.array([[inf, 5, inf]], dtype=np.float32), 2).tolist() == [[0, 2]]


def test_c_abi_rejects_bad_arguments():
    from qsa_b200 import capi

    a = capi.TopkArgs()
    a.rows, a.ctx, a.k, a.score_stride, a.out_stride = 2, 100, 0, 100, 1
    assert capi.topk_select(a) == capi.ERR_BAD_VALUE
    a.k, a.out_stride = 4, 3
    assert capi.topk_select(a) != 0
    a.out_stride, a.ctx = 4, 0
    assert capi.topk_select(a) != 0


def _scores(rows, ctx, kind, seed):
    import torch

    g = torch.Generator(device="cpu").manual_seed(seed)
    if kind == "ties":
        s = torch.randint(0, 8, (rows, ctx), generator=g).float()
    else:
        s = torch.randn(rows, ctx, generator=g)
    if kind == "subnormal":
        # float32 subnormals of both signs with many ties, +0 and -0 mixed
        s = torch.randint(-3, 4, (rows, ctx), generator=g).float() * 1e-42
        zero = s == 0
        flip = torch.rand(rows, ctx, generator=g) < 0.5
        s[zero & flip] = -0.0
    if kind.startswith("bucket"):
        # 1000 scores above the threshold bucket, then n keys sharing the top
        # 11 key bits of 1.5 (the bucket holding the k-th score: exactly the
        # kernel's shared-memory candidate buffer at n = 8192, one past it at
        # 8193), the rest far below, in random positions
        n = int(kind[len("bucket"):])
        v = torch.cat([100.0 + torch.randperm(1000, generator=g).float(),
                       1.5 + 0.2 * torch.rand(n, generator=g),
                       -10.0 - torch.rand(ctx - 1000 - n, generator=g)])
        s = torch.stack([v[torch.randperm(ctx, generator=g)] for _ in range(rows)])
    if kind == "sorted":
        s = torch.sort(s, dim=1).values
    if kind.startswith("strided"):
        # every 32nd score far below (or above) the rest: a strided sample of
        # the row sees a distribution unlike the row's
        s[:, ::32] = -50.0 if kind == "strided_low" else 50.0 + s[:, ::32]
    if kind == "special":
        m = torch.rand(rows, ctx, generator=g)
        s[m < 0.05] = float("-inf")
        s[(m >= 0.05) & (m < 0.08)] = float("nan")
        s[(m >= 0.08) & (m < 0.10)] = float("inf")
        s[(m >= 0.10) & (m < 0.12)] = -0.0
    return s


@pytest.mark.gpu
@pytest.mark.parametrize("rows,ctx,k,kind", [
    (5, 1000, 17, "randn"), (4, 4096, 512, "ties"), (3, 5000, 2048, "special"),
    (2, 32768, 2048, "randn"), (3, 2048, 2048, "ties"), (6, 300, 1, "special"), (2, 64, 100, "randn"),
    (4, 5000, 1500, "subnormal"), (3, 700, 300, "subnormal"), (1, (1 << 20) - 3, 2048, "randn"),
    (1, 1 << 20, 2048, "ties"), (2, 32768, 2048, "bucket8192"), (2, 32768, 2048, "bucket8193"),
    (2, 32771, 2048, "bucket8192"), (2, 32768, 2048, "sorted"), (2, 32768, 2048, "strided_low"),
    (2, 32768, 2048, "strided_high"), (3, 65536, 4096, "randn"), (2, 65540, 64, "randn"),
    (2, 1000, 1000, "randn"), (2, 1500, 1499, "ties"),
])
def test_kernel_matches_oracle(rows, ctx, k, kind):
    import torch

    from qsa_b200 import qsa_topk_select

    s = _scores(rows, ctx, kind, seed=rows * 7 + k)
    out = qsa_topk_select(s.cuda(), k)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), O.topk_select(s.numpy(), k))


@pytest.mark.gpu
def test_kernel_row_lengths_and_strides():
    import torch

    from qsa_b200 import qsa_topk_select

    s = _scores(6, 3000, "ties", seed=11)
    wide = torch.zeros(6, 3100)
    wide[:, :3000] = s
    lengths = torch.tensor([0, 1, 700, 3000, 5000, -3], dtype=torch.int32)
    out = torch.full((6, 300), 77, dtype=torch.int32, device="cuda")
    qsa_topk_select(wide.cuda()[:, :3000], 300, lengths=lengths.cuda(), out=out)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), O.topk_select(s.numpy(), 300, lengths=lengths.numpy()))
    # two calls in a row give the same answer
    again = qsa_topk_select(wide.cuda()[:, :3000], 300, lengths=lengths.cuda())
    torch.cuda.synchronize()
    assert torch.equal(again, out)


@pytest.mark.gpu
def test_produced_indices_feed_the_decode():
    """Scores -> Top-K indices -> decode, against the oracle's attention over
    the oracle's indices."""
    import torch

    from gpu_helpers import bits, check_close, u8
    from qsa_b200 import qsa_decode, qsa_topk_select
    from qsa_b200.inputs import make_workload

    w = make_workload(0, "cuda", seed=5, rows=4, ppr=40, topk=640, mode="sample")
    ctx = 40 * 16
    s = _scores(4, ctx, "randn", seed=3)
    idx = qsa_topk_select(s.cuda(), 200)
    out = qsa_decode(w.q, w.k, w.v, 1.0, 1.0, w.btable, w.t2r, idx, w.gate)
    torch.cuda.synchronize()
    ref_idx = O.topk_select(s.numpy(), 200)
    ref = O.attention(bits(w.q), u8(w.k).reshape(w.k.shape), u8(w.v).reshape(w.v.shape), 1.0, 1.0,
                      w.btable.cpu().numpy(), w.t2r.cpu().numpy(), ref_idx, bits(w.gate))
    check_close(bits(out), ref, what="topk -> decode")


def test_oracle_orders_subnormals_and_signed_zeros():
    """Subnormal scores order by value, and -0 ties +0 (lower position wins)."""
    d = np.float32(1e-42)
    s = np.array([[0.0, -0.0, d, -d, 2 * d, -0.0, 0.0]], dtype=np.float32)
    assert O.topk_select(s, 1).tolist() == [[4]]
    assert O.topk_select(s, 2).tolist() == [[2, 4]]
    # the third-highest score is 0: positions 0 and 1 (+0, -0) win over 5, 6
    assert O.topk_select(s, 4).tolist() == [[0, 1, 2, 4]]


@pytest.mark.gpu
def test_rejects_tensors_on_another_device():
    """lengths / out must live on the scores' device (a host pointer handed to
    the kernel would fault it)."""
    import torch

    from qsa_b200 import qsa_topk_select

    s = torch.randn(2, 100, device="cuda")
    with pytest.raises(ValueError, match="lengths"):
        qsa_topk_select(s, 5, lengths=torch.full((2,), 50, dtype=torch.int32))
    with pytest.raises(ValueError, match="out"):
        qsa_topk_select(s, 5, out=torch.empty(2, 5, dtype=torch.int32))
