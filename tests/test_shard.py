"""CPU: the request sharding of the multi-GPU path (qsa_b200.shard), as unit
tests and as two gloo ranks that plan, compute their shard with the CPU
oracle and gather the rows on rank 0 -- the same host-side steps the GPU
ranks take around the decode, with no data-path collective in between."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import qsa_oracle as O


def test_contiguous_shards_cover_every_row_once():
    from qsa_b200.shard import contiguous_shards

    for n, world in [(2048, 8), (256, 1), (7, 3), (3, 4), (0, 2)]:
        shards = contiguous_shards(n, world)
        assert len(shards) == world
        assert shards[0][0] == 0 and shards[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(shards, shards[1:]))
        sizes = [e - s for s, e in shards]
        assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        contiguous_shards(4, 0)


def test_lpt_bins_balance_and_determinism():
    from qsa_b200.inputs import CONFIGS, ragged_lengths
    from qsa_b200.shard import bin_loads, lpt_bins

    lengths = ragged_lengths(CONFIGS[4], 1024, seed=0)
    bins = lpt_bins(lengths, 8)
    flat = sorted(i for b in bins for i in b)
    assert flat == list(range(1024))
    loads = bin_loads(lengths, bins)
    # LPT: no bin exceeds the mean by more than the longest single request
    assert max(loads) - sum(loads) / 8 <= int(lengths.max())
    assert bins == lpt_bins(lengths.tolist(), 8)  # same plan from any rank
    for b in bins:  # longest-first order inside a bin
        lb = [int(lengths[i]) for i in b]
        assert lb == sorted(lb, reverse=True)


def _small_case(seed=3):
    """A ragged batch small enough for the float64 oracle: 6 requests,
    Hq 8 / Hkv 2, page 16, 4 pages per request, Top-K up to 64 with -1
    padding."""
    rng = np.random.default_rng(seed)
    B, hq, hkv, P, ppr, K = 6, 8, 2, 16, 4, 64
    num_pages = B * ppr
    e4 = O.e4m3fn_table()
    finite = np.nonzero(np.isfinite(e4) & (np.abs(e4) < 4))[0].astype(np.uint8)
    q = O.f32_to_bf16(rng.standard_normal((B, hq, 128)).astype(np.float32))
    gate = O.f32_to_bf16(rng.standard_normal((B, hq, 128)).astype(np.float32))
    k = rng.choice(finite, size=(num_pages, P, hkv, 128))
    v = rng.choice(finite, size=(num_pages, P, hkv, 128))
    btable = rng.permutation(num_pages).reshape(B, ppr).astype(np.int32)
    lens = rng.integers(1, K + 1, size=B)
    indices = np.full((B, K), -1, dtype=np.int32)
    for r in range(B):
        indices[r, : lens[r]] = rng.choice(ppr * P, size=lens[r], replace=False)
    return dict(q=q, gate=gate, k=k, v=v, btable=btable, t2r=np.arange(B, dtype=np.int32), indices=indices,
                lens=lens)


def _oracle_rows(c, rows):
    rows = np.asarray(rows, dtype=np.int64)
    return O.attention(c["q"][rows], c["k"], c["v"], 1.0, 1.0, c["btable"], c["t2r"][rows], c["indices"][rows],
                       c["gate"][rows])


def _rank_main(rank, world, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from qsa_b200.shard import gather_rows, lpt_bins

        c = _small_case()
        bins = lpt_bins(c["lens"], world)
        plans = [None] * world
        dist.all_gather_object(plans, bins)
        assert all(p == bins for p in plans), "ranks disagree on the plan"
        mine = bins[rank]
        local = torch.from_numpy(_oracle_rows(c, mine).astype(np.float32))
        counts = [len(b) for b in bins]
        got = gather_rows(local, counts, dst=0)
        if rank == 0:
            order = [i for b in bins for i in b]
            ref = _oracle_rows(c, order).astype(np.float32)
            np.save(out_path, np.stack([got.numpy(), ref]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_gloo_shard_compute_gather(tmp_path):
    out = tmp_path / "gathered.npy"
    mp.start_processes(_rank_main, args=(2, _free_port(), str(out)), nprocs=2, join=True, start_method="spawn")
    got, ref = np.load(out)
    assert got.shape == ref.shape == (6, 8, 128)
    np.testing.assert_array_equal(got, ref)


def _plan_rank_main(rank, world, port, out_path):
    """One rank of the bench's plan: its requests of configs[3] and [4] and
    the config object its line would carry, gathered on every rank."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench

        mine = {cfg: bench.rank_rows(cfg, rank, world)[1] for cfg in (3, 4)}
        conf = {cfg: bench.bench_config(cfg, world, *bench.config_rows(cfg, world)) for cfg in (1, 3, 4)}
        everyone = bench.gather_objects({"rows": mine, "config": conf}, world)
        if rank == 0:
            import json

            with open(out_path, "w") as f:
                json.dump(everyone, f)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_bench_plan_over_gloo_ranks(tmp_path, world):
    """contiguous ranges covering the 2048 requests once;
    LPT bins covering the 1024 ragged requests once, each bin's
    Top-K entries within one request of the mean; every rank prints the same
    ``config``."""
    import json

    from qsa_b200.inputs import CONFIGS, ragged_lengths

    out = tmp_path / "plan.json"
    mp.start_processes(_plan_rank_main, args=(world, _free_port(), str(out)), nprocs=world, join=True,
                       start_method="spawn")
    everyone = json.loads(out.read_text())
    assert len(everyone) == world
    rows3 = [r["rows"]["3"] for r in everyone]
    assert [i for rr in rows3 for i in rr] == list(range(2048))
    rows4 = [r["rows"]["4"] for r in everyone]
    assert sorted(i for rr in rows4 for i in rr) == list(range(1024))
    lengths = ragged_lengths(CONFIGS[4], 1024, seed=0)
    loads = [int(lengths[rr].sum()) for rr in rows4]
    assert max(loads) - sum(loads) / world <= int(lengths.max())
    assert all(r["config"] == everyone[0]["config"] for r in everyone)
    assert everyone[0]["config"]["3"]["rows_per_gpu"] == 2048 // world
    assert everyone[0]["config"]["1"]["rows_total"] == 256 * world
