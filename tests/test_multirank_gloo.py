"""The multi-GPU host logic of bench.py, on CPU: two and four gloo ranks run the
helpers the NCCL ranks run on B200s.  Each rank takes its own shard of the batch (weak
scaling: the same amount of work, different items); the only data-path collective is the
all_gather of the ranks' outputs; the timed region is bracketed by the barrier and reduced
to the slowest rank's time; the reported value is the units all ranks processed over that
time.  The strong-scaling leg splits one fixed global batch into contiguous ranges.  The
reference arm runs on rank 0 alone.
"""
import argparse
import datetime
import json
import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
import bench  # noqa: E402


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_worker(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        barrier, max_over_ranks = bench.make_rank_sync(world, torch.device("cpu"))
        batch, seq, vocab, layers = 2, 16, 1000, 12
        ids = bench.rank_shard_ids(rank, batch, seq, vocab)
        shards = [torch.empty_like(ids) for _ in range(world)]
        dist.all_gather(shards, ids)
        assert all(tuple(sh.shape) == (batch, seq) for sh in shards)      # same work per rank
        assert not torch.equal(shards[0], shards[1])                       # on items of its own
        assert torch.equal(ids, bench.rank_shard_ids(rank, batch, seq, vocab))   # a function of the rank
        barrier()
        ms = 17.5 if rank == 1 else 10.0 + rank * 0.5                     # rank 1 is the slow one
        slowest = max_over_ranks(ms)
        assert slowest == 17.5
        rate = bench.whole_job_rate(world, batch * seq * layers, slowest)
        assert abs(rate - world * batch * seq * layers / 17.5e-3) <= 1e-9 * rate
        # the data-path collective: every rank receives all ranks' outputs, in rank order
        out = torch.full((batch, 3), float(rank))
        got = bench.gather_outputs(world, out)
        assert tuple(got.shape) == (world * batch, 3)
        assert torch.equal(got, torch.cat([torch.full((batch, 3), float(r)) for r in range(world)]))
        # strong scaling: a fixed global batch split into contiguous, disjoint, covering ranges
        lo, hi = bench.strong_shard(rank, world, 256)
        ranges = [torch.tensor([lo, hi]) for _ in range(world)]
        dist.all_gather(ranges, torch.tensor([lo, hi]))
        assert [tuple(r.tolist()) for r in ranges] == [(i * 256 // world, (i + 1) * 256 // world)
                                                       for i in range(world)]
        barrier()
    finally:
        dist.destroy_process_group()


def _segment_worker(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        bench._load_package()      # registers the package in this spawned process
        from verace_v1_b200 import ranges
        g = torch.Generator().manual_seed(7)
        Ts = [torch.randn(2, 3, 5, 5, generator=g, dtype=torch.float64) for _ in range(world)]
        Tc = [torch.randn(2, 5, 5, generator=g, dtype=torch.complex128) for _ in range(world)]
        S0 = torch.randn(2, 3, 5, 5, generator=g, dtype=torch.float64)
        S0c = torch.randn(2, 5, 5, generator=g, dtype=torch.complex128)
        # the state entering this rank's segment: the earlier segments' products, in order
        S = ranges._prior_product(Ts[rank], S0, dist.group.WORLD)
        Sc = ranges._prior_product(Tc[rank], S0c, dist.group.WORLD)
        want, wantc = S0, S0c
        for j in range(rank):
            want, wantc = Ts[j] @ want, Tc[j] @ wantc
        assert torch.allclose(S, want, rtol=1e-12, atol=1e-12)
        assert torch.allclose(Sc, wantc, rtol=1e-12, atol=1e-12)
        # a segment's product of its ranges, newest on the left
        P = torch.randn(2, 4, 3, 3, generator=g, dtype=torch.float64)
        T = ranges._segment_product(P)
        assert torch.allclose(T, P[:, 3] @ P[:, 2] @ P[:, 1] @ P[:, 0])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sequence_segments_carry_state_across_gloo_ranks(world):
    mp.start_processes(_segment_worker, args=(world, _free_port()), nprocs=world, start_method="spawn", join=True)


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_ranks_shard_and_time_like_the_nccl_ranks(world):
    mp.start_processes(_rank_worker, args=(world, _free_port()), nprocs=world, start_method="spawn", join=True)


def test_single_rank_needs_no_process_group():
    barrier, max_over_ranks = bench.make_rank_sync(1, torch.device("cpu"))
    barrier()
    assert max_over_ranks(3.25) == 3.25
    t = torch.arange(6.0).view(2, 3)
    assert bench.gather_outputs(1, t) is t
    assert bench.strong_shard(0, 1, 256) == (0, 256)
    assert [bench.strong_shard(r, 8, 256) for r in (0, 7)] == [(0, 32), (224, 256)]
    assert bench.whole_job_rate(1, 1000, 2.0) == 500000.0
    assert torch.equal(bench.rank_shard_ids(0, 3, 5, 50), bench.rank_shard_ids(0, 3, 5, 50))


def _fake_sample(calls):
    def sample(tokens):
        calls.append(tokens)
        return {"value": 1.0, "unit": bench.UNIT, "cores": 1, "kind": "port", "sample": "fake"}
    return sample


def test_reference_arm_runs_on_rank_zero_only(monkeypatch, capsys):
    args = argparse.Namespace(warmup=1, steps=2, ref_tokens=4)
    calls = []
    monkeypatch.setattr(bench, "cpu_sample", _fake_sample(calls))
    monkeypatch.setenv("WORLD_SIZE", "2")
    monkeypatch.setenv("RANK", "1")
    bench.run_reference(args)
    assert calls == [] and capsys.readouterr().out == ""                  # no work, no line
    monkeypatch.setenv("RANK", "0")
    bench.run_reference(args)
    assert calls == [4, 4, 4]                                              # warm-up + 2 timed steps
    line = json.loads(capsys.readouterr().out.strip())
    assert line["impl"] == "reference" and line["n_gpus"] == 2 and line["steps"] == 2
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["kind"] == "port"
