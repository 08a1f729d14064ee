"""The multi-rank path of the benchmark harness on CPU ranks (gloo, world size 2; no GPU).

The GPU path shards tokens across ranks with no collective on the data path; NCCL only carries the
barrier, the max over ranks of the timings, and (in checking runs) the gather of outputs. Here the
same harness code runs on gloo ranks, with the oracle standing in for the kernels:
  * shard() gives contiguous, covering, balanced slices;
  * each rank's slice of a ragged batch, processed alone and gathered, equals the whole batch
    processed in one process, bit for bit (the ops are per token);
  * Dist.max returns the maximum over ranks and all_gather_object collects per-rank summaries;
  * a rank that fails before a collective makes the others' next collective fail within the process
    group timeout instead of hanging (failure detection on the host, no GPU involved).
"""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _env(rank: int, world: int, port: int) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    for p in (str(ROOT), str(ROOT / "tests")):
        if p not in sys.path:
            sys.path.insert(0, p)


def _worker_sharded_chain(rank: int, world: int, port: int, q) -> None:
    _env(rank, world, port)
    import datetime

    import torch.distributed as dist

    import bench
    import oracle

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        d = bench.Dist(backend="none")
        d.pg = True  # use the process group initialised above
        T, H, D, Hq, Hkv, I = 37, 64, 32, 2, 1, 48
        g = torch.Generator().manual_seed(0)
        x = torch.randn(T, H, generator=g).to(torch.bfloat16)
        r = torch.randn(T, H, generator=g).to(torch.bfloat16)
        w = torch.randn(H, generator=g).to(torch.bfloat16)
        qkv = torch.randn(T, (Hq + 2 * Hkv) * D, generator=g).to(torch.bfloat16)
        gu = torch.randn(T, 2 * I, generator=g).to(torch.bfloat16)
        cache = torch.randn(64, D, generator=g)
        pos = torch.randint(0, 64, (T,), generator=g).to(torch.int32)
        s, e = bench.shard(T, world, rank)
        xs, rs, qs = x[s:e].clone(), r[s:e].clone(), qkv[s:e].clone()
        oracle.fused_add_rmsnorm(xs, rs, w, 1e-5)
        oracle.apply_rope_with_cos_sin_cache_inplace(pos[s:e], qs[:, : Hq * D], qs[:, Hq * D: (Hq + Hkv) * D], D, cache)
        act = oracle.silu_and_mul(gu[s:e].contiguous())
        parts = d.gather_objects({"rank": rank, "x": xs, "r": rs, "qkv": qs, "act": act})
        slowest = d.max(float(rank + 1) * 0.5, "cpu")
        if rank == 0:
            xa, ra, qa = x.clone(), r.clone(), qkv.clone()
            oracle.fused_add_rmsnorm(xa, ra, w, 1e-5)
            oracle.apply_rope_with_cos_sin_cache_inplace(pos, qa[:, : Hq * D], qa[:, Hq * D: (Hq + Hkv) * D], D, cache)
            aa = oracle.silu_and_mul(gu)
            ok = all(torch.equal(torch.cat([p[k] for p in parts]).view(torch.int16), ref.view(torch.int16))
                     for k, ref in (("x", xa), ("r", ra), ("qkv", qa), ("act", aa)))
            q.put((ok, [p["rank"] for p in parts], slowest))
        d.barrier()
    finally:
        dist.destroy_process_group()


def _worker_rank_dies(rank: int, world: int, port: int, q) -> None:
    _env(rank, world, port)
    import datetime

    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    dist.barrier()
    if rank == 1:
        os._exit(0)  # leaves between steps, nothing in flight
    try:
        t = torch.ones(1)
        dist.all_reduce(t)
        q.put("no-error")
    except Exception as exc:  # the survivor's collective fails instead of hanging
        q.put(type(exc).__name__)
    finally:
        os._exit(0)


def test_shard_contiguous_and_balanced():
    import bench

    for total in (0, 1, 7, 4352, 4353):
        for world in (1, 2, 3, 8):
            spans = [bench.shard(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1


def test_sharded_ranks_match_whole_batch():
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_sharded_chain, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    ok, ranks, slowest = q.get()
    assert ok and ranks == [0, 1] and slowest == 1.0


def test_dead_rank_fails_the_next_collective():
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_rank_dies, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert not any(p.is_alive() for p in procs)
    assert q.get() != "no-error"


def test_weak_scaling_slices_are_whole_mixed_steps():
    from mas_b200 import workloads as wl

    ids, pos = wl.chain_host_inputs(replicas=4)
    per = ids.shape[0] // 4
    one, one_pos = wl.chain_host_inputs(replicas=1)
    assert per == 4352 and torch.equal(ids[:per], one) and torch.equal(pos[:per], one_pos)
    for r in range(4):
        sl = pos[r * per: (r + 1) * per]
        assert torch.equal(sl[256 + 1: 256 + 2048] - sl[256: 256 + 2047], torch.ones(2047, dtype=torch.int32))
