"""Expert-parallel host logic on CPU with two gloo ranks (no GPU).

Each rank draws the same seeded global routing, takes its contiguous expert
shard (``shard_experts`` / ``shard_routing``, the split ``bench.py`` uses under
torchrun), computes its experts' weight gradients with the CPU oracle, and the
shards are gathered to rank 0, which checks them against the single-process
result expert by expert (exact: an expert's blocks never depend on other
experts). The max-over-ranks / sum-over-ranks reductions that ``bench.py``
applies to the per-rank times and FLOPs are checked on the same group.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

EXPERTS, TOP_K, HIDDEN, INTER, TOKENS = 8, 2, 64, 32, 512


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return int(s.getsockname()[1])


def _inputs(counts):
    rows = int(sum(counts))
    rng = np.random.Generator(np.random.PCG64(5))
    lhs = rng.standard_normal((rows, HIDDEN), dtype=np.float32) * np.float32(0.01)
    rhs = rng.standard_normal((rows, INTER), dtype=np.float32)
    return lhs, rhs


def _wgrad(counts, lhs, rhs):
    import wgrad_oracle as O

    cu = np.concatenate([[0], np.cumsum(np.asarray(counts, np.int64))]).astype(np.int64)
    meta = O.build_meta(cu)
    return O.ref_scaled_wgrad(O.quantize_1x128(lhs, meta), O.quantize_1x128(rhs, meta), meta)


def _worker(rank: int, world: int, port: int, route: str, q) -> None:
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    for p in (root / "sm90-fp8-wgrad_b200", root / "oracle", root):
        sys.path.insert(0, str(p))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench
        from sm90_fp8_wgrad.routing import make_routing, shard_experts, shard_routing

        routing = make_routing(tokens=TOKENS, experts=EXPERTS, top_k=TOP_K, route=route, seed=0)
        e0, e1 = shard_experts(EXPERTS, world, rank)
        local = shard_routing(routing, e0, e1)
        lhs, rhs = _inputs(routing.counts)
        cu = np.concatenate([[0], np.cumsum(routing.counts)])
        r0, r1 = int(cu[e0]), int(cu[e1])
        assert list(local.counts) == list(routing.counts[e0:e1])
        assert torch.equal(local.gather_idx, routing.gather_idx[r0:r1])
        shard = _wgrad(local.counts, lhs[r0:r1], rhs[r0:r1])

        gathered = [None] * world if rank == 0 else None
        dist.gather_object((e0, e1, shard), gathered, dst=0)
        cpu = torch.device("cpu")
        t_max = bench._max_over_ranks(float(rank + 1) * 1.5, world, cpu)
        f_sum = bench._sum_over_ranks(float(shard.sum(dtype=np.float64)), world, cpu)
        if rank == 0:
            full = _wgrad(routing.counts, lhs, rhs)
            spans = sorted((a, b) for a, b, _ in gathered)
            assert spans[0][0] == 0 and spans[-1][1] == EXPERTS
            assert all(spans[i][1] == spans[i + 1][0] for i in range(len(spans) - 1))
            for a, b, part in gathered:
                np.testing.assert_array_equal(part, full[a:b])
            assert t_max == pytest.approx(1.5 * world)
            assert f_sum == pytest.approx(float(full.sum(dtype=np.float64)), rel=1e-6)
        q.put((rank, "ok"))
    except Exception as exc:  # report to the parent instead of hanging it
        q.put((rank, repr(exc)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("route", ["uniform", "zipf"])
def test_expert_sharded_wgrad_two_gloo_ranks(route):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, route, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, status = q.get(timeout=240)
        results[rank] = status
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results == {r: "ok" for r in range(world)}, results


def _failing_worker(rank: int, world: int, port: int, q) -> None:
    import datetime

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        if rank == 1:
            raise RuntimeError("injected failure on rank 1")   # this rank never reaches the barrier
        dist.barrier()                                           # the timing barrier of bench.py
        q.put((rank, "ok"))
    except Exception as exc:
        q.put((rank, type(exc).__name__))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_failed_rank_is_detected_not_hung():
    """A rank that fails before the timing barrier: the other rank's barrier ends
    with an error after the process-group timeout instead of hanging, and the
    parent sees both failures (host-side failure detection; no GPU involved)."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, status = q.get(timeout=120)
        results[rank] = status
    for p in procs:
        p.join(timeout=60)
    assert results[1] == "RuntimeError"
    assert results[0] != "ok"
