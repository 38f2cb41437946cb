"""CPU: the N-sharded wrapper's host logic on world_size-2 gloo ranks.

The local GEMM is replaced by the CPU oracle (test infrastructure), so this
checks sharding, padding and the all-gather reassembly, not the kernel."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.parametrize("n,world", [(5120, 2), (16384, 8), (300, 2), (100, 4), (3, 2),
                                     (129, 3), (1, 2)])
def test_shard_bounds_cover_exactly(n, world):
    from tinym_b200.sharded import shard_bounds

    bounds = [shard_bounds(n, world, r) for r in range(world)]
    assert bounds[0][0] == 0 and bounds[-1][1] == n
    for (a0, b0), (a1, b1) in zip(bounds, bounds[1:]):
        assert b0 == a1 and a0 <= b0
    if -(-n // 128) >= world:
        assert all(a % 128 == 0 for a, _ in bounds)
        sizes = [b - a for a, b in bounds]
        assert max(sizes) - min(sizes) <= 128


def _worker(rank, world, port, m, k, n, q):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        import sys
        from pathlib import Path

        root = Path(__file__).resolve().parents[1]
        sys.path.insert(0, str(root))
        sys.path.insert(0, str(root / "sm120-fp8-gemm-submit_b200"))
        from oracle import fp8_oracle as orc
        from tinym_b200.sharded import ShardedFp8Gemm

        xq, wq, sx, sw, alpha = orc.make_case(m, k, n, seed=42, dist="normal")

        def cpu_gemm(x, w_local, a, out):
            ref = orc.reference(x.numpy(), w_local.numpy(), a.numpy())
            out.copy_(torch.from_numpy(ref).to(torch.bfloat16))
            return out

        g = ShardedFp8Gemm.from_full_weight(torch.from_numpy(wq), local_gemm=cpu_gemm)
        y = g(torch.from_numpy(xq), torch.from_numpy(alpha))
        full = orc.reference(xq, wq, alpha)
        rel = orc.max_rel_err(y.float().numpy(), full)
        q.put((rank, tuple(y.shape), rel, g.start, g.stop))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, "error", repr(e), 0, 0))


@pytest.mark.parametrize("m,k,n", [(9, 256, 640), (1, 128, 300), (16, 128, 5)])
def test_sharded_gather_gloo_world2(m, k, n):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, m, k, n, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, shape, rel, a, b in res:
        assert shape == (m, n), (rank, shape, rel)
        assert rel <= 4e-3
    spans = sorted((a, b) for _, _, _, a, b in res)
    assert spans[0][0] == 0 and spans[-1][1] == n and spans[0][1] == spans[1][0]


def test_fused_requires_enable():
    """fused() on a wrapper whose peer buffers are not mapped raises on the
    host (the epilogue would otherwise store to unmapped peer memory)."""
    import torch

    from tinym_b200.sharded import ShardedFp8Gemm

    g = ShardedFp8Gemm(torch.zeros(4, 16), 4, 0, 4)
    with pytest.raises(RuntimeError, match="not enabled"):
        g.fused(torch.zeros(1, 16), 1.0)


def _worker_refuse(rank, world, port, q):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        import sys
        from pathlib import Path

        root = Path(__file__).resolve().parents[1]
        sys.path.insert(0, str(root / "sm120-fp8-gemm-submit_b200"))
        from tinym_b200.sharded import ShardedFp8Gemm

        g = ShardedFp8Gemm.from_full_weight(torch.zeros(1, 16))  # N = 1 < world
        try:
            g.enable_fused_gather(device=torch.device("cpu"))
            outcome = "enabled"
        except ValueError as e:
            outcome = "refused" if "N >= world" in str(e) else repr(e)
        dist.barrier()  # every rank is still in step after the refusal
        q.put((rank, outcome))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e)))


def test_fused_gather_refused_on_every_rank_when_n_below_world():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_refuse, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res == [(0, "refused"), (1, "refused")]


def _worker_rank_leaves(rank, world, port, q):
    """One gathered call on every rank, then rank 1 leaves between steps (the
    process ends with nothing in flight) while rank 0 makes the next call."""
    import datetime
    import time

    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    outcome = "no result"
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=10))
        import sys
        from pathlib import Path

        root = Path(__file__).resolve().parents[1]
        sys.path.insert(0, str(root / "sm120-fp8-gemm-submit_b200"))
        from tinym_b200.sharded import ShardedFp8Gemm

        def cpu_gemm(x, w_local, a, out):  # stands in for the kernel
            out.copy_((x.float() @ w_local.float().t() * a).to(torch.bfloat16))
            return out

        w = torch.randn(256, 32)
        x = torch.randn(2, 32)
        g = ShardedFp8Gemm.from_full_weight(w, local_gemm=cpu_gemm)
        y = g(x, 1.0)
        assert tuple(y.shape) == (2, 256)
        dist.barrier()
        if rank == 1:
            outcome = "left"
        else:
            time.sleep(1.0)  # rank 1 is gone by now
            t0 = time.monotonic()
            try:
                g(x, 1.0)
                outcome = "no error"
            except Exception as e:  # the collective ends with an error
                outcome = f"error after {time.monotonic() - t0:.1f} s: {type(e).__name__}"
    except Exception as e:  # pragma: no cover - reported to the parent
        outcome = repr(e)
    q.put((rank, outcome))
    q.close()
    q.join_thread()
    os._exit(0)  # no teardown collective with a rank that has left


def test_rank_leaving_between_steps_ends_peers_next_gather_with_error():
    """Failure detection on the host: a rank that leaves between steps makes
    the next gathered call of the other rank raise (the process group's short
    timeout or the closed connection) instead of waiting for good."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_rank_leaves, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.exitcode is None:  # pragma: no cover - never expected
            p.kill()
        assert p.exitcode == 0
    assert res[1] == "left", res
    assert res[0].startswith("error after "), res
    assert float(res[0].split()[2]) < 30.0, res


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_bench_rank_slabs(world):
    """The multi-GPU bench's slab arithmetic: weak scaling keeps every rank's
    slab at the workload's N (the sharded GEMM grows), strong scaling splits
    the workload's N; the shard bounds of the sharded wrapper tile the
    GEMM's N exactly with those slabs at the official N."""
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import bench
    from tinym_b200.sharded import shard_bounds

    for n in (5120, 8192, 16384):
        n_local, n_total = bench.rank_slab(n, world, "weak")
        assert (n_local, n_total) == (n, n * world)
        assert [shard_bounds(n_total, world, r) for r in range(world)] == \
            [(r * n, (r + 1) * n) for r in range(world)]
        n_local, n_total = bench.rank_slab(n, world, "strong")
        assert n_local * world == n_total == n
    with pytest.raises(ValueError):
        bench.rank_slab(5120, 3, "strong")
    with pytest.raises(ValueError):
        bench.rank_slab(5120, world, "diagonal")


def test_bench_replay_sizes():
    """The bench times exactly K steps as CUDA-graph replays of at least 40
    launches (one replay below 80 steps), about five replays otherwise."""
    import bench

    for steps in (1, 20, 79, 80, 100, 200, 1000, 12345):
        sizes = bench.replay_sizes(steps)
        assert sum(sizes) == steps
        if steps < 80:
            assert sizes == [steps]
        else:
            assert min(sizes[:-1] or sizes) >= 40 and len(sizes) <= 6
    with pytest.raises(ValueError):
        bench.replay_sizes(0)
