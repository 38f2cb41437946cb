"""Fused all-gather of the N-sharded wrapper on 2+ GPUs.

Two processes, one per GPU: each GEMM epilogue stores its rows into every
rank's full Y through CUDA IPC peer mappings (plain stores over NVLink, no
TMA on peer memory) and signals the per-rank arrival counters; the handles
are exchanged over a gloo group (no NCCL).  Every rank's result must equal,
bit for bit, the plain single-GPU GEMM of each rank's slab, for several
calls in a row (both buffers, growing counters).  Skipped with fewer than
two GPUs.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, shapes, errq):
    try:
        import datetime

        import torch
        import torch.distributed as dist

        import tinym_b200
        from oracle import fp8_oracle as orc
        from tinym_b200.sharded import ShardedFp8Gemm, shard_bounds

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=60))
        for (m_max, k, n, calls) in shapes:
            _, wq, _, sw, _ = orc.make_case(1, k, n, seed=n + k, dist="normal")
            w_full = torch.from_numpy(wq).to(dev).view(torch.float8_e4m3fn)
            g = ShardedFp8Gemm.from_full_weight(w_full)
            g.enable_fused_gather(m_max=16)
            for call in range(calls):
                m = 1 + (call * 7) % m_max
                xq, _, _, _, alpha = orc.make_case(m, k, 1, seed=100 * call + k, dist="normal")
                x = torch.from_numpy(xq).to(dev).view(torch.float8_e4m3fn)
                a = torch.from_numpy(alpha).to(dev)
                y = g.fused(x, a).clone()
                torch.cuda.synchronize()
                exp = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
                for r in range(world):
                    s0, s1 = shard_bounds(n, world, r)
                    if s1 > s0:
                        exp[:, s0:s1] = tinym_b200.gemm(x, w_full[s0:s1].contiguous(), a)
                assert torch.equal(y, exp), (rank, m, k, n, call)
                # every rank finishes reading before anyone starts the call after next
                dist.barrier()
            assert tinym_b200.device_status() == 0
            g.close_fused_gather()
        dist.destroy_process_group()
    except BaseException as e:  # report to the parent, which fails the test
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.parametrize("world", [2, 4])
def test_fused_allgather_matches_slab_gemms(world):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    # (m_max, K, N, calls): tile-aligned slabs, ragged N, and a K split
    shapes = [(9, 1024, 1024, 6), (16, 512, 1000, 5), (4, 6144, 5120, 4)]
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, shapes, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not alive, "a rank did not finish"
    assert not errs and all(p.exitcode == 0 for p in procs), errs
