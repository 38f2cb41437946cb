"""Fused all-gather of the N-sharded wrapper on 2+ GPUs.

Two processes, one per GPU: each GEMM epilogue stores its rows into every
rank's full Y through CUDA IPC peer mappings (plain stores over NVLink, no
TMA on peer memory) and signals the per-rank arrival counters; the handles
are exchanged over a gloo group (no NCCL).  Every rank's gathered Y must
meet the oracle bar against the FP32 oracle of the whole problem and equal,
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
                xq, _, sx, _, _ = orc.make_case(m, k, 1, seed=100 * call + k, dist="normal")
                alpha = (sx * sw).astype(np.float32).reshape(1)
                x = torch.from_numpy(xq).to(dev).view(torch.float8_e4m3fn)
                a = torch.from_numpy(alpha).to(dev)
                y = g.fused(x, a).clone()
                torch.cuda.synchronize()
                # the gathered Y against the FP32 oracle of the whole problem
                out = y.float().cpu().numpy()
                ref = orc.reference(xq, wq, alpha)
                assert orc.max_rel_err(out, ref) <= orc.MAX_REL_TOL, (rank, m, k, n, call)
                assert orc.mismatches(out, ref) == 0, (rank, m, k, n, call)
                # and bit for bit against the single-GPU GEMM of every slab
                exp = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
                for r in range(world):
                    s0, s1 = shard_bounds(n, world, r)
                    if s1 > s0:
                        exp[:, s0:s1] = tinym_b200.gemm(x, w_full[s0:s1].contiguous(), a)
                assert torch.equal(y, exp), (rank, m, k, n, call)
                # every rank has read this call's Y before anyone starts its next call
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


def _single_rank_desc(y_full, counter, m, n, target):
    import tinym_b200

    d = tinym_b200.GatherDesc()
    d.world, d.rank, d.n_full, d.col0 = 1, 0, n, 0
    d.y_full[0] = y_full.data_ptr()
    d.flag[0] = counter.data_ptr()
    d.target = target
    return d


def test_fused_gather_epilogue_single_rank(cuda_device, oracle):
    """World size 1: the fused-gather epilogue (store into the full Y, count,
    wait) gives the plain GEMM's bits, call after call."""
    import torch

    import tinym_b200

    k, n = 2048, 1000
    _, wq, _, sw, _ = oracle.make_case(1, k, n, seed=9, dist="normal")
    w = torch.from_numpy(wq).to(cuda_device).view(torch.float8_e4m3fn)
    y_full = torch.empty((16, n), dtype=torch.bfloat16, device=cuda_device)
    counter = torch.zeros(1, dtype=torch.int64, device=cuda_device)
    total = 0
    for call, m in enumerate((1, 9, 16, 4)):
        xq, _, sx, _, _ = oracle.make_case(m, k, 1, seed=call, dist="normal")
        alpha = (sx * sw).astype(np.float32).reshape(1)
        x = torch.from_numpy(xq).to(cuda_device).view(torch.float8_e4m3fn)
        a = torch.from_numpy(alpha).to(cuda_device)
        total += m * n
        d = _single_rank_desc(y_full, counter, m, n, total)
        tinym_b200.gemm_allgather_ptr(x.data_ptr(), w.data_ptr(), m, n, k, d,
                                      alpha_ptr=a.data_ptr(),
                                      stream=torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        out = y_full[:m].float().cpu().numpy()
        ref = oracle.reference(xq, wq, alpha)
        assert oracle.max_rel_err(out, ref) <= oracle.MAX_REL_TOL
        assert oracle.mismatches(out, ref) == 0
        assert torch.equal(y_full[:m], tinym_b200.gemm(x, w, a))
        assert int(counter.item()) == total
    assert tinym_b200.device_status() == 0


def test_fused_gather_wait_timeout_reports(cuda_device, oracle):
    """A counter that never reaches its target: the GEMM's bounded wait gives
    up (1 s), sets bit 0x40 of the device error word and the context stays
    usable (no fault, no hang)."""
    import torch

    import tinym_b200

    k, n, m = 1024, 512, 9
    xq, wq, _, _, alpha = oracle.make_case(m, k, n, seed=4, dist="normal")
    x = torch.from_numpy(xq).to(cuda_device).view(torch.float8_e4m3fn)
    w = torch.from_numpy(wq).to(cuda_device).view(torch.float8_e4m3fn)
    a = torch.from_numpy(alpha).to(cuda_device)
    y_full = torch.empty((m, n), dtype=torch.bfloat16, device=cuda_device)
    counter = torch.zeros(1, dtype=torch.int64, device=cuda_device)
    d = _single_rank_desc(y_full, counter, m, n, m * n + 1)  # one element never arrives
    tinym_b200.gemm_allgather_ptr(x.data_ptr(), w.data_ptr(), m, n, k, d,
                                  alpha_ptr=a.data_ptr(),
                                  stream=torch.cuda.current_stream().cuda_stream)
    assert tinym_b200.device_status() & 0x40
    assert tinym_b200.device_status() == 0  # read-and-clear
    assert torch.equal(y_full, tinym_b200.gemm(x, w, a))  # the rows themselves were stored
    assert tinym_b200.device_status() == 0
