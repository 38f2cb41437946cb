"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle.

Bar (build contract): max harness-relative error <= 4e-3 and zero elements
above 0.02, against the FP32 oracle of fp8_gemm_task_harness.py:63-65
(restated in oracle/fp8_oracle.py).  Every test calls the kernels through
libtinym_b200.so (ctypes) or through the torch op that wraps it.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

OFFICIAL = [(1, 5120, 16384), (9, 5120, 16384), (1, 6144, 5120), (9, 6144, 5120),
            (1, 5120, 8192), (9, 5120, 8192)]
MAX_REL = 4e-3


def _to_dev(codes: np.ndarray, device):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(codes)).to(device)
    return t.view(torch.float8_e4m3fn)


def _check(oracle, out_bf16, xq, wq, alpha, tol=MAX_REL):
    import torch

    out = out_bf16.float().cpu().numpy()
    ref = oracle.reference(xq, wq, alpha)
    rel = oracle.max_rel_err(out, ref)
    mism = oracle.mismatches(out, ref)
    assert np.isfinite(out).all(), "non-finite output"
    assert rel <= tol, f"max_rel {rel:.3e} > {tol}"
    assert mism == 0, f"{mism} mismatches above 0.02"
    return rel


def _run(x, w, alpha_dev, plan=None, out=None):
    import tinym_b200

    return tinym_b200.gemm(x, w, alpha_dev, plan=plan, out=out)


@pytest.mark.parametrize("m,k,n", OFFICIAL)
def test_official_points_normal(cuda_device, oracle, m, k, n):
    import torch

    xq, wq, sx, sw, alpha = oracle.make_case(m, k, n, seed=1000 + m + k + n, dist="normal")
    x, w = _to_dev(xq, cuda_device), _to_dev(wq, cuda_device)
    a = torch.from_numpy(alpha).to(cuda_device)
    y = _run(x, w, a)
    torch.cuda.synchronize()
    _check(oracle, y, xq, wq, alpha)


@pytest.mark.parametrize("m,k,n", OFFICIAL)
def test_official_points_harness_data(cuda_device, oracle, m, k, n):
    """The harness's own make_case on the GPU (CUDA generator, seed
    20260822+m+k+n, fp8_gemm_task_harness.py:47-60,124), through the
    drop-in candidate_kernel.fp8_gemm, against the oracle and against the
    harness's self-calibrating bar relative to torch._scaled_mm."""
    import torch

    import candidate_kernel

    seed = 20260822 + m + k + n
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn(m, k, device="cuda", dtype=torch.float32, generator=g) * 2.0
    wf = torch.randn(n, k, device="cuda", dtype=torch.float32, generator=g) * 0.03
    a.view(-1)[::37] = 30.0
    a.view(-1)[17::74] = -30.0
    wf.view(-1)[::1531] = 25.0
    wf.view(-1)[733::3062] = -25.0
    # quantise on the CPU oracle (bit-exact with the harness's quantiser)
    xq, sx = oracle.quantize_per_tensor(a.cpu().numpy())
    wq, sw = oracle.quantize_per_tensor(wf.cpu().numpy())
    alpha = (sx * sw).astype(np.float32)
    x, w = _to_dev(xq, cuda_device), _to_dev(wq, cuda_device)
    al = torch.from_numpy(alpha).to(cuda_device)
    out = candidate_kernel.fp8_gemm(x, candidate_kernel.prepare_weights(w), al)
    assert out.dtype == torch.bfloat16 and tuple(out.shape) == (m, n)
    cand_rel = _check(oracle, out, xq, wq, alpha)
    base = torch._scaled_mm(x, w.t(), scale_a=torch.from_numpy(sx).to(cuda_device),
                            scale_b=torch.from_numpy(sw).to(cuda_device),
                            out_dtype=torch.bfloat16)
    base_rel = oracle.max_rel_err(base.float().cpu().numpy(), oracle.reference(xq, wq, alpha))
    assert oracle.harness_bar(cand_rel, base_rel), (cand_rel, base_rel)


@pytest.mark.parametrize("dist", ["uniform", "student_t3"])
@pytest.mark.parametrize("k,n", [(6144, 5120), (5120, 8192), (5120, 16384)])
def test_m_sweep(cuda_device, oracle, dist, k, n):
    """M = 1..16 on each (K, N): the M-row problem uses the first M rows of
    one quantised 16-row X (same scale), so one oracle call covers all M."""
    import torch

    xq, wq, sx, sw, alpha = oracle.make_case(16, k, n, seed=7 + k + n, dist=dist)
    ref = oracle.reference(xq, wq, alpha)
    w = _to_dev(wq, cuda_device)
    a = torch.from_numpy(alpha).to(cuda_device)
    for m in range(1, 17):
        x = _to_dev(xq[:m], cuda_device)
        y = _run(x, w, a).float().cpu().numpy()
        assert np.isfinite(y).all()
        rel = oracle.max_rel_err(y, ref[:m])
        assert rel <= MAX_REL, (m, rel)
        assert oracle.mismatches(y, ref[:m]) == 0, m


def test_golden_fixtures(cuda_device, oracle, golden_cases):
    """The reference's own outputs (tests/golden) reproduced by the kernel."""
    import torch

    for c in golden_cases:
        x, w = _to_dev(c["aq"], cuda_device), _to_dev(c["wq"], cuda_device)
        y = _run(x, w, torch.from_numpy(c["alpha"]).to(cuda_device)).float().cpu().numpy()
        assert oracle.max_rel_err(y, c["ref"]) <= MAX_REL
        assert oracle.mismatches(y, c["ref"]) == 0
        # the kernel's BF16 output differs from the reference's BF16 rounding
        # of its FP32 oracle only where FP32 summation order moves a tie.
        diff = np.count_nonzero(oracle.bf16_round(y) != c["ref_bf16"])
        assert diff <= max(2, y.size // 200), (c["m"], c["k"], c["n"], diff)


@pytest.mark.parametrize("m,k,n", [(1, 16, 1), (1, 48, 127), (3, 144, 129), (16, 272, 200),
                                   (9, 1040, 300), (2, 4096, 1), (13, 128, 1000),
                                   (16, 8192, 640), (5, 2064, 4100)])
def test_ragged_shapes(cuda_device, oracle, m, k, n):
    """K not a multiple of 128 (TMA zero fill), N not a multiple of 128,
    tiny N and K; output prefilled with NaN to prove every element is written."""
    import torch

    xq, wq, sx, sw, alpha = oracle.make_case(m, k, n, seed=m * 31 + k + n, dist="harness")
    x, w = _to_dev(xq, cuda_device), _to_dev(wq, cuda_device)
    out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    _run(x, w, torch.from_numpy(alpha).to(cuda_device), out=out)
    _check(oracle, out, xq, wq, alpha)


@pytest.mark.parametrize("m,k,n", [(9, 5120, 2048), (1, 5120, 2048), (9, 5120, 4096),
                                   (9, 6144, 640), (16, 5120, 1024)])
def test_sharded_slab_shapes(cuda_device, oracle, m, k, n):
    """The per-rank slabs of the N-sharded bench (16384 / 8 or / 4, 5120 / 8):
    the dispatch's K split is large there, and when the device cannot hold
    every cluster at once the launcher shrinks the split to the next value
    that still gives every CTA of a cluster some K."""
    import torch

    xq, wq, sx, sw, alpha = oracle.make_case(m, k, n, seed=m * 7 + n, dist="normal")
    x, w = _to_dev(xq, cuda_device), _to_dev(wq, cuda_device)
    out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    _run(x, w, torch.from_numpy(alpha).to(cuda_device), out=out)
    _check(oracle, out, xq, wq, alpha)


@pytest.mark.parametrize("m,k,n", [(9, 5120, 2048), (1, 6144, 5120), (9, 5120, 16384)])
def test_launch_plan_is_what_runs(cuda_device, oracle, m, k, n):
    """tinym_launch_plan reports the plan a call without a plan runs: the
    table's plan, with the K split lowered where the device cannot hold
    every cluster; running it explicitly gives the same bits."""
    import torch

    import tinym_b200

    sms = torch.cuda.get_device_properties(cuda_device).multi_processor_count
    table = tinym_b200.select_plan(m, n, k, sms)
    lp = tinym_b200.launch_plan(m, n, k)
    assert lp.split_k <= table.split_k and lp.block_k == table.block_k
    assert tinym_b200.max_active_clusters(m, n, k, lp) >= lp.tiles_n
    if tinym_b200.max_active_clusters(m, n, k, table) >= table.tiles_n:
        assert lp.as_dict() == table.as_dict()
    xq, wq, sx, sw, alpha = oracle.make_case(m, k, n, seed=m + n, dist="normal")
    x, w = _to_dev(xq, cuda_device), _to_dev(wq, cuda_device)
    a = torch.from_numpy(alpha).to(cuda_device)
    y_default = _run(x, w, a)
    y_plan = _run(x, w, a, plan=lp)
    assert torch.equal(y_default, y_plan)
    _check(oracle, y_default, xq, wq, alpha)


def _valid(tinym_b200, m, k, n, plan):
    try:
        tinym_b200.check_plan(m, n, k, plan)
        return True
    except tinym_b200.TinymError:
        return False


def _plans_for(tinym_b200, m, k, n):
    plans = []
    kb = (k + 127) // 128
    for split in (1, 2, 3, 4, 5, 6, 7, 8):
        per = (kb + split - 1) // split
        if (split - 1) * per >= kb:
            continue
        for stages in (2, 4, 7):
            for mma_n in ((8, 16) if m <= 8 else (16,)):
                for bk in ((128, 256, 512) if k % 128 == 0 else (128,)):
                    for tm in (64, 128):
                        plans.append(tinym_b200.make_plan(tinym_b200.KERNEL_TC, split, stages,
                                                          mma_n, block_k=bk, tile_m=tm))
            if m == 1:
                for cw in (4, 8):
                    plans.append(tinym_b200.make_plan(tinym_b200.KERNEL_SIMT_M1, split, stages,
                                                      0, cw))
    return plans


@pytest.mark.parametrize("m,k,n", [(1, 1024, 384), (7, 1152, 256), (16, 896, 300), (9, 1040, 200)])
def test_explicit_plans(cuda_device, oracle, m, k, n):
    """Every kernel family, split-K cluster size, ring depth and MMA N."""
    import torch

    import tinym_b200

    xq, wq, sx, sw, alpha = oracle.make_case(m, k, n, seed=99 + m, dist="normal")
    x, w = _to_dev(xq, cuda_device), _to_dev(wq, cuda_device)
    a = torch.from_numpy(alpha).to(cuda_device)
    ran = 0
    for plan in _plans_for(tinym_b200, m, k, n):
        try:
            tinym_b200.check_plan(m, n, k, plan)
        except tinym_b200.TinymError as e:
            assert e.status == 7  # e.g. a ring too deep for the shared memory
            continue
        out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda_device)
        _run(x, w, a, plan=plan, out=out)
        _check(oracle, out, xq, wq, alpha)
        ran += 1
    assert ran >= 10


@pytest.mark.parametrize("m,k,n", [(1, 6144, 5120), (9, 5120, 8192)])
def test_simt_m1_and_splits_full_size(cuda_device, oracle, m, k, n):
    import torch

    import tinym_b200

    xq, wq, sx, sw, alpha = oracle.make_case(m, k, n, seed=5, dist="normal")
    x, w = _to_dev(xq, cuda_device), _to_dev(wq, cuda_device)
    a = torch.from_numpy(alpha).to(cuda_device)
    plans = [tinym_b200.make_plan(tinym_b200.KERNEL_TC, s, st, 16, block_k=bk, tile_m=tm)
             for s in (1, 2, 4, 8) for (st, bk) in ((6, 128), (5, 256), (3, 512))
             for tm in (64, 128)]
    plans = [p for p in plans if _valid(tinym_b200, m, k, n, p)]
    if m == 1:
        plans += [tinym_b200.make_plan(tinym_b200.KERNEL_SIMT_M1, s, 6, 0, cw)
                  for s in (1, 3) for cw in (4, 8)]
    for plan in plans:
        _check(oracle, _run(x, w, a, plan=plan), xq, wq, alpha)


def test_deterministic(cuda_device, oracle):
    """Split-K reduces in fixed K order: repeated runs are bit-identical."""
    import torch

    xq, wq, sx, sw, alpha = oracle.make_case(9, 6144, 5120, seed=3, dist="normal")
    x, w = _to_dev(xq, cuda_device), _to_dev(wq, cuda_device)
    a = torch.from_numpy(alpha).to(cuda_device)
    y0 = _run(x, w, a)
    for _ in range(5):
        assert torch.equal(_run(x, w, a).view(torch.int16), y0.view(torch.int16))


def test_host_alpha_and_ldy(cuda_device, oracle):
    """tinym_fp8_gemm (x_scale, w_scale by value) and a strided Y slab."""
    import torch

    import tinym_b200

    m, k, n = 5, 640, 384
    xq, wq, sx, sw, alpha = oracle.make_case(m, k, n, seed=8, dist="normal")
    x, w = _to_dev(xq, cuda_device), _to_dev(wq, cuda_device)
    y = torch.empty((m, n), dtype=torch.bfloat16, device=cuda_device)
    lib = tinym_b200.capi()
    st = lib.tinym_fp8_gemm(x.data_ptr(), w.data_ptr(), y.data_ptr(), m, n, k, float(sx[0]),
                            float(sw[0]), torch.cuda.current_stream().cuda_stream)
    assert st == 0
    _check(oracle, y, xq, wq, alpha)
    wide = torch.full((m, 3 * n), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    tinym_b200.gemm_ptr(x.data_ptr(), w.data_ptr(), wide[:, n:].data_ptr(), m, n, k, ldy=3 * n,
                        alpha=float(alpha[0]), stream=torch.cuda.current_stream().cuda_stream)
    _check(oracle, wide[:, n:2 * n], xq, wq, alpha)
    assert torch.isnan(wide[:, :n].float()).all() and torch.isnan(wide[:, 2 * n:].float()).all()


def test_torch_op_schemas(cuda_device, oracle):
    """torch.ops.sm120_fp8_gemm.run keeps the reference schema (float alpha)."""
    import torch

    import candidate_kernel

    candidate_kernel.build()
    xq, wq, sx, sw, alpha = oracle.make_case(9, 6144, 5120, seed=4, dist="harness")
    x, w = _to_dev(xq, cuda_device), _to_dev(wq, cuda_device)
    y1 = torch.ops.sm120_fp8_gemm.run(x, w, float(alpha[0]))
    y2 = torch.ops.sm120_fp8_gemm.run_alpha_tensor(x, w, torch.from_numpy(alpha).to(cuda_device))
    assert torch.equal(y1.view(torch.int16), y2.view(torch.int16))
    _check(oracle, y1, xq, wq, alpha)


def test_error_paths(cuda_device, oracle):
    """Rejected inputs raise before any launch (mirrors check_inputs,
    src/torch_candidate_extension.cu:17-46, and the C ABI status codes)."""
    import torch

    import candidate_kernel
    import tinym_b200

    dev = cuda_device
    f8 = torch.float8_e4m3fn
    a = torch.zeros(17, 256, device=dev).to(f8)
    b = torch.zeros(128, 256, device=dev).to(f8)
    al = torch.ones(1, device=dev)
    with pytest.raises(RuntimeError, match="UNSUPPORTED_SHAPE"):
        candidate_kernel.fp8_gemm(a, b, al)
    with pytest.raises(RuntimeError, match="same K"):
        candidate_kernel.fp8_gemm(torch.zeros(1, 128, device=dev).to(f8), b, al)
    with pytest.raises(RuntimeError, match="float8_e4m3fn"):
        candidate_kernel.fp8_gemm(torch.zeros(1, 256, device=dev, dtype=torch.bfloat16), b, al)
    with pytest.raises(ValueError):
        candidate_kernel.fp8_gemm(b[:1], b, al.double())
    # non-finite alpha: the reference op's "alpha must be finite"
    # (src/torch_candidate_extension.cu:30), also after an in-place change of
    # an alpha tensor that was already accepted
    for v in (float("nan"), float("inf")):
        with pytest.raises(RuntimeError, match="alpha must be finite"):
            candidate_kernel.fp8_gemm(b[:1], b, torch.full((1,), v, device=dev))
    ok = torch.ones(1, device=dev)
    candidate_kernel.fp8_gemm(b[:1], b, ok)
    ok.fill_(float("nan"))
    with pytest.raises(RuntimeError, match="alpha must be finite"):
        candidate_kernel.fp8_gemm(b[:1], b, ok)
    with pytest.raises(RuntimeError, match="alpha must be finite"):
        torch.ops.sm120_fp8_gemm.run(b[:1], b, float("nan"))
    with pytest.raises(RuntimeError, match="UNSUPPORTED_SHAPE"):
        candidate_kernel.fp8_gemm(torch.zeros(1, 40, device=dev).to(f8),
                                  torch.zeros(8, 40, device=dev).to(f8), al)
    raw = torch.zeros(2 * 256 + 16, device=dev, dtype=torch.uint8)
    x_mis = raw[1:257].view(f8).view(1, 256)
    y = torch.empty(1, 128, device=dev, dtype=torch.bfloat16)
    with pytest.raises(tinym_b200.TinymError, match="MISALIGNED"):
        tinym_b200.gemm_ptr(x_mis.data_ptr(), b.data_ptr(), y.data_ptr(), 1, 128, 256)
    bad = tinym_b200.make_plan(tinym_b200.KERNEL_SIMT_M1, 1, 4, 0, 4)
    with pytest.raises(tinym_b200.TinymError, match="BAD_PLAN"):
        tinym_b200.gemm(torch.zeros(2, 256, device=dev).to(f8), b, 1.0, plan=bad)
    assert tinym_b200.device_status() == 0


def test_static_w_flag_honours_x_dependency(cuda_device, oracle):
    """TINYM_FLAG_STATIC_W streams W before the dependency wait but must still
    read X only after the kernel that writes it: each GEMM follows a copy
    kernel that rewrites X, back to back and inside a CUDA graph."""
    import torch

    import tinym_b200

    m, k, n = 9, 6144, 5120
    _, wq, _, _, alpha = oracle.make_case(m, k, n, seed=77, dist="normal")
    w = _to_dev(wq, cuda_device)
    a = torch.from_numpy(alpha).to(cuda_device)
    xq_list = [oracle.make_case(m, k, 1, seed=300 + i, dist="normal")[0] for i in range(4)]
    xs = [_to_dev(xq, cuda_device) for xq in xq_list]
    # the flag changes the dispatch (more, smaller CTAs), so the bit-exact
    # reference is the same plan run without the flag
    plan = tinym_b200.select_plan(m, n, k, torch.cuda.get_device_properties(cuda_device)
                                  .multi_processor_count, static_w=True)
    refs = [tinym_b200.gemm(x, w, a, plan=plan) for x in xs]
    for xq, r in zip(xq_list, refs):
        _check(oracle, r, xq, wq, alpha)
    x = torch.empty_like(xs[0])
    y = torch.empty((m, n), dtype=torch.bfloat16, device=cuda_device)
    for rep in range(3):
        for i in range(4):
            x.view(torch.uint8).copy_(xs[i].view(torch.uint8))
            tinym_b200.gemm(x, w, a, out=y, static_w=True)
            assert torch.equal(y, refs[i]), (rep, i)
    # the same chain captured in a graph: copy -> GEMM, four times per replay
    outs = [torch.empty_like(y) for _ in range(4)]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        tinym_b200.gemm(x, w, a, out=outs[0], static_w=True)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(4):
            x.view(torch.uint8).copy_(xs[i].view(torch.uint8))
            tinym_b200.gemm(x, w, a, out=outs[i], static_w=True)
    for _ in range(3):
        for o in outs:
            o.zero_()
        g.replay()
        torch.cuda.synchronize()
        for i in range(4):
            assert torch.equal(outs[i], refs[i])
    assert tinym_b200.device_status() == 0
    lib = tinym_b200.capi()
    assert lib.tinym_fp8_gemm_ex2(x.data_ptr(), w.data_ptr(), y.data_ptr(), n, m, n, k,
                                  a.data_ptr(), 0.0, None, 2, None) == 1  # unknown flag
