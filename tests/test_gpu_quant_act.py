"""GPU tests of the fused activation path (quantise prologue + GEMM).

tinym_fp8_gemm_quant_act quantises a BF16 / FP32 activation per tensor on
the device -- the harness's quantize_per_tensor (fp8_gemm_task_harness.py:
41-44), restated in oracle/fp8_oracle.py -- and runs the GEMM on the codes.
The codes, x_scale and alpha must equal the oracle's bit for bit, and Y must
equal the plain GEMM on those codes bit for bit (same kernel arithmetic).
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _activation(m, k, seed, kind):
    rng = np.random.default_rng(seed)
    if kind == "spiky":  # harness make_case: 2*N(0,1) with planted +-30
        x = (rng.standard_normal((m, k), dtype=np.float32) * 2.0).astype(np.float32)
        f = x.reshape(-1)
        f[::37] = 30.0
        f[17::74] = -30.0
    elif kind == "tiny":  # amax/448 below 1e-12: the scale clamps
        x = (rng.standard_normal((m, k), dtype=np.float32) * 1e-10).astype(np.float32)
    elif kind == "zeros":
        x = np.zeros((m, k), dtype=np.float32)
    else:
        x = rng.standard_normal((m, k), dtype=np.float32)
    return x


def _run(oracle, cuda_device, m, k, n, dtype, kind, plan=None, seed=3):
    import torch

    import tinym_b200

    x32 = _activation(m, k, seed + m + k, kind)
    x = torch.from_numpy(x32).to(cuda_device).to(dtype)
    xw = x.float().cpu().numpy()  # the values the device sees (BF16-rounded)
    _, wq, _, sw, _ = oracle.make_case(1, k, n, seed=seed + n, dist="normal")
    w = torch.from_numpy(wq).to(cuda_device).view(torch.float8_e4m3fn)
    w_scale = torch.from_numpy(sw.astype(np.float32)).to(cuda_device)
    y, ws = tinym_b200.gemm_quant_act(x, w, w_scale, plan=plan)
    torch.cuda.synchronize()
    wsh = ws.cpu().numpy()
    codes = wsh[256:256 + m * k].reshape(m, k)
    hdr = wsh[:8].view(np.float32)
    xq_ref, sx_ref = oracle.quantize_per_tensor(xw)
    return x, w, w_scale, y, codes, hdr, xq_ref, sx_ref, wq, sw


@pytest.mark.parametrize("dtype_name", ["bfloat16", "float32"])
@pytest.mark.parametrize("m,k,n,kind", [(1, 6144, 5120, "normal"), (9, 6144, 5120, "spiky"),
                                        (16, 5120, 1024, "normal"), (3, 144, 129, "spiky"),
                                        (9, 1040, 300, "tiny"), (4, 256, 200, "zeros"),
                                        (1, 16, 1, "normal")])
def test_quant_act_bit_exact(cuda_device, oracle, dtype_name, m, k, n, kind):
    import torch

    import tinym_b200

    dtype = getattr(torch, dtype_name)
    x, w, w_scale, y, codes, hdr, xq_ref, sx_ref, wq, sw = _run(
        oracle, cuda_device, m, k, n, dtype, kind)
    assert np.array_equal(codes, xq_ref), "E4M3 codes differ from quantize_per_tensor"
    assert hdr[0].tobytes() == sx_ref[0].tobytes(), (hdr[0], sx_ref[0])
    alpha_ref = np.float32(sx_ref[0]) * np.float32(sw[0])
    assert hdr[1].tobytes() == np.float32(alpha_ref).tobytes()
    # the GEMM part equals the plain GEMM on the same codes, bit for bit
    xq_dev = torch.from_numpy(codes.copy()).to(cuda_device).view(torch.float8_e4m3fn)
    alpha_dev = torch.tensor([alpha_ref], dtype=torch.float32, device=cuda_device)
    assert torch.equal(y, tinym_b200.gemm(xq_dev, w, alpha_dev))
    out = y.float().cpu().numpy()
    ref = oracle.reference(xq_ref, wq, np.array([alpha_ref], dtype=np.float32))
    assert oracle.max_rel_err(out, ref) <= 4e-3
    assert oracle.mismatches(out, ref) == 0


@pytest.mark.parametrize("m,k,n", [(1, 1024, 384), (9, 2048, 640)])
def test_quant_act_explicit_plans(cuda_device, oracle, m, k, n):
    """The early-W GEMM under every plan family (and the SIMT kernel at M=1)."""
    import torch

    import tinym_b200

    plans = []
    for split in (1, 2, 4):
        for bk, st in ((128, 4), (256, 3), (512, 2)):
            for tm in (64, 128):
                plans.append(tinym_b200.make_plan(tinym_b200.KERNEL_TC, split, st,
                                                  8 if m <= 8 else 16, block_k=bk, tile_m=tm))
    if m == 1:
        plans.append(tinym_b200.make_plan(tinym_b200.KERNEL_SIMT_M1, 2, 4, 0, 4))
    ran = 0
    for plan in plans:
        try:
            tinym_b200.check_plan(m, n, k, plan)
        except tinym_b200.TinymError:
            continue
        x, w, w_scale, y, codes, hdr, xq_ref, sx_ref, wq, sw = _run(
            oracle, cuda_device, m, k, n, torch.bfloat16, "spiky", plan=plan)
        assert np.array_equal(codes, xq_ref)
        xq_dev = torch.from_numpy(codes.copy()).to(cuda_device).view(torch.float8_e4m3fn)
        alpha_dev = torch.from_numpy(hdr[1:2].copy()).to(cuda_device)
        assert torch.equal(y, tinym_b200.gemm(xq_dev, w, alpha_dev, plan=plan)), plan.as_dict()
        ran += 1
    assert ran >= 10
    assert tinym_b200.device_status() == 0


def test_quant_act_torch_op_and_adapter(cuda_device, oracle):
    import torch

    import candidate_kernel as ck

    x, w, w_scale, y, codes, hdr, xq_ref, sx_ref, wq, sw = _run(
        oracle, cuda_device, 9, 6144, 5120, torch.bfloat16, "spiky")
    y2, xs = ck.fp8_gemm_act(x, w, w_scale)
    assert torch.equal(y2, y)
    assert xs.dtype == torch.float32 and xs.item() == float(sx_ref[0])
    with pytest.raises(RuntimeError):
        ck.fp8_gemm_act(x.to(torch.float16), w, w_scale)  # unsupported activation dtype
    with pytest.raises(RuntimeError):
        ck.fp8_gemm_act(x[:, :6128].contiguous(), w, w_scale)  # K mismatch


def test_quant_act_rejected_plan_leaves_workspace_untouched(cuda_device):
    """The GEMM is validated before the quantise prologue is queued: a call
    whose plan is rejected writes neither the workspace nor Y."""
    import torch

    import tinym_b200

    m, k, n = 9, 1024, 512
    x = torch.randn((m, k), device=cuda_device).to(torch.bfloat16)
    w = torch.zeros((n, k), dtype=torch.uint8, device=cuda_device).view(torch.float8_e4m3fn)
    w_scale = torch.ones(1, dtype=torch.float32, device=cuda_device)
    ws = torch.full((tinym_b200.quant_workspace_bytes(m, k),), 0xA5, dtype=torch.uint8,
                    device=cuda_device)
    y = torch.full((m, n), 7.0, dtype=torch.bfloat16, device=cuda_device)
    bad = [tinym_b200.make_plan(tinym_b200.KERNEL_TC, 1, 4, 8),      # MMA N 8 < M 9
           tinym_b200.make_plan(tinym_b200.KERNEL_TC, 9, 4, 16)]     # cluster of 9
    for plan in bad:
        with pytest.raises(tinym_b200.TinymError):
            tinym_b200.gemm_quant_act(x, w, w_scale, out=y, workspace=ws, plan=plan)
    torch.cuda.synchronize()
    assert bool((ws == 0xA5).all())
    assert bool((y == 7.0).all())
    assert tinym_b200.device_status() == 0


def test_quant_act_back_to_back_in_a_graph(cuda_device, oracle):
    """Repeated fused calls captured in a CUDA graph keep giving the same bits
    (the quantise kernel and the early-W GEMM chain through programmatic
    dependent launch)."""
    import torch

    import tinym_b200

    x, w, w_scale, y, codes, hdr, xq_ref, sx_ref, wq, sw = _run(
        oracle, cuda_device, 9, 6144, 5120, torch.bfloat16, "normal")
    out = torch.empty_like(y)
    ws = torch.empty(tinym_b200.quant_workspace_bytes(9, 6144), dtype=torch.uint8,
                     device=cuda_device)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        tinym_b200.gemm_quant_act(x, w, w_scale, out=out, workspace=ws)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(4):
            tinym_b200.gemm_quant_act(x, w, w_scale, out=out, workspace=ws)
    for _ in range(3):
        out.zero_()
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, y)
    assert tinym_b200.device_status() == 0
