"""The no-allocation entry point of the fused activation path.

tinym_fp8_gemm_quant_act_noalloc runs the quantise prologue + GEMM with its
workspace in a static device array inside the library (address from
cudaGetSymbolAddress, per device) instead of a caller-provided buffer.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest


def test_noalloc_symbol_exported():
    import tinym_b200

    lib = tinym_b200.capi()
    assert hasattr(lib, "tinym_fp8_gemm_quant_act_noalloc")
    assert "tinym_fp8_gemm_quant_act_noalloc" in tinym_b200.EXPORTED


def test_noalloc_rejects_oversized_activation_on_host():
    """M*K beyond the static workspace is refused before any CUDA call."""
    import tinym_b200

    lib = tinym_b200.capi()
    st = lib.tinym_fp8_gemm_quant_act_noalloc(16, tinym_b200.ACT_BF16, 16, 16, 16, 128,
                                              16, 128, 65536, None, None)
    assert st == 2 and b"static workspace" in lib.tinym_last_error()
    st = lib.tinym_fp8_gemm_quant_act_noalloc(16, tinym_b200.ACT_BF16, 16, 16, 16, 128,
                                              17, 128, 128, None, None)
    assert st == 2  # M > 16


def _noalloc(x, w, w_scale, out, plan=None):
    import torch

    import tinym_b200

    dt = tinym_b200.ACT_BF16 if x.dtype == torch.bfloat16 else tinym_b200.ACT_F32
    m, k = x.shape
    n = w.shape[0]
    lib = tinym_b200.capi()
    st = lib.tinym_fp8_gemm_quant_act_noalloc(
        x.data_ptr(), dt, w.data_ptr(), w_scale.data_ptr(), out.data_ptr(), out.stride(0),
        m, n, k, ctypes.byref(plan) if plan is not None else None,
        torch.cuda.current_stream(x.device).cuda_stream)
    if st:
        raise tinym_b200.TinymError(st, lib.tinym_last_error().decode())
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("dtype_name", ["bfloat16", "float32"])
@pytest.mark.parametrize("m,k,n", [(9, 6144, 5120), (1, 5120, 1024), (16, 272, 200)])
def test_noalloc_matches_workspace_form(cuda_device, oracle, dtype_name, m, k, n):
    import torch

    import tinym_b200

    rng = np.random.default_rng(m + k + n)
    x = torch.from_numpy(rng.standard_normal((m, k), dtype=np.float32) * 2.0).to(cuda_device)
    x = x.to(getattr(torch, dtype_name))
    _, wq, _, sw, _ = oracle.make_case(1, k, n, seed=n, dist="normal")
    w = torch.from_numpy(wq).to(cuda_device).view(torch.float8_e4m3fn)
    w_scale = torch.from_numpy(sw.astype(np.float32)).to(cuda_device)
    y_ws, ws = tinym_b200.gemm_quant_act(x, w, w_scale)
    y_na = _noalloc(x, w, w_scale, torch.full_like(y_ws, float("nan")))
    assert torch.equal(y_na, y_ws)
    xq_ref, sx_ref = oracle.quantize_per_tensor(x.float().cpu().numpy())
    alpha = np.float32(sx_ref[0]) * np.float32(sw[0])
    ref = oracle.reference(xq_ref, wq, np.array([alpha], dtype=np.float32))
    out = y_na.float().cpu().numpy()
    assert oracle.max_rel_err(out, ref) <= 4e-3 and oracle.mismatches(out, ref) == 0
    assert tinym_b200.device_status() == 0


@pytest.mark.gpu
def test_noalloc_stream_ordered_reuse(cuda_device, oracle):
    """Back-to-back calls on one stream reuse the static workspace safely:
    each result matches its own workspace-form result."""
    import torch

    import tinym_b200

    k, n = 2048, 640
    _, wq, _, sw, _ = oracle.make_case(1, k, n, seed=5, dist="normal")
    w = torch.from_numpy(wq).to(cuda_device).view(torch.float8_e4m3fn)
    w_scale = torch.from_numpy(sw.astype(np.float32)).to(cuda_device)
    xs = [torch.randn(m, k, device=cuda_device).to(torch.bfloat16) * s
          for m, s in ((9, 1.0), (3, 100.0), (16, 1e-3), (1, 7.0))]
    outs = [torch.empty((x.shape[0], n), dtype=torch.bfloat16, device=cuda_device) for x in xs]
    for _ in range(3):
        for x, o in zip(xs, outs):
            _noalloc(x, w, w_scale, o)
    torch.cuda.synchronize()
    for x, o in zip(xs, outs):
        y_ws, _ = tinym_b200.gemm_quant_act(x, w, w_scale)
        assert torch.equal(o, y_ws)
    assert tinym_b200.device_status() == 0


@pytest.mark.gpu
def test_noalloc_interleaved_with_early_weight_gemms(cuda_device, oracle):
    """The static workspace stays consistent when no-allocation calls are
    interleaved on one stream with plain GEMMs launched under programmatic
    dependent launch with TINYM_FLAG_STATIC_W (the kernels that start
    streaming before the previous kernel completes): the quantise prologue
    is an ordinarily ordered launch, so it never overwrites the workspace
    while an earlier GEMM still reads it."""
    import torch

    import tinym_b200

    k, n = 2048, 640
    _, wq, _, sw, _ = oracle.make_case(1, k, n, seed=6, dist="normal")
    w = torch.from_numpy(wq).to(cuda_device).view(torch.float8_e4m3fn)
    w_scale = torch.from_numpy(sw.astype(np.float32)).to(cuda_device)
    xs = [torch.randn(m, k, device=cuda_device).to(torch.bfloat16) * s
          for m, s in ((9, 1.0), (16, 50.0), (2, 1e-2))]
    xq, _, _, _, alpha = oracle.make_case(9, k, 1, seed=7, dist="normal")
    x8 = torch.from_numpy(xq).to(cuda_device).view(torch.float8_e4m3fn)
    a8 = torch.from_numpy(alpha).to(cuda_device)
    outs = [torch.empty((x.shape[0], n), dtype=torch.bfloat16, device=cuda_device) for x in xs]
    plain = [torch.empty((9, n), dtype=torch.bfloat16, device=cuda_device) for _ in xs]
    for _ in range(2):
        for x, o, yp in zip(xs, outs, plain):
            _noalloc(x, w, w_scale, o)
            tinym_b200.gemm(x8, w, a8, out=yp, static_w=True)
    torch.cuda.synchronize()
    # the same plan as the static-W launches, without the flag: identical bits
    sms = torch.cuda.get_device_properties(cuda_device).multi_processor_count
    y_plain = tinym_b200.gemm(x8, w, a8, plan=tinym_b200.select_plan(9, n, k, sms, static_w=True))
    for x, o, yp in zip(xs, outs, plain):
        y_ws, _ = tinym_b200.gemm_quant_act(x, w, w_scale)
        assert torch.equal(o, y_ws)
        assert torch.equal(yp, y_plain)
    assert tinym_b200.device_status() == 0
