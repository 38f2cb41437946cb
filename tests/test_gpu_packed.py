"""GPU tests of the packed (tile-contiguous) weight layout.

tinym_pack_weights repacks W [N, K] into [tile][K chunk][128 rows][128 B]
blocks (include/tinym_b200.h).  The packed GEMM must give exactly the bits
of the row-major GEMM under the same plan (only the load addresses differ),
and both must meet the oracle bar.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _packed_layout(wq: np.ndarray) -> np.ndarray:
    """numpy restatement of the packed layout: zero-padded to whole 128-row
    tiles and a multiple of four 128-byte chunks, then [tile][chunk][row][byte]."""
    n, k = wq.shape
    tiles = (n + 127) // 128
    kc = ((k + 127) // 128 + 3) // 4 * 4
    pad = np.zeros((tiles * 128, kc * 128), dtype=np.uint8)
    pad[:n, :k] = wq
    return pad.reshape(tiles, 128, kc, 128).transpose(0, 2, 1, 3).reshape(-1)


def _pack(w):
    import torch

    import tinym_b200

    n, k = w.shape
    out = torch.empty(tinym_b200.packed_weight_bytes(n, k), dtype=torch.uint8, device=w.device)
    tinym_b200.pack_weights_ptr(w.data_ptr(), out.data_ptr(), n, k,
                                torch.cuda.current_stream(w.device).cuda_stream)
    return out


def _gemm_packed(x, wp, n, alpha, plan=None):
    import torch

    import tinym_b200

    m, k = x.shape
    y = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=x.device)
    tinym_b200.gemm_packed_ptr(x.data_ptr(), wp.data_ptr(), y.data_ptr(), m, n, k,
                               alpha_ptr=alpha.data_ptr(), plan=plan,
                               stream=torch.cuda.current_stream(x.device).cuda_stream)
    return y


def _dev(codes, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(codes)).to(device).view(torch.float8_e4m3fn)


@pytest.mark.parametrize("n,k", [(1, 16), (127, 144), (129, 272), (5120, 6144), (300, 1040)])
def test_pack_layout_bit_exact(cuda_device, oracle, n, k):
    xq, wq, sx, sw, alpha = oracle.make_case(1, k, n, seed=n + k, dist="normal")
    got = _pack(_dev(wq, cuda_device)).cpu().numpy()
    assert np.array_equal(got, _packed_layout(wq))


@pytest.mark.parametrize("m,k,n", [(1, 6144, 5120), (9, 6144, 5120), (9, 5120, 8192),
                                   (1, 5120, 16384), (16, 5120, 16384), (3, 144, 129),
                                   (9, 1040, 300), (16, 272, 200), (5, 2064, 4100)])
def test_packed_matches_row_major_and_oracle(cuda_device, oracle, m, k, n):
    import torch

    import tinym_b200

    xq, wq, sx, sw, alpha = oracle.make_case(m, k, n, seed=7 * m + k + n, dist="harness")
    x, w = _dev(xq, cuda_device), _dev(wq, cuda_device)
    a = torch.from_numpy(alpha).to(cuda_device)
    wp = _pack(w)
    y_p = _gemm_packed(x, wp, n, a)
    y_r = tinym_b200.gemm(x, w, a)
    assert torch.equal(y_p, y_r)
    out = y_p.float().cpu().numpy()
    ref = oracle.reference(xq, wq, alpha)
    assert oracle.max_rel_err(out, ref) <= 4e-3
    assert oracle.mismatches(out, ref) == 0


@pytest.mark.parametrize("m,k,n", [(1, 1024, 384), (9, 1152, 300), (16, 2048, 640)])
def test_packed_explicit_plans(cuda_device, oracle, m, k, n):
    """Every TC tiling the packed path accepts: block_k, tile_m, K split."""
    import torch

    import tinym_b200

    xq, wq, sx, sw, alpha = oracle.make_case(m, k, n, seed=11 + m, dist="normal")
    x, w = _dev(xq, cuda_device), _dev(wq, cuda_device)
    a = torch.from_numpy(alpha).to(cuda_device)
    wp = _pack(w)
    ran = 0
    for split in (1, 2, 3, 4):
        for bk, st in ((128, 4), (256, 3), (512, 2)):
            for tm in (64, 128):
                plan = tinym_b200.make_plan(tinym_b200.KERNEL_TC, split, st, 8 if m <= 8 else 16,
                                            block_k=bk, tile_m=tm)
                try:
                    tinym_b200.check_plan(m, n, k, plan)
                except tinym_b200.TinymError:
                    continue
                y_p = _gemm_packed(x, wp, n, a, plan=plan)
                y_r = tinym_b200.gemm(x, w, a, plan=plan)
                assert torch.equal(y_p, y_r), plan.as_dict()
                ran += 1
    assert ran >= 12
    assert tinym_b200.device_status() == 0


def test_packed_rejects_simt_plan(cuda_device, oracle):
    import torch

    import tinym_b200

    xq, wq, sx, sw, alpha = oracle.make_case(1, 1024, 256, seed=3, dist="normal")
    x, w = _dev(xq, cuda_device), _dev(wq, cuda_device)
    a = torch.from_numpy(alpha).to(cuda_device)
    plan = tinym_b200.make_plan(tinym_b200.KERNEL_SIMT_M1, 1, 4, 0, 4)
    with pytest.raises(tinym_b200.TinymError) as ei:
        _gemm_packed(x, _pack(w), 256, a, plan=plan)
    assert ei.value.status == 7


def test_adapter_packed_layout(cuda_device, oracle, monkeypatch):
    """prepare_weights(layout="packed") through the harness-facing adapter
    and torch ops gives the row-major result bit for bit."""
    import torch

    import candidate_kernel as ck

    xq, wq, sx, sw, alpha = oracle.make_case(9, 6144, 5120, seed=21, dist="harness")
    a, w = _dev(xq, cuda_device), _dev(wq, cuda_device)
    al = torch.from_numpy(alpha).to(cuda_device)
    ref = ck.fp8_gemm(a, ck.prepare_weights(w), al)
    pw = ck.prepare_weights(w, layout="packed")
    assert isinstance(pw, ck.PackedWeight) and pw.shape == (5120, 6144)
    assert torch.equal(ck.fp8_gemm(a, pw, al), ref)
    monkeypatch.setenv("TINYM_WEIGHT_LAYOUT", "packed")
    assert isinstance(ck.prepare_weights(w), ck.PackedWeight)
    with pytest.raises(ValueError):
        ck.prepare_weights(w, layout="bogus")
    with pytest.raises(RuntimeError):  # K mismatch is caught by the op
        torch.ops.sm120_fp8_gemm.run_packed(a, pw.data, 5120, 6128, al)
