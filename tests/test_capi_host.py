"""CPU: the C-ABI library loads, exports every declared symbol, and its
host-side logic (shape gate, dispatch table, plan validation, argument
checks) behaves as documented.  No kernel is launched here."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

HEADER = Path(__file__).resolve().parents[1] / "include" / "tinym_b200.h"

OFFICIAL = [(1, 5120, 16384), (9, 5120, 16384), (1, 6144, 5120), (9, 6144, 5120),
            (1, 5120, 8192), (9, 5120, 8192)]


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"TINYM_API\s+[\w\s\*]+?\b(tinym_\w+)\s*\(", text)))


def test_header_and_binding_agree():
    import tinym_b200

    assert declared_symbols() == sorted(tinym_b200.EXPORTED)


def test_library_exports_every_declared_symbol():
    import tinym_b200

    lib = tinym_b200.capi()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.tinym_abi_version() == 8


def test_status_strings():
    import tinym_b200

    lib = tinym_b200.capi()
    for code, name in tinym_b200.STATUS_NAMES.items():
        assert lib.tinym_status_string(code).decode() == name
    assert lib.tinym_status_string(99).decode() == "TINYM_ERR_UNKNOWN"


def test_plan_struct_layout():
    import tinym_b200

    assert ctypes.sizeof(tinym_b200.Plan) == 44


@pytest.mark.parametrize("m,k,n", OFFICIAL)
def test_dispatch_table_official_points(m, k, n):
    """Every official point gets a plan that fits 227 KiB of shared memory and
    one wave on 148 SMs (two CTAs per SM when each fits half an SM's 228 KiB)."""
    import tinym_b200

    p = tinym_b200.select_plan(m, n, k, 148)
    assert p.smem_bytes <= 232448
    per_sm = 2 if p.smem_bytes <= (233472 - 2048) // 2 else 1
    assert p.grid_ctas <= per_sm * 148
    assert p.tiles_n == (n + p.tile_m - 1) // p.tile_m
    kb = (k + 127) // 128
    per = -(-kb // p.split_k)
    assert (p.split_k - 1) * per < kb  # no empty K range
    if p.kernel == tinym_b200.KERNEL_TC:
        assert p.mma_n >= m and p.mma_n in (8, 16)
    else:
        assert m == 1


def test_dispatch_fills_small_sm_counts():
    import tinym_b200

    p = tinym_b200.select_plan(9, 5120, 6144, 40)
    assert p.grid_ctas <= 2 * 40 or p.split_k == 1
    p = tinym_b200.select_plan(1, 128, 128, 148)
    assert p.split_k == 1  # one K block cannot be split


@pytest.mark.parametrize("m", list(range(1, 17)))
def test_dispatch_every_m(m):
    import tinym_b200

    for k, n in ((6144, 5120), (5120, 8192), (5120, 16384), (16, 1), (4096, 100000)):
        p = tinym_b200.select_plan(m, n, k, 148)
        assert p.grid_ctas >= 1 and p.stages >= 2


def test_shape_gate():
    import tinym_b200

    for m, n, k, status in [(17, 128, 128, 2), (0, 128, 128, 1), (1, 0, 128, 1),
                            (1, 128, 40, 2), (1, 128, 0, 1)]:
        with pytest.raises(tinym_b200.TinymError) as ei:
            tinym_b200.select_plan(m, n, k, 148)
        assert ei.value.status == status


def test_check_plan_rejects_bad_plans():
    import tinym_b200 as t

    good = t.check_plan(1, 1024, 1024, t.make_plan(t.KERNEL_SIMT_M1, 2, 4, 0, 8))
    assert good.threads == 288 and good.grid_ctas == 16
    bad = [
        (2, t.make_plan(t.KERNEL_SIMT_M1, 1, 4, 0, 4)),    # SIMT needs M == 1
        (9, t.make_plan(t.KERNEL_TC, 1, 4, 8)),             # MMA N < M
        (1, t.make_plan(t.KERNEL_TC, 9, 4, 8)),             # cluster > 8
        (1, t.make_plan(t.KERNEL_TC, 1, 1, 8)),             # ring too shallow
        (1, t.make_plan(t.KERNEL_TC, 1, 4, 12)),            # MMA N not 8/16
        (1, t.make_plan(7, 1, 4, 8)),                       # unknown kernel
        (1, t.make_plan(t.KERNEL_TC, 8, 4, 8)),             # 8 splits of 7 K blocks
        (1, t.make_plan(t.KERNEL_SIMT_M1, 1, 4, 0, 4, 256)),  # SIMT stages are 128 B of K
        (9, t.make_plan(t.KERNEL_TC, 1, 4, 16, 0, 384)),      # block_k not 128/256/512
        (1, t.make_plan(t.KERNEL_SIMT_M1, 1, 4, 0, 4, 128, 64)),  # SIMT tiles are 128 rows
        (9, t.make_plan(t.KERNEL_TC, 1, 4, 16, 0, 128, 32)),  # tile_m not 64/128
    ]
    for m, plan in bad:
        with pytest.raises(t.TinymError) as ei:
            t.check_plan(m, 1024, 896, plan)
        assert ei.value.status == 7, (m, plan.as_dict())


def test_zero_plan_fields_mean_defaults():
    import tinym_b200 as t

    p = t.make_plan(t.KERNEL_TC, 1, 4, 16, 0, 0, 0)
    q = t.check_plan(9, 512, 1024, p)
    assert q.block_k == 128 and q.tile_m == 128 and q.tiles_n == 4


def test_dispatch_tiles_for_official_points():
    """The measured winners on B200: 128-row tiles, 64 KiB stages (128 rows x
    512 B) three deep, K split 3 / 2 / 1 for N = 5120 / 8192 / 16384; 32 KiB
    stages four deep where a CTA would keep fewer than four 64 KiB stages."""
    import tinym_b200 as t

    for m in (1, 8, 9, 16):
        for k, n, want in ((6144, 5120, (128, 3, 512, 3)), (5120, 8192, (128, 2, 512, 3)),
                           (5120, 16384, (128, 1, 512, 3)), (5120, 4096, (128, 4, 256, 4))):
            p = t.select_plan(m, n, k, 148)
            assert (p.tile_m, p.split_k, p.block_k, p.stages) == want, p.as_dict()


def test_block_k_needs_whole_chunks():
    import tinym_b200 as t

    t.check_plan(9, 512, 1024, t.make_plan(t.KERNEL_TC, 1, 2, 16, 0, 512))
    with pytest.raises(t.TinymError):
        t.check_plan(9, 512, 1040, t.make_plan(t.KERNEL_TC, 1, 4, 16, 0, 256))


def test_argument_checks_before_any_cuda_call():
    """Null / misaligned pointers and bad ldy are rejected on the host."""
    import tinym_b200 as t

    lib = t.capi()
    st = lib.tinym_fp8_gemm_ex(None, 16, 16, 128, 1, 128, 128, None, 1.0, None, None)
    assert st == 1
    st = lib.tinym_fp8_gemm_ex(17, 32, 64, 128, 1, 128, 128, None, 1.0, None, None)
    assert st == 3 and b"16-byte" in lib.tinym_last_error()
    st = lib.tinym_fp8_gemm_ex(16, 32, 65, 128, 1, 128, 128, None, 1.0, None, None)
    assert st == 3
    st = lib.tinym_fp8_gemm_ex(16, 32, 64, 64, 1, 128, 128, None, 1.0, None, None)
    assert st == 1 and b"ldy" in lib.tinym_last_error()
    st = lib.tinym_fp8_gemm_ex(16, 32, 64, 128, 1, 128, 128, None, float("inf"), None, None)
    assert st == 1
    st = lib.tinym_fp8_gemm_dev_alpha(16, 32, 64, 1, 128, 128, None, None)
    assert st == 1
    st = lib.tinym_fp8_gemm(16, 32, 64, 20, 128, 128, 1.0, 1.0, None)
    assert st == 2


def test_torch_op_registers_reference_schema():
    import torch

    import tinym_b200

    tinym_b200.load_torch_op()
    schema = str(torch.ops.sm120_fp8_gemm.run.default._schema)
    assert schema == "sm120_fp8_gemm::run(Tensor a, Tensor b, float alpha) -> Tensor"
    assert "run_alpha_tensor" in str(torch.ops.sm120_fp8_gemm.run_alpha_tensor.default._schema)


def test_candidate_kernel_surface():
    """Same public names and validation as the reference adapter."""
    import torch

    import candidate_kernel

    assert candidate_kernel.__all__ == ["build", "prepare_weights", "fp8_gemm"]
    with pytest.raises(ValueError):
        candidate_kernel.prepare_weights(torch.zeros(4, 4))
    assert candidate_kernel.build() is True
    # alpha that is not a one-element CUDA float32 tensor: ValueError before
    # any launch, as the reference's _host_alpha
    for bad in (1.0, None, torch.ones(1)):
        with pytest.raises(ValueError, match="alpha"):
            candidate_kernel.fp8_gemm(torch.zeros(1, 16), torch.zeros(16, 16), bad)


@pytest.mark.parametrize("m", [1, 3, 9, 16])
def test_dispatch_plans_always_validate(m):
    """The dispatch table never emits a plan its own validator rejects."""
    import tinym_b200

    for k in (16, 48, 128, 144, 272, 1040, 2064, 4096, 5120, 6144, 8192):
        for n in (1, 127, 129, 300, 640, 1000, 4100, 5120, 8192, 16384):
            for sms in (148, 132, 40):
                p = tinym_b200.select_plan(m, n, k, sms)
                tinym_b200.check_plan(m, n, k, p)


def test_packed_weight_bytes():
    """Packed weights are whole 128-row tiles x a multiple of four 128-byte
    K chunks."""
    import tinym_b200 as t

    assert t.packed_weight_bytes(5120, 6144) == 5120 * 6144
    assert t.packed_weight_bytes(16384, 5120) == 16384 * 5120
    assert t.packed_weight_bytes(129, 144) == 2 * 4 * 128 * 128
    assert t.packed_weight_bytes(1, 16) == 4 * 128 * 128
    assert t.packed_weight_bytes(300, 1152) == 3 * 12 * 128 * 128
    with pytest.raises(t.TinymError):
        t.packed_weight_bytes(4, 24)  # K % 16 != 0


def test_gather_descriptor_layout_and_host_checks():
    """tinym_gather_desc mirrors the header, and a bad descriptor is refused
    before any CUDA call."""
    import tinym_b200 as t

    assert ctypes.sizeof(t.GatherDesc) == 4 + 4 + 8 + 8 + 64 + 64 + 8
    lib = t.capi()
    d = t.GatherDesc()
    d.world, d.rank, d.n_full, d.col0 = 0, 0, 128, 0
    assert lib.tinym_fp8_gemm_allgather(16, 16, 1, 128, 128, None, 1.0, ctypes.byref(d),
                                        None, None) == 1
    d.world, d.rank = 2, 0
    d.y_full[0] = d.y_full[1] = 256
    d.flag[0], d.flag[1] = 512, 516  # second counter not 8-byte aligned
    assert lib.tinym_fp8_gemm_allgather(16, 16, 1, 128, 128, None, 1.0, ctypes.byref(d),
                                        None, None) == 1
    d.flag[1] = 520
    d.col0 = 64  # 64 + 128 > N_full
    assert lib.tinym_fp8_gemm_allgather(16, 16, 1, 128, 128, None, 1.0, ctypes.byref(d),
                                        None, None) == 1


def test_static_w_dispatch_packs_two_ctas_per_sm():
    """TINYM_FLAG_STATIC_W: 64 KiB rings (two CTAs fit an SM) and twice the K
    split of the default table at the official points."""
    import tinym_b200 as t

    for m in (1, 9, 16):
        for k, n, split in ((6144, 5120, 6), (5120, 8192, 4), (5120, 16384, 2)):
            p = t.select_plan(m, n, k, 148, static_w=True)
            assert (p.block_k, p.stages, p.split_k) == (256, 2, split), p.as_dict()
            assert p.smem_bytes <= (233472 - 2048) // 2
            assert p.grid_ctas <= 2 * 148
    lib = t.capi()
    out = t.Plan()
    assert lib.tinym_select_plan_ex(9, 5120, 6144, 148, 4, ctypes.byref(out)) == 1  # bad flag


def test_quant_act_host_checks():
    """Workspace size and the fused activation path's argument checks run on
    the host, before any CUDA call."""
    import tinym_b200 as t

    assert t.quant_workspace_bytes(9, 6144) == 256 + 55296
    assert t.quant_workspace_bytes(1, 16) == 256 + 256  # codes rounded to 256 bytes
    with pytest.raises(t.TinymError):
        t.quant_workspace_bytes(17, 128)
    lib = t.capi()
    # null workspace, bad dtype, misaligned X, misaligned workspace: every call
    # fails before any pointer is used
    # (x, dtype, w, w_scale, y, ldy, m, n, k, workspace, plan, stream)
    assert lib.tinym_fp8_gemm_quant_act(256, 1, 256, 256, 256, 128, 1, 128, 128, None, None,
                                        None) == 1
    assert lib.tinym_fp8_gemm_quant_act(256, 3, 256, 256, 256, 128, 1, 128, 128, 512, None,
                                        None) == 1
    assert lib.tinym_fp8_gemm_quant_act(264, 1, 256, 256, 256, 128, 1, 128, 128, 512, None,
                                        None) == 3
    assert lib.tinym_fp8_gemm_quant_act(256, 1, 256, 256, 256, 128, 1, 128, 128, 528, None,
                                        None) == 3
    # the GEMM's own checks (misaligned W, ldy < N) also run before the
    # quantise prologue is queued
    assert lib.tinym_fp8_gemm_quant_act(256, 1, 264, 256, 256, 128, 1, 128, 128, 512, None,
                                        None) == 3
    assert lib.tinym_fp8_gemm_quant_act(256, 1, 256, 256, 256, 64, 1, 128, 128, 512, None,
                                        None) == 1


def test_ipc_export_rejects_null_arguments():
    import tinym_b200 as t

    lib = t.capi()
    off = ctypes.c_int64(0)
    h = ctypes.create_string_buffer(64)
    assert lib.tinym_ipc_export(None, h, ctypes.byref(off)) == 1
    base = ctypes.c_void_p(0)
    assert lib.tinym_ipc_open(None, ctypes.byref(base)) == 1


def test_bench_reference_arm_prints_one_line():
    """The driver's reference arm: the CPU oracle on the host cores, one JSON
    line with the contract's keys.  Run with OMP_NUM_THREADS=1, as torchrun
    sets it for every rank: the arm still uses every CPU it may run on."""
    import json
    import os
    import subprocess
    import sys

    root = Path(__file__).resolve().parents[1]
    env = dict(os.environ, OMP_NUM_THREADS="1")
    res = subprocess.run([sys.executable, str(root / "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "3"],
                         capture_output=True, text=True, timeout=240, cwd=root, env=env)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.strip().splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "GB/s" and d["value"] > 0
    assert d["cpu_baseline"]["kind"] in ("port", "reference")
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["gpu_launches"] == 0
    assert d["cpu_baseline"]["cores"] == len(os.sched_getaffinity(0))


def test_torch_wrappers_validate_before_launch():
    """tinym_b200.gemm / gemm_quant_act refuse operands the kernel would read
    or write out of bounds (K mismatch, strided views, a short out or
    workspace) and host tensors, before any pointer reaches the C ABI."""
    import torch

    import tinym_b200 as t

    f8 = torch.float8_e4m3fn
    x = torch.zeros(2, 32).to(f8)
    w = torch.zeros(8, 32).to(f8)
    with pytest.raises(ValueError, match="same K"):
        t.gemm(x, torch.zeros(8, 16).to(f8), 1.0)
    with pytest.raises(ValueError, match="contiguous"):
        t.gemm(x, torch.zeros(32, 8).to(f8).t(), 1.0)
    with pytest.raises(ValueError, match=r"\[2, 8\]"):
        t.gemm(x, w, 1.0, out=torch.empty(2, 4, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match=r"\[2, 8\]"):
        t.gemm(x, w, 1.0, out=torch.empty(8, 2, dtype=torch.bfloat16).t())
    with pytest.raises(ValueError, match="CUDA"):
        t.gemm(x, w, 1.0)
    xa = torch.zeros(2, 32, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="workspace"):
        t.gemm_quant_act(xa, w, torch.ones(1), workspace=torch.empty(300, dtype=torch.uint8))
    with pytest.raises(ValueError, match="w_scale"):
        t.gemm_quant_act(xa, w, torch.ones(2))
    with pytest.raises(ValueError, match="CUDA"):
        t.gemm_quant_act(xa, w, torch.ones(1))


def test_plain_c_caller(tmp_path):
    """A C99 program (tests/c_abi_host.c) compiles against include/tinym_b200.h,
    links libtinym_b200.so and runs the host-side entry points: the boundary
    needs neither Python nor torch."""
    import shutil
    import subprocess

    import tinym_b200

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    lib = tinym_b200.capi()  # builds the library if it is missing
    assert lib is not None
    root = Path(__file__).resolve().parents[1]
    libdir = tinym_b200.CORE_SO.parent
    exe = tmp_path / "c_abi_host"
    subprocess.run([cc, "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic",
                    "-I", str(root / "include"), str(root / "tests" / "c_abi_host.c"),
                    "-o", str(exe), "-L", str(libdir), "-ltinym_b200",
                    f"-Wl,-rpath,{libdir}"], check=True, capture_output=True, text=True)
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, run.stderr
    lines = run.stdout.strip().splitlines()
    assert lines[-1] == "c abi host checks ok"
    assert "M=9 K=6144 N=5120 split=3 stages=3 block_k=512 tile_m=128 ctas=120" in lines
