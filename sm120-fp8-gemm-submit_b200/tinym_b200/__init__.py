"""B200-native tiny-M FP8 GEMM: Python side of the C ABI.

Loads the in-tree native libraries and exposes

* ``capi()``            -- the ctypes handle of ``libtinym_b200.so`` with the
  signatures of ``include/tinym_b200.h``;
* ``load_torch_op()``   -- registers ``torch.ops.sm120_fp8_gemm`` (the
  reference's op namespace, src/torch_candidate_extension.cu:85-91);
* ``gemm_ptr(...)``     -- one call through the C ABI on raw pointers (used by
  the parity tests and the N-sharded wrapper);
* ``select_plan(...)``  -- the shape-dispatch table (host only);
* ``Plan``              -- ``tinym_plan`` as a ctypes structure.

There is no CPU fallback: if the native library is missing or the GPU is
not an sm_100 device, calls raise.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from . import build as _build

PKG = Path(__file__).resolve().parent
CORE_SO = _build.CORE_SO
TORCH_SO = _build.TORCH_SO

TINYM_OK = 0
STATUS_NAMES = {
    0: "TINYM_OK",
    1: "TINYM_ERR_INVALID_ARGUMENT",
    2: "TINYM_ERR_UNSUPPORTED_SHAPE",
    3: "TINYM_ERR_MISALIGNED",
    4: "TINYM_ERR_CUDA",
    5: "TINYM_ERR_UNSUPPORTED_DEVICE",
    6: "TINYM_ERR_DEVICE_TIMEOUT",
    7: "TINYM_ERR_BAD_PLAN",
}
KERNEL_TC = 1
KERNEL_SIMT_M1 = 2

# Every symbol include/tinym_b200.h declares (checked by the CPU tests).
EXPORTED = (
    "tinym_fp8_gemm",
    "tinym_fp8_gemm_dev_alpha",
    "tinym_fp8_gemm_ex",
    "tinym_fp8_gemm_ex2",
    "tinym_select_plan_ex",
    "tinym_select_plan",
    "tinym_check_plan",
    "tinym_device_status",
    "tinym_pending_errors",
    "tinym_plan_max_active_clusters",
    "tinym_launch_plan",
    "tinym_selftest_wait_timeout",
    "tinym_packed_weight_bytes",
    "tinym_pack_weights",
    "tinym_fp8_gemm_packed",
    "tinym_quant_workspace_bytes",
    "tinym_fp8_gemm_quant_act",
    "tinym_fp8_gemm_quant_act_noalloc",
    "tinym_fp8_gemm_allgather",
    "tinym_ipc_export",
    "tinym_ipc_open",
    "tinym_ipc_close",
    "tinym_status_string",
    "tinym_last_error",
    "tinym_abi_version",
)


class Plan(ctypes.Structure):
    """Mirror of ``tinym_plan`` (include/tinym_b200.h)."""

    _fields_ = [
        ("kernel", ctypes.c_int32),
        ("split_k", ctypes.c_int32),
        ("stages", ctypes.c_int32),
        ("mma_n", ctypes.c_int32),
        ("consumer_warps", ctypes.c_int32),
        ("block_k", ctypes.c_int32),
        ("tile_m", ctypes.c_int32),
        ("tiles_n", ctypes.c_int32),
        ("grid_ctas", ctypes.c_int32),
        ("smem_bytes", ctypes.c_int32),
        ("threads", ctypes.c_int32),
    ]

    def as_dict(self) -> dict:
        return {name: int(getattr(self, name)) for name, _ in self._fields_}

    def __repr__(self) -> str:  # pragma: no cover - debugging aid
        return f"Plan({self.as_dict()})"


class GatherDesc(ctypes.Structure):
    """Mirror of ``tinym_gather_desc`` (include/tinym_b200.h)."""

    _fields_ = [
        ("world", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("n_full", ctypes.c_int64),
        ("col0", ctypes.c_int64),
        ("y_full", ctypes.c_void_p * 8),
        ("flag", ctypes.c_void_p * 8),
        ("target", ctypes.c_uint64),
    ]


class TinymError(RuntimeError):
    """A non-zero tinym_status from the C ABI."""

    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")


_lock = threading.Lock()
_capi = None
_torch_op_loaded = False


def capi() -> ctypes.CDLL:
    """Load libtinym_b200.so (building it first if it is missing; a stale
    library is rebuilt by build.build_all, which __graft_entry__.build runs)."""
    global _capi
    if _capi is not None:
        return _capi
    with _lock:
        if _capi is None:
            if not CORE_SO.exists():
                _build.build_core()
            lib = ctypes.CDLL(str(CORE_SO))
            vp, i64, f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float
            lib.tinym_fp8_gemm.argtypes = [vp, vp, vp, i64, i64, i64, f32, f32, vp]
            lib.tinym_fp8_gemm.restype = ctypes.c_int
            lib.tinym_fp8_gemm_dev_alpha.argtypes = [vp, vp, vp, i64, i64, i64, vp, vp]
            lib.tinym_fp8_gemm_dev_alpha.restype = ctypes.c_int
            lib.tinym_fp8_gemm_ex.argtypes = [vp, vp, vp, i64, i64, i64, i64, vp, f32,
                                              ctypes.POINTER(Plan), vp]
            lib.tinym_fp8_gemm_ex.restype = ctypes.c_int
            lib.tinym_fp8_gemm_ex2.argtypes = [vp, vp, vp, i64, i64, i64, i64, vp, f32,
                                               ctypes.POINTER(Plan), ctypes.c_uint32, vp]
            lib.tinym_fp8_gemm_ex2.restype = ctypes.c_int
            lib.tinym_select_plan_ex.argtypes = [i64, i64, i64, ctypes.c_int32, ctypes.c_uint32,
                                                 ctypes.POINTER(Plan)]
            lib.tinym_select_plan_ex.restype = ctypes.c_int
            lib.tinym_select_plan.argtypes = [i64, i64, i64, ctypes.c_int32, ctypes.POINTER(Plan)]
            lib.tinym_select_plan.restype = ctypes.c_int
            lib.tinym_check_plan.argtypes = [i64, i64, i64, ctypes.POINTER(Plan)]
            lib.tinym_check_plan.restype = ctypes.c_int
            lib.tinym_device_status.argtypes = [ctypes.POINTER(ctypes.c_uint32), ctypes.c_int32]
            lib.tinym_device_status.restype = ctypes.c_int
            lib.tinym_pending_errors.argtypes = [ctypes.POINTER(ctypes.c_uint32), ctypes.c_int32]
            lib.tinym_pending_errors.restype = ctypes.c_int
            lib.tinym_selftest_wait_timeout.argtypes = [vp, vp, vp, i64, i64, i64,
                                                        ctypes.POINTER(Plan), ctypes.c_uint64, vp]
            lib.tinym_selftest_wait_timeout.restype = ctypes.c_int
            lib.tinym_plan_max_active_clusters.argtypes = [i64, i64, i64, ctypes.POINTER(Plan),
                                                           ctypes.POINTER(ctypes.c_int32)]
            lib.tinym_plan_max_active_clusters.restype = ctypes.c_int
            lib.tinym_launch_plan.argtypes = [i64, i64, i64, ctypes.c_uint32, ctypes.POINTER(Plan)]
            lib.tinym_launch_plan.restype = ctypes.c_int
            lib.tinym_packed_weight_bytes.argtypes = [i64, i64, ctypes.POINTER(i64)]
            lib.tinym_packed_weight_bytes.restype = ctypes.c_int
            lib.tinym_pack_weights.argtypes = [vp, vp, i64, i64, vp]
            lib.tinym_pack_weights.restype = ctypes.c_int
            lib.tinym_fp8_gemm_packed.argtypes = [vp, vp, vp, i64, i64, i64, i64, vp, f32,
                                                  ctypes.POINTER(Plan), vp]
            lib.tinym_fp8_gemm_packed.restype = ctypes.c_int
            lib.tinym_quant_workspace_bytes.argtypes = [i64, i64, ctypes.POINTER(i64)]
            lib.tinym_quant_workspace_bytes.restype = ctypes.c_int
            lib.tinym_fp8_gemm_quant_act.argtypes = [vp, ctypes.c_int32, vp, vp, vp, i64, i64, i64,
                                                     i64, vp, ctypes.POINTER(Plan), vp]
            lib.tinym_fp8_gemm_quant_act.restype = ctypes.c_int
            lib.tinym_fp8_gemm_quant_act_noalloc.argtypes = [vp, ctypes.c_int32, vp, vp, vp, i64,
                                                             i64, i64, i64,
                                                             ctypes.POINTER(Plan), vp]
            lib.tinym_fp8_gemm_quant_act_noalloc.restype = ctypes.c_int
            lib.tinym_fp8_gemm_allgather.argtypes = [vp, vp, i64, i64, i64, vp, f32,
                                                     ctypes.POINTER(GatherDesc),
                                                     ctypes.POINTER(Plan), vp]
            lib.tinym_fp8_gemm_allgather.restype = ctypes.c_int
            lib.tinym_ipc_export.argtypes = [vp, vp, ctypes.POINTER(i64)]
            lib.tinym_ipc_export.restype = ctypes.c_int
            lib.tinym_ipc_open.argtypes = [vp, ctypes.POINTER(vp)]
            lib.tinym_ipc_open.restype = ctypes.c_int
            lib.tinym_ipc_close.argtypes = [vp]
            lib.tinym_ipc_close.restype = ctypes.c_int
            lib.tinym_status_string.argtypes = [ctypes.c_int32]
            lib.tinym_status_string.restype = ctypes.c_char_p
            lib.tinym_last_error.argtypes = []
            lib.tinym_last_error.restype = ctypes.c_char_p
            lib.tinym_abi_version.argtypes = []
            lib.tinym_abi_version.restype = ctypes.c_int32
            _capi = lib
    return _capi


def _check(status: int) -> None:
    if status != TINYM_OK:
        msg = capi().tinym_last_error().decode(errors="replace")
        raise TinymError(status, msg)


def load_torch_op() -> None:
    """Register torch.ops.sm120_fp8_gemm from the in-tree shim."""
    global _torch_op_loaded
    if _torch_op_loaded:
        return
    with _lock:
        if not _torch_op_loaded:
            import torch

            if not TORCH_SO.exists():
                _build.build_torch_op()
            torch.ops.load_library(str(TORCH_SO))
            _torch_op_loaded = True


def select_plan(m: int, n: int, k: int, sm_count: int = 148, static_w: bool = False) -> Plan:
    """The shape-dispatch table's choice for (m, n, k) on sm_count SMs
    (with TINYM_FLAG_STATIC_W's two-CTA-per-SM variant when static_w)."""
    p = Plan()
    if static_w:
        _check(capi().tinym_select_plan_ex(m, n, k, sm_count, 1, ctypes.byref(p)))
    else:
        _check(capi().tinym_select_plan(m, n, k, sm_count, ctypes.byref(p)))
    return p


def check_plan(m: int, n: int, k: int, plan: Plan) -> Plan:
    """Validate an explicit plan and fill its derived fields."""
    p = Plan.from_buffer_copy(plan)
    _check(capi().tinym_check_plan(m, n, k, ctypes.byref(p)))
    return p


def make_plan(kernel: int = KERNEL_TC, split_k: int = 1, stages: int = 4, mma_n: int = 16,
              consumer_warps: int = 0, block_k: int = 128, tile_m: int = 128) -> Plan:
    """An explicit plan (derived fields are filled by check_plan / the launch)."""
    p = Plan()
    p.kernel, p.split_k, p.stages, p.mma_n = kernel, split_k, stages, mma_n
    p.consumer_warps, p.block_k, p.tile_m = consumer_warps, block_k, tile_m
    return p


FLAG_STATIC_W = 1


def gemm_ptr(x_ptr: int, w_ptr: int, y_ptr: int, m: int, n: int, k: int, *,
             ldy: int | None = None, alpha: float = 1.0, alpha_ptr: int | None = None,
             plan: Plan | None = None, stream: int = 0, static_w: bool = False) -> None:
    """Y = alpha * X . W^T through tinym_fp8_gemm_ex on raw device pointers
    (tinym_fp8_gemm_ex2 with TINYM_FLAG_STATIC_W when static_w)."""
    lib = capi()
    pl = ctypes.byref(plan) if plan is not None else None
    if static_w:
        st = lib.tinym_fp8_gemm_ex2(x_ptr, w_ptr, y_ptr, n if ldy is None else ldy, m, n, k,
                                    alpha_ptr, alpha, pl, FLAG_STATIC_W, stream)
    else:
        st = lib.tinym_fp8_gemm_ex(x_ptr, w_ptr, y_ptr, n if ldy is None else ldy, m, n, k,
                                   alpha_ptr, alpha, pl, stream)
    _check(st)


def packed_weight_bytes(n: int, k: int) -> int:
    """Bytes of the packed (tile-contiguous) form of an [N, K] weight."""
    out = ctypes.c_int64(0)
    _check(capi().tinym_packed_weight_bytes(n, k, ctypes.byref(out)))
    return int(out.value)


def pack_weights_ptr(w_ptr: int, packed_ptr: int, n: int, k: int, stream: int = 0) -> None:
    """Repack row-major W [N, K] at w_ptr into the packed layout at packed_ptr."""
    _check(capi().tinym_pack_weights(w_ptr, packed_ptr, n, k, stream))


def gemm_packed_ptr(x_ptr: int, wp_ptr: int, y_ptr: int, m: int, n: int, k: int, *,
                    ldy: int | None = None, alpha: float = 1.0, alpha_ptr: int | None = None,
                    plan: Plan | None = None, stream: int = 0) -> None:
    """Y = alpha * X . W^T with W in the packed layout (tinym_fp8_gemm_packed)."""
    pl = ctypes.byref(plan) if plan is not None else None
    _check(capi().tinym_fp8_gemm_packed(x_ptr, wp_ptr, y_ptr, n if ldy is None else ldy, m, n,
                                        k, alpha_ptr, alpha, pl, stream))


ACT_BF16 = 1
ACT_F32 = 2


def quant_workspace_bytes(m: int, k: int) -> int:
    """Workspace bytes of the fused activation path for an [M, K] activation."""
    out = ctypes.c_int64(0)
    _check(capi().tinym_quant_workspace_bytes(m, k, ctypes.byref(out)))
    return int(out.value)


def _check_operands(x, w) -> tuple[int, int, int]:
    """(M, K, N) of contiguous row-major x [M, K] and w [N, K]; the kernels
    read them as dense matrices, so views with other strides are refused."""
    if x.dim() != 2 or w.dim() != 2:
        raise ValueError("x and w must be rank-2 tensors")
    if not x.is_contiguous() or not w.is_contiguous():
        raise ValueError("x and w must be contiguous row-major tensors")
    if x.shape[1] != w.shape[1]:
        raise ValueError(f"x and w must have the same K (got {x.shape[1]} and {w.shape[1]})")
    return int(x.shape[0]), int(x.shape[1]), int(w.shape[0])


def _check_out(out, m: int, n: int, x):
    """A fresh [M, N] BF16 output, or the caller's after checking that the
    kernel's writes (M rows of N, row stride out.stride(0)) stay inside it."""
    import torch

    if out is None:
        return torch.empty((m, n), dtype=torch.bfloat16, device=x.device)
    if out.dtype != torch.bfloat16 or out.dim() != 2 or tuple(out.shape) != (m, n) or \
            out.stride(1) != 1 or out.stride(0) < n:
        raise ValueError(f"out must be a [{m}, {n}] bfloat16 tensor with unit column stride")
    return out


def _check_devices(*tensors) -> None:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("every tensor argument must be a CUDA tensor")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("every tensor argument must be on the same CUDA device")


def gemm_quant_act(x, w, w_scale, *, out=None, workspace=None, plan: Plan | None = None):
    """Fused activation path: quantise BF16 / FP32 x per tensor on the device,
    then Y = alpha * q(x) . W^T.  Returns (Y, workspace); the workspace holds
    x_scale, alpha and the E4M3 codes (see include/tinym_b200.h)."""
    import torch

    if x.dtype == torch.bfloat16:
        dt = ACT_BF16
    elif x.dtype == torch.float32:
        dt = ACT_F32
    else:
        raise ValueError("x must be bfloat16 or float32")
    if w.dtype != torch.float8_e4m3fn:
        raise ValueError("w must be float8_e4m3fn")
    m, k, n = _check_operands(x, w)
    if not isinstance(w_scale, torch.Tensor) or w_scale.dtype != torch.float32 or \
            w_scale.numel() != 1:
        raise ValueError("w_scale must be a one-element float32 tensor")
    need = quant_workspace_bytes(m, k)
    if workspace is not None and (workspace.dtype != torch.uint8 or workspace.dim() != 1 or
                                  not workspace.is_contiguous() or workspace.numel() < need):
        raise ValueError(f"workspace must be a contiguous uint8 vector of >= {need} bytes")
    out = _check_out(out, m, n, x)
    _check_devices(x, w, w_scale, out, workspace)
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    stream = torch.cuda.current_stream(x.device).cuda_stream
    pl = ctypes.byref(plan) if plan is not None else None
    _check(capi().tinym_fp8_gemm_quant_act(x.data_ptr(), dt, w.data_ptr(), w_scale.data_ptr(),
                                           out.data_ptr(), out.stride(0), m, n, k,
                                           workspace.data_ptr(), pl, stream))
    return out, workspace


def ipc_export(ptr: int) -> tuple[bytes, int]:
    """CUDA IPC handle (64 bytes) of the allocation holding device pointer
    ptr, and ptr's byte offset in that allocation."""
    h = ctypes.create_string_buffer(64)
    off = ctypes.c_int64(0)
    _check(capi().tinym_ipc_export(ptr, h, ctypes.byref(off)))
    return h.raw, int(off.value)


def ipc_open(handle: bytes) -> int:
    """Map a peer process's allocation into this one; returns its base."""
    base = ctypes.c_void_p(0)
    _check(capi().tinym_ipc_open(ctypes.create_string_buffer(handle, 64), ctypes.byref(base)))
    return int(base.value)


def ipc_close(base: int) -> None:
    _check(capi().tinym_ipc_close(base))


def gemm_allgather_ptr(x_ptr: int, w_ptr: int, m: int, n_local: int, k: int, desc: GatherDesc,
                       *, alpha: float = 1.0, alpha_ptr: int | None = None,
                       plan: Plan | None = None, stream: int = 0) -> None:
    """N-sharded GEMM whose epilogue stores into every rank's full Y
    (tinym_fp8_gemm_allgather)."""
    pl = ctypes.byref(plan) if plan is not None else None
    _check(capi().tinym_fp8_gemm_allgather(x_ptr, w_ptr, m, n_local, k, alpha_ptr, alpha,
                                           ctypes.byref(desc), pl, stream))


def launch_plan(m: int, n: int, k: int, static_w: bool = False) -> Plan:
    """The plan a call without an explicit plan runs on the current GPU:
    the dispatch table's choice with the K split lowered, as the launcher
    does, until every cluster is resident at once (queries the device)."""
    p = Plan()
    _check(capi().tinym_launch_plan(m, n, k, 1 if static_w else 0, ctypes.byref(p)))
    return p


def max_active_clusters(m: int, n: int, k: int, plan: Plan) -> int:
    """Clusters of `plan` the current GPU can hold resident at once."""
    out = ctypes.c_int32(0)
    _check(capi().tinym_plan_max_active_clusters(m, n, k, ctypes.byref(plan), ctypes.byref(out)))
    return int(out.value)


def device_status(clear: bool = True) -> int:
    """Device error word (bounded-wait timeouts); synchronises the device."""
    flags = ctypes.c_uint32(0)
    st = capi().tinym_device_status(ctypes.byref(flags), 1 if clear else 0)
    if st not in (TINYM_OK, 6):
        _check(st)
    return int(flags.value)


def pending_errors(clear: bool = True) -> int:
    """Bits of bounded device waits that ran out in kernels that have already
    finished on the current device (0 = none), read without synchronising."""
    flags = ctypes.c_uint32(0)
    st = capi().tinym_pending_errors(ctypes.byref(flags), 1 if clear else 0)
    if st not in (TINYM_OK, 6):
        _check(st)
    return int(flags.value)


def raise_pending() -> None:
    """Raise TinymError if an earlier GEMM on the current device timed out
    (its output is unspecified); clears the report."""
    flags = ctypes.c_uint32(0)
    st = capi().tinym_pending_errors(ctypes.byref(flags), 1)
    if st != TINYM_OK:
        _check(st)


def gemm(x, w, alpha, *, out=None, plan: Plan | None = None, static_w: bool = False):
    """torch convenience wrapper over the C ABI (device alpha, current stream).
    Raises TinymError first if an earlier GEMM on the device timed out."""
    import torch

    if x.dtype != torch.float8_e4m3fn or w.dtype != torch.float8_e4m3fn:
        raise ValueError("x and w must be float8_e4m3fn")
    m, k, n = _check_operands(x, w)
    if isinstance(alpha, torch.Tensor) and (alpha.dtype != torch.float32 or alpha.numel() < 1):
        raise ValueError("a tensor alpha must be float32 with at least one element")
    out = _check_out(out, m, n, x)
    _check_devices(x, w, alpha if isinstance(alpha, torch.Tensor) else None, out)
    with torch.cuda.device(x.device):
        raise_pending()
    stream = torch.cuda.current_stream(x.device).cuda_stream
    if isinstance(alpha, torch.Tensor):
        gemm_ptr(x.data_ptr(), w.data_ptr(), out.data_ptr(), m, n, k, ldy=out.stride(0),
                 alpha_ptr=alpha.data_ptr(), plan=plan, stream=stream, static_w=static_w)
    else:
        gemm_ptr(x.data_ptr(), w.data_ptr(), out.data_ptr(), m, n, k, ldy=out.stride(0),
                 alpha=float(alpha), plan=plan, stream=stream, static_w=static_w)
    return out


__all__ = [
    "capi", "load_torch_op", "select_plan", "check_plan", "make_plan", "gemm_ptr", "gemm",
    "device_status", "pending_errors", "raise_pending", "Plan", "TinymError", "EXPORTED", "KERNEL_TC", "KERNEL_SIMT_M1",
    "packed_weight_bytes", "pack_weights_ptr", "gemm_packed_ptr", "quant_workspace_bytes",
    "gemm_quant_act", "ACT_BF16", "ACT_F32", "GatherDesc", "ipc_export", "ipc_open", "ipc_close",
    "gemm_allgather_ptr",
]
