"""Harness entry point for the B200-native tiny-M FP8 GEMM (drop-in).

Same module name and functions as the reference's candidate_kernel.py
(``build``, ``prepare_weights``, ``fp8_gemm``; candidate_kernel.py:33-105),
so ``fp8_gemm_task_harness.py --impl candidate_kernel`` runs unchanged:

    out = fp8_gemm(a, prepare_weights(b), alpha)
    # a: [M,K] float8_e4m3fn CUDA, b: [N,K] float8_e4m3fn CUDA,
    # alpha: [1] float32 CUDA  ->  [M,N] bfloat16 CUDA

Differences from the reference adapter:

* ``build()`` loads the in-tree sm_100a libraries (building them with nvcc
  if they are missing) instead of JIT-compiling for sm_120a.
* alpha stays on the device: the op reads it inside the kernel.  The host
  reads it only to keep the reference's error behaviour (``alpha must be
  finite``, src/torch_candidate_extension.cu:30), once per alpha tensor and
  version as the reference's ``_host_alpha`` cache does
  (candidate_kernel.py:77-94); calls with an alpha already checked do not
  synchronise, and a call made while the stream is being captured into a
  CUDA graph skips the read.
* any 1 <= M <= 16 and K % 16 == 0 is accepted, not only the six official
  points (reference src/torch_candidate_extension.cu:40-46).
* ``prepare_weights`` may repack W (the harness runs it once, untimed,
  fp8_gemm_task_harness.py:13-19): with ``TINYM_WEIGHT_LAYOUT=packed`` (or
  ``prepare_weights(b, layout="packed")``) it returns a ``PackedWeight`` in
  the tile-contiguous layout of tinym_pack_weights, which ``fp8_gemm``
  accepts in place of the [N,K] tensor.  The default keeps the reference's
  identity.
* ``fp8_gemm_act(x, b, w_scale)`` takes the activation before quantisation
  (BF16 or FP32): the per-tensor E4M3 quantisation of the harness's
  ``quantize_per_tensor`` (fp8_gemm_task_harness.py:41-44) runs on the device
  as a prologue overlapped with the GEMM's weight stream.

There is no fallback: if the native library cannot be loaded, ``build()``
raises.
"""

from __future__ import annotations

import math
import os
import sys
import threading
from pathlib import Path
from typing import Any

import torch

_ROOT = Path(__file__).resolve().parent
_SRC = _ROOT / "sm120-fp8-gemm-submit_b200"
if str(_SRC) not in sys.path:
    sys.path.insert(0, str(_SRC))

import tinym_b200  # noqa: E402  (package lives in the source root above)

_BUILT = False
_BUILD_LOCK = threading.Lock()
_run_alpha_tensor = None
_run_packed = None
_pack = None
_run_quant_act = None
# The alpha tensor (and its version counter) last checked finite.
_ALPHA_TENSOR = None
_ALPHA_VERSION = None


class PackedWeight:
    """W [N, K] repacked into the tile-contiguous layout (include/tinym_b200.h:
    tinym_pack_weights); returned by prepare_weights(b, layout="packed")."""

    __slots__ = ("data", "n", "k")

    def __init__(self, data: torch.Tensor, n: int, k: int):
        self.data, self.n, self.k = data, n, k

    @property
    def shape(self):
        return (self.n, self.k)

    @property
    def device(self):
        return self.data.device


def build():
    """Load (building once if needed) the native op; returns True."""
    global _BUILT, _run_alpha_tensor, _run_packed, _pack, _run_quant_act
    if _BUILT:
        return True
    with _BUILD_LOCK:
        if not _BUILT:
            tinym_b200.load_torch_op()
            _run_alpha_tensor = torch.ops.sm120_fp8_gemm.run_alpha_tensor
            _run_packed = torch.ops.sm120_fp8_gemm.run_packed
            _pack = torch.ops.sm120_fp8_gemm.pack_weights
            _run_quant_act = torch.ops.sm120_fp8_gemm.run_quant_act
            _BUILT = True
    return True


def prepare_weights(b: torch.Tensor, layout: str | None = None) -> Any:
    """Validate W (reference :68-74) and return it unchanged, or repacked
    when layout (default: env TINYM_WEIGHT_LAYOUT, else "rowmajor") is
    "packed"."""
    if not b.is_cuda or b.dtype != torch.float8_e4m3fn or b.ndim != 2:
        raise ValueError("B must be a rank-2 CUDA float8_e4m3fn tensor")
    if not b.is_contiguous():
        raise ValueError("B must be contiguous row-major")
    layout = layout or os.environ.get("TINYM_WEIGHT_LAYOUT", "rowmajor")
    if layout == "rowmajor":
        return b
    if layout != "packed":
        raise ValueError(f"unknown weight layout {layout!r} (rowmajor | packed)")
    if not _BUILT:
        build()
    return PackedWeight(_pack(b), b.shape[0], b.shape[1])


def _check_alpha(alpha: torch.Tensor) -> None:
    """The reference's alpha checks: ValueError for a tensor that is not a
    one-element CUDA float32 (candidate_kernel.py:77-94), RuntimeError for a
    non-finite value (src/torch_candidate_extension.cu:30).  The value is read
    once per (tensor, version), like the reference's cache."""
    global _ALPHA_TENSOR, _ALPHA_VERSION
    if not isinstance(alpha, torch.Tensor):
        raise ValueError("alpha must be a one-element CUDA float32 tensor")
    try:
        version = alpha._version
    except RuntimeError:
        # inference-mode tensors have no version counter
        version = None
    if alpha is _ALPHA_TENSOR and version == _ALPHA_VERSION:
        return
    if not alpha.is_cuda or alpha.dtype != torch.float32 or alpha.numel() != 1:
        raise ValueError("alpha must be a one-element CUDA float32 tensor")
    if torch.cuda.is_current_stream_capturing():
        return  # no host read inside a capture; the kernel reads the device value
    if not math.isfinite(float(alpha.item())):
        raise RuntimeError("alpha must be finite")
    _ALPHA_TENSOR, _ALPHA_VERSION = alpha, version


def fp8_gemm(a: torch.Tensor, b: torch.Tensor, alpha: torch.Tensor) -> torch.Tensor:
    """Return (a.float() @ b.float().T) * alpha as BF16 on CUDA."""
    if not _BUILT:
        build()
    _check_alpha(alpha)
    if isinstance(b, PackedWeight):
        return _run_packed(a, b.data, b.n, b.k, alpha)
    return _run_alpha_tensor(a, b, alpha)


def fp8_gemm_act(x: torch.Tensor, b: torch.Tensor, w_scale: torch.Tensor):
    """Quantise the activation x (BF16/FP32 [M,K]) per tensor on the device and
    return (bf16(alpha * q(x) @ b.float().T), x_scale) with alpha = x_scale *
    w_scale.  b is the [N,K] E4M3 weight, w_scale its one-element CUDA scale."""
    if not _BUILT:
        build()
    return _run_quant_act(x, b, w_scale)


__all__ = ["build", "prepare_weights", "fp8_gemm"]
