"""Build the native parts in-tree (no JIT cache outside the repository).

* ``lib/libtinym_b200.so``  -- kernels + C ABI (nvcc, sm_100a only, static
  CUDA runtime, no libcuda link: the driver entry point is resolved at run
  time, so the library also loads on machines without a GPU driver).
* ``lib/tinym_torch_op.so`` -- the ``torch.ops.sm120_fp8_gemm`` shim (g++
  against the installed torch; links the C ABI library via $ORIGIN).

The reference JIT-compiles through ``torch.utils.cpp_extension.load`` with
arch 12.0a (candidate_kernel.py:33-65); this build targets
``-gencode arch=compute_100a,code=sm_100a`` and writes next to the package so
the built files travel with the source tree.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
SRC_ROOT = PKG.parent
CSRC = SRC_ROOT / "csrc"
INCLUDE = SRC_ROOT.parent / "include"
LIBDIR = PKG / "lib"
CORE_SO = LIBDIR / "libtinym_b200.so"
TORCH_SO = LIBDIR / "tinym_torch_op.so"

GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]
CORE_SOURCES = [CSRC / "tinym_capi.cu"]
CORE_DEPS = CORE_SOURCES + [CSRC / "tinym_kernels.cuh", CSRC / "tinym_ptx.cuh",
                            CSRC / "tinym_quant.cuh",
                            INCLUDE / "tinym_b200.h"]
TORCH_SOURCES = [CSRC / "tinym_torch_op.cpp"]


def _cuda_home() -> Path:
    for cand in (os.environ.get("CUDA_HOME"), "/usr/local/cuda"):
        if cand and (Path(cand) / "bin" / "nvcc").exists():
            return Path(cand)
    nvcc = shutil.which("nvcc")
    if nvcc:
        return Path(nvcc).resolve().parent.parent
    raise RuntimeError("nvcc not found: set CUDA_HOME")


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def _run(cmd, verbose: bool) -> str:
    if verbose:
        print(" ".join(str(c) for c in cmd), flush=True)
    proc = subprocess.run([str(c) for c in cmd], capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"build step failed ({proc.returncode}):\n{' '.join(map(str, cmd))}\n"
                           f"{proc.stdout}\n{proc.stderr}")
    return proc.stdout + proc.stderr


def build_core(force: bool = False, verbose: bool = False) -> Path:
    """Compile the kernels and the C ABI into lib/libtinym_b200.so."""
    if not force and not _stale(CORE_SO, CORE_DEPS):
        return CORE_SO
    LIBDIR.mkdir(parents=True, exist_ok=True)
    nvcc = _cuda_home() / "bin" / "nvcc"
    tmp = CORE_SO.with_suffix(".so.tmp")
    out = _run([nvcc, *GENCODE, "-O3", "-std=c++17", "-lineinfo", "-Xptxas", "-v",
                "-Xcompiler", "-fPIC,-fvisibility=hidden", "-shared",
                "-I", INCLUDE, "-o", tmp, *CORE_SOURCES], verbose)
    os.replace(tmp, CORE_SO)
    (LIBDIR / "ptxas_core.txt").write_text(out)
    return CORE_SO


def build_torch_op(force: bool = False, verbose: bool = False) -> Path:
    """Compile the torch.ops.sm120_fp8_gemm shim into lib/tinym_torch_op.so."""
    core = build_core(force=force, verbose=verbose)
    if not force and not _stale(TORCH_SO, TORCH_SOURCES + [core, INCLUDE / "tinym_b200.h"]):
        return TORCH_SO
    import torch
    from torch.utils import cpp_extension

    cuda = _cuda_home()
    torch_lib = Path(torch.__file__).resolve().parent / "lib"
    incs = []
    for p in cpp_extension.include_paths():
        incs += ["-I", p]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cxx = os.environ.get("CXX", "g++")
    tmp = TORCH_SO.with_suffix(".so.tmp")
    _run([cxx, "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
          "-DTORCH_API_INCLUDE_EXTENSION_H", "-I", sysconfig.get_paths()["include"], *incs,
          "-I", cuda / "include", "-I", INCLUDE, *TORCH_SOURCES, "-o", tmp,
          "-L", LIBDIR, "-ltinym_b200", "-L", torch_lib, "-lc10", "-lc10_cuda", "-ltorch",
          "-ltorch_cpu", "-ltorch_cuda", f"-Wl,-rpath,$ORIGIN:{torch_lib}"], verbose)
    os.replace(tmp, TORCH_SO)
    return TORCH_SO


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_core(force=force, verbose=verbose)
    build_torch_op(force=force, verbose=verbose)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose=True)
    print("built", CORE_SO, TORCH_SO)
