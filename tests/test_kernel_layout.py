"""CPU check of the kernels' index arithmetic.

tests/kernel_layout_host.cu includes csrc/tinym_kernels.cuh and checks, on
the host, the functions the kernels and the launcher share: split-K row
ownership, the shared-memory carve-up (1024-byte stage alignment for the
128-byte swizzle, 16-byte receive blocks, room for every mbarrier), the K
ranges of a cluster and the packed layout's chunk count, over every plan
shape the launcher accepts.  nvcc builds it for sm_100a; it runs on the CPU.
"""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
CSRC = ROOT / "sm120-fp8-gemm-submit_b200" / "csrc"


def _nvcc():
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    return None


def test_kernel_index_arithmetic(tmp_path):
    nvcc = _nvcc()
    if nvcc is None:
        pytest.skip("nvcc not found")
    exe = tmp_path / "kernel_layout_host"
    build = subprocess.run(
        [nvcc, "-std=c++17", "-O1", "-gencode", "arch=compute_100a,code=sm_100a",
         "-I", str(CSRC), "-I", str(ROOT / "include"),
         str(ROOT / "tests" / "kernel_layout_host.cu"), "-o", str(exe)],
        capture_output=True, text=True, timeout=300)
    assert build.returncode == 0, build.stderr[-4000:]
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout[-4000:]
    last = run.stdout.strip().splitlines()[-1]
    assert last.startswith("kernel layout checks ok ("), last
    assert int(last.split("(")[1].split()[0]) > 50000  # every plan shape was visited
