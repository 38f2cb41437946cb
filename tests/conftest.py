"""Shared fixtures for the tiny-M FP8 GEMM tests.

Marker ``gpu``: needs an sm_100 GPU (run on the B200 box with ``-m gpu``).
Everything else runs on CPU only.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
SRC = ROOT / "sm120-fp8-gemm-submit_b200"
for p in (str(ROOT), str(SRC)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: requires an sm_100 (B200) GPU")


@pytest.fixture(scope="session")
def oracle():
    from oracle import fp8_oracle

    return fp8_oracle


@pytest.fixture(scope="session")
def golden_cases():
    data = np.load(GOLDEN / "cases.npz")
    cases = []
    for i in range(int(data["num_cases"])):
        p = f"c{i}_"
        m, k, n, seed = (int(v) for v in data[p + "shape"])
        case = {"m": m, "k": k, "n": n, "seed": seed}
        for key in ("a", "w", "aq", "wq", "sa", "sw", "alpha", "ref", "ref_bf16"):
            if p + key in data:
                case[key] = data[p + key]
        cases.append(case)
    return cases


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.skip(f"needs sm_100, found sm_{major}{minor}")
    return torch.device("cuda:0")
