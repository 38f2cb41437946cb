"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a container where the reference checkout is present:

    python tests/golden/make_golden.py --reference-root <path to the reference>

It imports the reference harness ``fp8_gemm_task_harness.py`` and runs its
own ``quantize_per_tensor`` (lines 41-44), ``reference`` (lines 63-65) and
``max_rel_err`` (lines 72-73) on CPU torch.  The harness's ``make_case``
(lines 47-60) hard-codes a CUDA generator, so the operands are drawn here
with a CPU ``torch.Generator`` using the same statements (same distribution,
same planted +-30/+-25 spikes).  Outputs:

* ``e4m3_codes.npz``  -- torch's float8_e4m3fn decode of all 256 codes and
  torch's encode of a probe vector (ties, subnormals, saturation edges);
* ``cases.npz``       -- per case: raw FP32 operands, the reference's FP8
  codes and scales, alpha, the reference's FP32 oracle output and the
  reference's BF16-rounded output.

The fixtures are small (tens of KB) and committed; the GPU box never reads
the reference checkout.
"""

from __future__ import annotations

import argparse
import importlib.util
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

# (M, K, N, seed, keep_raw) -- small enough for the CPU suite, shaped to
# cover one and several K blocks of 128, ragged N and every M class (1, odd,
# 8, 9, 16).  keep_raw stores the FP32 operands too (they pin the quantiser);
# the others store only the reference's FP8 codes, scales and outputs, which
# keeps the fixture file small.
CASES = [
    (1, 128, 128, 11, True),
    (1, 640, 72, 12, False),
    (3, 256, 136, 13, True),
    (8, 384, 64, 14, False),
    (9, 512, 96, 15, False),
    (16, 256, 130, 16, True),
    (9, 6144, 8, 17, False),
    (1, 5120, 8, 18, False),
]


def load_harness(reference_root: Path):
    path = reference_root / "fp8_gemm_task_harness.py"
    spec = importlib.util.spec_from_file_location("ref_harness", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def make_operands_cpu(m: int, k: int, n: int, seed: int):
    """fp8_gemm_task_harness.py:48-56 on a CPU generator."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    a = torch.randn(m, k, dtype=torch.float32, generator=g) * 2.0
    w = torch.randn(n, k, dtype=torch.float32, generator=g) * 0.03
    a.view(-1)[::37] = 30.0
    a.view(-1)[17::74] = -30.0
    w.view(-1)[::1531] = 25.0
    w.view(-1)[733::3062] = -25.0
    return a, w


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-root", type=Path, required=True)
    args = ap.parse_args()
    h = load_harness(args.reference_root)

    # 1. Code table and encoder probe, straight from torch's float8_e4m3fn.
    codes = torch.arange(256, dtype=torch.int32).to(torch.uint8)
    decoded = codes.view(torch.float8_e4m3fn).float().numpy()
    grid = decoded[:0x7F]
    mids = (grid[1:] + grid[:-1]) / 2.0  # exact ties between neighbours
    probe = np.concatenate([
        grid, -grid, mids, -mids,
        np.nextafter(mids, np.float32(0)), np.nextafter(mids, np.float32(1e9)),
        np.float32([0.0, -0.0, 2.0 ** -10, 2.0 ** -11, 3 * 2.0 ** -11, 447.9, 448.0, -448.0]),
        np.random.default_rng(5).uniform(-448, 448, 4096).astype(np.float32),
        np.random.default_rng(6).standard_normal(4096).astype(np.float32) * 1e-2,
    ]).astype(np.float32)
    probe_codes = torch.from_numpy(probe).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.savez_compressed(HERE / "e4m3_codes.npz", decoded=decoded, probe=probe,
                        probe_codes=probe_codes)

    # 2. End-to-end cases through the reference's own functions.
    out = {}
    for i, (m, k, n, seed, keep_raw) in enumerate(CASES):
        a, w = make_operands_cpu(m, k, n, seed)
        aq, sa = h.quantize_per_tensor(a)
        wq, sw = h.quantize_per_tensor(w)
        alpha = (sa * sw).to(torch.float32).reshape(1)
        ref = h.reference(aq, wq, alpha)
        ref_bf16 = ref.to(torch.bfloat16)
        assert h.max_rel_err(ref_bf16, ref) <= 4e-3
        p = f"c{i}_"
        out[p + "shape"] = np.array([m, k, n, seed], dtype=np.int64)
        if keep_raw:
            out[p + "a"] = a.numpy()
            out[p + "w"] = w.numpy()
        out[p + "aq"] = aq.view(torch.uint8).numpy()
        out[p + "wq"] = wq.view(torch.uint8).numpy()
        out[p + "sa"] = sa.numpy().astype(np.float32)
        out[p + "sw"] = sw.numpy().astype(np.float32)
        out[p + "alpha"] = alpha.numpy().astype(np.float32)
        out[p + "ref"] = ref.numpy().astype(np.float32)
        out[p + "ref_bf16"] = ref_bf16.view(torch.int16).numpy().view(np.uint16)
    out["num_cases"] = np.array(len(CASES), dtype=np.int64)
    np.savez_compressed(HERE / "cases.npz", **out)
    print("wrote", HERE / "e4m3_codes.npz", HERE / "cases.npz")


if __name__ == "__main__":
    main()
