"""Calibrate the tolerance constant ``c`` against the vendor fp16 GEMM and freeze it.

    python -m tests.numerics.calibrate --device cuda --write

Same procedure as the reference (tests/numerics/calibrate.py:26-68): ``c`` is the worst
``max|y_vendor - y_ref| / error_scale`` over every (shape, M, seed) the numerics tests use,
with ``y_vendor = x16 @ w16^T`` from cuBLAS (torch defaults) and ``y_ref`` the fp64 product of
the same fp16 inputs, rounded up to two significant figures. The fp16 weights are the oracle's
dequantization of the seeded AWQ layers; the fp64 reference product runs on the device.
"""

from __future__ import annotations

import argparse
import json
import math

import torch

from oracle import oracle
from tests.numerics import cases
from tests.numerics.shapes import M_SUITE, linear_shapes
from tests.numerics.tolerance import TOLERANCES_PATH, error_scale


def calibrate(device: str) -> dict[str, object]:
    worst, worst_case, n_cases = 0.0, (), 0
    for shape in linear_shapes():
        for seed in cases.CALIBRATION_SEEDS:
            w = cases.layer_weights(shape.n, shape.k, seed)
            w16 = oracle.dequantize_tf(w.qweight_t, w.scales, w.qzeros, w.group_size)
            w_dev = w16.to(device)
            w64 = w_dev.to(torch.float64)
            for m in M_SUITE:
                x16 = cases.activations(m, shape.k, seed)
                x_dev = x16.to(device)
                ref = (x_dev.to(torch.float64) @ w64.t()).cpu()
                y = (x_dev @ w_dev.t()).cpu().to(torch.float64)
                ratio = float((y - ref).abs().max()) / error_scale(x16, w16)
                n_cases += 1
                if ratio > worst:
                    worst, worst_case = ratio, (shape.layer, shape.n, shape.k, m, seed)
            del w_dev, w64
        cases.layer_weights.cache_clear()
    exp = math.floor(math.log10(worst))
    c = math.ceil(worst / 10 ** (exp - 1)) * 10 ** (exp - 1)
    return {
        "c": round(c, 6),
        "observed_max": worst,
        "worst_case": list(worst_case),
        "cases": n_cases,
        "suite": "full",
        "vendor_gemm": "cublas" if device == "cuda" else "aten-cpu-fp16",
        "device_name": torch.cuda.get_device_name() if device == "cuda" else "cpu",
        "torch": torch.__version__,
    }


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--device", choices=["cuda"], default="cuda")
    ap.add_argument("--write", action="store_true", help="freeze the result in tolerances.json")
    args = ap.parse_args()
    result = calibrate(args.device)
    print(json.dumps(result, indent=2))
    if args.write:
        data = json.loads(TOLERANCES_PATH.read_text()) if TOLERANCES_PATH.exists() else {}
        data.setdefault("w4a16", {})[args.device] = result
        TOLERANCES_PATH.write_text(json.dumps(data, indent=2, sort_keys=True) + "\n")


if __name__ == "__main__":
    main()
