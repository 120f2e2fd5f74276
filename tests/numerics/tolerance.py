"""Derived tolerance for W4A16 outputs (the reference's rule, tests/numerics/tolerance.py:24-46).

With fp32 accumulation the error grows like sqrt(K):

    atol = c * sqrt(K) * eps_fp16 * max|x| * max|w|

``c`` is calibrated per device type against the vendor fp16 GEMM (cuBLAS on CUDA) by
``python -m tests.numerics.calibrate --device cuda --write`` and frozen in tolerances.json; a
kernel that needs a looser constant than the vendor GEMM fails.
"""

from __future__ import annotations

import json
import math
from pathlib import Path

import torch

EPS_FP16 = float(torch.finfo(torch.float16).eps)  # 2**-10
TOLERANCES_PATH = Path(__file__).with_name("tolerances.json")


def error_scale(x: torch.Tensor, w: torch.Tensor) -> float:
    """``sqrt(K) * eps_fp16 * max|x| * max|w|`` over finite entries."""
    k = x.shape[-1]
    xf = x.to(torch.float64)
    wf = w.to(torch.float64)
    finite = torch.isfinite(xf)
    xmax = float(xf[finite].abs().max()) if finite.any() else 0.0
    wmax = float(wf.abs().max()) if wf.numel() else 0.0
    return math.sqrt(k) * EPS_FP16 * xmax * wmax


def load_constant(device_type: str) -> float:
    data = json.loads(TOLERANCES_PATH.read_text())
    entry = data["w4a16"].get(device_type)
    if entry is None:
        raise LookupError(
            f"no calibrated tolerance for device '{device_type}'; run "
            f"`python -m tests.numerics.calibrate --device {device_type} --write` once and commit it"
        )
    return float(entry["c"])


def atol(x: torch.Tensor, w: torch.Tensor, device_type: str) -> float:
    return load_constant(device_type) * error_scale(x, w)
