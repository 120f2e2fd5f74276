"""Generate the golden vectors that pin the CPU oracle to the reference implementation.

Runs the reference (saransh-debugs/TokenForge) itself: its torch functions
(tokenforge/kernels/pack.py, tokenforge/kernels/reference.py) and its Triton kernels under the
CPU interpreter (TRITON_INTERPRET=1; tokenforge/kernels/triton/*.py), on small seeded inputs,
and writes the inputs and outputs to ``tests/golden/*.npz``. The reference is needed only
here; the committed ``.npz`` files are what the tests read.

    python tests/golden/make_golden.py --reference /path/to/TokenForge
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _np(t):  # type: ignore[no-untyped-def]
    import torch

    t = t.detach().cpu()
    if t.dtype == torch.float16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy()
    return t.numpy()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of saransh-debugs/TokenForge")
    args = ap.parse_args()
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, str(Path(args.reference).resolve()))

    import torch

    from tests.numerics import cases  # reference's own seeded case generators
    from tokenforge.kernels import pack, reference
    from tokenforge.kernels.config import default_config, m_bucket
    from tokenforge.kernels.triton.rmsnorm_fp8 import rmsnorm_fp8_quant
    from tokenforge.kernels.triton.w4a16 import w4a16_gemm

    out: dict[str, dict[str, np.ndarray]] = {}

    # --- nibble codec and repack (pack.py:42-67, 141-148)
    gen = torch.Generator().manual_seed(1234)
    codec: dict[str, np.ndarray] = {}
    for tag, (k, n) in {"a": (256, 64), "b": (64, 200), "c": (24, 8)}.items():
        qweight = torch.randint(-(2**31), 2**31 - 1, (k, n // 8), generator=gen, dtype=torch.int32)
        qweight_t = pack.repack_awq_to_tf(qweight)
        codec[f"{tag}_qweight"] = _np(qweight)
        codec[f"{tag}_qweight_t"] = _np(qweight_t)
        codec[f"{tag}_back"] = _np(pack.repack_tf_to_awq(qweight_t))
        codec[f"{tag}_unpacked"] = _np(pack.unpack_int4(qweight))
    ints = torch.randint(0, 16, (6, 40), generator=gen, dtype=torch.int32)
    codec["ints"] = _np(ints)
    codec["ints_packed"] = _np(pack.pack_int4(ints))
    sign = torch.zeros((1, 8), dtype=torch.int32)
    sign[0, pack.AWQ_ORDER[7]] = 15
    codec["sign_values"] = _np(sign)
    codec["sign_packed"] = _np(pack.pack_int4(sign))
    out["codec"] = codec

    # --- awq_quantize fixture generator (pack.py:83-107) and dequant (pack.py:189-194)
    deq: dict[str, np.ndarray] = {}
    gen = torch.Generator().manual_seed(99)
    weight = torch.randn((64, 256), generator=gen) * 0.02
    qweight, qzeros, scales = pack.awq_quantize(weight, 128)
    deq["quant_weight"] = _np(weight)
    deq["quant_qweight"], deq["quant_qzeros"], deq["quant_scales"] = map(_np, (qweight, qzeros, scales))
    for g in (32, 64, 128):
        w = cases.layer_weights(200, 384, 0, g)
        deq[f"g{g}_qweight_t"] = _np(w.qweight_t)
        deq[f"g{g}_scales"] = _np(w.scales)
        deq[f"g{g}_qzeros"] = _np(w.qzeros)
        deq[f"g{g}_dequant"] = _np(pack.dequantize_tf(w))
    out["dequant"] = deq

    # --- W4A16 linear: fp64 reference, torch CPU path and the Triton kernel (interpreter)
    lin: dict[str, np.ndarray] = {}
    n, k, g = 200, 512, 128
    w = cases.layer_weights(n, k, 0, g)
    b = cases.bias(n, 0)
    lin["qweight_t"], lin["scales"], lin["qzeros"], lin["bias"] = map(
        _np, (w.qweight_t, w.scales, w.qzeros, b)
    )
    for m in (1, 3, 8, 16, 33):
        x = cases.activations(m, k, 0)
        lin[f"m{m}_x"] = _np(x)
        lin[f"m{m}_ref64"] = _np(reference.w4a16_reference(x, w, b))
        lin[f"m{m}_torch"] = _np(reference.w4a16_torch(x, w, b))
        if m in (1, 3, 16):
            cfg = default_config(m_bucket(m), n, k, g)
            lin[f"m{m}_triton"] = _np(
                w4a16_gemm(x, w.qweight_t, w.scales, w.qzeros, g, cfg, b)
            )
    out["w4a16"] = lin

    # --- RMSNorm + FP8 (reference.py:35-56; triton/rmsnorm_fp8.py)
    rms: dict[str, np.ndarray] = {}
    eps = 1e-6
    for tag, (t, h, scale) in {"a": (7, 896, 2.0), "b": (3, 1000, 2.0), "c": (16, 896, 3.0)}.items():
        gen = torch.Generator().manual_seed(t * h)
        x = (torch.randn((t, h), generator=gen) * scale).to(torch.float16)
        wt = (torch.rand((h,), generator=gen) + 0.5).to(torch.float16)
        static = torch.tensor([2e-3], dtype=torch.float32) if tag == "c" else None
        q_ref, s_ref = reference.rmsnorm_fp8_reference(x, wt, eps, static)
        q_tri, s_tri = rmsnorm_fp8_quant(x, wt, eps, static)
        rms[f"{tag}_x"], rms[f"{tag}_w"] = _np(x), _np(wt)
        rms[f"{tag}_q_ref"], rms[f"{tag}_s_ref"] = _np(q_ref), _np(s_ref)
        rms[f"{tag}_q_triton"], rms[f"{tag}_s_triton"] = _np(q_tri), _np(s_tri)
        rms[f"{tag}_y16"] = _np(reference.rmsnorm(x, wt, eps))
        if static is not None:
            rms[f"{tag}_static"] = _np(static)
    out["rmsnorm_fp8"] = rms

    # --- e4m3 known-answer set: every code, every midpoint, and its fp32 neighbours, both
    # signs and +-0 (the probe set of tests/numerics/test_rmsnorm_fp8.py:89-101); the answer is
    # torch's float8_e4m3fn cast, the reference's arithmetic for this step.
    values = torch.arange(0, 0x7F, dtype=torch.uint8).view(torch.float8_e4m3fn).float()
    mids = (values[1:] + values[:-1]) / 2
    probe = torch.cat([values, mids, mids.nextafter(torch.tensor(1e9)), mids.nextafter(torch.tensor(-1e9))])
    probe = torch.cat([probe, -probe, torch.tensor([0.0, -0.0])])
    out["e4m3_kat"] = {"probe": _np(probe), "codes": _np(probe.to(torch.float8_e4m3fn))}

    for name, arrays in out.items():
        np.savez_compressed(HERE / f"{name}.npz", **arrays)
        print(name, sum(a.nbytes for a in arrays.values()), "bytes")


if __name__ == "__main__":
    main()
