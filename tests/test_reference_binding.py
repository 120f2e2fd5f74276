"""The drop-in ``_C`` boundary, seen from the reference's side (CPU only).

Installing ``tokenforge_b200._C`` as ``tokenforge.kernels._C`` must do exactly one thing to the
reference: make its extension probe (tokenforge/kernels/ops.py:29-40) report the CUDA
extension as available, so decode-sized calls with ``backend="cuda"`` on GPU tensors reach
``_C.w4a16_gemv``. It must not touch the reference's own ``torch.ops.tokenforge.*``
registrations: a CPU call of ``torch.ops.tokenforge.w4a16_linear`` still runs the reference's
torch path. Both packages register the same op names, so the check runs in a fresh interpreter
with the reference's checkout first on the path. It needs that checkout and skips without it.
"""

from __future__ import annotations

import os
import subprocess
import sys
import textwrap
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
# The TokenForge checkout: $TOKENFORGE_REFERENCE, else a `reference` directory beside this repo.
REFERENCE = Path(os.environ.get("TOKENFORGE_REFERENCE", str(ROOT.parent / "reference")))

SCRIPT = textwrap.dedent(
    """
    import sys

    import torch

    import tokenforge_b200._C as shim

    # Route 1 of the integration notes: the shim installed as the reference's _C module.
    sys.modules["tokenforge.kernels._C"] = shim
    import tokenforge.kernels as tk

    tk._C = shim
    from tokenforge.kernels import ops as ref_ops
    from tokenforge.kernels.pack import W4A16Weights, awq_pack, repack_awq_to_tf
    from tokenforge.kernels.reference import w4a16_torch

    assert "tokenforge_b200.ops" not in sys.modules, "the shim registered tokenforge_b200's ops"
    assert ref_ops.cuda_ext_available(), "the reference's probe does not see the extension"
    assert ref_ops._cuda_ext() is shim

    gen = torch.Generator().manual_seed(0)
    n, k, g = 64, 256, 128
    q = torch.randint(0, 16, (k, n), generator=gen, dtype=torch.int32)
    z = torch.randint(0, 16, (k // g, n), generator=gen, dtype=torch.int32)
    s = (torch.rand((k // g, n), generator=gen) * 0.018 + 0.002).half()
    qweight, qzeros = awq_pack(q, z)
    w = W4A16Weights(repack_awq_to_tf(qweight), s, qzeros, g)
    x = torch.randn((3, k), generator=gen).half()
    for backend in ("cuda", "triton"):
        y = torch.ops.tokenforge.w4a16_linear(x, w.qweight_t, w.scales, w.qzeros, None, g, backend)
        assert torch.equal(y, w4a16_torch(x, w, None)), backend
    print("ok")
    """
)


@pytest.mark.skipif(not (REFERENCE / "tokenforge" / "kernels" / "ops.py").exists(),
                    reason="needs the reference checkout")
def test_shim_keeps_the_reference_ops() -> None:
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([str(REFERENCE), str(ROOT)])
    env["PYTHONDONTWRITEBYTECODE"] = "1"
    env["CUDA_VISIBLE_DEVICES"] = ""
    proc = subprocess.run([sys.executable, "-c", SCRIPT], env=env, capture_output=True,
                          text=True, timeout=600, cwd=str(ROOT))
    assert proc.returncode == 0, proc.stdout + proc.stderr
    assert proc.stdout.strip().endswith("ok")
