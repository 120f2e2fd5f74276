"""The vLLM plugin's weight processing and apply on the GPU: the repacked weight equals the
oracle's repack_awq_to_tf bit for bit, and apply matches the oracle's fp64 product within the
W4A16 tolerance."""

from __future__ import annotations

import pytest
import torch

from oracle import oracle
from tests.numerics import cases
from tests.numerics.tolerance import atol

pytestmark = pytest.mark.gpu
pytest.importorskip("vllm")


@pytest.mark.parametrize("m", [1, 32])
def test_process_and_apply(m: int, device: torch.device, monkeypatch: pytest.MonkeyPatch) -> None:
    plugin = pytest.importorskip("tokenforge_b200.vllm_plugin")
    import vllm.model_executor.parameter as vparam

    # vLLM's parameter classes ask for the tensor-parallel rank; one process is rank 0 of 1.
    monkeypatch.setattr(vparam, "get_tensor_model_parallel_rank", lambda: 0, raising=False)
    monkeypatch.setattr(vparam, "get_tensor_model_parallel_world_size", lambda: 1, raising=False)
    n, k, g = 256, 1024, 128
    cfg = plugin.TokenForgeConfig(4, g, True)
    method = plugin.TokenForgeLinearMethod(cfg)
    layer = torch.nn.Module()
    method.create_weights(layer, k, [n], k, n, torch.float16, weight_loader=None)
    gen = torch.Generator().manual_seed(m)
    qweight, qzeros, scales = oracle.awq_quantize(torch.randn((n, k), generator=gen) * 0.02, g)
    layer.qweight.data = qweight.to(device)
    layer.qzeros.data = qzeros.to(device)
    layer.scales.data = scales.to(device)
    method.process_weights_after_loading(layer)
    qweight_t = oracle.repack_awq_to_tf(qweight)
    assert torch.equal(layer.qweight_t.cpu(), qweight_t)
    assert not hasattr(layer, "qweight")
    x = cases.activations(m, k, m)
    bias = cases.bias(n, m)
    y = method.apply(layer, x.to(device), bias.to(device))
    ref = oracle.w4a16_reference(x, qweight_t, scales, qzeros, g, bias)
    w16 = oracle.dequantize_tf(qweight_t, scales, qzeros, g)
    assert float((y.cpu().double() - ref).abs().max()) <= atol(x, w16, "cuda")
