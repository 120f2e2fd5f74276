"""The vLLM out-of-tree quantization backend (tokenforge_b200.vllm_plugin) on CPU: registration
under the name "tokenforge", the AWQ config keys, the version guard and the checkpoint-layout
parameters create_weights registers. (Repack and apply run on the GPU: test_gpu_vllm_plugin.)"""

from __future__ import annotations

import pytest
import torch

vllm = pytest.importorskip("vllm")
plugin = pytest.importorskip("tokenforge_b200.vllm_plugin")


@pytest.fixture(autouse=True)
def _single_rank(monkeypatch: pytest.MonkeyPatch) -> None:
    """vLLM's parameter classes ask for the tensor-parallel rank; one process is rank 0 of 1."""
    import vllm.model_executor.parameter as vparam

    monkeypatch.setattr(vparam, "get_tensor_model_parallel_rank", lambda: 0, raising=False)
    monkeypatch.setattr(vparam, "get_tensor_model_parallel_world_size", lambda: 1, raising=False)


def test_registered_as_a_quantization_method() -> None:
    from vllm.model_executor.layers.quantization import (
        QUANTIZATION_METHODS,
        get_quantization_config,
    )

    assert "tokenforge" in QUANTIZATION_METHODS
    assert get_quantization_config("tokenforge") is plugin.TokenForgeConfig


def test_reads_awq_config_keys() -> None:
    cfg = plugin.TokenForgeConfig.from_config(
        {"quant_method": "awq", "w_bit": 4, "q_group_size": 128, "zero_point": True,
         "version": "gemm"})
    assert (cfg.weight_bits, cfg.group_size, cfg.zero_point) == (4, 128, True)
    assert cfg.get_name() == "tokenforge"
    assert cfg.get_min_capability() == 100
    alt = plugin.TokenForgeConfig.from_config({"bits": 4, "group_size": 64, "zero_point": True,
                                               "modules_to_not_convert": ["lm_head"]})
    assert alt.group_size == 64 and alt.modules_to_not_convert == ["lm_head"]


@pytest.mark.parametrize("bad", [{"w_bit": 8, "q_group_size": 128, "zero_point": True},
                                 {"w_bit": 4, "q_group_size": 128, "zero_point": False},
                                 {"w_bit": 4, "q_group_size": 96, "zero_point": True}])
def test_rejects_what_the_kernels_do_not_serve(bad: dict) -> None:  # type: ignore[type-arg]
    with pytest.raises(ValueError):
        plugin.TokenForgeConfig.from_config(bad)


def test_awq_checkpoints_switch_only_on_request() -> None:
    cls = plugin.TokenForgeConfig
    assert cls.override_quantization_method({"quant_method": "awq"}, "tokenforge") == "tokenforge"
    assert cls.override_quantization_method({"quant_method": "awq"}, None) is None
    assert cls.override_quantization_method({"quant_method": "gptq"}, "tokenforge") is None


def test_version_guard() -> None:
    plugin.check_vllm_version("0.22.0")
    for bad in ("0.9.2", "0.23.0", "1.0.0"):
        with pytest.raises(RuntimeError, match="supports vLLM"):
            plugin.check_vllm_version(bad)
    plugin.register()


def test_create_weights_registers_the_checkpoint_layout() -> None:
    cfg = plugin.TokenForgeConfig(4, 128, True)
    method = cfg.get_quant_method(torch.nn.Linear(4, 4), "model.layers.0.mlp.down_proj")
    assert method is None  # not a vLLM LinearBase
    layer = torch.nn.Module()
    plugin.TokenForgeLinearMethod(cfg).create_weights(
        layer, input_size_per_partition=512, output_partition_sizes=[64, 64], input_size=512,
        output_size=128, params_dtype=torch.float16, weight_loader=lambda *a, **k: None)
    assert tuple(layer.qweight.shape) == (512, 16) and layer.qweight.dtype == torch.int32
    assert tuple(layer.qzeros.shape) == (4, 16) and layer.qzeros.dtype == torch.int32
    assert tuple(layer.scales.shape) == (4, 128) and layer.scales.dtype == torch.float16
    with pytest.raises(ValueError, match="group"):
        plugin.TokenForgeLinearMethod(cfg).create_weights(
            torch.nn.Module(), 500, [64], 500, 64, torch.float16, weight_loader=None)
