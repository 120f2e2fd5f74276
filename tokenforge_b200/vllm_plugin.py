"""vLLM out-of-tree quantization backend: AWQ checkpoints served by the B200 kernels.

The reference plans this plugin (docs/design.md:95-101: a ``vllm.general_plugins`` entry
point, a version guard, AWQ checkpoints loaded unchanged, ``apply`` calling
``w4a16_linear(..., "cuda")``) but does not ship it. Here:

* :class:`TokenForgeConfig` is registered as quantization method ``"tokenforge"``. It reads the
  AWQ ``quant_config.json`` keys (4-bit, zero point, group size 32/64/128), so an AWQ model
  loads with ``LLM(model, quantization="tokenforge")``.
* :class:`TokenForgeLinearMethod` registers the checkpoint tensors in AWQ layout
  (``qweight`` [K, N/8], ``qzeros`` [K/G, N/8], ``scales`` [K/G, N]) with vLLM's packed and
  group-scale parameter classes, so vLLM's own loaders shard them for tensor parallelism;
  ``process_weights_after_loading`` repacks ``qweight`` once on the GPU
  (``tokenforge::awq_repack``, bit-exact with the reference's ``repack_awq_to_tf``) and
  ``apply`` is one ``tokenforge::w4a16_linear`` call: no host syncs, CUDA-graph capturable.
* :func:`register` is the entry point; it refuses vLLM versions outside the tested range.

vLLM is an optional dependency: importing this module imports vLLM.
"""

from __future__ import annotations

from typing import Any

import torch

SUPPORTED_VLLM = ((0, 10), (0, 23))  # [low, high) major.minor range this module was written for


def _version_tuple(version: str) -> tuple[int, int]:
    parts = version.split(".")
    return int(parts[0]), int("".join(ch for ch in parts[1] if ch.isdigit()) or 0)


def check_vllm_version(version: str | None = None) -> None:
    """Raise if the installed vLLM is outside :data:`SUPPORTED_VLLM` (API churn then fails at
    start-up instead of producing wrong outputs)."""
    if version is None:
        import vllm

        version = vllm.__version__
    low, high = SUPPORTED_VLLM
    v = _version_tuple(version)
    if not (low <= v < high):
        raise RuntimeError(
            f"tokenforge_b200 vLLM plugin supports vLLM {low[0]}.{low[1]} <= version < "
            f"{high[0]}.{high[1]}, found {version}"
        )


check_vllm_version()

from vllm.model_executor.layers.linear import (  # noqa: E402
    LinearBase,
    LinearMethodBase,
    UnquantizedLinearMethod,
)
from vllm.model_executor.layers.quantization import register_quantization_config  # noqa: E402
from vllm.model_executor.layers.quantization.base_config import QuantizationConfig  # noqa: E402
from vllm.model_executor.parameter import (  # noqa: E402
    GroupQuantScaleParameter,
    PackedvLLMParameter,
)

PACK_FACTOR = 8


@register_quantization_config("tokenforge")
class TokenForgeConfig(QuantizationConfig):
    """AWQ (4-bit, zero point) checkpoint executed by the tokenforge_b200 kernels."""

    def __init__(self, weight_bits: int, group_size: int, zero_point: bool,
                 modules_to_not_convert: list[str] | None = None) -> None:
        super().__init__()
        if weight_bits != 4:
            raise ValueError(f"tokenforge serves 4-bit AWQ weights, got {weight_bits} bits")
        if not zero_point:
            raise ValueError("tokenforge serves AWQ weights with zero points")
        if group_size not in (32, 64, 128):
            raise ValueError(f"group size {group_size} must be 32, 64 or 128")
        self.weight_bits = weight_bits
        self.group_size = group_size
        self.zero_point = zero_point
        self.modules_to_not_convert = list(modules_to_not_convert or [])

    def __repr__(self) -> str:
        return (f"TokenForgeConfig(weight_bits={self.weight_bits}, group_size={self.group_size}, "
                f"modules_to_not_convert={self.modules_to_not_convert})")

    def get_name(self) -> str:  # type: ignore[override]
        return "tokenforge"

    def get_supported_act_dtypes(self) -> list[torch.dtype]:
        return [torch.half]

    @classmethod
    def get_min_capability(cls) -> int:
        return 100  # sm_100 (B200)

    @staticmethod
    def get_config_filenames() -> list[str]:
        return ["quant_config.json", "quantize_config.json"]

    @classmethod
    def from_config(cls, config: dict[str, Any]) -> TokenForgeConfig:
        return cls(
            weight_bits=cls.get_from_keys(config, ["w_bit", "bits"]),
            group_size=cls.get_from_keys(config, ["q_group_size", "group_size"]),
            zero_point=cls.get_from_keys(config, ["zero_point"]),
            modules_to_not_convert=cls.get_from_keys_or(config, ["modules_to_not_convert"], None),
        )

    @classmethod
    def override_quantization_method(cls, hf_quant_cfg, user_quant):  # type: ignore[no-untyped-def]
        """An AWQ checkpoint runs here when the user asks for ``quantization="tokenforge"``."""
        method = (hf_quant_cfg or {}).get("quant_method", "").lower()
        if user_quant == "tokenforge" and method == "awq":
            return "tokenforge"
        return None

    def get_quant_method(self, layer: torch.nn.Module, prefix: str):  # type: ignore[no-untyped-def]
        if not isinstance(layer, LinearBase):
            return None
        if any(name in prefix for name in self.modules_to_not_convert):
            return UnquantizedLinearMethod()
        return TokenForgeLinearMethod(self)


class TokenForgeLinearMethod(LinearMethodBase):
    """Linear layers of an AWQ checkpoint on the tokenforge_b200 kernels."""

    def __init__(self, quant_config: TokenForgeConfig) -> None:
        self.quant_config = quant_config

    def create_weights(self, layer: torch.nn.Module, input_size_per_partition: int,  # type: ignore[override]
                       output_partition_sizes: list[int], input_size: int, output_size: int,
                       params_dtype: torch.dtype, **extra_weight_attrs: Any) -> None:
        g = self.quant_config.group_size
        n = sum(output_partition_sizes)
        k = input_size_per_partition
        if k % g:
            raise ValueError(f"input size per partition {k} is not a multiple of the group "
                             f"size {g} (tensor-parallel degree too large?)")
        if n % PACK_FACTOR:
            raise ValueError(f"output size per partition {n} is not a multiple of {PACK_FACTOR}")
        loader = extra_weight_attrs.get("weight_loader")
        qweight = PackedvLLMParameter(
            data=torch.empty(k, n // PACK_FACTOR, dtype=torch.int32), input_dim=0, output_dim=1,
            packed_dim=1, packed_factor=PACK_FACTOR, weight_loader=loader)
        qzeros = PackedvLLMParameter(
            data=torch.empty(k // g, n // PACK_FACTOR, dtype=torch.int32), input_dim=0,
            output_dim=1, packed_dim=1, packed_factor=PACK_FACTOR, weight_loader=loader)
        scales = GroupQuantScaleParameter(
            data=torch.empty(k // g, n, dtype=params_dtype), input_dim=0, output_dim=1,
            weight_loader=loader)
        layer.register_parameter("qweight", qweight)
        layer.register_parameter("qzeros", qzeros)
        layer.register_parameter("scales", scales)

    def process_weights_after_loading(self, layer: torch.nn.Module) -> None:
        import tokenforge_b200.ops  # noqa: F401  (registers torch.ops.tokenforge)

        qweight_t = torch.ops.tokenforge.awq_repack(layer.qweight.data.contiguous())
        layer.qweight_t = torch.nn.Parameter(qweight_t, requires_grad=False)
        layer.scales = torch.nn.Parameter(layer.scales.data.contiguous(), requires_grad=False)
        layer.qzeros = torch.nn.Parameter(layer.qzeros.data.contiguous(), requires_grad=False)
        del layer.qweight  # the AWQ-layout copy is not needed after the repack

    def apply(self, layer: torch.nn.Module, x: torch.Tensor,
              bias: torch.Tensor | None = None) -> torch.Tensor:
        return torch.ops.tokenforge.w4a16_linear(x, layer.qweight_t, layer.scales, layer.qzeros,
                                                 bias, self.quant_config.group_size, "cuda")


def register() -> None:
    """``vllm.general_plugins`` entry point: importing this module registered the config."""
    check_vllm_version()


__all__ = ["TokenForgeConfig", "TokenForgeLinearMethod", "check_vllm_version", "register"]
