"""AWQ checkpoint loader on the GPU: a synthetic two-layer Qwen2-style checkpoint (sharded, with
q/k/v biases) loads into kernel-layout layers whose packed weights equal the oracle's repack of
the fused projections bit for bit, and whose linear outputs match the oracle's fp64 reference
of the unfused projections side by side."""

from __future__ import annotations

import pytest
import torch

import tokenforge_b200.ops  # noqa: F401  (registers torch.ops.tokenforge)
from oracle import oracle
from tests.awq_checkpoint import HIDDEN, KV, write_checkpoint
from tests.numerics.tolerance import atol
from tokenforge_b200.checkpoint import CheckpointError, load_decoder_layers

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("g", [64, 128])
def test_loaded_layers_are_the_fused_projections(tmp_path, g: int, device: torch.device) -> None:  # type: ignore[no-untyped-def]
    tensors = write_checkpoint(tmp_path, layers=2, g=g, shards=2)
    layers = load_decoder_layers(tmp_path, device)
    assert len(layers) == 2
    fused = {"qkv": ("self_attn", ("q_proj", "k_proj", "v_proj")), "o": ("self_attn", ("o_proj",)),
             "gate_up": ("mlp", ("gate_proj", "up_proj")), "down": ("mlp", ("down_proj",))}
    for i, layer in enumerate(layers):
        for name, w in layer.linears().items():
            block, projs = fused[name]
            pre = [f"model.layers.{i}.{block}.{p}" for p in projs]
            qweight = torch.cat([tensors[p + ".qweight"] for p in pre], dim=1)
            assert torch.equal(w.qweight_t.cpu(), oracle.repack_awq_to_tf(qweight))
            assert torch.equal(w.scales.cpu(), torch.cat([tensors[p + ".scales"] for p in pre], 1))
            assert torch.equal(w.qzeros.cpu(), torch.cat([tensors[p + ".qzeros"] for p in pre], 1))
            assert w.group_size == g
            # One linear call on the fused layer = the projections' references side by side.
            # (a seed apart from the checkpoint's, whose weight streams start at seed * 1000 + i)
            x = torch.randn((3, w.k), generator=torch.Generator().manual_seed(7919 + i)).half()
            y = torch.ops.tokenforge.w4a16_linear(x.to(device), w.qweight_t, w.scales, w.qzeros,
                                                  None, g, "cuda").cpu().double()
            refs = []
            for p in pre:
                qt = oracle.repack_awq_to_tf(tensors[p + ".qweight"])
                refs.append(oracle.w4a16_reference(x, qt, tensors[p + ".scales"],
                                                   tensors[p + ".qzeros"], g))
            w16 = oracle.dequantize_tf(w.qweight_t.cpu(), w.scales.cpu(), w.qzeros.cpu(), g)
            assert float((y - torch.cat(refs, dim=1)).abs().max()) <= atol(x, w16, "cuda")
        bias = torch.cat([tensors[f"model.layers.{i}.self_attn.{p}.bias"]
                          for p in ("q_proj", "k_proj", "v_proj")])
        assert layer.qkv_bias is not None and torch.equal(layer.qkv_bias.cpu(), bias)
        assert layer.qkv.n == HIDDEN + 2 * KV
        assert torch.equal(layer.input_norm.cpu(),
                           tensors[f"model.layers.{i}.input_layernorm.weight"])
        assert torch.equal(layer.post_attention_norm.cpu(),
                           tensors[f"model.layers.{i}.post_attention_layernorm.weight"])


def test_selected_layers_and_unsupported_checkpoints(tmp_path, device: torch.device) -> None:  # type: ignore[no-untyped-def]
    write_checkpoint(tmp_path / "a", layers=3)
    assert len(load_decoder_layers(tmp_path / "a", device, layers=[2])) == 1
    write_checkpoint(tmp_path / "b", layers=1, config={"zero_point": True, "q_group_size": 128,
                                                       "w_bit": 4, "version": "GEMV"})
    with pytest.raises(CheckpointError, match="packing"):
        load_decoder_layers(tmp_path / "b", device)


def test_tensor_parallel_load_equals_sharding_the_full_load(tmp_path, device: torch.device) -> None:  # type: ignore[no-untyped-def]
    """load_decoder_layers(rank=r, world=2) slices before the repack; the result equals
    tp's shards of the full load (q|k|v and gate|up projection by projection, o/down by K)."""
    from tokenforge_b200 import tp

    write_checkpoint(tmp_path, layers=1, g=128)
    full = load_decoder_layers(tmp_path, device)[0]
    for rank in range(2):
        part = load_decoder_layers(tmp_path, device, rank=rank, world=2)[0]
        want = {
            "qkv": tp.shard_fused_columns(full.qkv, (HIDDEN, KV, KV), rank, 2, full.qkv_bias),
            "o": tp.shard_layer(full.o, "row", rank, 2),
            "gate_up": tp.shard_fused_columns(full.gate_up, (full.gate_up.n // 2,) * 2, rank, 2,
                                              group_aligned=True),
            "down": tp.shard_layer(full.down, "row", rank, 2),
        }
        for name, w in part.linears().items():
            ws = want[name].weights
            assert torch.equal(w.qweight_t, ws.qweight_t), name
            assert torch.equal(w.scales, ws.scales) and torch.equal(w.qzeros, ws.qzeros), name
        assert part.qkv_bias is not None and torch.equal(part.qkv_bias, want["qkv"].bias)
        assert torch.equal(part.input_norm, full.input_norm)
