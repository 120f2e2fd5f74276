"""AWQ checkpoint loader on the GPU: a synthetic two-layer Qwen2-style checkpoint (sharded, with
q/k/v biases) loads into kernel-layout layers whose packed weights equal the oracle's repack of
the fused projections bit for bit, and whose linear outputs match the oracle's fp64 reference
of the unfused projections side by side."""

from __future__ import annotations

import pytest
import torch

import tokenforge_b200.ops  # noqa: F401  (registers torch.ops.tokenforge)
from oracle import oracle
from tests.awq_checkpoint import HEAD_DIM, HEADS, HIDDEN, KV, KV_HEADS, write_checkpoint
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


@pytest.mark.parametrize(("g", "world"), [(128, 2), (64, 2), (64, 4)])
def test_tensor_parallel_load_equals_sharding_the_full_load(tmp_path, g: int, world: int,  # type: ignore[no-untyped-def]
                                                            device: torch.device) -> None:
    """load_decoder_layers(rank=r, world=w) slices before the repack; the result equals tp's
    shards of the full load: q|k|v and o on whole heads (the one KV head replicated), gate|up
    projection by projection, down by K. Each rank's q width is its o shard's K."""
    from tokenforge_b200 import tp

    write_checkpoint(tmp_path, layers=1, g=g)
    full = load_decoder_layers(tmp_path, device)[0]
    heads = tp.AttentionHeads(HEADS, KV_HEADS, HEAD_DIM)
    for rank in range(world):
        part = load_decoder_layers(tmp_path, device, rank=rank, world=world)[0]
        qkv_s, o_s = tp.shard_attention(full.qkv, full.o, heads, rank, world, full.qkv_bias)
        q_piece = qkv_s.pieces[0]
        assert q_piece[1] - q_piece[0] == part.o.k
        want = {
            "qkv": qkv_s,
            "o": o_s,
            "gate_up": tp.shard_fused_columns(full.gate_up, (full.gate_up.n // 2,) * 2, rank,
                                              world, group_aligned=True),
            "down": tp.shard_layer(full.down, "row", rank, world),
        }
        for name, w in part.linears().items():
            ws = want[name].weights
            assert torch.equal(w.qweight_t, ws.qweight_t), name
            assert torch.equal(w.scales, ws.scales) and torch.equal(w.qzeros, ws.qzeros), name
        assert part.qkv_bias is not None and torch.equal(part.qkv_bias, want["qkv"].bias)
        assert torch.equal(part.input_norm, full.input_norm)
