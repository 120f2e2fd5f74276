"""Synthetic AWQ Qwen2-style checkpoints for the loader tests, written with the `safetensors`
package (an independent writer of the format the loader reads). Shapes are a scaled-down
Qwen2.5 decoder layer (hidden 256, q 256 = 4 heads of 64, k/v 64 each = one KV head,
intermediate 512), with a model config.json giving the head counts. Like a real AWQ
checkpoint, each projection is real-valued weights (randn * 0.02) quantised min-max per group by
the oracle's restatement of the reference's awq_quantize, in the AWQ 'gemm' packing."""

from __future__ import annotations

import json
from pathlib import Path

import torch

from oracle import oracle

HIDDEN, KV, INTER = 256, 64, 512
HEADS, KV_HEADS, HEAD_DIM = 4, 1, 64  # q 4 x 64 = HIDDEN, k and v 1 x 64 = KV
PROJS = {  # name -> (K, N)
    "self_attn.q_proj": (HIDDEN, HIDDEN),
    "self_attn.k_proj": (HIDDEN, KV),
    "self_attn.v_proj": (HIDDEN, KV),
    "self_attn.o_proj": (HIDDEN, HIDDEN),
    "mlp.gate_proj": (HIDDEN, INTER),
    "mlp.up_proj": (HIDDEN, INTER),
    "mlp.down_proj": (INTER, HIDDEN),
}


def awq_projection(k: int, n: int, g: int, gen: torch.Generator) -> dict[str, torch.Tensor]:
    weight = torch.randn((n, k), generator=gen) * 0.02
    qweight, qzeros, scales = oracle.awq_quantize(weight, g)
    return {"qweight": qweight, "qzeros": qzeros, "scales": scales}


def layer_tensors(layer: int, g: int, seed: int) -> dict[str, torch.Tensor]:
    gen = torch.Generator().manual_seed(seed * 1000 + layer)
    out: dict[str, torch.Tensor] = {}
    for name, (k, n) in PROJS.items():
        for key, t in awq_projection(k, n, g, gen).items():
            out[f"model.layers.{layer}.{name}.{key}"] = t
        if name in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"):
            out[f"model.layers.{layer}.{name}.bias"] = (torch.randn(n, generator=gen) * 0.1).half()
    for norm in ("input_layernorm", "post_attention_layernorm"):
        out[f"model.layers.{layer}.{norm}.weight"] = (1 + 0.1 * torch.randn(HIDDEN, generator=gen)).half()
    return out


def write_checkpoint(root: Path, layers: int = 2, g: int = 128, seed: int = 0, shards: int = 1,
                     config: dict | None = None) -> dict[str, torch.Tensor]:
    """Writes the model (optionally sharded with an index) and its quant config under root;
    returns every tensor written."""
    from safetensors.torch import save_file

    root.mkdir(parents=True, exist_ok=True)
    tensors: dict[str, torch.Tensor] = {}
    for i in range(layers):
        tensors.update(layer_tensors(i, g, seed))
    tensors["model.embed_tokens.weight"] = torch.zeros((8, HIDDEN), dtype=torch.float16)
    names = sorted(tensors)
    if shards == 1:
        save_file({k: tensors[k] for k in names}, str(root / "model.safetensors"),
                  metadata={"format": "pt"})
    else:
        weight_map = {}
        for s in range(shards):
            part = names[s::shards]
            fname = f"model-{s + 1:05d}-of-{shards:05d}.safetensors"
            save_file({k: tensors[k] for k in part}, str(root / fname))
            weight_map.update({k: fname for k in part})
        (root / "model.safetensors.index.json").write_text(
            json.dumps({"metadata": {}, "weight_map": weight_map}))
    cfg = config if config is not None else {
        "zero_point": True, "q_group_size": g, "w_bit": 4, "version": "GEMM"}
    (root / "quant_config.json").write_text(json.dumps(cfg))
    (root / "config.json").write_text(json.dumps({
        "architectures": ["Qwen2ForCausalLM"], "hidden_size": HIDDEN, "intermediate_size": INTER,
        "num_attention_heads": HEADS, "num_key_value_heads": KV_HEADS,
        "num_hidden_layers": layers}))
    return tensors
