"""AWQ checkpoint loader, host side: the safetensors reader against files written by the
`safetensors` package, sharded checkpoints, the quantisation-config rules and the q/k/v and
gate/up fusion checked nibble by nibble with the oracle's unpack."""

from __future__ import annotations

import json
import struct

import pytest
import torch

from oracle import oracle
from tests.awq_checkpoint import HIDDEN, INTER, KV, write_checkpoint
from tokenforge_b200.checkpoint import (
    AWQConfig, Checkpoint, CheckpointError, SafetensorsFile, fused_awq_tensors, num_layers,
)

safetensors_torch = pytest.importorskip("safetensors.torch")


def test_reader_matches_the_reference_writer(tmp_path) -> None:  # type: ignore[no-untyped-def]
    gen = torch.Generator().manual_seed(0)
    tensors = {
        "f16": torch.randn((3, 5), generator=gen).half(),
        "bf16": torch.randn(4, generator=gen).bfloat16(),
        "f32": torch.tensor(1.5),
        "i32": torch.randint(-(2**31), 2**31 - 1, (2, 3), generator=gen, dtype=torch.int32),
        "i64": torch.arange(3, dtype=torch.int64) - 7,
        "u8": torch.empty(0, dtype=torch.uint8),
        "b": torch.tensor([True, False, True]),
    }
    path = tmp_path / "t.safetensors"
    safetensors_torch.save_file(tensors, str(path), metadata={"format": "pt", "note": "x"})
    f = SafetensorsFile(path)
    assert sorted(f.keys()) == sorted(tensors)
    assert f.metadata == {"format": "pt", "note": "x"}
    for name, t in tensors.items():
        got = f.get(name)
        assert got.dtype == t.dtype and got.shape == t.shape
        assert torch.equal(got, t)
    # Views are copy-on-write: writing one leaves the file as it was.
    f.get("i32").zero_()
    assert torch.equal(SafetensorsFile(path).get("i32"), tensors["i32"])


def test_reader_rejects_corrupt_files(tmp_path) -> None:  # type: ignore[no-untyped-def]
    p = tmp_path / "short.safetensors"
    p.write_bytes(b"\x01\x02")
    with pytest.raises(CheckpointError, match="too short"):
        SafetensorsFile(p)
    header = json.dumps({"a": {"dtype": "F16", "shape": [4], "data_offsets": [0, 8]}}).encode()
    p = tmp_path / "trunc.safetensors"
    p.write_bytes(struct.pack("<Q", len(header)) + header + b"\0" * 4)  # 4 of 8 data bytes
    with pytest.raises(CheckpointError, match="data_offsets"):
        SafetensorsFile(p)
    header = json.dumps({"a": {"dtype": "F8_E9", "shape": [1], "data_offsets": [0, 1]}}).encode()
    p = tmp_path / "dtype.safetensors"
    p.write_bytes(struct.pack("<Q", len(header)) + header + b"\0")
    with pytest.raises(CheckpointError, match="unsupported dtype"):
        SafetensorsFile(p)


@pytest.mark.parametrize("shards", [1, 3])
def test_checkpoint_reads_single_and_sharded_models(tmp_path, shards: int) -> None:  # type: ignore[no-untyped-def]
    tensors = write_checkpoint(tmp_path, layers=3, shards=shards)
    ck = Checkpoint(tmp_path)
    assert sorted(ck.keys()) == sorted(tensors)
    for name in ("model.layers.2.mlp.down_proj.qweight", "model.layers.0.self_attn.q_proj.bias"):
        assert torch.equal(ck.get(name), tensors[name])
    assert num_layers(ck) == 3
    with pytest.raises(KeyError, match="no tensor"):
        ck.get("model.layers.3.mlp.down_proj.qweight")


def test_quant_config_rules(tmp_path) -> None:  # type: ignore[no-untyped-def]
    autoawq = {"zero_point": True, "q_group_size": 128, "w_bit": 4, "version": "GEMM"}
    assert AWQConfig.from_dict(autoawq) == AWQConfig(4, 128, True, "gemm")
    hf = {"quant_method": "awq", "bits": 4, "group_size": 64, "zero_point": True,
          "version": "gemm", "modules_to_not_convert": ["visual"]}
    assert AWQConfig.from_dict(hf).modules_to_not_convert == ("visual",)
    (tmp_path / "config.json").write_text(json.dumps({"quantization_config": hf}))
    assert AWQConfig.from_dir(tmp_path).group_size == 64
    for bad, match in (({**autoawq, "w_bit": 8}, "8-bit"), ({**autoawq, "zero_point": False}, "zero points"),
                       ({**autoawq, "q_group_size": 96}, "group size"), ({**autoawq, "version": "GEMV"}, "packing"),
                       ({**hf, "quant_method": "gptq"}, "not AWQ")):
        with pytest.raises(CheckpointError, match=match):
            AWQConfig.from_dict(bad)


def test_fusion_concatenates_projections_along_n(tmp_path) -> None:  # type: ignore[no-untyped-def]
    tensors = write_checkpoint(tmp_path, layers=1, g=64)
    ck = Checkpoint(tmp_path)
    pre = "model.layers.0.self_attn."
    qw, qz, sc, bias = fused_awq_tensors(ck, [pre + p for p in ("q_proj", "k_proj", "v_proj")])
    n = HIDDEN + 2 * KV
    assert qw.shape == (HIDDEN, n // 8) and qz.shape == (HIDDEN // 64, n // 8)
    assert sc.shape == (HIDDEN // 64, n) and bias is not None and bias.shape == (n,)
    # Nibble by nibble: the fused matrix's integer weights are the projections' side by side.
    ints = oracle.unpack_int4(qw)
    parts = [oracle.unpack_int4(tensors[pre + p + ".qweight"]) for p in ("q_proj", "k_proj", "v_proj")]
    assert torch.equal(ints, torch.cat(parts, dim=1))
    zs = oracle.unpack_int4(qz)
    assert torch.equal(zs, torch.cat([oracle.unpack_int4(tensors[pre + p + ".qzeros"])
                                      for p in ("q_proj", "k_proj", "v_proj")], dim=1))
    gu = fused_awq_tensors(ck, ["model.layers.0.mlp.gate_proj", "model.layers.0.mlp.up_proj"])
    assert gu[0].shape == (HIDDEN, 2 * INTER // 8) and gu[3] is None


def test_fusion_rejects_inconsistent_projections(tmp_path) -> None:  # type: ignore[no-untyped-def]
    write_checkpoint(tmp_path, layers=1)
    ck = Checkpoint(tmp_path)
    with pytest.raises(CheckpointError, match="disagree on K"):
        fused_awq_tensors(ck, ["model.layers.0.mlp.gate_proj", "model.layers.0.mlp.down_proj"])
    with pytest.raises(CheckpointError, match="bias present on some"):
        fused_awq_tensors(ck, ["model.layers.0.self_attn.q_proj", "model.layers.0.self_attn.o_proj"])
    with pytest.raises(CheckpointError, match="no tensor"):
        fused_awq_tensors(ck, ["model.layers.0.mlp.missing_proj"])


@pytest.mark.parametrize("world", [2, 4])
def test_awq_shards_match_the_kernel_layout_partition(tmp_path, world: int) -> None:  # type: ignore[no-untyped-def]
    """Slicing the AWQ-layout tensors and then repacking (what each rank's loader does) gives
    exactly tp's shard of the repacked full layer, for every linear of a Qwen2 layer."""
    from tokenforge_b200 import tp
    from tokenforge_b200.checkpoint import QWEN2_LINEARS, QWEN2_TP, shard_awq
    from tokenforge_b200.pack import W4A16Weights

    write_checkpoint(tmp_path, layers=1, g=64)
    ck = Checkpoint(tmp_path)
    for name, (block, projs) in QWEN2_LINEARS.items():
        pre = [f"model.layers.0.{block}.{p}" for p in projs]
        qw, qz, sc, bias = fused_awq_tensors(ck, pre)
        parts = tuple(int(ck.get(p + ".scales").shape[1]) for p in pre)
        full = W4A16Weights(oracle.repack_awq_to_tf(qw), sc, qz, 64)
        kind, aligned = QWEN2_TP[name]
        for rank in range(world):
            s_qw, s_qz, s_sc, s_b = shard_awq(qw, qz, sc, bias, kind, rank, world, 64,
                                              parts if kind == "column" else None, aligned)
            if kind == "column":
                want = tp.shard_fused_columns(full, parts, rank, world, bias, aligned)
            else:
                want = tp.shard_layer(full, "row", rank, world, bias)
            assert torch.equal(oracle.repack_awq_to_tf(s_qw), want.weights.qweight_t)
            assert torch.equal(s_sc, want.weights.scales) and torch.equal(s_qz, want.weights.qzeros)
            assert (s_b is None) == (want.bias is None)
            if s_b is not None:
                assert torch.equal(s_b, want.bias)


def test_layer_gaps_and_unquantised_linears_are_refused(tmp_path) -> None:  # type: ignore[no-untyped-def]
    """Errors that stop a load before anything reaches the GPU: a checkpoint whose layer ids have
    a gap, and one that leaves a served linear unquantised (modules_to_not_convert)."""
    from tokenforge_b200.checkpoint import load_decoder_layers

    tensors = write_checkpoint(tmp_path / "gap", layers=1)
    extra = {k.replace("layers.0.", "layers.2."): v for k, v in tensors.items()
             if k.startswith("model.layers.0.")}
    safetensors_torch.save_file(extra, str(tmp_path / "gap" / "extra.safetensors"))
    with pytest.raises(CheckpointError, match="missing \\[1\\]"):
        num_layers(Checkpoint(tmp_path / "gap"))

    write_checkpoint(tmp_path / "skip", layers=1, config={
        "zero_point": True, "q_group_size": 128, "w_bit": 4, "version": "GEMM",
        "modules_to_not_convert": ["mlp.down_proj"]})
    with pytest.raises(CheckpointError, match="unquantised"):
        load_decoder_layers(tmp_path / "skip", "cpu")
    with pytest.raises(ValueError, match="rank"):
        load_decoder_layers(tmp_path / "skip", "cpu", rank=2, world=2)


def test_tensor_parallel_load_refuses_worlds_the_heads_do_not_split(tmp_path) -> None:  # type: ignore[no-untyped-def]
    """Attention splits on whole heads: 4 q heads do not split over 3 ranks, one q head of 64
    columns is not a whole group of 128 at world 4, and a checkpoint without the model config
    has no head counts. All are refused before any tensor reaches a device."""
    import json

    from tokenforge_b200.checkpoint import load_decoder_layers

    write_checkpoint(tmp_path / "a", layers=1, g=128)
    with pytest.raises(CheckpointError, match="attention heads do not split"):
        load_decoder_layers(tmp_path / "a", "cpu", rank=0, world=3)
    with pytest.raises(CheckpointError, match="whole groups"):
        load_decoder_layers(tmp_path / "a", "cpu", rank=0, world=4)
    (tmp_path / "a" / "config.json").unlink()
    with pytest.raises(CheckpointError, match="head counts"):
        load_decoder_layers(tmp_path / "a", "cpu", rank=0, world=2)
    write_checkpoint(tmp_path / "b", layers=1, g=64)
    cfg = json.loads((tmp_path / "b" / "config.json").read_text())
    assert cfg["num_attention_heads"] * 64 == cfg["hidden_size"]


def test_head_shards_in_awq_layout_match_the_kernel_layout(tmp_path) -> None:  # type: ignore[no-untyped-def]
    """Slicing q|k|v and o on heads in AWQ layout and then repacking (what each rank's loader
    does) gives exactly tp.shard_attention of the repacked full layers."""
    from tests.awq_checkpoint import HEAD_DIM, HEADS, KV_HEADS
    from tokenforge_b200 import tp
    from tokenforge_b200.checkpoint import slice_awq_columns, slice_awq_rows
    from tokenforge_b200.pack import W4A16Weights

    write_checkpoint(tmp_path, layers=1, g=64)
    ck = Checkpoint(tmp_path)
    heads = tp.AttentionHeads(HEADS, KV_HEADS, HEAD_DIM)
    qw, qz, sc, bias = fused_awq_tensors(
        ck, [f"model.layers.0.self_attn.{p}" for p in ("q_proj", "k_proj", "v_proj")])
    ow, oz, osc, _ = fused_awq_tensors(ck, ["model.layers.0.self_attn.o_proj"])
    full_qkv = W4A16Weights(oracle.repack_awq_to_tf(qw), sc, qz, 64)
    full_o = W4A16Weights(oracle.repack_awq_to_tf(ow), osc, oz, 64)
    for world in (2, 4):
        for rank in range(world):
            want_qkv, want_o = tp.shard_attention(full_qkv, full_o, heads, rank, world, bias)
            pieces, (k0, k1) = tp.attention_bounds(heads, rank, world, 64)
            s_qw, s_qz, s_sc, s_b = slice_awq_columns(qw, qz, sc, bias, pieces)
            assert torch.equal(oracle.repack_awq_to_tf(s_qw), want_qkv.weights.qweight_t)
            assert torch.equal(s_sc, want_qkv.weights.scales)
            assert torch.equal(s_qz, want_qkv.weights.qzeros)
            assert s_b is not None and torch.equal(s_b, want_qkv.bias)
            r_qw, r_qz, r_sc, _ = slice_awq_rows(ow, oz, osc, None, k0, k1, 64, rank == 0)
            assert torch.equal(oracle.repack_awq_to_tf(r_qw), want_o.weights.qweight_t)
            assert torch.equal(r_sc, want_o.weights.scales) and torch.equal(r_qz, want_o.weights.qzeros)
