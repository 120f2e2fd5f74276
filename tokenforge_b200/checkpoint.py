"""AWQ checkpoint loader: safetensors files of an AWQ-quantised Qwen2-family model (for example
Qwen2.5-7B-Instruct-AWQ, the model the reference's design names) into the kernel layout.

The reference plans this step (it loads AWQ checkpoints "unchanged" into ``pack_awq``,
``tokenforge/kernels/pack.py:171-181``, and names the checkpoint in ``infra/versions.lock``) but
ships no reader. Here:

* :class:`SafetensorsFile` / :class:`Checkpoint` read the safetensors format (an 8-byte
  little-endian header length, a JSON header of ``{name: {dtype, shape, data_offsets}}``, then
  the raw little-endian tensor bytes) through a copy-on-write memory map, so a tensor is a
  zero-copy CPU view until it is moved to the GPU. A directory with
  ``model.safetensors.index.json`` is read across its shards.
* :class:`AWQConfig` reads the quantisation config (``quant_config.json``,
  ``quantize_config.json`` or ``config.json``'s ``quantization_config``) and accepts what the
  kernels serve: 4 bits, zero points, group size 32/64/128, AutoAWQ's ``gemm`` packing (the
  layout of ``pack.awq_pack``; the ``gemv`` packings order nibbles differently).
* :func:`fused_awq_tensors` concatenates projections that run as one GEMM along N, as vLLM
  does for Qwen2 (q/k/v -> qkv, gate/up -> gate_up): packed words hold 8 consecutive output
  columns, so ``qweight``/``qzeros`` concatenate along their packed dimension and ``scales``
  along N.
* :func:`load_decoder_layers` returns each decoder layer's four linear layers as
  :class:`~tokenforge_b200.pack.W4A16Weights` (repacked once on the GPU by the bit-exact
  ``tokenforge::awq_repack``), the q/k/v bias and the two RMSNorm weights. With ``world > 1``
  it returns tensor-parallel rank ``rank``'s shards instead (:func:`shard_awq`, the partition
  of :mod:`tokenforge_b200.tp`): the AWQ-layout tensors are sliced before the repack, so each
  rank repacks only its own part.
"""

from __future__ import annotations

import json
import mmap
import os
import struct
from dataclasses import dataclass
from pathlib import Path

import torch

from tokenforge_b200.pack import SUPPORTED_GROUP_SIZES, W4A16Weights, pack_awq, validate_awq

_DTYPES = {
    "F64": torch.float64, "F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16,
    "I64": torch.int64, "I32": torch.int32, "I16": torch.int16, "I8": torch.int8,
    "U8": torch.uint8, "BOOL": torch.bool,
}
_MAX_HEADER = 100 << 20  # a larger header is a corrupt file, not a checkpoint


class CheckpointError(ValueError):
    """A checkpoint that cannot be read or is not a supported AWQ model."""


class SafetensorsFile:
    """One ``.safetensors`` file, memory-mapped copy-on-write (the file is never modified)."""

    def __init__(self, path: str | os.PathLike[str]) -> None:
        self.path = Path(path)
        with open(self.path, "rb") as f:
            head = f.read(8)
            if len(head) != 8:
                raise CheckpointError(f"{self.path}: too short for a safetensors header")
            (n,) = struct.unpack("<Q", head)
            if n > _MAX_HEADER:
                raise CheckpointError(f"{self.path}: header of {n} bytes")
            try:
                header = json.loads(f.read(n))
            except ValueError as e:
                raise CheckpointError(f"{self.path}: header is not JSON ({e})") from None
            size = os.fstat(f.fileno()).st_size
            self._map = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_COPY) if size else None
        self._base = 8 + n
        self.metadata: dict[str, str] = header.pop("__metadata__", None) or {}
        self._entries: dict[str, tuple[torch.dtype, tuple[int, ...], int, int]] = {}
        for name, e in header.items():
            try:
                dtype = _DTYPES[e["dtype"]]
            except KeyError:
                raise CheckpointError(f"{self.path}: {name} has unsupported dtype "
                                      f"{e.get('dtype')!r}") from None
            shape = tuple(int(d) for d in e["shape"])
            b, end = (int(v) for v in e["data_offsets"])
            numel = 1
            for d in shape:
                numel *= d
            if end - b != numel * dtype.itemsize or b < 0 or self._base + end > size:
                raise CheckpointError(f"{self.path}: {name} has data_offsets {b}..{end} that do "
                                      f"not hold {shape} {e['dtype']} inside the file")
            self._entries[name] = (dtype, shape, b, end)

    def keys(self) -> list[str]:
        return list(self._entries)

    def __contains__(self, name: str) -> bool:
        return name in self._entries

    def get(self, name: str) -> torch.Tensor:
        """The tensor as a CPU view of the mapped file (copy-on-write: writes stay private)."""
        try:
            dtype, shape, b, end = self._entries[name]
        except KeyError:
            raise KeyError(f"{self.path}: no tensor {name!r}") from None
        if end == b:
            return torch.empty(shape, dtype=dtype)
        assert self._map is not None
        flat = torch.frombuffer(self._map, dtype=dtype, count=(end - b) // dtype.itemsize,
                                offset=self._base + b)
        return flat.reshape(shape)


class Checkpoint:
    """A single safetensors file, or a directory of them (with or without an index file)."""

    def __init__(self, path: str | os.PathLike[str]) -> None:
        p = Path(path)
        self.root = p if p.is_dir() else p.parent
        self._where: dict[str, SafetensorsFile] = {}
        if p.is_file():
            files = [SafetensorsFile(p)]
        else:
            index = p / "model.safetensors.index.json"
            if index.exists():
                weight_map = json.loads(index.read_text())["weight_map"]
                shards = {f: SafetensorsFile(p / f) for f in sorted(set(weight_map.values()))}
                for name, f in weight_map.items():
                    if name not in shards[f]:
                        raise CheckpointError(f"index lists {name} in {f}, which lacks it")
                    self._where[name] = shards[f]
                return
            files = [SafetensorsFile(f) for f in sorted(p.glob("*.safetensors"))]
            if not files:
                raise CheckpointError(f"{p}: no .safetensors files")
        for f in files:
            for name in f.keys():
                if name in self._where:
                    raise CheckpointError(f"{name} appears in {self._where[name].path} and {f.path}")
                self._where[name] = f

    def keys(self) -> list[str]:
        return list(self._where)

    def __contains__(self, name: str) -> bool:
        return name in self._where

    def get(self, name: str) -> torch.Tensor:
        try:
            return self._where[name].get(name)
        except KeyError:
            raise KeyError(f"checkpoint has no tensor {name!r}") from None


@dataclass(frozen=True)
class AWQConfig:
    bits: int
    group_size: int
    zero_point: bool
    version: str
    modules_to_not_convert: tuple[str, ...] = ()

    @classmethod
    def from_dict(cls, cfg: dict) -> AWQConfig:
        def pick(*keys: str, default=None):  # type: ignore[no-untyped-def]
            for k in keys:
                if k in cfg:
                    return cfg[k]
            return default

        method = str(pick("quant_method", default="awq")).lower()
        if method != "awq":
            raise CheckpointError(f"quantisation method {method!r} is not AWQ")
        out = cls(
            bits=int(pick("w_bit", "bits", default=0)),
            group_size=int(pick("q_group_size", "group_size", default=0)),
            zero_point=bool(pick("zero_point", default=False)),
            version=str(pick("version", default="gemm")).lower(),
            modules_to_not_convert=tuple(pick("modules_to_not_convert", default=None) or ()),
        )
        if out.bits != 4:
            raise CheckpointError(f"{out.bits}-bit AWQ; the kernels serve 4-bit weights")
        if not out.zero_point:
            raise CheckpointError("AWQ without zero points is not served")
        if out.group_size not in SUPPORTED_GROUP_SIZES:
            raise CheckpointError(f"group size {out.group_size} not in {SUPPORTED_GROUP_SIZES}")
        if out.version != "gemm":
            raise CheckpointError(f"AWQ packing {out.version!r}: only the 'gemm' packing "
                                  f"(nibble order 0,2,4,6,1,3,5,7 along N) is served")
        return out

    @classmethod
    def from_dir(cls, root: str | os.PathLike[str]) -> AWQConfig:
        root = Path(root)
        for name in ("quant_config.json", "quantize_config.json"):
            if (root / name).exists():
                return cls.from_dict(json.loads((root / name).read_text()))
        if (root / "config.json").exists():
            qc = json.loads((root / "config.json").read_text()).get("quantization_config")
            if qc:
                return cls.from_dict(qc)
        raise CheckpointError(f"{root}: no AWQ quantisation config found")


# Qwen2 decoder layer: fused linear -> (projections in N order), attention or MLP prefix.
QWEN2_LINEARS: dict[str, tuple[str, tuple[str, ...]]] = {
    "qkv": ("self_attn", ("q_proj", "k_proj", "v_proj")),
    "o": ("self_attn", ("o_proj",)),
    "gate_up": ("mlp", ("gate_proj", "up_proj")),
    "down": ("mlp", ("down_proj",)),
}


def fused_awq_tensors(
    ckpt: Checkpoint, prefixes: list[str]
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor | None]:
    """``(qweight [K, N/8], qzeros [K/G, N/8], scales [K/G, N], bias [N] | None)`` of the
    projections ``prefixes`` concatenated along N (CPU tensors). Bias is returned when every
    projection has one; a partial set is an error."""
    parts = []
    for pre in prefixes:
        try:
            parts.append((ckpt.get(pre + ".qweight"), ckpt.get(pre + ".qzeros"),
                          ckpt.get(pre + ".scales"),
                          ckpt.get(pre + ".bias") if pre + ".bias" in ckpt else None))
        except KeyError as e:
            raise CheckpointError(f"{pre}: {e}") from None
    ks = {p[0].shape[0] for p in parts}
    if len(ks) != 1:
        raise CheckpointError(f"{prefixes}: projections disagree on K ({sorted(ks)})")
    with_bias = [p[3] is not None for p in parts]
    if any(with_bias) and not all(with_bias):
        raise CheckpointError(f"{prefixes}: bias present on some projections only")
    cat = (lambda i: parts[0][i]) if len(parts) == 1 else (
        lambda i: torch.cat([p[i] for p in parts], dim=-1))
    bias = cat(3) if all(with_bias) else None
    return cat(0), cat(1), cat(2), bias


def slice_awq_columns(
    qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor, bias: torch.Tensor | None,
    pieces: list[tuple[int, int]],
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor | None]:
    """The global column ranges ``pieces`` (multiples of 8) of an AWQ-layout layer,
    concatenated in order."""
    qw = torch.cat([qweight[:, a // 8:b // 8] for a, b in pieces], dim=1)
    qz = torch.cat([qzeros[:, a // 8:b // 8] for a, b in pieces], dim=1)
    sc = torch.cat([scales[:, a:b] for a, b in pieces], dim=1)
    bs = None if bias is None else torch.cat([bias[a:b] for a, b in pieces])
    return qw.contiguous(), qz.contiguous(), sc.contiguous(), bs


def slice_awq_rows(
    qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor, bias: torch.Tensor | None,
    k0: int, k1: int, group_size: int, keep_bias: bool,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor | None]:
    """K range [k0, k1) (whole groups) of an AWQ-layout layer; the bias only where kept."""
    if k0 % group_size or k1 % group_size:
        raise CheckpointError(f"K range [{k0}, {k1}) is not whole groups of {group_size}")
    g0, g1 = k0 // group_size, k1 // group_size
    return (qweight[k0:k1].contiguous(), qzeros[g0:g1].contiguous(), scales[g0:g1].contiguous(),
            bias if keep_bias else None)


def shard_awq(
    qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor, bias: torch.Tensor | None,
    kind: str, rank: int, world: int, group_size: int, parts: tuple[int, ...] | None = None,
    group_aligned: bool = False,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor | None]:
    """Rank ``rank``'s slice of an AWQ-layout layer (qweight [K, N/8], qzeros [K/G, N/8],
    scales [K/G, N], bias [N]), the same partition as :mod:`tokenforge_b200.tp` applies to the
    kernel layout: ``"column"`` takes the rank's pieces of each projection of width ``parts``
    (the whole N when None; :func:`~tokenforge_b200.tp.fused_column_bounds`), concatenated;
    ``"row"`` takes the rank's K range in whole groups (bias on rank 0 only). Attention layers
    of a real model are split on heads instead (:func:`load_decoder_layers`)."""
    from tokenforge_b200 import tp

    n = scales.shape[1]
    if kind == "column":
        if sum(parts or (n,)) != n:
            raise CheckpointError(f"parts {parts} do not add up to N={n}")
        pieces = tp.fused_column_bounds(parts or (n,), rank, world,
                                        group_size if group_aligned else None)
        return slice_awq_columns(qweight, qzeros, scales, bias, pieces)
    if kind == "row":
        k0, k1 = tp.row_bounds(qweight.shape[0], group_size, world)[rank]
        return slice_awq_rows(qweight, qzeros, scales, bias, k0, k1, group_size, rank == 0)
    raise ValueError(f"kind must be 'column' or 'row', got {kind!r}")


def attention_heads(root: str | os.PathLike[str]):  # type: ignore[no-untyped-def]
    """The model's attention head layout from its ``config.json`` (``num_attention_heads``,
    ``num_key_value_heads`` (default: as many as the q heads), ``head_dim`` (default:
    ``hidden_size / num_attention_heads``))."""
    from tokenforge_b200.tp import AttentionHeads

    path = Path(root) / "config.json"
    if not path.exists():
        raise CheckpointError(f"{root}: no config.json; a tensor-parallel load splits attention "
                              f"on heads and needs the model's head counts")
    cfg = json.loads(path.read_text())
    try:
        h = int(cfg["num_attention_heads"])
        kv = int(cfg.get("num_key_value_heads", h))
        hd = int(cfg.get("head_dim") or int(cfg["hidden_size"]) // h)
    except (KeyError, TypeError, ValueError) as e:
        raise CheckpointError(f"{path}: cannot read the attention head layout ({e})") from None
    return AttentionHeads(h, kv, hd)


# How the MLP's fused linears of a Qwen2 layer shard: column-parallel projections keep every
# rank's slice of each part (gate/up on whole groups, so gate_r is the K range of down's row
# shard). q|k|v and o split on attention heads (load_decoder_layers); their entries here are the
# head-agnostic split of shard_awq.
QWEN2_TP = {"qkv": ("column", False), "o": ("row", False), "gate_up": ("column", True),
            "down": ("row", False)}


@dataclass
class DecoderLayer:
    """One Qwen2 decoder layer's weights in kernel layout (on the load device)."""

    qkv: W4A16Weights
    qkv_bias: torch.Tensor | None
    o: W4A16Weights
    gate_up: W4A16Weights
    down: W4A16Weights
    input_norm: torch.Tensor  # fp16 [hidden], RMSNorm before attention
    post_attention_norm: torch.Tensor  # fp16 [hidden], RMSNorm before the MLP

    def linears(self) -> dict[str, W4A16Weights]:
        return {"qkv": self.qkv, "o": self.o, "gate_up": self.gate_up, "down": self.down}


def num_layers(ckpt: Checkpoint, prefix: str = "model.layers.") -> int:
    ids = {int(k[len(prefix):].split(".", 1)[0]) for k in ckpt.keys()
           if k.startswith(prefix) and k[len(prefix):].split(".", 1)[0].isdigit()}
    if not ids:
        raise CheckpointError(f"no tensors under {prefix!r}")
    if ids != set(range(len(ids))):
        raise CheckpointError(f"layer ids are not 0..{len(ids) - 1}: missing "
                              f"{sorted(set(range(max(ids) + 1)) - ids)}")
    return len(ids)


def load_decoder_layers(path: str | os.PathLike[str], device: torch.device | str = "cuda",
                        layers: list[int] | None = None, prefix: str = "model.layers.",
                        rank: int = 0, world: int = 1) -> list[DecoderLayer]:
    """Each requested decoder layer (all by default) of an AWQ Qwen2 checkpoint, its linear
    layers repacked on ``device`` (a CUDA device: the repack is a GPU kernel). With
    ``world > 1``: tensor-parallel rank ``rank``'s shards. q|k|v and o split on whole attention
    heads (:func:`tokenforge_b200.tp.attention_bounds`, head counts from ``config.json``): the
    rank's q heads, their KV heads (replicated when there are more ranks than KV heads) and o's
    K range over the same q heads, so the rank's attention output feeds its own o shard; a
    world size the heads do not divide is refused. gate|up split projection by projection in
    whole groups and down by the matching K groups. The q/k/v bias is sliced with its columns."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    ckpt = Checkpoint(path)
    cfg = AWQConfig.from_dir(ckpt.root)
    ids = list(range(num_layers(ckpt, prefix))) if layers is None else layers
    attn = None
    if world > 1:
        from tokenforge_b200 import tp

        heads = attention_heads(ckpt.root)
        try:
            attn = tp.attention_bounds(heads, rank, world, cfg.group_size)
        except ValueError as e:
            raise CheckpointError(f"tensor parallel over {world} ranks: {e}") from None
    # Refuse unserved checkpoints before any tensor is read or moved to the device.
    for i in ids:
        for block, projs in QWEN2_LINEARS.values():
            for p in projs:
                if any(m in f"{prefix}{i}.{block}.{p}" for m in cfg.modules_to_not_convert):
                    raise CheckpointError(f"{prefix}{i}.{block}.{p}: left unquantised by the "
                                          f"checkpoint (modules_to_not_convert); only AWQ "
                                          f"linears are served")
    dev = torch.device(device)
    out = []
    for i in ids:
        lp = f"{prefix}{i}."
        ws: dict[str, W4A16Weights] = {}
        qkv_bias = None
        for name, (block, projs) in QWEN2_LINEARS.items():
            qw, qz, sc, bias = fused_awq_tensors(ckpt, [f"{lp}{block}.{p}" for p in projs])
            try:
                validate_awq(qw, qz, sc, cfg.group_size)
            except ValueError as e:
                raise CheckpointError(f"{lp}{block} ({name}): {e}") from None
            if world > 1 and name == "qkv":
                pieces, _ = attn  # type: ignore[misc]
                if sc.shape[1] != sum(heads.parts):
                    raise CheckpointError(f"{lp}{block}: q|k|v N={sc.shape[1]} does not match "
                                          f"the head layout {heads}")
                qw, qz, sc, bias = slice_awq_columns(qw, qz, sc, bias, pieces)
            elif world > 1 and name == "o":
                _, (k0, k1) = attn  # type: ignore[misc]
                if qw.shape[0] != heads.parts[0]:
                    raise CheckpointError(f"{lp}{block}: o_proj K={qw.shape[0]} does not match "
                                          f"the head layout {heads}")
                qw, qz, sc, bias = slice_awq_rows(qw, qz, sc, bias, k0, k1, cfg.group_size,
                                                  rank == 0)
            elif world > 1:
                kind, aligned = QWEN2_TP[name]
                parts = tuple(int(ckpt.get(f"{lp}{block}.{p}.scales").shape[1]) for p in projs)
                qw, qz, sc, bias = shard_awq(qw, qz, sc, bias, kind, rank, world, cfg.group_size,
                                             parts if kind == "column" else None, aligned)
            ws[name] = pack_awq(qw.to(dev), qz.to(dev), sc.to(dev), cfg.group_size)
            if name == "qkv" and bias is not None:
                qkv_bias = bias.to(device=dev, dtype=torch.float16)
            elif bias is not None:
                raise CheckpointError(f"{lp}{block} ({name}): unexpected bias")
        norms = []
        for n in ("input_layernorm", "post_attention_layernorm"):
            try:
                norms.append(ckpt.get(f"{lp}{n}.weight").to(device=dev, dtype=torch.float16))
            except KeyError as e:
                raise CheckpointError(str(e)) from None
        out.append(DecoderLayer(ws["qkv"], qkv_bias, ws["o"], ws["gate_up"], ws["down"],
                                norms[0], norms[1]))
    return out


__all__ = [
    "AWQConfig", "Checkpoint", "CheckpointError", "DecoderLayer", "QWEN2_LINEARS", "QWEN2_TP",
    "SafetensorsFile", "attention_heads", "fused_awq_tensors", "load_decoder_layers",
    "num_layers", "shard_awq", "slice_awq_columns", "slice_awq_rows",
]
