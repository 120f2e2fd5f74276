"""Benchmark of the quantized-linear hot path on B200 (one JSON line on rank 0).

Headline workload (BASELINE config 3 at M = 1): the Qwen2.5-7B decode linear-layer sweep,
28 layers x {qkv 3584->4608, o 3584->3584, gate_up 3584->37888, down 18944->3584}, W4A16
group-128 AWQ weights with random codes (q, z uniform in [0, 15], scales uniform(0.002, 0.02)),
repacked once by the awq_repack kernel. A "step" is one pass over all 112 layers. At N GPUs
the layers are tensor-parallel (column-split qkv/gate_up, row-split o/down + NCCL all-reduce
of the fp16 partials), so the total work is fixed and ``scaling`` is "strong".

    python bench.py [--gpus N] [--steps K] [--warmup W] [--m M] [--impl ours|reference]

Metric: achieved W4A16 HBM GB/s, i.e. algorithmic bytes of every layer in the step
(N*K/2 + (K/G)*N*2 + (K/G)*N/2 + M*K*2 + M*N*2 per layer, the reference's formula in
tokenforge/bench/micro.py:82-86, summed over ranks) divided by the device time of the step,
max over ranks. The step streams 3.4 GB of weights, far more than the 126 MB L2, so no layer's
weights are cache-resident when it runs (no separate L2 flush).
The same line carries the W4A16 GEMM TFLOP/s at M = 1024 (config 2, gate_up + down).

``--impl reference`` times the reference's CPU path (dequantize + fp32 matmul, w4a16_torch of
tokenforge/kernels/reference.py:24-32) through the oracle's C port on all host cores, on one
decoder layer of the same workload per step.
"""

from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
HIDDEN, INTER, LAYERS, G = 3584, 18944, 28, 128
# name, N, K, parallel kind
LAYER_SHAPES = [
    ("qkv", 4608, HIDDEN, "column"),
    ("o", HIDDEN, HIDDEN, "row"),
    ("gate_up", 2 * INTER, HIDDEN, "column"),
    ("down", HIDDEN, INTER, "row"),
]
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def _qwen7b_heads():  # type: ignore[no-untyped-def]
    from tokenforge_b200.tp import AttentionHeads

    return AttentionHeads(28, 4, 128)


def algorithmic_bytes(m: int, n: int, k: int, g: int = G) -> int:
    return n * k // 2 + (k // g) * n * 2 + (k // g) * n // 2 + m * k * 2 + m * n * 2


def metric_name(m: int) -> str:
    return f"W4A16 GEMV HBM GB/s at M={m} (Qwen2.5-7B decode sweep, 28 layers)"


TRAFFIC_FILE = ROOT / "profiles" / "w4a16_gemv_decode_dram.json"


def dram_traffic(kinds: list[str], n_layers: int, m: int, world: int) -> dict | None:
    """DRAM bytes (read + write) per launch of each layer type, from the committed ncu capture
    (dram__bytes_read.sum + dram__bytes_write.sum), scaled to one step of this sweep."""
    if not TRAFFIC_FILE.exists():
        return None
    d = json.loads(TRAFFIC_FILE.read_text())
    per = d.get("dram_bytes_per_launch", {})
    if d.get("m") != m or d.get("tp") != world or any(k not in per for k in kinds):
        return None
    return {"bytes_per_step": int(sum(per[k] for k in kinds) * n_layers),
            "per_launch": {k: per[k] for k in kinds}}


def peaks() -> tuple[dict[str, float], str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"])}, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# ----------------------------------------------------------------------------- clocks


class ClockSampler:
    """Samples SM clock and throttle reasons with nvidia-smi while the GPU is under load.

    Polls every ~50 ms from a background thread. :meth:`window` brackets the timed region; the
    summary reports the samples taken inside it, and when the region is shorter than one poll,
    the samples of the untimed settle phase that runs the same graph immediately before it
    (``"window"`` says which).
    """

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, index: int) -> None:
        self.index = index
        self.samples: list[tuple[float, list[str]]] = []  # (host time at the poll's midpoint, fields)
        self.t0 = self.t1 = 0.0
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True)

    def _run(self) -> None:
        while not self._stop.is_set():
            t = time.monotonic()
            try:
                out = subprocess.run(
                    ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                     "--format=csv,noheader,nounits"],
                    capture_output=True, text=True, timeout=5,
                ).stdout.strip()
            except (OSError, subprocess.SubprocessError):
                return
            if out:
                self.samples.append((0.5 * (t + time.monotonic()), [v.strip() for v in out.split(",")]))
            self._stop.wait(0.05)

    def __enter__(self) -> ClockSampler:
        self._thread.start()
        return self

    def __exit__(self, *exc: object) -> None:
        self._stop.set()
        self._thread.join(timeout=10)

    def window(self, start: bool) -> None:
        if start:
            self.t0 = time.monotonic()
        else:
            self.t1 = time.monotonic()

    def summary(self) -> dict[str, object]:
        inside = [f for t, f in self.samples if self.t0 <= t <= self.t1]
        where = "timed region"
        if not inside:
            inside = [f for t, f in self.samples if t <= self.t1]
            where = "settle phase before the timed region (same graph) + timed region"
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}

        def num(v: str) -> float | None:
            try:
                return float(v)
            except ValueError:
                return None

        sm = [x for x in (num(f[0]) for f in inside) if x is not None]
        mx = [x for x in (num(f[1]) for f in inside) if x is not None]
        pw = [x for x in (num(f[2]) for f in inside) if x is not None]
        reasons = sorted({self.NAMES[i] for f in inside for i in range(4)
                          if len(f) > 3 + i and f[3 + i].lower() == "active"})
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(mx) if mx else None,
            "power_w": round(statistics.median(pw), 1) if pw else None,
            "reasons": reasons,
            "samples": len(inside),
            "window": where,
        }


# ----------------------------------------------------------------------------- workload


class DecodeSweep:
    """This rank's shards of the 28-layer sweep plus the C-ABI argument tuples of a step."""

    def __init__(self, m: int, rank: int, world: int, device: torch.device, seed: int = 0,
                 kinds: tuple[str, ...] | None = None, n_layers: int = LAYERS,
                 peers=None) -> None:  # type: ignore[no-untyped-def]
        from tokenforge_b200 import _lib, tp
        from tokenforge_b200.pack import W4A16Weights

        self.m, self.rank, self.world, self.device = m, rank, world, device
        self.n_layers = n_layers
        # Row-parallel layers whose all-reduce runs fused in the GEMV (same decision on every
        # rank: it depends on the global shape only).
        self.peers = peers
        self.fused = {name: bool(peers is not None and peers.supports(m, n, k, G))
                      for name, n, k, kind in LAYER_SHAPES if kind == "row"}
        shapes = [s for s in LAYER_SHAPES if kinds is None or s[0] in kinds]
        self.kinds = [s[0] for s in shapes]
        self.lib = _lib.lib()
        gen = torch.Generator(device=device).manual_seed(seed * 7919 + rank)
        self.layers: list[list[tuple[str, W4A16Weights, tuple[int, int]]]] = []
        self.bytes_per_step = 0  # this rank's algorithmic bytes
        self.shard_shapes: dict[str, tuple[int, int]] = {}
        for _ in range(n_layers):
            row = []
            for name, n, k, kind in shapes:
                if kind == "column":
                    n0, n1 = tp.column_bounds(n, world)[rank]
                    nn, kk, bounds = n1 - n0, k, (n0, n1)
                else:
                    k0, k1 = tp.row_bounds(k, G, world)[rank]
                    nn, kk, bounds = n, k1 - k0, (k0, k1)
                qweight = torch.randint(-(2**31), 2**31 - 1, (kk, nn // 8), generator=gen,
                                        dtype=torch.int32, device=device)
                qzeros = torch.randint(-(2**31), 2**31 - 1, (kk // G, nn // 8), generator=gen,
                                       dtype=torch.int32, device=device)
                scales = (torch.rand((kk // G, nn), generator=gen, device=device) * 0.018
                          + 0.002).to(torch.float16)
                qweight_t = torch.ops.tokenforge.awq_repack(qweight)
                del qweight
                row.append((name, W4A16Weights(qweight_t, scales, qzeros, G), bounds))
                self.bytes_per_step += algorithmic_bytes(m, nn, kk)
                self.shard_shapes[name] = (nn, kk)
            self.layers.append(row)
        xg = torch.Generator(device=device).manual_seed(seed + 17)
        self.x_h = torch.randn((m, HIDDEN), generator=xg, device=device).to(torch.float16)
        self.x_o = torch.randn((m, HIDDEN), generator=xg, device=device).to(torch.float16)
        self.x_d = torch.randn((m, INTER), generator=xg, device=device).to(torch.float16)
        self.y = {name: torch.empty((m, self.shard_shapes[name][0]), dtype=torch.float16,
                                    device=device) for name in self.kinds}
        ws = max(int(self.lib.tf_w4a16_workspace_bytes(m, nn, kk, G))
                 for nn, kk in self.shard_shapes.values())
        self.ws = torch.empty(max(ws, 16), dtype=torch.uint8, device=device)
        self.ws_bytes = ws
        self.calls: list[tuple[str, tuple]] = []
        for row in self.layers:
            for name, w, bounds in row:
                if name in ("qkv", "gate_up"):
                    x, ldx = self.x_h, HIDDEN
                    xp = x.data_ptr()
                else:
                    x = self.x_o if name == "o" else self.x_d
                    ldx = x.stride(0)
                    xp = x.data_ptr() + bounds[0] * 2  # this rank's K slice
                y = self.y[name]
                args = (xp, m, w.k, ldx, w.qweight_t.data_ptr(), w.scales.data_ptr(),
                        w.qzeros.data_ptr(), None, w.n, G, y.data_ptr(), w.n,
                        self.ws.data_ptr(), self.ws_bytes)
                self.calls.append((name, args))
        self.launches_per_step = 0
        for name, (nn, kk) in self.shard_shapes.items():
            out = (ctypes.c_int32 * 9)()
            self.lib.tf_launch_plan(m, nn, kk, G, ctypes.addressof(out))
            outer_split = out[4] // max(out[8], 1)
            self.launches_per_step += n_layers * (1 + (1 if outer_split > 1 else 0))

    def step(self, only: str | None = None, allreduce: bool = True) -> None:
        import torch.distributed as dist

        stream = torch.cuda.current_stream(self.device).cuda_stream
        fn = self.lib.tf_w4a16_linear
        for name, args in self.calls:
            if only is not None and name != only:
                continue
            if self.world > 1 and self.fused.get(name, False):
                st = self.lib.tf_w4a16_linear_allreduce(*args, ctypes.byref(self.peers.peers),
                                                         stream)
                if st != 0:
                    raise RuntimeError(f"tf_w4a16_linear_allreduce({name}) failed with status {st}")
                continue
            st = fn(*args, stream)
            if st != 0:
                raise RuntimeError(f"tf_w4a16_linear({name}) failed with status {st}")
            if allreduce and self.world > 1 and name in ("o", "down"):
                dist.all_reduce(self.y[name])


def random_w4a16(n: int, k: int, gen: torch.Generator, device: torch.device):  # type: ignore[no-untyped-def]
    """A synthetic AWQ layer (uniform int4 codes and zeros, scales in [0.002, 0.02]) repacked on
    the GPU into the kernel layout."""
    from tokenforge_b200.pack import W4A16Weights

    qweight = torch.randint(-(2**31), 2**31 - 1, (k, n // 8), generator=gen, dtype=torch.int32,
                            device=device)
    qzeros = torch.randint(-(2**31), 2**31 - 1, (k // G, n // 8), generator=gen,
                           dtype=torch.int32, device=device)
    scales = (torch.rand((k // G, n), generator=gen, device=device) * 0.018 + 0.002).to(torch.float16)
    return W4A16Weights(torch.ops.tokenforge.awq_repack(qweight), scales, qzeros, G)


def capture(fn, device: torch.device) -> torch.cuda.CUDAGraph:  # type: ignore[no-untyped-def]
    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream(device).wait_stream(s)
    torch.cuda.synchronize(device)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize(device)
    return g


def time_graph(g: torch.cuda.CUDAGraph, reps: int, device: torch.device, barrier=None,  # type: ignore[no-untyped-def]
               clocks: ClockSampler | None = None) -> float:
    """Milliseconds for ``reps`` back-to-back replays, timed with CUDA events on the current
    stream (the one the graph is replayed on), with a synchronize (and barrier) on both sides."""
    torch.cuda.synchronize(device)
    if barrier:
        barrier()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    if clocks:
        clocks.window(True)
    start.record()
    for _ in range(reps):
        g.replay()
    end.record()
    torch.cuda.synchronize(device)
    if clocks:
        clocks.window(False)
    if barrier:
        barrier()
    return start.elapsed_time(end)


# ----------------------------------------------------------------------------- CPU baseline


class CpuLayerSample:
    """One decoder layer (qkv, o, gate_up, down) at M tokens for the oracle's C port of the
    reference CPU path (dequantize + fp32 matmul, all host cores)."""

    def __init__(self, m: int) -> None:
        self.m = m
        self.cores = os.cpu_count() or 1
        gen = torch.Generator().manual_seed(5)
        self.tensors, self.bytes = [], 0
        for _, n, k, _ in LAYER_SHAPES:
            qw = torch.randint(-(2**31), 2**31 - 1, (n, k // 8), generator=gen, dtype=torch.int32)
            z = torch.randint(-(2**31), 2**31 - 1, (k // G, n // 8), generator=gen, dtype=torch.int32)
            s = (torch.rand((k // G, n), generator=gen) * 0.018 + 0.002).to(torch.float16)
            x = torch.randn((m, k), generator=gen).to(torch.float16)
            self.tensors.append((x, qw, s, z))
            self.bytes += algorithmic_bytes(m, n, k)

    def run(self) -> float:
        """Seconds for one pass over the layer."""
        from oracle import oracle

        t0 = time.perf_counter()
        for x, qw, s, z in self.tensors:
            oracle.w4a16_cpu(x, qw, s, z, G, threads=self.cores)
        return time.perf_counter() - t0

    def describe(self, reps: int) -> str:
        return (f"one decoder layer (qkv, o, gate_up, down) at M={self.m}, {self.bytes} algorithmic "
                f"bytes per pass, median of {reps} passes")


def cpu_baseline(m: int, min_seconds: float = 10.0) -> dict[str, object]:
    """The CPU port timed for about ``min_seconds`` (at least 3 passes), median pass."""
    sample = CpuLayerSample(m)
    sample.run()  # first touch of the inputs
    times: list[float] = []
    while len(times) < 3 or sum(times) < min_seconds:
        times.append(sample.run())
    sec = statistics.median(times)
    return {
        "value": round(sample.bytes / sec / 1e9, 4),
        "unit": "GB/s",
        "cores": sample.cores,
        "kind": "port",
        "sample": sample.describe(len(times)),
        "seconds_per_sample": round(sec, 4),
    }


def run_reference(args: argparse.Namespace) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    t_all = time.perf_counter()
    sample = CpuLayerSample(args.m)
    for _ in range(args.warmup):
        sample.run()
    times = [sample.run() for _ in range(args.steps)]
    sec = statistics.median(times)
    value = round(sample.bytes / sec / 1e9, 4)
    cb = {"value": value, "unit": "GB/s", "cores": sample.cores, "kind": "port",
          "sample": sample.describe(len(times))}
    line = {
        "impl": "reference",
        "metric": metric_name(args.m),
        "value": value,
        "unit": "GB/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(sec * 1e3, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int4xfp16->fp32",
        "data": "synthetic",
        "config": {"workload": f"config3 decode sweep: 28 layers x (qkv, o, gate_up, down), "
                               f"M={args.m}; each step times one of its decoder layers on the CPU",
                   "m": args.m, "group_size": G},
        "cpu_baseline": cb,
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": round(time.perf_counter() - t_all, 2),
    }
    print(json.dumps(line), flush=True)


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def _median_seconds(fn, min_seconds: float) -> tuple[float, int]:  # type: ignore[no-untyped-def]
    fn()  # first touch
    times: list[float] = []
    while len(times) < 3 or sum(times) < min_seconds:
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    return statistics.median(times), len(times)


def cpu_aux_baselines(min_seconds: float = 4.0) -> dict[str, dict]:
    """The reference's CPU path for the other legs, through the oracle's C ports on bounded samples:
    the GEMM (w4a16_torch, reference.py:24-32, at M = 1024 on a 1024-column slice of gate_up),
    the AWQ repack (repack_awq_to_tf, pack.py:141-143, on the whole down layer) and RMSNorm + FP8
    (rmsnorm_fp8_reference, reference.py:53-56, at T = 4096, H = 3584)."""
    from oracle import oracle

    cores = os.cpu_count() or 1
    gen = torch.Generator().manual_seed(11)
    out: dict[str, dict] = {}
    m, n, k = 1024, 1024, HIDDEN
    qw = torch.randint(-(2**31), 2**31 - 1, (n, k // 8), generator=gen, dtype=torch.int32)
    z = torch.randint(-(2**31), 2**31 - 1, (k // G, n // 8), generator=gen, dtype=torch.int32)
    s = (torch.rand((k // G, n), generator=gen) * 0.018 + 0.002).to(torch.float16)
    x = torch.randn((m, k), generator=gen).to(torch.float16)
    sec, reps = _median_seconds(lambda: oracle.w4a16_cpu(x, qw, s, z, G, threads=cores), min_seconds)
    out["gemm"] = {"value": round(2 * m * n * k / sec / 1e12, 5), "unit": "TFLOP/s", "cores": cores,
                   "kind": "port", "sample": f"w4a16_torch at M={m}, N={n} (a slice of gate_up), "
                                             f"K={k}; median of {reps}"}
    qweight = torch.randint(-(2**31), 2**31 - 1, (INTER, HIDDEN // 8), generator=gen,
                            dtype=torch.int32)
    sec, reps = _median_seconds(lambda: oracle.repack_awq_to_tf(qweight), min_seconds)
    out["repack"] = {"value": round(2 * qweight.numel() * 4 / sec / 1e9, 4), "unit": "GB/s",
                     "cores": 1, "kind": "port",
                     "sample": f"repack_awq_to_tf of down [{INTER}, {HIDDEN // 8}] int32, one "
                               f"thread; median of {reps}"}
    t = 4096
    xr = torch.randn((t, HIDDEN), generator=gen).to(torch.float16)
    gamma = (1 + 0.1 * torch.randn(HIDDEN, generator=gen)).to(torch.float16)
    sec, reps = _median_seconds(lambda: oracle.rmsnorm_fp8(xr, gamma, 1e-6), min_seconds)
    per_call = t * HIDDEN * 2 + HIDDEN * 2 + t * HIDDEN + t * 4
    out["rmsnorm_fp8"] = {"value": round(per_call / sec / 1e9, 4), "unit": "GB/s", "cores": cores,
                          "kind": "port",
                          "sample": f"rmsnorm_fp8_reference at T={t}, H={HIDDEN}; median of {reps}"}
    return out


def _w4a16_tol(x: torch.Tensor, w16: torch.Tensor) -> float:
    """The W4A16 tolerance rule c * sqrt(K) * 2^-10 * max|x| * max|w| with the calibrated cuda
    constant (tests/numerics/tolerances.json), the reference's rule (tests/numerics/tolerance.py)."""
    c = json.loads((ROOT / "tests" / "numerics" / "tolerances.json").read_text())["w4a16"]["cuda"]["c"]
    return float(c) * x.shape[-1] ** 0.5 * 2.0**-10 * float(x.abs().max()) * float(w16.abs().max())


def decode_parity(device: torch.device, rank: int, world: int, peers, m: int) -> dict:  # type: ignore[no-untyped-def]
    """Correctness of the timed decode paths at this N, checked in the bench run itself with the
    product's own kernels: the o and down layers of Qwen2.5-7B (weights from one seed, identical
    on every rank) against the fp64 product of their dequantized weights (tokenforge dequant
    kernel, bit-exact with the reference's dequant), full width.
      N = 1: the decode GEMV (tf_w4a16_linear) of each layer within the W4A16 tolerance.
      N > 1: each rank's row shard through the all-reduce fused into the GEMV
      (tf_w4a16_linear_allreduce) and through the GEMV + NCCL all-reduce; the fused result must
      be bit-identical on every rank and across repeated calls, within the tolerance of the
      fp64 product of the unsharded layer (NCCL path: twice the tolerance, fp16 partials)."""
    import torch.distributed as dist

    import tokenforge_b200.ops as ops
    from tokenforge_b200 import tp

    gen = torch.Generator(device=device).manual_seed(2027)
    res: dict[str, object] = {"m": m, "layers": {}}
    ok = True
    for name, n, k in (("o", HIDDEN, HIDDEN), ("down", HIDDEN, INTER)):
        w = random_w4a16(n, k, gen, device)
        x = torch.randn((m, k), generator=gen, device=device).to(torch.float16)
        w16 = torch.ops.tokenforge.w4a16_dequant(w.qweight_t, w.scales, w.qzeros, G)
        ref = x.double() @ w16.double().t()
        tol = _w4a16_tol(x, w16)
        entry: dict[str, object] = {"tol": tol}
        if world == 1:
            y = ops.w4a16_gemm(x, w.qweight_t, w.scales, w.qzeros, G)
            err = float((y.double() - ref).abs().max())
            entry["gemv_err"] = err
            ok &= err <= tol
        else:
            shard = tp.shard_layer(w, "row", rank, world)
            fused = [tp.linear_shard(x, shard, peers=peers) for _ in range(2)] if peers else []
            plain = tp.linear_shard(x, shard)
            if fused:
                gathered = [torch.empty_like(fused[0]) for _ in range(world)]
                dist.all_gather(gathered, fused[0])
                same = all(torch.equal(g, gathered[0]) for g in gathered) and torch.equal(
                    fused[0], fused[1])
                err = float((fused[0].double() - ref).abs().max())
                entry.update({"fused_err": err, "ranks_bit_identical": same})
                ok &= same and err <= tol
            err_p = float((plain.double() - ref).abs().max())
            entry["nccl_err"] = err_p
            ok &= err_p <= 2 * tol
        res["layers"][name] = entry  # type: ignore[index]
        del w16, ref
    if world > 1:
        flags = torch.tensor([1 if ok else 0], device=device)
        dist.all_reduce(flags, op=dist.ReduceOp.MIN)
        ok = bool(flags.item())
        res["peer_error"] = peers.error() if peers else 0
        ok &= res["peer_error"] == 0
    res["ok"] = bool(ok)
    return res


def peer_trace_leg(device: torch.device, rank: int, world: int, peers, m: int,  # type: ignore[no-untyped-def]
                   reps: int = 20) -> dict:
    """Where the fused all-reduce GEMV spends its time (N > 1; tf_peer_trace): for o and down of
    Qwen2.5-7B, `reps` times, eight back-to-back fused calls of the layer with the last one
    traced. Every 32-row tile's storing warp stamps %globaltimer at the exchange's entry (its
    partial sums done), after its stores to every peer, when the last peer word has arrived, and
    after writing y. The eight calls are one CUDA graph (the last captured with the trace
    buffer), so the traced launch runs in a device-side stream of exchanges, as in the sweep.
    Reported in us, medians over the replays:
      entry_spread: last tile's entry minus first tile's entry on this rank (compute imbalance);
      store: entry -> stores issued; wait: stores issued -> last peer word here (median tile,
      and the slowest tile); tail: arrived -> y written.
    The GPUs' timers are not aligned with each other (offsets of seconds were seen), so skew
    between ranks shows only inside `wait` (the peer's matching tile stored later, plus the
    store's flight over NVLink). The timer ticks in 256 ns steps on this B200 pool."""
    import torch.distributed as dist

    from tokenforge_b200 import _lib, tp

    gen = torch.Generator(device=device).manual_seed(2028)
    lib = _lib.lib()
    out: dict[str, object] = {"m": m, "reps": reps}
    for name, n, k in (("o", HIDDEN, HIDDEN), ("down", HIDDEN, INTER)):
        w = random_w4a16(n, k, gen, device)
        x = torch.randn((m, k), generator=gen, device=device).to(torch.float16)
        shard = tp.shard_layer(w, "row", rank, world)
        tiles = -(-n // 32)
        rec = torch.zeros(4 * tiles, dtype=torch.int64, device=device)

        def calls() -> None:
            for i in range(8):
                if i == 7:
                    lib.tf_peer_trace(ctypes.c_void_p(rec.data_ptr()))
                tp.linear_shard(x, shard, peers=peers)
                if i == 7:
                    lib.tf_peer_trace(None)

        for _ in range(3):
            tp.linear_shard(x, shard, peers=peers)
        torch.cuda.synchronize(device)
        graph = capture(calls, device)
        rows = []
        for _ in range(reps):
            dist.barrier(device_ids=[device.index])
            graph.replay()
            torch.cuda.synchronize(device)
            t = rec.view(tiles, 4).cpu().double()
            first = t[:, 0].min()
            rows.append([float(t[:, 0].max() - first), float((t[:, 1] - t[:, 0]).median()),
                         float((t[:, 2] - t[:, 1]).median()), float((t[:, 2] - t[:, 1]).max()),
                         float((t[:, 3] - t[:, 2]).median())])
        del graph
        med = torch.tensor(rows).median(dim=0).values.tolist()
        keys = ("entry_spread", "store", "wait", "wait_max", "tail")
        out[name] = {kk: round(v / 1e3, 3) for kk, v in zip(keys, med)}
        del w, shard
    return out


def e2e_graph(sweep: DecodeSweep, device: torch.device, steps: int, barrier, world: int) -> dict:  # type: ignore[no-untyped-def]
    """The sweep end to end through the C ABI, as a user serves it: every step copies the step's
    activations from pinned host memory to the device, runs the 112 tf_w4a16_linear calls (plus
    the row-parallel all-reduces) and copies the last output back to pinned host memory; the
    whole step is one CUDA graph (the calls captured once), replayed once per step."""
    import torch.distributed as dist

    h_in = [torch.empty_like(x, device="cpu").pin_memory() for x in (sweep.x_h, sweep.x_o, sweep.x_d)]
    for hbuf, x in zip(h_in, (sweep.x_h, sweep.x_o, sweep.x_d)):
        hbuf.copy_(x.cpu())
    y_last = sweep.y[sweep.kinds[-1]]
    h_out = torch.empty_like(y_last, device="cpu").pin_memory()
    h2d = sum(h.numel() * h.element_size() for h in h_in)
    d2h = h_out.numel() * h_out.element_size()

    def e2e_step() -> None:
        for hbuf, x in zip(h_in, (sweep.x_h, sweep.x_o, sweep.x_d)):
            x.copy_(hbuf, non_blocking=True)
        sweep.step()
        h_out.copy_(y_last, non_blocking=True)

    g = capture(e2e_step, device)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize(device)
    if barrier:
        barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    e0.record()
    for _ in range(steps):
        g.replay()
    e1.record()
    torch.cuda.synchronize(device)
    wall_ms = (time.perf_counter() - w0) * 1e3 / steps
    t = torch.tensor([max(e0.elapsed_time(e1) / steps, wall_ms)], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    del g
    return {"ms_per_step": float(t.item()), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "host_matches_device": bool(torch.equal(h_out, y_last.cpu()))}


def chain_leg(sweep: DecodeSweep, device: torch.device, steps: int) -> dict | None:
    """The same sweep as one persistent decode chain (tokenforge_b200.chain.DecodeChain), every op
    waiting for the one before (as the layers of a real decode step do), timed with CUDA events."""
    from tokenforge_b200.chain import ChainLinear, DecodeChain

    xs = {"qkv": sweep.x_h, "gate_up": sweep.x_h, "o": sweep.x_o, "down": sweep.x_d}
    ops_ = [ChainLinear(xs[name], w, sweep.y[name], wait=i > 0)
            for i, (name, w, _) in enumerate(e for row in sweep.layers for e in row)]
    try:
        ch = DecodeChain(ops_)
    except Exception as e:  # noqa: BLE001 - a shape outside the chain's limits: report, not fail
        return {"unavailable": str(e)}
    with ch:
        for _ in range(3):
            ch.run()
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            ch.run()
        e1.record()
        torch.cuda.synchronize(device)
        ms = e0.elapsed_time(e1) / steps
        err = ch.error()
    return {"ms_per_step": round(ms, 4), "gbs": round(sweep.bytes_per_step / (ms * 1e-3) / 1e9, 1),
            "device_error": err, "dependent_ops": True}


# ----------------------------------------------------------------------------- block stack (config 4)


def block_metric(sweep: DecodeSweep, device: torch.device, ms: tuple[int, ...], steps: int,
                 fuse_norm: bool = True, rank: int = 0, world: int = 1, peers=None,  # type: ignore[no-untyped-def]
                 barrier=None, fuse_silu: bool = True) -> dict:
    """the Qwen2.5-7B-shaped quantized block stack on the sweep's 28 layers of
    weights. Per layer: rmsnorm_fp8_quant of the fp16 residual -> W4A16 qkv on the e4m3
    activations -> the v slice (512 channels) repeated 7x stands in for attention -> W4A16 o ->
    residual add -> rmsnorm_fp8_quant -> W4A16 gate_up on e4m3 -> SiLU * up -> W4A16 down ->
    residual add. One step = the 28 layers on M tokens, replayed as a CUDA graph; tokens/s =
    M / step time. With fuse_norm, each RMSNorm + quant + linear pair is the one fused op
    (rmsnorm_fp8_w4a16_linear: one kernel at decode sizes, bit-identical; two ops otherwise)."""
    import tokenforge_b200.ops as ops

    gen = torch.Generator(device=device).manual_seed(123)
    gammas = [((1 + 0.1 * torch.randn((2, HIDDEN), generator=gen, device=device))
               .to(torch.float16)) for _ in sweep.layers]
    out: dict[str, object] = {
        "metric": f"Qwen2.5-7B quantized block stack tokens/s (config 4, 28 layers, TP={world})",
        "unit": "tokens/s",
        "fused_norm_linear": fuse_norm,
        "fused_silu_linear": fuse_silu and world == 1,
        "per_m": {},
    }
    if world > 1:
        return block_tp_metric(out, gammas, device, ms, steps, fuse_norm, rank, world, peers,
                               barrier)
    for m in ms:
        h0 = torch.randn((m, HIDDEN), generator=gen, device=device).to(torch.float16)

        def norm_linear(h: torch.Tensor, gamma: torch.Tensor, wt) -> torch.Tensor:  # type: ignore[no-untyped-def]
            if fuse_norm:
                return torch.ops.tokenforge.rmsnorm_fp8_w4a16_linear(
                    h, gamma, 1e-6, None, wt.qweight_t, wt.scales, wt.qzeros, None, G)
            q, sc = torch.ops.tokenforge.rmsnorm_fp8_quant(h, gamma, 1e-6, None)
            return torch.ops.tokenforge.w4a16_linear_fp8(q, sc, wt.qweight_t, wt.scales,
                                                         wt.qzeros, None, G)

        def step() -> None:
            h = h0
            for row, gamma in zip(sweep.layers, gammas):
                w = {name: wt for name, wt, _ in row}
                qkv = norm_linear(h, gamma[0], w["qkv"])
                v = qkv[:, 4096:].repeat(1, 7)
                h = h + ops.w4a16_gemm(v, w["o"].qweight_t, w["o"].scales, w["o"].qzeros, G)
                gu = norm_linear(h, gamma[1], w["gate_up"])
                if fuse_silu:
                    h = h + torch.ops.tokenforge.silu_mul_w4a16_linear(
                        gu, w["down"].qweight_t, w["down"].scales, w["down"].qzeros, None, G)
                else:
                    a = ops.silu_mul(gu)
                    h = h + ops.w4a16_gemm(a, w["down"].qweight_t, w["down"].scales,
                                           w["down"].qzeros, G)
            step.out = h  # type: ignore[attr-defined]

        g = capture(step, device)
        g.replay()
        torch.cuda.synchronize(device)
        reps = max(2, steps if m <= 64 else steps // 4)
        ms_step = time_graph(g, reps, device) / reps
        finite = bool(torch.isfinite(step.out).all())  # type: ignore[attr-defined]
        out["per_m"][str(m)] = {  # type: ignore[index]
            "tokens_per_s": round(m / (ms_step * 1e-3), 1),
            "ms_per_step": round(ms_step, 4),
            "output_finite": finite,
        }
        del g
    return out


def block_tp_metric(out: dict, gammas: list, device: torch.device, ms: tuple[int, ...], steps: int,  # type: ignore[type-arg]
                    fuse_norm: bool, rank: int, world: int, peers, barrier) -> dict:  # type: ignore[no-untyped-def]
    """The config-4 block stack over ``world`` GPUs (tensor parallel, one rank per GPU): this
    rank's shards of every layer, synthetic like the single-GPU leg. qkv holds [q_r | k_r | v_r]
    and gate_up [gate_r | up_r] (tp.fused_column_bounds, gate/up on 128-column groups so that
    gate_r is down's K shard); o and down are row shards whose partials are summed through the
    all-reduce fused into the GEMV (M <= 8, when ``peers`` is given) or NCCL. The attention
    stand-in tiles the rank's v slice to o's K shard width. The residual stream is replicated.
    tokens/s = M / step time (max over ranks)."""
    import torch.distributed as dist

    import tokenforge_b200.ops as ops
    from tokenforge_b200 import tp

    q_w, kv_w = HIDDEN, 512
    try:  # q|k|v and o on whole heads (28 q heads, 4 KV heads of 128): TP 1, 2 and 4
        qkv_pieces, (o0, o1) = tp.attention_bounds(_qwen7b_heads(), rank, world, G)
        attn_split = "heads"
    except ValueError:  # TP 8: 28 heads do not split 8 ways; the stand-in has no real heads
        qkv_pieces = tp.fused_column_bounds((q_w, kv_w, kv_w), rank, world)
        o0, o1 = tp.row_bounds(HIDDEN, G, world)[rank]
        attn_split = (f"8-column words (Qwen2.5-7B's 28 heads do not split over {world} ranks; "
                      f"the attention stand-in tiles the rank's v slice to o's K shard)")
    widths = [b - a for a, b in qkv_pieces]
    i0, i1 = tp.row_bounds(INTER, G, world)[rank]
    o_k, i_r = o1 - o0, i1 - i0
    gen = torch.Generator(device=device).manual_seed(4242 + rank)
    layers = [{"qkv": random_w4a16(sum(widths), HIDDEN, gen, device),
               "o": random_w4a16(HIDDEN, o_k, gen, device),
               "gate_up": random_w4a16(2 * i_r, HIDDEN, gen, device),
               "down": random_w4a16(HIDDEN, i_r, gen, device)} for _ in gammas]
    reps_of = max(1, -(-o_k // max(widths[2], 1)))
    out["tp"] = world
    out["sharding"] = (f"qkv [q_r|k_r|v_r] widths {widths}, o K {o_k}, gate_up [gate_r|up_r] "
                       f"2x{i_r}, down K {i_r} (rank {rank}); attention split on {attn_split}")
    for m in ms:
        fused_ok = {"o": peers is not None and peers.supports(m, HIDDEN, HIDDEN, G),
                    "down": peers is not None and peers.supports(m, HIDDEN, INTER, G)}
        h0 = torch.randn((m, HIDDEN), generator=torch.Generator(device=device).manual_seed(9),
                         device=device).to(torch.float16)

        def norm_linear(h: torch.Tensor, gamma: torch.Tensor, wt) -> torch.Tensor:  # type: ignore[no-untyped-def]
            if fuse_norm:
                return torch.ops.tokenforge.rmsnorm_fp8_w4a16_linear(
                    h, gamma, 1e-6, None, wt.qweight_t, wt.scales, wt.qzeros, None, G)
            q, sc = torch.ops.tokenforge.rmsnorm_fp8_quant(h, gamma, 1e-6, None)
            return torch.ops.tokenforge.w4a16_linear_fp8(q, sc, wt.qweight_t, wt.scales,
                                                         wt.qzeros, None, G)

        def row_parallel(x: torch.Tensor, wt, name: str) -> torch.Tensor:  # type: ignore[no-untyped-def]
            if fused_ok[name]:
                y = peers.linear(x, wt, None)
                if y is None:
                    raise RuntimeError(f"fused all-reduce refused {name} at M={m}")
                return y
            y = ops.w4a16_gemm(x, wt.qweight_t, wt.scales, wt.qzeros, G, None)
            dist.all_reduce(y)
            return y

        def step() -> None:
            h = h0
            for w, gamma in zip(layers, gammas):
                qkv = norm_linear(h, gamma[0], w["qkv"])
                v = qkv[:, widths[0] + widths[1]:]
                attn = v.repeat(1, reps_of)[:, :o_k].contiguous()
                h = h + row_parallel(attn, w["o"], "o")
                gu = norm_linear(h, gamma[1], w["gate_up"])
                h = h + row_parallel(ops.silu_mul(gu), w["down"], "down")
            step.out = h  # type: ignore[attr-defined]

        if barrier:
            barrier()
        g = capture(step, device)
        g.replay()
        torch.cuda.synchronize(device)
        reps = max(2, steps if m <= 64 else steps // 4)
        t = torch.tensor([time_graph(g, reps, device, barrier) / reps], device=device,
                         dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_step = float(t.item())
        finite = bool(torch.isfinite(step.out).all())  # type: ignore[attr-defined]
        out["per_m"][str(m)] = {  # type: ignore[index]
            "tokens_per_s": round(m / (ms_step * 1e-3), 1),
            "ms_per_step": round(ms_step, 4),
            "output_finite": finite,
            "allreduce": {k: ("fused" if v else "nccl") for k, v in fused_ok.items()},
        }
        del g
    return out


# ----------------------------------------------------------------------------- GEMM (config 2)


def gemm_metric(device: torch.device, ms: tuple[int, ...], steps: int, warmup: int, pk: dict,
                src: str, headline_m: int = 1024) -> dict:
    """gate_up + down W4A16 GEMM at each M, one CUDA graph per M."""
    from tokenforge_b200 import _lib
    from tokenforge_b200.config import launch_plan

    lib = _lib.lib()
    gen = torch.Generator(device=device).manual_seed(3)
    layers = []
    for name, n, k, _ in (LAYER_SHAPES[2], LAYER_SHAPES[3]):
        qweight = torch.randint(-(2**31), 2**31 - 1, (k, n // 8), generator=gen, dtype=torch.int32, device=device)
        qz = torch.randint(-(2**31), 2**31 - 1, (k // G, n // 8), generator=gen, dtype=torch.int32, device=device)
        s = (torch.rand((k // G, n), generator=gen, device=device) * 0.018 + 0.002).to(torch.float16)
        layers.append((name, n, k, torch.ops.tokenforge.awq_repack(qweight), qz, s))
        del qweight
    per_m = {}
    for m in ms:
        calls, flops, names, keep = [], 0, [], []
        for name, n, k, qt, qz, s in layers:
            x = torch.randn((m, k), generator=gen, device=device).to(torch.float16)
            y = torch.empty((m, n), dtype=torch.float16, device=device)
            ws_b = int(lib.tf_w4a16_workspace_bytes(m, n, k, G))
            ws = torch.empty(max(ws_b, 16), dtype=torch.uint8, device=device)
            keep += [x, y, ws]
            calls.append((x.data_ptr(), m, k, k, qt.data_ptr(), s.data_ptr(), qz.data_ptr(), None,
                          n, G, y.data_ptr(), n, ws.data_ptr(), ws_b))
            flops += 2 * m * n * k
            names.append(f"{name} {launch_plan(m, n, k, G).kernel}")

        def step() -> None:
            st = torch.cuda.current_stream(device).cuda_stream
            for a in calls:
                rc = lib.tf_w4a16_linear(*a, st)
                if rc != 0:
                    raise RuntimeError(f"gemm failed: {rc}")

        g = capture(step, device)
        for _ in range(warmup):
            g.replay()
        reps = steps if m <= 1024 else max(3, steps // 4)
        t_ms = time_graph(g, reps, device) / reps
        del g
        tflops = flops / (t_ms * 1e-3) / 1e12
        per_m[str(m)] = {"tflops": round(tflops, 2), "ms_per_step": round(t_ms, 4),
                         "frac": round(tflops / pk["bf16_tflops"], 4), "kernels": names}
    head = per_m[str(headline_m)]
    return {
        "metric": f"W4A16 GEMM TFLOP/s at M={headline_m} (Qwen2.5-7B gate_up + down, config 2)",
        "value": head["tflops"],
        "unit": "TFLOP/s",
        "ms_per_step": head["ms_per_step"],
        "kernels": head["kernels"],
        "roofline": {"bound": "tensor", "achieved": head["tflops"], "peak": pk["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": head["frac"],
                     "peak_source": f"{src} bf16_tflops (burst)", "traffic": None},
        "per_m": per_m,
        "l2": "weights 105 MB, x and y re-used across replays (tensor-bound above M ~ 256)",
    }


def repack_metric(device: torch.device, steps: int, pk: dict) -> dict:
    """BASELINE config 2's load-time step: AWQ repack of gate_up and down (int32 read + write),
    two copies of each alternated so that consecutive launches do not hit L2."""
    gen = torch.Generator(device=device).manual_seed(4)
    jobs, nbytes = [], 0
    for _, n, k, _ in (LAYER_SHAPES[2], LAYER_SHAPES[3]):
        for _ in range(2):
            jobs.append(torch.randint(-(2**31), 2**31 - 1, (k, n // 8), generator=gen,
                                      dtype=torch.int32, device=device))
        nbytes += 2 * k * (n // 8) * 4  # read + write of one layer
    outs: list[torch.Tensor] = []

    def step() -> None:
        outs.clear()
        for q in jobs[0::2]:
            outs.append(torch.ops.tokenforge.awq_repack(q))
        for q in jobs[1::2]:
            outs.append(torch.ops.tokenforge.awq_repack(q))

    g = capture(step, device)
    g.replay()
    t_ms = time_graph(g, steps, device) / steps / 2  # each step repacks every layer twice
    gbs = nbytes / (t_ms * 1e-3) / 1e9
    return {"metric": "AWQ repack GB/s (gate_up + down, read + write, config 2)",
            "value": round(gbs, 1), "unit": "GB/s", "ms_per_step": round(t_ms, 4),
            "frac_of_hbm": round(gbs / pk["hbm_gbs"], 4)}


def rmsnorm_metric(device: torch.device, steps: int, pk: dict) -> dict:
    """fused RMSNorm + per-token e4m3 quant, H = 3584, T in {1, 256, 4096};
    inputs fp16 ~N(0, 1) with 8 outlier channels x20, gamma ~N(1, 0.1). Enough input copies are
    rotated that the bytes touched per replay exceed L2 for T = 4096."""
    gen = torch.Generator(device=device).manual_seed(6)
    out: dict[str, object] = {"metric": "RMSNorm + FP8 e4m3 quant GB/s (config 1, H = 3584)",
                              "unit": "GB/s", "per_t": {}}
    hidden = HIDDEN
    outliers = torch.randperm(hidden, generator=torch.Generator().manual_seed(6))[:8]
    gamma = (1 + 0.1 * torch.randn(hidden, generator=gen, device=device)).to(torch.float16)
    for t in (1, 256, 4096):
        per_call = t * hidden * 2 + hidden * 2 + t * hidden + t * 4
        copies = max(2, min(64, -(-(256 << 20) // per_call)))
        xs = []
        for _ in range(copies):
            x = torch.randn((t, hidden), generator=gen, device=device)
            x[:, outliers.to(device)] *= 20
            xs.append(x.to(torch.float16))

        def step() -> None:
            for x in xs:
                torch.ops.tokenforge.rmsnorm_fp8_quant(x, gamma, 1e-6, None)

        g = capture(step, device)
        g.replay()
        t_ms = time_graph(g, max(3, steps // 2), device) / max(3, steps // 2) / copies
        out["per_t"][str(t)] = {  # type: ignore[index]
            "gbs": round(per_call / (t_ms * 1e-3) / 1e9, 1), "us_per_call": round(t_ms * 1e3, 3),
            "frac_of_hbm": round(per_call / (t_ms * 1e-3) / 1e9 / pk["hbm_gbs"], 4)}
        del g, xs
    return out


# ----------------------------------------------------------------------------- main


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--m", type=int, default=1)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--gemm-m", type=int, default=1024, help="M of the GEMM headline")
    ap.add_argument("--gemm-ms", type=str, default="16,64,256,1024,4096",
                    help="comma-separated M values of the GEMM leg (config 2)")
    ap.add_argument("--no-pdl", action="store_true", help="launch without programmatic dependent launch")
    ap.add_argument("--no-fuse", action="store_true",
                    help="N > 1: all-reduce o/down with NCCL instead of inside the GEMV")
    ap.add_argument("--skip-cpu", action="store_true", help="omit the CPU baseline leg")
    ap.add_argument("--skip-gemm", action="store_true", help="omit the GEMM M=1024 leg")
    ap.add_argument("--skip-block", action="store_true", help="omit the config-4 block-stack leg")
    ap.add_argument("--skip-aux", action="store_true",
                    help="omit the AWQ repack and RMSNorm+FP8 legs (configs 1 and 2)")
    ap.add_argument("--block-ms", type=str, default="1,64,2048",
                    help="token counts M of the config-4 block-stack leg")
    ap.add_argument("--skip-chain", action="store_true",
                    help="omit the persistent decode-chain leg (N = 1)")
    ap.add_argument("--no-fuse-silu", action="store_true",
                    help="block stack: separate SiLU-product and down-projection launches")
    ap.add_argument("--no-fuse-norm", action="store_true",
                    help="block stack: separate RMSNorm+FP8 and linear launches")
    ap.add_argument("--layer", choices=[s[0] for s in LAYER_SHAPES], action="append",
                    help="restrict the sweep to these layer types (profiling a small case)")
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="decoder layers in the sweep (28 = Qwen2.5-7B; fewer for a small case)")
    ap.add_argument("--peer-trace", action="store_true",
                    help="N > 1: trace the fused all-reduce's exchange on o and down (peer_trace)")
    ap.add_argument("--aux", action="store_true",
                    help="run the AWQ repack and RMSNorm+FP8 legs with a restricted sweep too "
                         "(profiling them on a small case)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        print("warmup must be >= 3", file=sys.stderr)
        sys.exit(2)
    if args.impl == "reference":
        run_reference(args)
        return

    import torch.distributed as dist

    import tokenforge_b200.ops  # noqa: F401
    from tokenforge_b200 import _lib

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=300))
    if world != args.gpus:
        print(f"--gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)
    _lib.set_launch_flags(0 if args.no_pdl else _lib.TF_LAUNCH_PDL)
    pk, src = peaks()

    full = args.layer is None and args.layers == LAYERS
    peers = None
    if world > 1 and not args.no_fuse:
        from tokenforge_b200.tp import PeerMailbox

        peers = PeerMailbox(max_m=8, max_n=HIDDEN, device=device)
    sweep = DecodeSweep(args.m, rank, world, device,
                        kinds=tuple(args.layer) if args.layer else None, n_layers=args.layers,
                        peers=peers)
    if world > 1:
        warm = torch.ones(1, device=device)
        dist.all_reduce(warm)
    barrier = (lambda: dist.barrier(device_ids=[local])) if world > 1 else None

    graph = capture(sweep.step, device)
    for _ in range(args.warmup):
        graph.replay()
    # Settle phase: about one second of untimed replays so the clocks seen by the sampler are
    # the ones under sustained load. The count is agreed over ranks (the graph holds NCCL calls).
    one = torch.tensor([time_graph(graph, 1, device, barrier)], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(one, op=dist.ReduceOp.MAX)
    settle = int(min(2000, max(3, 1000.0 / max(float(one.item()), 1e-3))))
    with ClockSampler(local) as clocks:
        time_graph(graph, settle, device, barrier)
        ms_total = time_graph(graph, args.steps, device, barrier, clocks)
    ms = ms_total / args.steps
    t = torch.tensor([ms], device=device, dtype=torch.float64)
    b = torch.tensor([sweep.bytes_per_step], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(b, op=dist.ReduceOp.SUM)
    ms_max = float(t.item())
    total_bytes = float(b.item())
    value = total_bytes / (ms_max * 1e-3) / 1e9

    # Roofline of the dominant kernel (the W4A16 GEMV): each layer type's 28 launches replayed
    # back to back as a graph, timed with CUDA events; algorithmic bytes / mean launch time.
    per_kind = {}
    kind_bytes = kind_ms = 0.0
    for name in sweep.kinds:
        g = capture(lambda name=name: sweep.step(only=name, allreduce=False), device)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize(device)
        reps = max(3, args.steps // 2)
        kms = time_graph(g, reps, device, barrier) / reps / sweep.n_layers
        nn, kk = sweep.shard_shapes[name]
        kb = algorithmic_bytes(args.m, nn, kk)
        per_kind[name] = {"n": nn, "k": kk, "us_per_launch": round(kms * 1e3, 3),
                          "gbs": round(kb / (kms * 1e-3) / 1e9, 1)}
        kind_bytes += kb * sweep.n_layers
        kind_ms += kms * sweep.n_layers
        del g
    achieved = kind_bytes / (kind_ms * 1e-3) / 1e9
    traffic = dram_traffic(sweep.kinds, sweep.n_layers, args.m, world)
    if traffic:
        for name in sweep.kinds:
            per_kind[name]["dram_bytes"] = traffic["per_launch"][name]

    # End to end through the C ABI with host buffers (pinned H2D of the step's activations, the
    # calls, D2H of the last output), captured once as a graph and replayed per step.
    e2e = e2e_graph(sweep, device, args.steps, barrier, world)
    e2e_value = total_bytes / (e2e["ms_per_step"] * 1e-3) / 1e9
    # Correctness of the timed paths at this N (fused all-reduce across ranks at N > 1).
    parity = decode_parity(device, rank, world, peers, min(args.m, 8))
    peer_trace = (peer_trace_leg(device, rank, world, peers, min(args.m, 8))
                  if args.peer_trace and world > 1 and peers is not None else None)
    chain = None
    if world == 1 and full and not args.skip_chain and args.m <= 8:
        chain = chain_leg(sweep, device, args.steps)

    gemm = None
    if world == 1 and not args.skip_gemm:
        gemm_ms = {int(v) for v in args.gemm_ms.split(",") if v} | {args.gemm_m}
        gemm = gemm_metric(device, tuple(sorted(gemm_ms)),
                           max(3, args.steps // 2), 3, pk, src, headline_m=args.gemm_m)
    extra = {}
    if world == 1 and (full or args.aux) and not args.skip_aux:
        extra["repack"] = repack_metric(device, max(3, args.steps // 2), pk)
        extra["rmsnorm_fp8"] = rmsnorm_metric(device, max(3, args.steps // 2), pk)
    block = None
    if full and not args.skip_block:
        block = block_metric(sweep, device, tuple(int(v) for v in args.block_ms.split(",")),
                             max(3, args.steps // 2), fuse_norm=not args.no_fuse_norm,
                             rank=rank, world=world, peers=peers, barrier=barrier,
                             fuse_silu=not args.no_fuse_silu)
    cpu = None
    if rank == 0 and world == 1 and full and not args.skip_cpu:
        cpu = cpu_baseline(args.m, min_seconds=10.0)
        cpu["cpu_model"] = cpu_model()
        aux_cpu = cpu_aux_baselines()
        if gemm is not None:
            gemm["cpu_baseline"] = aux_cpu["gemm"]
        for leg in ("repack", "rmsnorm_fp8"):
            if leg in extra:
                extra[leg]["cpu_baseline"] = aux_cpu[leg]

    if rank == 0:
        line = {
            "metric": metric_name(args.m),
            "value": round(value, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_max, 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "int4xfp16->fp32",
            "data": "synthetic",
            "config": {
                "workload": f"config3 decode sweep: {sweep.n_layers} layers x ({', '.join(sweep.kinds)}), "
                            f"M={args.m}, TP={world}, CUDA-graph replay",
                "m": args.m, "group_size": G, "tp": world,
                "parallelism": f"tp{world}" + ("" if world == 1 else (
                    " (o/down all-reduce fused into the GEMV over NVLink peer stores: "
                    + ", ".join(k for k, v in sweep.fused.items() if v) + "; NCCL for the rest)")),
                "l2": f"inputs larger than L2 ({total_bytes / 1e9:.2f} GB of weights streamed per step)",
                "pdl": not args.no_pdl,
                "bytes_per_step": int(total_bytes),
            },
            "roofline": {
                "bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / pk["hbm_gbs"], 4),
                "traffic": traffic["bytes_per_step"] if traffic else None,
                "algorithmic_bytes": int(kind_bytes),
                "per": "step (all GEMV launches of one sweep; achieved = algorithmic bytes / summed "
                       "per-launch device time)",
                "peak_source": f"{src} hbm_gbs",
                "kernel": ("w4a16_gemv_kernel (decode GEMV, M<=8)" if args.m <= 8 else
                           "w4a16_gemv16_kernel (16-token decode GEMV, M 9-16)" if args.m <= 16 else
                           "w4a16_tc_kernel (tcgen05 GEMM)"),
                "per_layer": per_kind,
            },
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": e2e["h2d_bytes_per_step"],
                    "d2h_bytes_per_step": e2e["d2h_bytes_per_step"],
                    "ms_per_step": round(e2e["ms_per_step"], 4),
                    "host_matches_device": e2e["host_matches_device"],
                    "path": "tf_w4a16_linear C ABI calls with pinned H2D / D2H copies, the step "
                            "captured as one CUDA graph and replayed per step"},
            "parity": parity,
            **({"peer_trace": peer_trace} if peer_trace else {}),
            "chain": chain,
            "gpu_launches": sweep.launches_per_step * args.steps,
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
            "gemm": gemm,
            "block": block,
            **extra,
        }
        print(json.dumps(line), flush=True)
    del graph
    if not parity["ok"]:
        print(f"parity check failed: {json.dumps(parity)}", file=sys.stderr)
    if peers is not None:
        if peers.error():
            print("peer all-reduce: a wait timed out", file=sys.stderr)
        peers.close()
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if not parity["ok"]:
        sys.exit(3)


if __name__ == "__main__":
    main()
