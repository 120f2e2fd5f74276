"""Kernel-path counters, same names and labels as the reference (tokenforge/kernels/metrics.py).

``tokenforge_kernel_calls_total{kernel,bucket}`` counts dispatch decisions per kernel and M
bucket (kernel labels here: ``cuda_gemv``, ``cuda_gemm``); ``tokenforge_fallback_total{reason}``
counts layers or calls routed away from the requested path. Counting happens on the host at
dispatch time, so a call captured in a CUDA graph is counted once, when it is captured.
When ``prometheus_client`` is importable every increment is mirrored into it.
"""

from __future__ import annotations

import threading
from typing import Any


class LabeledCounter:
    """A monotonically increasing counter keyed by a fixed tuple of label names."""

    def __init__(self, name: str, documentation: str, labelnames: tuple[str, ...]) -> None:
        self.name = name
        self.labelnames = labelnames
        self._counts: dict[tuple[str, ...], float] = {}
        self._lock = threading.Lock()
        self._prom = _prometheus_counter(name, documentation, labelnames)

    def _labels(self, labels: dict[str, str]) -> tuple[str, ...]:
        if sorted(labels) != sorted(self.labelnames):
            raise ValueError(f"{self.name} expects labels {self.labelnames}, got {sorted(labels)}")
        return tuple(str(labels[name]) for name in self.labelnames)

    def inc(self, amount: float = 1.0, **labels: str) -> None:
        key = self._labels(labels)
        with self._lock:
            self._counts[key] = self._counts.get(key, 0.0) + amount
        if self._prom is not None:
            self._prom.labels(*key).inc(amount)

    def value(self, **labels: str) -> float:
        key = self._labels(labels)
        with self._lock:
            return self._counts.get(key, 0.0)

    def total(self) -> float:
        with self._lock:
            return float(sum(self._counts.values()))

    def snapshot(self) -> dict[tuple[str, ...], float]:
        with self._lock:
            return dict(self._counts)

    def reset(self) -> None:
        """Forget the in-process counts (tests); exported Prometheus series stay monotonic."""
        with self._lock:
            self._counts.clear()


def _prometheus_counter(name: str, documentation: str, labelnames: tuple[str, ...]) -> Any:
    try:
        import prometheus_client
    except ImportError:
        return None
    try:
        return prometheus_client.Counter(name, documentation, labelnames)
    except ValueError:  # registered by an earlier import of this module
        return prometheus_client.REGISTRY._names_to_collectors.get(name)


KERNEL_CALLS = LabeledCounter(
    "tokenforge_kernel_calls",
    "TokenForge kernel dispatches by kernel and M bucket",
    ("kernel", "bucket"),
)
FALLBACKS = LabeledCounter(
    "tokenforge_fallback",
    "TokenForge fallbacks away from the requested kernel path, by reason",
    ("reason",),
)
