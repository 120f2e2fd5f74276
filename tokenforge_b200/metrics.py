"""Dispatch counters of the CUDA backend, exported under the reference's metric names.

The names and label sets are the reference's contract (tokenforge/kernels/metrics.py:67-76):
``tokenforge_kernel_calls_total{kernel,bucket}`` counts dispatch decisions (kernel labels here:
``cuda_gemv``, ``cuda_gemm``) and ``tokenforge_fallback_total{reason}`` counts layers or calls
routed away from the requested path. Counting happens on the host when a call is dispatched,
so a call captured in a CUDA graph counts once, at capture.

Every counter writes into one process-wide tally, a ``collections.Counter`` per metric behind
a single lock. Nothing is mirrored per increment: when ``prometheus_client`` is importable, one
collector registered with its default registry reads the tally at scrape time and reports each
metric as a counter family.
"""

from __future__ import annotations

import collections
import threading
from collections.abc import Iterator
from typing import Any

_LOCK = threading.Lock()
_TALLY: dict[str, collections.Counter[tuple[str, ...]]] = {}
_DECLARED: dict[str, CounterMetric] = {}


class CounterMetric:
    """Handle on one metric of the tally: a name, a help text and its ordered label names."""

    def __init__(self, name: str, documentation: str, labelnames: tuple[str, ...]) -> None:
        self.name = name
        self.documentation = documentation
        self.labelnames = tuple(labelnames)
        with _LOCK:
            _TALLY.setdefault(name, collections.Counter())
            _DECLARED[name] = self

    def _series(self, labels: dict[str, Any]) -> tuple[str, ...]:
        missing = set(self.labelnames) - labels.keys()
        extra = labels.keys() - set(self.labelnames)
        if missing or extra:
            raise ValueError(f"metric {self.name} takes labels {self.labelnames}; "
                             f"missing {sorted(missing)}, unknown {sorted(extra)}")
        return tuple(str(labels[k]) for k in self.labelnames)

    def inc(self, amount: float = 1.0, **labels: Any) -> None:
        if amount < 0:
            raise ValueError(f"metric {self.name} only increases (amount {amount})")
        series = self._series(labels)
        with _LOCK:
            _TALLY[self.name][series] += amount

    def value(self, **labels: Any) -> float:
        series = self._series(labels)
        with _LOCK:
            return float(_TALLY[self.name].get(series, 0.0))

    def total(self) -> float:
        with _LOCK:
            return float(sum(_TALLY[self.name].values()))

    def snapshot(self) -> dict[tuple[str, ...], float]:
        with _LOCK:
            return {k: float(v) for k, v in _TALLY[self.name].items()}

    def reset(self) -> None:
        """Zero this metric (tests). A scrape afterwards sees the counter restart, as after a
        process restart."""
        with _LOCK:
            _TALLY[self.name].clear()


class _TallyCollector:
    """``prometheus_client`` custom collector over the tally (read at scrape time)."""

    def collect(self) -> Iterator[Any]:
        from prometheus_client.core import CounterMetricFamily

        with _LOCK:
            rows = [(m, dict(_TALLY[m.name])) for m in _DECLARED.values()]
        for metric, series in rows:
            family = CounterMetricFamily(metric.name, metric.documentation,
                                         labels=list(metric.labelnames))
            for key, v in sorted(series.items()):
                family.add_metric(list(key), float(v))
            yield family


def _export_once() -> None:
    try:
        from prometheus_client import REGISTRY
    except ImportError:
        return
    if getattr(REGISTRY, "_tokenforge_b200_tally", False):
        return
    try:
        REGISTRY.register(_TallyCollector())
    except ValueError:  # the same series names were registered by another exporter
        return
    REGISTRY._tokenforge_b200_tally = True  # type: ignore[attr-defined]


KERNEL_CALLS = CounterMetric(
    "tokenforge_kernel_calls",
    "TokenForge kernel dispatches by kernel and M bucket",
    ("kernel", "bucket"),
)
FALLBACKS = CounterMetric(
    "tokenforge_fallback",
    "TokenForge fallbacks away from the requested kernel path, by reason",
    ("reason",),
)
_export_once()
