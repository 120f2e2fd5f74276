"""M buckets and the fixed launch table (replaces tokenforge/kernels/config.py and autotune.py).

The reference picks a Triton launch config per ``(M bucket, N, K, G)`` from a persistent
autotune cache with a heuristic default (config.py:71-92, autotune.py:190-193). This backend has
no runtime tuning: the table and the K-split rule are compiled into the kernel library
(``csrc/capi.cu``) and are the same on every run, so there is no cache to load, validate or
corrupt. :func:`launch_plan` reads the table back for inspection and tests.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

from tokenforge_b200 import _lib

# The reference's buckets 1..128 (config.py:8) extended to the prefill sizes of the benchmark.
M_BUCKETS: tuple[int, ...] = (1, 2, 4, 8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096)
MAX_GEMV_M = 8
KERNEL_NAMES = {0: "gemv", 1: "mma_gemm", 2: "tcgen05_gemm"}


def m_bucket(m: int) -> int:
    """Smallest bucket >= m; M above the last bucket shares the last bucket's launch."""
    if m < 1:
        raise ValueError(f"M must be >= 1, got {m}")
    for b in M_BUCKETS:
        if m <= b:
            return b
    return M_BUCKETS[-1]


def bucket_label(m: int) -> str:
    return f">{M_BUCKETS[-1]}" if m > M_BUCKETS[-1] else str(m_bucket(m))


@dataclass(frozen=True)
class LaunchPlan:
    kernel: str
    m_bucket: int
    tile_n: int
    warps_k: int
    split_k: int
    tile_m: int
    grid_x: int
    grid_z: int
    cluster: int


def launch_plan(m: int, n: int, k: int, group_size: int) -> LaunchPlan:
    """The launch the kernel library will use for ``y[m, n] = x[m, k] W[n, k]^T``."""
    out = (ctypes.c_int32 * 9)()
    status = _lib.lib().tf_launch_plan(m, n, k, group_size, ctypes.addressof(out))
    if status != _lib.TF_OK:
        raise ValueError(
            f"no launch for M={m}, N={n}, K={k}, group_size={group_size}: "
            f"{_lib.status_string(status)}"
        )
    v = list(out)
    return LaunchPlan(KERNEL_NAMES[v[0]], v[1], v[2], v[3], v[4], v[5], v[6], v[7], v[8])


def workspace_bytes(m: int, n: int, k: int, group_size: int) -> int:
    return int(_lib.lib().tf_w4a16_workspace_bytes(m, n, k, group_size))
