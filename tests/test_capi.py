"""The C ABI surface of the kernel library, checked without a GPU: the shared object loads,
exports every function ``include/tokenforge_b200.h`` declares, and its host-only entry points
(status strings, launch planning, argument validation) behave as documented."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from tokenforge_b200 import _lib
from tokenforge_b200.config import launch_plan, m_bucket, workspace_bytes

HEADER = Path(__file__).resolve().parent.parent / "include" / "tokenforge_b200.h"


def _declared() -> list[str]:
    return re.findall(r"^TF_API [\w\s\*]+?\b(tf_\w+)\(", HEADER.read_text(), flags=re.M)


def test_header_declares_the_boundary() -> None:
    names = set(_declared())
    for required in ("tf_awq_repack", "tf_w4a16_dequant", "tf_w4a16_gemv", "tf_w4a16_gemm",
                     "tf_w4a16_linear", "tf_rmsnorm_fp8_quant", "tf_launch_plan"):
        assert required in names


def test_library_exports_every_declared_symbol() -> None:
    lib = _lib.lib()
    for name in _declared():
        assert hasattr(lib, name), name
    assert set(_declared()) <= set(_lib.SIGNATURES)


def test_status_strings_and_version() -> None:
    assert _lib.status_string(0) == "ok"
    assert "aligned" in _lib.status_string(_lib.TF_ERR_ALIGNMENT)
    assert _lib.status_string(999) == "unknown status"
    assert _lib.lib().tf_abi_version() == 1


def test_launch_flags_roundtrip() -> None:
    old = _lib.get_launch_flags()
    try:
        _lib.set_launch_flags(_lib.TF_LAUNCH_PDL)
        assert _lib.get_launch_flags() == _lib.TF_LAUNCH_PDL
    finally:
        _lib.set_launch_flags(old)


@pytest.mark.parametrize("m", [1, 2, 3, 4, 5, 8])
def test_decode_sizes_use_the_gemv(m: int) -> None:
    plan = launch_plan(m, 4608, 3584, 128)
    assert plan.kernel == "gemv"
    assert plan.m_bucket == m_bucket(m)
    assert plan.tile_m == 8


@pytest.mark.parametrize("m", [17, 32, 64, 129, 1024, 4096, 5000])
def test_prefill_sizes_use_a_gemm(m: int) -> None:
    plan = launch_plan(m, 37888, 3584, 128)
    assert plan.kernel in ("tcgen05_gemm", "mma_gemm")


@pytest.mark.parametrize("m", [9, 12, 16])
def test_batched_decode_uses_the_16_token_gemv(m: int) -> None:
    """M = 9..16 with group size 128: the GEMV with two 8-token n-tiles (8-warp CTAs, two per
    SM, activations at most 96 KB per CTA); other group sizes take a GEMM."""
    for n, k in [(4608, 3584), (3584, 3584), (37888, 3584), (3584, 18944)]:
        plan = launch_plan(m, n, k, 128)
        assert plan.kernel == "gemv" and plan.tile_m == 16 and plan.m_bucket == 16
        assert plan.warps_k in (1, 2, 4, 8)  # no 16-warp CTA at 16 tokens
        per_split = -(-(-(-k // 128)) // plan.split_k)
        assert 2 * m * (per_split * 128 + 8) <= 96 * 1024
    assert launch_plan(m, 4608, 3584, 64).kernel in ("tcgen05_gemm", "mma_gemm")


@pytest.mark.parametrize(("n", "k"), [(4608, 3584), (3584, 3584), (37888, 3584), (3584, 18944),
                                      (200, 256), (1000, 1024), (896, 4864), (1152, 896)])
def test_plan_covers_every_k_block_once(n: int, k: int) -> None:
    plan = launch_plan(1, n, k, 128)
    assert plan.kernel == "gemv"
    kblocks = -(-k // 128)  # the decode GEMV walks 128-wide K blocks
    assert plan.warps_k in (1, 2, 4, 8, 16)
    assert plan.cluster in (1, 2, 4, 8) and plan.split_k % plan.cluster == 0
    if plan.warps_k == 16:  # one 16-warp CTA per row tile, no cluster
        assert plan.cluster == 1 and plan.split_k == 1
    warps_n = 1 if plan.warps_k == 16 else 8 // plan.warps_k
    assert plan.grid_x * warps_n * 32 >= n
    per = -(-kblocks // plan.split_k)
    assert (plan.split_k - 1) * per < kblocks <= plan.split_k * per  # no empty split
    outer = plan.split_k // plan.cluster
    ws = workspace_bytes(1, n, k, 128)
    assert ws >= (outer * n * 4 if outer > 1 else 0)


def test_decode_plan_fills_the_gpu_without_a_reduce_launch() -> None:
    for n, k in [(4608, 3584), (3584, 3584), (37888, 3584), (3584, 18944)]:
        plan = launch_plan(1, n, k, 128)
        # Warps on the GPU: 16 per SM at most (two 8-warp CTAs or one 16-warp CTA per SM),
        # at least half of that.
        warps = plan.grid_x * plan.split_k * (16 if plan.warps_k == 16 else 8)
        assert 148 * 16 // 2 <= warps <= 148 * 16, (n, k, plan)
        if plan.warps_k == 16:
            assert plan.grid_x <= 148  # one wave of one-per-SM CTAs
        assert plan.split_k == plan.cluster  # any K split is reduced inside the CTA or cluster


@pytest.mark.parametrize(("m", "n", "k"), [(1024, 3584, 18944), (64, 3584, 18944), (32, 37888, 3584)])
def test_tensor_core_plan_splits_k_to_fill_the_gpu(m: int, n: int, k: int) -> None:
    plan = launch_plan(m, n, k, 128)
    assert plan.kernel == "tcgen05_gemm"
    base = plan.grid_x * plan.grid_z
    units = base * plan.split_k
    # Splitting K must not make the busiest persistent CTA's share of the work larger.
    assert -(-units // 148) / plan.split_k <= -(-base // 148)
    assert workspace_bytes(m, n, k, 128) >= (plan.split_k * m * n * 4 if plan.split_k > 1 else 0)


def test_plan_is_deterministic() -> None:
    assert launch_plan(3, 37888, 3584, 128) == launch_plan(3, 37888, 3584, 128)


def test_plan_rejects_bad_shapes() -> None:
    with pytest.raises(ValueError, match="no launch"):
        launch_plan(1, 4608, 3584, 256)
    with pytest.raises(ValueError, match="no launch"):
        launch_plan(1, 4604, 3584, 128)
    with pytest.raises(ValueError, match="no launch"):
        launch_plan(0, 4608, 3584, 128)


def test_entry_points_validate_before_touching_the_device() -> None:
    lib = _lib.lib()
    # Invalid group size / shapes are rejected on the host with no launch.
    st = lib.tf_w4a16_linear(None, 1, 3584, 3584, None, None, None, None, 4608, 96, None, 4608,
                             None, 0, None)
    assert st == _lib.TF_ERR_INVALID_ARG
    st = lib.tf_w4a16_gemv(None, 1, 3584, 3584, None, None, None, None, 4604, 128, None, 4604,
                           None, 0, None)
    assert st == _lib.TF_ERR_INVALID_ARG
    # M == 0 is a no-op.
    st = lib.tf_w4a16_linear(None, 0, 3584, 3584, None, None, None, None, 4608, 128, None, 4608,
                             None, 0, None)
    assert st == _lib.TF_OK
    # Misaligned activations are refused (the Python layer copies them first).
    st = lib.tf_w4a16_linear(2, 1, 256, 256, 16, 16, 16, None, 64, 128, 16, 64, None, 0, None)
    assert st == _lib.TF_ERR_ALIGNMENT
    # A split-K launch without its workspace is refused.
    plan = launch_plan(8, 65536, 65536, 128)
    assert plan.split_k // plan.cluster > 1  # splits beyond one cluster need the workspace
    st = lib.tf_w4a16_linear(16, 8, 65536, 65536, 16, 16, 16, None, 65536, 128, 16, 65536, None, 0,
                             None)
    assert st == _lib.TF_ERR_WORKSPACE
    st = lib.tf_awq_repack(None, 12, 8, None, None)
    assert st == _lib.TF_ERR_INVALID_ARG
    st = lib.tf_rmsnorm_fp8_quant(None, 0, 896, 896, None, ctypes.c_float(1e-6), None, None, None, None)
    assert st == _lib.TF_OK
    st = lib.tf_w4a16_dequant(None, None, None, 64, 256, 48, None, None)
    assert st == _lib.TF_ERR_INVALID_ARG
