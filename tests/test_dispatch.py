"""Host-side dispatch, counters and the CPU contract (no fallback), mirroring the reference's
tests/unit/test_dispatch.py for this backend's routing."""

from __future__ import annotations

import pytest
import torch
from hypothesis import given
from hypothesis import strategies as st

from tokenforge_b200 import dispatch
from tokenforge_b200.config import M_BUCKETS, m_bucket
from tokenforge_b200.metrics import FALLBACKS, KERNEL_CALLS, CounterMetric


@given(st.integers(1, 4096))
def test_m_bucket_is_tight(m: int) -> None:
    b = m_bucket(m)
    assert b in M_BUCKETS
    assert b >= m
    assert b == 1 or b // 2 < m


def test_m_bucket_rejects_zero() -> None:
    with pytest.raises(ValueError, match=">= 1"):
        m_bucket(0)


@pytest.mark.parametrize(
    ("n", "k", "group", "dtype", "sm", "backend", "expected"),
    [
        (1152, 896, 128, "float16", 100, "cuda", None),
        (1152, 896, 128, "torch.float16", None, "triton", None),
        (1152, 896 + 64, 128, "float16", 100, "cuda", "unsupported_shape"),
        (1150, 896, 128, "float16", 100, "cuda", "unsupported_shape"),
        (1152, 896, 256, "float16", 100, "cuda", "unsupported_group_size"),
        (1152, 896, 128, "bfloat16", 100, "cuda", "unsupported_dtype"),
        (1152, 896, 128, "float16", 90, "cuda", "unsupported_arch"),
        (1152, 896, 128, "float16", 100, "marlin", "kill_switch"),
    ],
)
def test_layer_support(n, k, group, dtype, sm, backend, expected) -> None:  # type: ignore[no-untyped-def]
    assert dispatch.layer_support(n, k, group, dtype, sm, backend) == expected


@pytest.mark.parametrize(
    ("m", "backend", "kernel", "bucket"),
    [
        (1, "cuda", "cuda_gemv", "1"),
        (3, "cuda", "cuda_gemv", "4"),
        (8, "triton", "cuda_gemv", "8"),
        (9, "cuda", "cuda_gemm", "16"),
        (129, "cuda", "cuda_gemm", "256"),
        (4096, "triton", "cuda_gemm", "4096"),
        (5000, "cuda", "cuda_gemm", ">4096"),
    ],
)
def test_select(m, backend, kernel, bucket) -> None:  # type: ignore[no-untyped-def]
    d = dispatch.select(m, backend=backend, on_gpu=True, cuda_ext_available=True)
    assert (d.kernel, d.bucket, d.fallback) == (kernel, bucket, None)


def test_select_has_no_cpu_fallback() -> None:
    with pytest.raises(dispatch.BackendUnavailableError, match="CUDA"):
        dispatch.select(1, backend="cuda", on_gpu=False, cuda_ext_available=True)
    with pytest.raises(dispatch.BackendUnavailableError, match="library"):
        dispatch.select(1, backend="cuda", on_gpu=True, cuda_ext_available=False)


def test_select_rejects_marlin_per_call() -> None:
    with pytest.raises(ValueError, match="per layer"):
        dispatch.select(1, backend="marlin", on_gpu=True, cuda_ext_available=True)


def test_record_counts_calls_and_fallbacks() -> None:
    d = dispatch.select(2, backend="cuda", on_gpu=True, cuda_ext_available=True)
    dispatch.record(d)
    dispatch.record(d)
    assert KERNEL_CALLS.value(kernel="cuda_gemv", bucket="2") == 2
    dispatch.record_layer_fallback("unsupported_shape")
    assert FALLBACKS.value(reason="unsupported_shape") == 1
    assert FALLBACKS.total() == 1


def test_counter_rejects_wrong_labels() -> None:
    c = CounterMetric("tf_test_counter_x", "doc", ("a",))
    with pytest.raises(ValueError, match="takes labels"):
        c.inc(b="1")
    with pytest.raises(ValueError, match="only increases"):
        c.inc(a="1", amount=-1.0)
    c.inc(a="1", amount=2.0)
    assert c.value(a="1") == 2.0
    assert c.snapshot() == {("1",): 2.0}


def test_counters_export_through_prometheus() -> None:
    prometheus_client = pytest.importorskip("prometheus_client")
    KERNEL_CALLS.inc(kernel="cuda_gemv", bucket="1")
    KERNEL_CALLS.inc(kernel="cuda_gemv", bucket="1")
    text = prometheus_client.generate_latest().decode()
    assert 'tokenforge_kernel_calls_total{bucket="1",kernel="cuda_gemv"} 2.0' in text
    assert "# TYPE tokenforge_fallback_total counter" in text or "tokenforge_fallback" in text


def test_backend_from_env(monkeypatch: pytest.MonkeyPatch) -> None:
    monkeypatch.delenv(dispatch.BACKEND_ENV, raising=False)
    assert dispatch.backend_from_env() == "cuda"
    monkeypatch.setenv(dispatch.BACKEND_ENV, " Marlin ")
    assert dispatch.backend_from_env() == "marlin"
    monkeypatch.setenv(dispatch.BACKEND_ENV, "cublas")
    with pytest.raises(ValueError, match="TOKENFORGE_BACKEND"):
        dispatch.backend_from_env()
    monkeypatch.setenv(dispatch.BACKEND_ENV, "triton")
    with pytest.raises(ValueError, match="no Triton path"):
        dispatch.backend_from_env()


def test_op_on_cpu_tensors_raises_instead_of_falling_back() -> None:
    import tokenforge_b200.ops  # noqa: F401
    from tests.numerics import cases

    w = cases.layer_weights(64, 256, 0)
    x = cases.activations(2, 256, 0)
    with pytest.raises(dispatch.BackendUnavailableError):
        torch.ops.tokenforge.w4a16_linear(x, w.qweight_t, w.scales, w.qzeros, None, 128, "cuda")
    with pytest.raises(RuntimeError, match="CUDA"):
        torch.ops.tokenforge.awq_repack(torch.zeros((16, 2), dtype=torch.int32))
    with pytest.raises(RuntimeError, match="CUDA"):
        torch.ops.tokenforge.rmsnorm_fp8_quant(x, torch.ones(256, dtype=torch.float16), 1e-6, None)


def test_error_messages_match_the_reference_contract() -> None:
    from tests.numerics import cases
    from tokenforge_b200.ops import w4a16_gemm

    w = cases.layer_weights(64, 256, 0)
    x = cases.activations(1, 256, 0)
    with pytest.raises(ValueError, match="contiguous"):
        w4a16_gemm(x, w.qweight_t.t().contiguous().t(), w.scales, w.qzeros, 128)
    with pytest.raises(ValueError, match="encodes K"):
        w4a16_gemm(x[:, :128], w.qweight_t, w.scales, w.qzeros, 128)
    with pytest.raises(TypeError, match="fp16"):
        w4a16_gemm(x.float(), w.qweight_t, w.scales, w.qzeros, 128)
    with pytest.raises(ValueError, match="divide"):
        w4a16_gemm(x, w.qweight_t, w.scales, w.qzeros, 256)
    with pytest.raises(ValueError, match="2-D"):
        w4a16_gemm(x.reshape(-1), w.qweight_t, w.scales, w.qzeros, 128)


def test_rejects_marlin_at_op_level() -> None:
    import tokenforge_b200.ops  # noqa: F401
    from tests.numerics import cases

    w = cases.layer_weights(64, 256, 0)
    with pytest.raises(ValueError, match="op level"):
        torch.ops.tokenforge.w4a16_linear(cases.activations(1, 256, 0), w.qweight_t, w.scales,
                                          w.qzeros, None, 128, "marlin")


def test_fake_tensor_shapes() -> None:
    import tokenforge_b200.ops  # noqa: F401
    from torch._subclasses.fake_tensor import FakeTensorMode

    from tests.numerics import cases

    w = cases.layer_weights(64, 256, 0)
    with FakeTensorMode() as mode:
        x = mode.from_tensor(cases.activations(2, 256, 0)).reshape(1, 2, 256)
        out = torch.ops.tokenforge.w4a16_linear(x, mode.from_tensor(w.qweight_t),
                                                mode.from_tensor(w.scales),
                                                mode.from_tensor(w.qzeros), None, 128, "cuda")
        assert out.shape == (1, 2, 64)
        assert out.dtype == torch.float16
        q, s = torch.ops.tokenforge.rmsnorm_fp8_quant(
            mode.from_tensor(torch.zeros((2, 3, 128), dtype=torch.float16)),
            mode.from_tensor(torch.ones(128, dtype=torch.float16)), 1e-6, None)
        assert q.shape == (2, 3, 128) and q.dtype == torch.float8_e4m3fn
        assert s.shape == (2, 3, 1)
        r = torch.ops.tokenforge.awq_repack(mode.from_tensor(torch.zeros((256, 8), dtype=torch.int32)))
        assert r.shape == (64, 32)
