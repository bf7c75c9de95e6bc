"""The runtime surface of the C ABI on a GPU: the caching allocator (the
replacement for candle's per-tensor cudarc allocation,
vendor/candle-core/src/cuda_backend/device.rs:78-90), the per-device current
stream (candle's one CudaStream per device, device.rs:388-389) and the
counters that mirror the reference's `_C._cuda_counters()`
(torch_c/src/device.rs:1671-1700)."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle
from tests import q4_exact

pytestmark = pytest.mark.gpu
P = ctypes.c_void_p


@pytest.fixture(scope="module")
def N(cuda_device):
    from torchnative_b200 import _native, build

    build.build()
    _native.lib()
    return _native


def _stats(N):
    a, r = ctypes.c_size_t(), ctypes.c_size_t()
    N.check(N.lib().tn_memory_stats(ctypes.byref(a), ctypes.byref(r)))
    return a.value, r.value


def test_allocator_reuses_a_rounded_size_per_stream_and_empty_cache_releases(N, cuda_device):
    L = N.lib()
    N.check(L.tn_empty_cache())
    s1 = torch.cuda.Stream()
    s2 = torch.cuda.Stream()
    a0, r0 = _stats(N)
    p = ctypes.c_void_p()
    N.check(L.tn_alloc(ctypes.byref(p), 1000, P(s1.cuda_stream)))
    first = p.value
    a1, r1 = _stats(N)
    assert a1 - a0 == 1024 and r1 - r0 == 1024  # rounded up to 512-byte multiples
    # the block holds data the device can write and read
    N.check(L.tn_free(p, P(s1.cuda_stream)))
    assert _stats(N) == (a0, r1)  # freed: no longer allocated, still reserved
    # a request of the same rounded size on the same stream gets the block back
    q = ctypes.c_void_p()
    N.check(L.tn_alloc(ctypes.byref(q), 900, P(s1.cuda_stream)))
    assert q.value == first and _stats(N) == (a1, r1)
    N.check(L.tn_free(q, P(s1.cuda_stream)))
    # on another stream it does not (stream-ordered reuse only)
    r_ = ctypes.c_void_p()
    N.check(L.tn_alloc(ctypes.byref(r_), 1000, P(s2.cuda_stream)))
    assert r_.value != first
    N.check(L.tn_free(r_, P(s2.cuda_stream)))
    # large sizes round to 2 MB
    big = ctypes.c_void_p()
    N.check(L.tn_alloc(ctypes.byref(big), (3 << 20) + 5, P(s1.cuda_stream)))
    assert _stats(N)[0] - a0 == 4 << 20
    N.check(L.tn_free(big, P(s1.cuda_stream)))
    free_before = torch.cuda.mem_get_info()[0]
    N.check(L.tn_empty_cache())
    a2, r2 = _stats(N)
    assert a2 == a0 and r2 == r0
    assert torch.cuda.mem_get_info()[0] >= free_before + (4 << 20)
    # a pointer the allocator does not own is refused
    with pytest.raises(RuntimeError, match="not allocated by tn_alloc"):
        N.check(L.tn_free(P(12345), None))


def test_null_stream_calls_run_on_the_devices_current_stream(N, cuda_device):
    from torchnative_b200 import quant

    L = N.lib()
    dev = cuda_device.index or 0
    side = torch.cuda.Stream()
    got = ctypes.c_void_p()
    N.check(L.tn_stream_get(dev, ctypes.byref(got)))
    assert got.value is None
    N.check(L.tn_stream_set(dev, P(side.cuda_stream)))
    try:
        N.check(L.tn_stream_get(dev, ctypes.byref(got)))
        assert got.value == side.cuda_stream
        rng = np.random.default_rng(4)
        blob = q4_exact.random_q4_0_blob(rng, 384, 1024)
        w = quant._quantized_from_blob(blob, (384, 1024), "q4_0", cuda_device)
        x_np = rng.standard_normal((3, 1024)).astype(np.float32)
        x = torch.from_numpy(x_np).to(cuda_device)
        y = torch.zeros((3, 384), device=cuda_device)
        side.wait_stream(torch.cuda.current_stream())
        # stream NULL: the call runs on `side`
        N.check(L.tn_q4_0_linear(P(x.data_ptr()), N.TN_F32, 1024, P(w.blob.data_ptr()), None, P(y.data_ptr()),
                                 N.TN_F32, 3, 384, 1024, N.TN_ACT_Q8_0, None))
        side.synchronize()
        exact, abs_sum, ref_err = q4_exact.exact_linear_q4_0(oracle.q8_0_quantize(x_np), blob, 3, 384, 1024)
        bound = q4_exact.linear_bound(1024, abs_sum, ref_err)
        assert float(np.max(np.abs(y.cpu().numpy().astype(np.float64) - exact) / bound)) <= 1.0
    finally:
        N.check(L.tn_stream_set(dev, None))
    with pytest.raises(RuntimeError, match="bad device index"):
        N.check(L.tn_stream_set(-1, None))
    N.device_status(reset=True)


def test_cuda_counters_have_the_reference_shape(N, cuda_device):
    from torchnative_b200 import quant

    before = N.cuda_counters()
    for key in ("resolves", "dispatches", "readback_refusals", "refusals", "ops", "device_free_bytes",
                "device_total_bytes"):
        assert key in before
    assert before["resolves"] >= 1 and before["device_total_bytes"] > 0
    with pytest.raises(NotImplementedError):
        quant._quantize(torch.zeros(4, 33, device=cuda_device), "q4_0")
    w = quant._quantize(torch.randn(64, 64, device=cuda_device), "q4_0")
    quant._quantized_linear(torch.randn(2, 64, device=cuda_device), w)
    after = N.cuda_counters()
    assert after["dispatches"] >= before["dispatches"] + 2
    with pytest.raises(NotImplementedError):
        N.check(N.lib().tn_q4_0_linear(None, N.TN_F64, 64, None, None, None, N.TN_F32, 1, 8, 64, 0, None))
    assert N.cuda_counters()["refusals"] >= before["refusals"] + 1
    N.device_status(reset=True)
