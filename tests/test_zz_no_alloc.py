"""tn_q4_0_linear_noalloc -- the Q4_0 linear for callers that cannot allow a
device allocation while they run (a preplanned HBM arena, recording a CUDA
graph under global capture, a loop that cannot absorb cudaMalloc's implicit
synchronisation). It keeps its activation blocks in a fixed device array in
the library instead of the allocator and runs the decode GEMV, so up to 8 rows
its results must be the allocating entry point's bit for bit, call after call,
while the shared array is reused; from 9 rows the allocating entry point takes
the tensor-core kernel (another summation order), and both must lie within the
counted bound of the exact value.

Collected last (test_zz_*) so a failure here stops a `-x` run only after every
other test has run; it also passes alone in a fresh process.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle
from tests import q4_exact

pytestmark = pytest.mark.gpu

P = ctypes.c_void_p


@pytest.fixture(scope="module")
def lib(cuda_device):
    from torchnative_b200 import _native, build

    build.build()
    return _native


def _call(N, fn, x, w, y, M, Nout, K, bias=None):
    stream = P(torch.cuda.current_stream().cuda_stream)
    args = [P(x.data_ptr()), N.TN_F32, K, P(w.data_ptr()), None if bias is None else P(bias.data_ptr()),
            P(y.data_ptr()), N.TN_F32, M, Nout, K]
    if fn == "tn_q4_0_linear":
        args.append(N.TN_ACT_Q8_0)
    args.append(stream)
    N.check(getattr(N.lib(), fn)(*args))


@pytest.mark.parametrize("M,Nout,K", [(1, 4096, 4096), (8, 1000, 4096), (16, 1000, 4096), (3, 517, 14336),
                                       (5, 64, 576)])
def test_noalloc_matches_the_allocating_entry_point_twice_in_a_row(lib, cuda_device, M, Nout, K):
    rng = np.random.default_rng(M + Nout + K)
    blob = q4_exact.random_q4_0_blob(rng, Nout, K)
    w = torch.frombuffer(bytearray(blob), dtype=torch.uint8).to(cuda_device)
    for call in range(2):  # the second call reuses the shared array with new activations
        x_np = (rng.standard_normal((M, K)) * (1.0 + call)).astype(np.float32)
        x = torch.from_numpy(x_np).to(cuda_device)
        want = torch.empty((M, Nout), device=cuda_device)
        got = torch.full((M, Nout), float("nan"), device=cuda_device)
        _call(lib, "tn_q4_0_linear", x, w, want, M, Nout, K)
        _call(lib, "tn_q4_0_linear_noalloc", x, w, got, M, Nout, K)
        torch.cuda.synchronize()
        # up to 8 rows the same kernels on the same blocks: identical; always
        # inside the counted bound
        if M <= 8:
            assert torch.equal(got, want), f"call {call}: differs from tn_q4_0_linear"
        exact, abs_sum, ref_err = q4_exact.exact_linear_q4_0(oracle.q8_0_quantize(x_np), blob, M, Nout, K)
        bound = q4_exact.linear_bound(K, abs_sum, ref_err)
        assert float(np.max(np.abs(got.cpu().numpy().astype(np.float64) - exact) / bound)) <= 1.0
        assert float(np.max(np.abs(want.cpu().numpy().astype(np.float64) - exact) / bound)) <= 1.0
    lib.device_status(reset=True)


def test_noalloc_allocates_nothing_and_refuses_oversize(lib, cuda_device):
    rng = np.random.default_rng(3)
    K, Nout = 4096, 256
    blob = q4_exact.random_q4_0_blob(rng, Nout, K)
    w = torch.frombuffer(bytearray(blob), dtype=torch.uint8).to(cuda_device)
    x = torch.randn((2, K), device=cuda_device)
    y = torch.empty((2, Nout), device=cuda_device)
    _call(lib, "tn_q4_0_linear_noalloc", x, w, y, 2, Nout, K)  # first call on the device does the set-up
    torch.cuda.synchronize()
    before = lib.counters()["bytes_allocated"]
    free_before = torch.cuda.mem_get_info()[0]
    _call(lib, "tn_q4_0_linear_noalloc", x, w, y, 2, Nout, K)
    torch.cuda.synchronize()
    assert lib.counters()["bytes_allocated"] == before
    assert torch.cuda.mem_get_info()[0] == free_before
    big = torch.randn((17, K), device=cuda_device)
    with pytest.raises(RuntimeError, match="exceed its fixed scratch"):
        _call(lib, "tn_q4_0_linear_noalloc", big, w, torch.empty((17, Nout), device=cuda_device), 17, Nout, K)


def test_noalloc_refuses_zero_in_features_and_counts_its_calls(lib, cuda_device):
    """K == 0 is refused by name (as tn_q4_0_linear refuses it) instead of
    reaching the kernel planner, and every call counts as a Q4 linear call."""
    x = torch.zeros((1, 32), device=cuda_device)
    w = torch.zeros(8 * 18, dtype=torch.uint8, device=cuda_device)
    y = torch.zeros((1, 8), device=cuda_device)
    before = lib.counters()["q4_linear_calls"]
    stream = P(torch.cuda.current_stream().cuda_stream)
    st = lib.lib().tn_q4_0_linear_noalloc(P(x.data_ptr()), lib.TN_F32, 0, P(w.data_ptr()), None, P(y.data_ptr()),
                                          lib.TN_F32, 1, 8, 0, stream)
    assert st == lib.TN_ERR_NOT_IMPLEMENTED
    assert "in_features == 0" in lib.last_error()
    assert lib.counters()["q4_linear_calls"] == before + 1


def test_noalloc_at_its_limits_bf16_bias_and_strided_rows(lib, cuda_device):
    """The largest call the fixed array takes (16 rows of 16384), bf16 in and
    out, a float32 bias and a row stride wider than K: the decode GEMV then
    runs in row chunks at several offsets into the array. Checked twice in a
    row against the counted bound of the exact value (the bf16 output adds
    one rounding: half a bf16 ulp of the result)."""
    M, Nout, K, stride = 16, 300, 16384, 16384 + 64
    rng = np.random.default_rng(99)
    blob = q4_exact.random_q4_0_blob(rng, Nout, K)
    w = torch.frombuffer(bytearray(blob), dtype=torch.uint8).to(cuda_device)
    bias_np = rng.standard_normal(Nout).astype(np.float32)
    bias = torch.from_numpy(bias_np).to(cuda_device)
    stream = P(torch.cuda.current_stream().cuda_stream)
    for call in range(2):
        xs = torch.from_numpy((rng.standard_normal((M, stride)) * (1 + call)).astype(np.float32))
        xb = xs.to(torch.bfloat16).to(cuda_device)
        y = torch.full((M, Nout), float("nan"), device=cuda_device, dtype=torch.bfloat16)
        lib.check(lib.lib().tn_q4_0_linear_noalloc(P(xb.data_ptr()), lib.TN_BF16, stride, P(w.data_ptr()),
                                                   P(bias.data_ptr()), P(y.data_ptr()), lib.TN_BF16, M, Nout, K,
                                                   stream))
        torch.cuda.synchronize()
        x_np = xb[:, :K].float().cpu().numpy()
        exact, abs_sum, ref_err = q4_exact.exact_linear_q4_0(oracle.q8_0_quantize(x_np), blob, M, Nout, K)
        exact = exact + bias_np.astype(np.float64)
        bound = q4_exact.linear_bound(K, abs_sum + np.abs(bias_np), ref_err) + np.abs(exact) * 2.0 ** -8
        got = y.float().cpu().numpy().astype(np.float64)
        assert float(np.max(np.abs(got - exact) / bound)) <= 1.0, f"call {call}"
    lib.device_status(reset=True)
