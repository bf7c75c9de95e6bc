"""The batched-decode Q4_0 linear (9 to 32 activation rows: the tcgen05 kernel
with the weights on the MMA's 128-row side, split over K when the weight has
few 128-row tiles) against the exact value of the quantised operands and the
oracle, under the counted bound the decode GEMV and the prefill GEMM meet
(tests/numerics/test_q4ref.py:203-289 of the reference: K/32 + 3
accumulations), and bit-exact for lossless integer operands
(tests/numerics/test_qgemm.py:102-137 of the reference)."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle
from tests import q4_exact

pytestmark = pytest.mark.gpu

P = ctypes.c_void_p


@pytest.fixture(scope="module")
def tn(cuda_device):
    from torchnative_b200 import _native, build, quant

    build.build()
    _native.lib()
    return quant


SHAPES = [
    # (M, N, K)
    (9, 128, 256),      # the smallest row count that takes the kernel, one chunk (no split)
    (10, 200, 2048),    # ragged weight tile, K split
    (12, 4096, 4096),   # BASELINE o_proj: 32 tiles, many splits
    (16, 6144, 4096),   # BASELINE q/k/v at decode batch 16
    (16, 4096, 14336),  # BASELINE down_proj
    (17, 333, 4096),    # the 32-column variant, ragged everything
    (32, 1024, 4096),   # the largest row count
]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_skinny_within_counted_bound_and_near_oracle(tn, cuda_device, M, N, K):
    from torchnative_b200 import _native

    rng = np.random.default_rng(M * 7 + N * 3 + K + 1)
    blob = q4_exact.random_q4_0_blob(rng, N, K)
    x = (rng.standard_normal((M, K)) * 1.3).astype(np.float32)
    w = tn._quantized_from_blob(blob, (N, K), "q4_0", cuda_device)
    before = _native.counters()
    got = tn._quantized_linear(torch.from_numpy(x).to(cuda_device), w).cpu().numpy().astype(np.float64)
    after = _native.counters()
    assert after["q4_skinny_launches"] == before["q4_skinny_launches"] + 1
    assert after["q4_gemv_launches"] == before["q4_gemv_launches"]
    xq = oracle.q8_0_quantize(x)
    exact, abs_sum, ref_err = q4_exact.exact_linear_q4_0(xq, blob, M, N, K)
    bound = q4_exact.linear_bound(K, abs_sum, ref_err)
    worst = float(np.max(np.abs(got - exact) / bound))
    assert worst <= 1.0, f"|gpu - exact| reaches {worst:.3g}x the counted bound"
    if M * N * K <= 16 * 6144 * 4096:
        ref = oracle.q4_0_linear(x, blob, N, threads=8).astype(np.float64)
        assert float(np.max(np.abs(got - ref) / (2 * bound))) <= 1.0
    _native.device_status(reset=True)


@pytest.mark.parametrize("M", [9, 24])
def test_skinny_lossless_integer_operands_give_the_exact_integer_matmul(tn, cuda_device, M):
    rng = np.random.default_rng(80 + M)
    N, K = 260, 4096
    codes = rng.integers(-8, 8, size=(N, K))
    blob = q4_exact.q4_0_blob_from_codes(codes, np.ones((N, K // 32), dtype=np.float16))
    x = rng.integers(-127, 128, size=(M, K)).astype(np.float32)
    x[:, ::32] = 127.0
    w = tn._quantized_from_blob(blob, (N, K), "q4_0", cuda_device)
    y = tn._quantized_linear(torch.from_numpy(x).to(cuda_device), w).cpu().numpy().astype(np.float64)
    assert (y == x.astype(np.float64) @ codes.T.astype(np.float64)).all()


def test_skinny_bias_and_reduced_precision_outputs(tn, cuda_device):
    rng = np.random.default_rng(81)
    M, N, K = 12, 520, 4096
    blob = q4_exact.random_q4_0_blob(rng, N, K)
    w = tn._quantized_from_blob(blob, (N, K), "q4_0", cuda_device)
    x = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(cuda_device)
    b = torch.from_numpy(rng.standard_normal(N).astype(np.float32)).to(cuda_device)
    y0 = tn._quantized_linear(x, w)
    assert torch.equal(tn._quantized_linear(x, w, b), y0 + b)
    for dt in (torch.bfloat16, torch.float16):
        xd = x.to(dt)
        y = tn._quantized_linear(xd, w)
        assert y.dtype == dt
        assert torch.equal(y, tn._quantized_linear(xd.float(), w).to(dt))


def test_skinny_repeated_calls_are_identical(tn, cuda_device):
    """The split-K tickets reset themselves: the same call gives the same bits
    every time (the last CTA of a tile adds the partials in split order)."""
    rng = np.random.default_rng(82)
    M, N, K = 16, 4096, 4096
    blob = q4_exact.random_q4_0_blob(rng, N, K)
    w = tn._quantized_from_blob(blob, (N, K), "q4_0", cuda_device)
    x = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(cuda_device)
    y0 = tn._quantized_linear(x, w)
    for _ in range(5):
        assert torch.equal(tn._quantized_linear(x, w), y0)


@pytest.mark.parametrize("M,I,K", [(16, 1792, 4096), (11, 256, 512)])
def test_skinny_silu_mul_pair_epilogue(tn, cuda_device, M, I, K):
    """Interleaved (gate, up) rows with TN_EPILOGUE_SILU_MUL_PAIRS: column i of
    the bf16 output is bf16(bf16(silu(bf16(gate_i))) * bf16(up_i)) of the same
    kernel's f32 sums (within one bf16 rounding of torch's silu)."""
    from torchnative_b200 import _native as N

    rng = np.random.default_rng(83 + M)
    dev = cuda_device
    blob = torch.frombuffer(bytearray(q4_exact.random_q4_0_blob(rng, 2 * I, K)), dtype=torch.uint8).to(dev)
    x = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(dev)
    nb = K // 32
    codes = torch.empty((M, K), dtype=torch.int8, device=dev)
    sc, of = torch.empty((M, nb), device=dev), torch.empty((M, nb), device=dev)
    s = P(torch.cuda.current_stream().cuda_stream)
    N.check(N.lib().tn_q8_0_quantize_planar(P(x.data_ptr()), N.TN_F32, K, P(codes.data_ptr()), K,
                                            P(sc.data_ptr()), P(of.data_ptr()), M, K, s))
    y = torch.full((M, 2 * I), float("nan"), device=dev)
    act = torch.full((M, I), float("nan"), device=dev, dtype=torch.bfloat16)
    before = N.counters()
    N.check(N.lib().tn_q4_0_linear_q8(P(codes.data_ptr()), K, P(sc.data_ptr()), P(of.data_ptr()),
                                      P(blob.data_ptr()), None, P(y.data_ptr()), N.TN_F32, M, 2 * I, K, 0, s))
    N.check(N.lib().tn_q4_0_linear_q8(P(codes.data_ptr()), K, P(sc.data_ptr()), P(of.data_ptr()),
                                      P(blob.data_ptr()), None, P(act.data_ptr()), N.TN_BF16, M, 2 * I, K,
                                      N.TN_EPILOGUE_SILU_MUL_PAIRS, s))
    torch.cuda.synchronize()
    assert N.counters()["q4_skinny_launches"] == before["q4_skinny_launches"] + 2
    g, u = y[:, 0::2].to(torch.bfloat16), y[:, 1::2].to(torch.bfloat16)
    want = (torch.nn.functional.silu(g.float()).to(torch.bfloat16).float() * u.float()).to(torch.bfloat16)
    diff = (act.float() - want.float()).abs()
    assert bool((diff <= want.float().abs() * 2.0 ** -7 + 1e-30).all()), float(diff.max())
    N.device_status(reset=True)


def test_eight_rows_still_take_the_decode_gemv(tn, cuda_device):
    from torchnative_b200 import _native

    rng = np.random.default_rng(84)
    N, K = 256, 4096
    blob = q4_exact.random_q4_0_blob(rng, N, K)
    w = tn._quantized_from_blob(blob, (N, K), "q4_0", cuda_device)
    before = _native.counters()
    tn._quantized_linear(torch.randn(8, K, device=cuda_device), w)
    after = _native.counters()
    assert after["q4_skinny_launches"] == before["q4_skinny_launches"]
    assert after["q4_gemv_launches"] == before["q4_gemv_launches"] + 1
