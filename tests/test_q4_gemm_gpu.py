"""The prefill Q4_0 linear (many activation rows: the tcgen05 GEMM) against the
exact value of the quantised operands and the oracle, under the same counted
bound as the decode GEMV (tests/numerics/test_q4ref.py:203-289 of the
reference: K = K_in/32 + 3 accumulations), and bit-exact for lossless integer
operands (tests/numerics/test_qgemm.py:102-137 of the reference)."""

import numpy as np
import pytest
import torch

from oracle import oracle
from tests import q4_exact

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tn(cuda_device):
    from torchnative_b200 import _native, build, quant

    build.build()
    _native.lib()
    return quant


GEMM_SHAPES = [
    # (M, N, K)
    (48, 128, 256),     # one 256-wide chunk, the smallest M that takes the GEMM
    (130, 200, 2048),   # ragged M and N tiles
    (256, 384, 4096),   # BASELINE K
    (64, 96, 14336),    # BASELINE down-projection K, N below one tile
    (2048, 128, 4096),  # BASELINE prefill M
]


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
def test_gemm_within_counted_bound_and_near_oracle(tn, cuda_device, M, N, K):
    from torchnative_b200 import _native

    rng = np.random.default_rng(M * 7 + N * 3 + K)
    blob = q4_exact.random_q4_0_blob(rng, N, K)
    x = (rng.standard_normal((M, K)) * 1.3).astype(np.float32)
    w = tn._quantized_from_blob(blob, (N, K), "q4_0", cuda_device)
    before = _native.counters()
    got = tn._quantized_linear(torch.from_numpy(x).to(cuda_device), w).cpu().numpy().astype(np.float64)
    after = _native.counters()
    assert after["q4_gemm_launches"] == before["q4_gemm_launches"] + 1
    assert after["q4_gemv_launches"] == before["q4_gemv_launches"]
    xq = oracle.q8_0_quantize(x)
    exact, abs_sum, ref_err = q4_exact.exact_linear_q4_0(xq, blob, M, N, K)
    bound = q4_exact.linear_bound(K, abs_sum, ref_err)
    worst = float(np.max(np.abs(got - exact) / bound))
    assert worst <= 1.0, f"|gpu - exact| reaches {worst:.3g}x the counted bound"
    if M * N * K <= 256 * 384 * 4096:
        ref = oracle.q4_0_linear(x, blob, N, threads=8).astype(np.float64)
        assert float(np.max(np.abs(got - ref) / (2 * bound))) <= 1.0
    _native.device_status(reset=True)


def test_gemm_lossless_integer_operands_give_the_exact_integer_matmul(tn, cuda_device):
    rng = np.random.default_rng(70)
    M, N, K = 200, 130, 4096
    codes = rng.integers(-8, 8, size=(N, K))
    blob = q4_exact.q4_0_blob_from_codes(codes, np.ones((N, K // 32), dtype=np.float16))
    x = rng.integers(-127, 128, size=(M, K)).astype(np.float32)
    x[:, ::32] = 127.0
    w = tn._quantized_from_blob(blob, (N, K), "q4_0", cuda_device)
    y = tn._quantized_linear(torch.from_numpy(x).to(cuda_device), w).cpu().numpy().astype(np.float64)
    assert (y == x.astype(np.float64) @ codes.T.astype(np.float64)).all()


def test_gemm_bias_and_reduced_precision_outputs(tn, cuda_device):
    rng = np.random.default_rng(71)
    M, N, K = 96, 264, 4096
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


def test_gemm_matches_row_chunks_of_the_decode_gemv(tn, cuda_device):
    """The same rows through the GEMV (16 at a time) and the GEMM agree within
    the bound of both (they round differently: one FMA per block each, in a
    different association)."""
    rng = np.random.default_rng(72)
    M, N, K = 64, 512, 4096
    blob = q4_exact.random_q4_0_blob(rng, N, K)
    w = tn._quantized_from_blob(blob, (N, K), "q4_0", cuda_device)
    x = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(cuda_device)
    y = tn._quantized_linear(x, w)
    ys = torch.cat([tn._quantized_linear(x[i:i + 16], w) for i in range(0, M, 16)])
    xq = oracle.q8_0_quantize(x.cpu().numpy())
    _, abs_sum, ref_err = q4_exact.exact_linear_q4_0(xq, blob, M, N, K)
    bound = torch.from_numpy(2 * q4_exact.linear_bound(K, abs_sum, ref_err)).to(cuda_device)
    assert bool(((y.double() - ys.double()).abs() <= bound).all())
