"""The Q4_0 operator family on the GPU against the oracle (the reference's CPU
arithmetic restated) and against the exact value of the quantised operands.

* integer / byte work is bit-exact: the Q4_0 writer's bytes, the Q4_0 reader's
  float32 bits, the Q8_0 activation quantiser's bytes;
* the linear is within the reference's counted float32 bound of the exact
  value of (Q8_0(x), Q4_0(W)) (tests/numerics/test_q4ref.py:203-289 of the
  reference, K = K_in/32 + 3), and within twice that bound of the oracle;
* lossless integer operands give the exact integer matmul, bit for bit;
* the kernels that ran are the ones the counters name.
"""

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


def _blob_tensor(blob: bytes, dev):
    return torch.frombuffer(bytearray(blob), dtype=torch.uint8).to(dev)


def test_q4_0_writer_is_byte_identical(tn, cuda_device):
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((67, 256)) * 0.05).astype(np.float32)
    w[3, :32] = 0.0
    w[4, 7] = -1.0  # negative signed maximum
    w[5, :32] = 1e-7  # f16-subnormal scale
    q = tn._quantize(torch.from_numpy(w).to(cuda_device))
    got = np.frombuffer(tn._quantized_blob(q), np.uint8).reshape(-1, 18)
    want = np.frombuffer(oracle.q4_0_quantize(w), np.uint8).reshape(-1, 18)
    bad = np.nonzero((got != want).any(axis=1))[0]
    assert bad.size == 0, [(int(i), got[i].tobytes().hex(), want[i].tobytes().hex()) for i in bad[:6]] + [bad.size]


def test_q4_0_reader_is_bit_identical(tn, cuda_device):
    rng = np.random.default_rng(1)
    n, k = 129, 512
    blob = q4_exact.random_q4_0_blob(rng, n, k)
    q = tn._quantized_from_blob(blob, (n, k), "q4_0", cuda_device)
    got = tn._dequantize(q).cpu().numpy()
    want = oracle.q4_0_dequantize(blob, n * k).reshape(n, k)
    assert got.tobytes() == want.tobytes()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_q8_0_activation_quantiser_is_byte_identical(tn, cuda_device, dtype):
    rng = np.random.default_rng(2)
    x = (rng.standard_normal((5, 4096)) * 1.7).astype(np.float32)
    x[0, :32] = 0.0
    x[1, 40] = 127.0 * 3  # a block whose values tie at .5 after scaling
    xt = torch.from_numpy(x).to(dtype)
    got = tn._q8_0_quantize(xt.to(cuda_device)).cpu().numpy().tobytes()
    assert got == oracle.q8_0_quantize(xt.float().numpy())


SHAPES = [
    # (M, N, K): decode rows, BASELINE shapes scaled to seconds, odd tails
    (1, 8, 64),
    (3, 12, 512),
    (2, 5, 1024),
    (1, 1, 256),
    (1, 14336, 4096),
    (4, 4096, 14336),
    (16, 6144, 4096),
    (7, 333, 4096),
    (17, 96, 2048),
    (1, 49, 576),  # K % 256 != 0: the unstaged path (SmolLM2's hidden size)
    (5, 64, 1536),
    (2, 31, 96),  # odd number of blocks
]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_linear_within_counted_bound_and_near_oracle(tn, cuda_device, M, N, K):
    rng = np.random.default_rng(M * 1000 + N + K)
    blob = q4_exact.random_q4_0_blob(rng, N, K)
    x = (rng.standard_normal((M, K)) * 1.7).astype(np.float32)
    w = tn._quantized_from_blob(blob, (N, K), "q4_0", cuda_device)
    got = tn._quantized_linear(torch.from_numpy(x).to(cuda_device), w).cpu().numpy().astype(np.float64)
    xq = oracle.q8_0_quantize(x)
    exact, abs_sum, ref_err = q4_exact.exact_linear_q4_0(xq, blob, M, N, K)
    bound = q4_exact.linear_bound(K, abs_sum, ref_err)
    worst = float(np.max(np.abs(got - exact) / bound))
    assert worst <= 1.0, f"|gpu - exact| reaches {worst:.3g}x the counted bound"
    ref = oracle.q4_0_linear(x, blob, N, threads=8).astype(np.float64)
    assert float(np.max(np.abs(got - ref) / (2 * bound))) <= 1.0


def test_linear_with_bias_is_one_float32_add(tn, cuda_device):
    rng = np.random.default_rng(9)
    M, N, K = 2, 300, 4096
    blob = q4_exact.random_q4_0_blob(rng, N, K)
    w = tn._quantized_from_blob(blob, (N, K), "q4_0", cuda_device)
    x = torch.from_numpy((rng.standard_normal((M, K))).astype(np.float32)).to(cuda_device)
    b = torch.from_numpy(rng.standard_normal(N).astype(np.float32)).to(cuda_device)
    y0 = tn._quantized_linear(x, w)
    y1 = tn._quantized_linear(x, w, b)
    assert torch.equal(y1, y0 + b)


def test_lossless_integer_operands_give_the_exact_integer_matmul(tn, cuda_device):
    rng = np.random.default_rng(7)
    M, N, K = 3, 70, 4096
    codes = rng.integers(-8, 8, size=(N, K))
    blob = q4_exact.q4_0_blob_from_codes(codes, np.ones((N, K // 32), dtype=np.float16))
    x = rng.integers(-127, 128, size=(M, K)).astype(np.float32)
    x[:, ::32] = 127.0
    w = tn._quantized_from_blob(blob, (N, K), "q4_0", cuda_device)
    y = tn._quantized_linear(torch.from_numpy(x).to(cuda_device), w).cpu().numpy().astype(np.float64)
    assert (y == x.astype(np.float64) @ codes.T.astype(np.float64)).all()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_reduced_precision_activations_are_widened_exactly(tn, cuda_device, dtype):
    """bf16/f16 input: the reference arithmetic on the exactly widened values,
    then one rounding of the result to the input dtype."""
    rng = np.random.default_rng(11)
    M, N, K = 4, 257, 4096
    blob = q4_exact.random_q4_0_blob(rng, N, K)
    w = tn._quantized_from_blob(blob, (N, K), "q4_0", cuda_device)
    x = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(dtype)
    y = tn._quantized_linear(x.to(cuda_device), w)
    assert y.dtype == dtype
    y32 = tn._quantized_linear(x.float().to(cuda_device), w)
    assert torch.equal(y, y32.to(dtype))


def test_leading_dims_and_strided_input(tn, cuda_device):
    rng = np.random.default_rng(12)
    N, K = 40, 512
    blob = q4_exact.random_q4_0_blob(rng, N, K)
    w = tn._quantized_from_blob(blob, (N, K), "q4_0", cuda_device)
    x = torch.from_numpy(rng.standard_normal((2, 3, 2 * K)).astype(np.float32)).to(cuda_device)[..., ::2]
    y = tn._quantized_linear(x, w)
    assert y.shape == (2, 3, N)
    assert torch.equal(y, tn._quantized_linear(x.contiguous(), w))


def test_refusals_in_the_reference_wording(tn, cuda_device):
    rng = np.random.default_rng(13)
    blob = q4_exact.random_q4_0_blob(rng, 8, 64)
    w = tn._quantized_from_blob(blob, (8, 64), "q4_0", cuda_device)
    with pytest.raises(RuntimeError, match="mat1 and mat2 shapes cannot be multiplied"):
        tn._quantized_linear(torch.zeros(2, 32, device=cuda_device), w)
    with pytest.raises(NotImplementedError, match="activation must be float32"):
        tn._quantized_linear(torch.zeros(2, 64, dtype=torch.float64, device=cuda_device), w)
    with pytest.raises(RuntimeError, match="Expected all tensors to be on the same device"):
        tn._quantized_linear(torch.zeros(2, 64), w)
    with pytest.raises(NotImplementedError, match="the bias must be float32"):
        tn._quantized_linear(torch.zeros(2, 64, device=cuda_device), w, torch.zeros(8, dtype=torch.float16,
                                                                                         device=cuda_device))
    with pytest.raises(ValueError, match="needs 288 bytes"):
        tn._quantized_from_blob(blob[:-1], (8, 64), "q4_0", cuda_device)
    assert tn._quantized_linear(torch.zeros(0, 64, device=cuda_device), w).shape == (0, 8)


def test_the_staged_kernel_ran_and_no_wait_timed_out(tn, cuda_device):
    from torchnative_b200 import _native

    rng = np.random.default_rng(14)
    blob = q4_exact.random_q4_0_blob(rng, 1024, 4096)
    w = tn._quantized_from_blob(blob, (1024, 4096), "q4_0", cuda_device)
    before = _native.counters()
    tn._quantized_linear(torch.randn(1, 4096, device=cuda_device), w)
    after = _native.counters()
    assert after["q4_gemv_launches"] == before["q4_gemv_launches"] + 1
    assert after["q8_quant_launches"] == before["q8_quant_launches"] + 1
    _native.device_status(reset=True)
