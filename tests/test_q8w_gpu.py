"""Q8_0 weights (GGML BlockQ8_0, k_quants.rs:652-756) on the same decode GEMV
as Q4_0, against the oracle and the exact value of the quantised operands:

* the Q8_0 writer's bytes and reader's float32 bits equal the oracle's (which
  is pinned to llama.cpp's gguf-py in test_oracle_q4.py);
* the linear is within the reference's counted float32 bound of the exact
  value of (Q8_0(x), Q8_0(W)), and within twice that bound of the oracle;
* lossless integer operands give the exact integer matmul, bit for bit;
* torch._C._quantize / _dequantize / _quantized_linear and QuantizedLinear
  take the format by name, as the reference's quant.rs does.
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


def test_q8_0_weight_writer_and_reader_equal_the_oracle(tn, cuda_device):
    rng = np.random.default_rng(31)
    w = (rng.standard_normal((45, 256)) * 0.05).astype(np.float32)
    w[2, :32] = 0.0
    w[5, 9] = -3.0
    q = tn._quantize(torch.from_numpy(w).to(cuda_device), "q8_0")
    assert q.format == "q8_0" and q.nbytes() == 45 * 8 * 34
    assert tn._quantized_blob(q) == oracle.q8_0_quantize(w)
    deq = tn._dequantize(q).cpu().numpy()
    assert deq.tobytes() == oracle.q8_0_dequantize(oracle.q8_0_quantize(w), w.size).reshape(45, 256).tobytes()


SHAPES = [
    (1, 4096, 4096),
    (1, 6144, 4096),
    (4, 4096, 14336),
    (16, 1000, 4096),
    (17, 96, 2048),   # two GEMV chunks
    (40, 64, 1024),
    (1, 49, 576),     # K % 256 != 0: the unstaged path
    (3, 31, 96),      # odd number of blocks
]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_q8_0_linear_within_counted_bound_and_near_oracle(tn, cuda_device, M, N, K):
    rng = np.random.default_rng(M * 977 + N + K)
    blob = q4_exact.random_q8_0_blob(rng, N, K)
    x = (rng.standard_normal((M, K)) * 1.7).astype(np.float32)
    w = tn._quantized_from_blob(blob, (N, K), "q8_0", cuda_device)
    got = tn._quantized_linear(torch.from_numpy(x).to(cuda_device), w).cpu().numpy().astype(np.float64)
    xq = oracle.q8_0_quantize(x)
    exact, abs_sum, ref_err = q4_exact.exact_linear_q8_0(xq, blob, M, N, K)
    bound = q4_exact.linear_bound(K, abs_sum, ref_err)
    worst = float(np.max(np.abs(got - exact) / bound))
    assert worst <= 1.0, f"|gpu - exact| reaches {worst:.3g}x the counted bound"
    ref = oracle.q8_0_linear(x, blob, N, threads=8).astype(np.float64)
    assert float(np.max(np.abs(got - ref) / (2 * bound))) <= 1.0


def test_q8_0_lossless_integer_operands_give_the_exact_integer_matmul(tn, cuda_device):
    rng = np.random.default_rng(33)
    M, N, K = 3, 70, 4096
    codes = rng.integers(-127, 128, size=(N, K))
    blob = q4_exact.q8_0_blob_from_codes(codes, np.ones((N, K // 32), dtype=np.float16))
    x = rng.integers(-127, 128, size=(M, K)).astype(np.float32)
    x[:, ::32] = 127.0
    w = tn._quantized_from_blob(blob, (N, K), "q8_0", cuda_device)
    y = tn._quantized_linear(torch.from_numpy(x).to(cuda_device), w).cpu().numpy().astype(np.float64)
    assert (y == x.astype(np.float64) @ codes.T.astype(np.float64)).all()


def test_q8_0_quantized_linear_module_with_bias(tn, cuda_device):
    torch.manual_seed(3)
    lin = torch.nn.Linear(512, 40).to(cuda_device)
    mod = tn.QuantizedLinear.from_linear(lin, "q8_0")
    assert mod.qweight.format == "q8_0" and "format=q8_0" in repr(mod)
    x = torch.randn(2, 5, 512, device=cuda_device)
    y = mod(x)
    blob = tn._quantized_blob(mod.qweight)
    want = oracle.q8_0_linear(x.reshape(-1, 512).cpu().numpy(), blob, 40, bias=lin.bias.detach().cpu().numpy())
    xq = oracle.q8_0_quantize(x.reshape(-1, 512).cpu().numpy())
    exact, abs_sum, ref_err = q4_exact.exact_linear_q8_0(xq, blob, 10, 40, 512)
    bound = q4_exact.linear_bound(512, abs_sum, ref_err)
    got = y.reshape(-1, 40).detach().cpu().numpy().astype(np.float64)
    bias = lin.bias.detach().cpu().numpy().astype(np.float64)
    assert y.shape == (2, 5, 40)
    assert float(np.max(np.abs(got - bias - exact) / (bound + np.abs(got) * 2.0 ** -23 + 1e-30))) <= 2.0
    assert float(np.max(np.abs(got - want.astype(np.float64)) / (2 * bound + np.abs(got) * 2.0 ** -23))) <= 1.0


def test_q8_0_staged_kernel_ran(tn, cuda_device):
    from torchnative_b200 import _native

    rng = np.random.default_rng(34)
    blob = q4_exact.random_q8_0_blob(rng, 1024, 4096)
    w = tn._quantized_from_blob(blob, (1024, 4096), "q8_0", cuda_device)
    before = _native.counters()
    tn._quantized_linear(torch.randn(1, 4096, device=cuda_device), w)
    after = _native.counters()
    assert after["q4_gemv_launches"] == before["q4_gemv_launches"] + 1
    _native.device_status(reset=True)
