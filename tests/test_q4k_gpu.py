"""Q4_K weights (GGML BlockQ4K, k_quants.rs:153-159) on the GPU against the
oracle (pinned to llama.cpp's Q4_K bytes in test_oracle_q4.py) and the exact
value of the quantised operands:

* the reader's float32 bits equal the oracle's and llama.cpp's golden case;
* the linear (Q8_K activations, BlockQ4K::vec_dot_unopt's arithmetic) is
  within the counted float32 bound of the exact value and within twice that
  bound of the oracle; lossless operands give the exact integer matmul;
* a Q4_K tensor of a GGUF file becomes a QuantizedLinear without re-encoding.
"""

import json
import os

import numpy as np
import pytest
import torch

from oracle import oracle
from tests import gguf_util, q4_exact

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tn(cuda_device):
    from torchnative_b200 import _native, build, quant

    build.build()
    _native.lib()
    return quant


def test_q4_k_reader_is_bit_identical(tn, cuda_device):
    with open(os.path.join(os.path.dirname(__file__), "golden", "q4_gguf_golden.json")) as fh:
        case = [c for c in json.load(fh)["cases"] if c["format"] == "q4_k"][0]
    q = tn._quantized_from_blob(bytes.fromhex(case["blob"]), (1, 768), "q4_k", cuda_device)
    assert tn._dequantize(q).cpu().numpy().tobytes() == bytes.fromhex(case["dequant_f32"])
    rng = np.random.default_rng(70)
    blob = q4_exact.q4_k_blob(rng, 5, 1024)
    q = tn._quantized_from_blob(blob, (5, 1024), "q4_k", cuda_device)
    assert tn._dequantize(q).cpu().numpy().tobytes() == oracle.q4_k_dequantize(blob, 5 * 1024).tobytes()


SHAPES = [
    (1, 4096, 4096),
    (1, 14336, 4096),
    (4, 4096, 14336),
    (16, 1000, 4096),
    (17, 64, 2048),  # two launches of rows
    (3, 31, 256),    # odd N, one super-block per row
    (2, 49, 512),
]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_q4_k_linear_within_counted_bound_and_near_oracle(tn, cuda_device, M, N, K):
    rng = np.random.default_rng(M * 991 + N + K)
    blob = q4_exact.q4_k_blob(rng, N, K)
    x = (rng.standard_normal((M, K)) * 1.3).astype(np.float32)
    w = tn._quantized_from_blob(blob, (N, K), "q4_k", cuda_device)
    got = tn._quantized_linear(torch.from_numpy(x).to(cuda_device), w).cpu().numpy().astype(np.float64)
    xq = oracle.q8_k_quantize(x)
    exact, abs_sum, ref_err = q4_exact.exact_linear_q4_k(xq, blob, M, N, K)
    bound = q4_exact.linear_bound_q4_k(K, abs_sum, ref_err)
    worst = float(np.max(np.abs(got - exact) / bound))
    assert worst <= 1.0, f"|gpu - exact| reaches {worst:.3g}x the counted bound"
    if M * N * K <= 16 * 4096 * 4096:
        ref = oracle.q4_k_linear(x, blob, N).astype(np.float64)
        assert float(np.max(np.abs(got - ref) / (2 * bound))) <= 1.0


def test_q4_k_lossless_operands_give_the_exact_integer_matmul(tn, cuda_device):
    rng = np.random.default_rng(71)
    M, N, K = 3, 70, 4096
    blob = q4_exact.q4_k_blob(rng, N, K, lossless=True)
    codes = oracle.q4_k_dequantize(blob, N * K).reshape(N, K).astype(np.float64)
    x = rng.integers(-127, 128, size=(M, K)).astype(np.float32)
    x[:, ::256] = 127.0
    w = tn._quantized_from_blob(blob, (N, K), "q4_k", cuda_device)
    y = tn._quantized_linear(torch.from_numpy(x).to(cuda_device), w).cpu().numpy().astype(np.float64)
    assert (y == x.astype(np.float64) @ codes.T).all()


def test_q4_k_from_gguf_and_refusals(tn, cuda_device, tmp_path):
    pytest.importorskip("gguf")
    from torchnative_b200 import gguf as G

    rng = np.random.default_rng(72)
    blob = q4_exact.q4_k_blob(rng, 24, 512)
    path = tmp_path / "k.gguf"
    gguf_util.write_gguf(path, {"w": (np.frombuffer(blob, np.uint8).reshape(24, -1), "Q4_K")})
    x = torch.randn(2, 512, device=cuda_device)
    with G.GGUFContainer(path) as f:
        mod = G.quantized_linear(f, "w", device=cuda_device)
        assert mod.format == "q4_k" and tn._quantized_blob(mod.qweight) == blob
        want = tn._quantized_linear(x, tn._quantized_from_blob(blob, (24, 512), "q4_k", cuda_device))
        assert torch.equal(mod(x), want)
    with pytest.raises(NotImplementedError, match="q4_k writer"):
        tn._quantize(torch.randn(4, 256, device=cuda_device), "q4_k")
    w = tn._quantized_from_blob(blob, (24, 512), "q4_k", cuda_device)
    from torchnative_b200 import _native
    with pytest.raises(RuntimeError, match="whole 256-element super-blocks"):
        _native.check(_native.lib().tn_q4_k_linear(None, 0, 384, None, None, None, 0, 1, 24, 384, 0, None))
    _native.device_status(reset=True)
    del w
