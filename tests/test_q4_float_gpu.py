"""The float-activation mode of the Q4_0 linear (TN_ACT_FLOAT): no activation
quantisation -- every weight dequantised exactly to f32 ((code - 8) * d, the
bits tn_q4_0_dequantize writes), times the activations widened exactly from
their dtype, f32 accumulate, f32 bias. Checked against the exact value in
float64 of the same dequantised weights and widened activations, within the
kernel's counted f32 bound: every term passes through at most 32 (a block's
sum) + ceil(K / 1024) (a lane's blocks) + 5 (the warp's butterfly) + 1 (the
bias) roundings, plus the rounding to the output dtype."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle
from tests import q4_exact

pytestmark = pytest.mark.gpu
P = ctypes.c_void_p
U = 2.0 ** -24  # unit roundoff of f32
DT = {"float32": (torch.float32, 0), "bfloat16": (torch.bfloat16, 2), "float16": (torch.float16, 1)}


@pytest.fixture(scope="module")
def N(cuda_device):
    from torchnative_b200 import _native, build

    build.build()
    _native.lib()
    return _native


def _gamma(k: int) -> float:
    return k * U / (1 - k * U)


@pytest.mark.parametrize("x_dtype", ["float32", "bfloat16", "float16"])
@pytest.mark.parametrize("M,Nout,K", [(1, 1024, 4096), (3, 300, 1056), (16, 257, 14336)])
def test_float_mode_within_its_f32_bound(N, cuda_device, x_dtype, M, Nout, K):
    rng = np.random.default_rng(M + K)
    blob = q4_exact.random_q4_0_blob(rng, Nout, K)
    w = oracle.q4_0_dequantize(np.frombuffer(blob, dtype=np.uint8), Nout * K).reshape(Nout, K).astype(np.float64)
    tdt, code = DT[x_dtype]
    stride = K + 32  # a row stride above K
    xbuf = torch.from_numpy(rng.standard_normal((M, stride)).astype(np.float32)).to(tdt)
    x = xbuf.to(cuda_device)
    bias = torch.from_numpy(rng.standard_normal(Nout).astype(np.float32)).to(cuda_device)
    wd = torch.from_numpy(np.frombuffer(blob, dtype=np.uint8).copy()).to(cuda_device)
    for y_dtype, ycode in (("float32", 0), ("bfloat16", 2)):
        y = torch.empty((M, Nout), dtype=DT[y_dtype][0], device=cuda_device)
        N.check(N.lib().tn_q4_0_linear(P(x.data_ptr()), code, stride, P(wd.data_ptr()), P(bias.data_ptr()),
                                       P(y.data_ptr()), ycode, M, Nout, K, N.TN_ACT_FLOAT,
                                       P(torch.cuda.current_stream().cuda_stream)))
        torch.cuda.synchronize()
        xs = xbuf[:, :K].float().numpy().astype(np.float64)
        exact = xs @ w.T + bias.cpu().numpy().astype(np.float64)
        absum = np.abs(xs) @ np.abs(w).T + np.abs(bias.cpu().numpy().astype(np.float64))
        depth = 32 + -(-K // 1024) + 6
        # the output's rounding: unit roundoff 2^-24 (f32) or 2^-8 (bf16, 8
        # significant bits) of the value
        out_u = 2.0 ** -24 if y_dtype == "float32" else 2.0 ** -8
        bound = _gamma(depth) * absum + np.abs(exact) * out_u * (1 + _gamma(depth)) + 1e-30
        got = y.float().cpu().numpy().astype(np.float64)
        worst = float(np.max(np.abs(got - exact) / bound))
        assert worst <= 1.0, f"{x_dtype} -> {y_dtype}: {worst:.3g}x the bound"
    N.device_status(reset=True)


def test_float_mode_refuses_more_than_16_rows_by_name(N, cuda_device):
    x = torch.zeros((17, 64), device=cuda_device)
    w = torch.zeros(8 * 2 * 18, dtype=torch.uint8, device=cuda_device)
    y = torch.empty((17, 8), device=cuda_device)
    with pytest.raises(NotImplementedError, match="float-activation mode runs at most 16"):
        N.check(N.lib().tn_q4_0_linear(P(x.data_ptr()), N.TN_F32, 64, P(w.data_ptr()), None, P(y.data_ptr()),
                                       N.TN_F32, 17, 8, 64, N.TN_ACT_FLOAT, None))
    N.device_status(reset=True)
