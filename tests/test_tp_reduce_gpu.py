"""The row-parallel GEMV's fused all-reduce (tn_tp_link.reduce) on one GPU.

A one-rank group runs the whole protocol with nothing to wait for across
GPUs: every CTA stores its f32 partial columns, each tagged with the launch's
epoch and slot in one 8-byte word, into the (own) region, polls the words of
its columns until every rank's -- here only its own -- carries the tag, and
writes y as the sum over ranks of the partials, 0 + p: the plain GEMV's f32
result, rounded once to y's dtype. A stale tag (the previous step's, or
another slot's in the same buffer) would make it wait, so equality step
after step also shows the tags advance. So y must equal the unlinked GEMV bit for bit, step after step
(tn_tp_step_end advances the epoch the counters are compared with), for
several rows, both partial buffers and a slot far into the table. The
multi-rank exchange itself runs in tests/test_tp_gpu.py (2+ GPUs)."""

import ctypes

import numpy as np
import pytest
import torch

from tests import q4_exact

pytestmark = pytest.mark.gpu
P = ctypes.c_void_p


@pytest.fixture(scope="module")
def N(cuda_device):
    from torchnative_b200 import _native, build

    build.build()
    _native.lib()
    return _native


def _planar(N, x, stream):
    M, K = x.shape
    codes = torch.empty((M, K), dtype=torch.int8, device=x.device)
    scales = torch.empty((M, K // 32), device=x.device)
    offs = torch.empty((M, K // 32), device=x.device)
    N.check(N.lib().tn_q8_0_quantize_planar(P(x.data_ptr()), N.TN_BF16, K, P(codes.data_ptr()), K,
                                            P(scales.data_ptr()), P(offs.data_ptr()), M, K, stream))
    return codes, scales, offs


@pytest.mark.parametrize("M,Nout,K", [(1, 4096, 512), (2, 1000, 1792), (4, 4096, 256)])
def test_one_rank_reduce_equals_the_plain_gemv(N, cuda_device, M, Nout, K):
    L = N.lib()
    N.device_status(reset=True)
    rng = np.random.default_rng(M * 7 + K)
    blob = torch.from_numpy(np.frombuffer(q4_exact.random_q4_0_blob(rng, Nout, K), dtype=np.uint8).copy())
    w = blob.to(cuda_device)
    stream = P(torch.cuda.current_stream().cuda_stream)
    base, handle = ctypes.c_void_p(), (ctypes.c_uint8 * 64)()
    part_bytes = M * Nout * 8  # tagged 8-byte words
    N.check(L.tn_tp_region_alloc(2 * part_bytes + 1024, ctypes.byref(base), handle))
    try:
        link = N.TpLink()
        link.world, link.rank = 1, 0
        link.bases[0] = base.value
        link.dst_row_stride, link.wait_slot, link.reduce = Nout, -1, 1
        for step in range(3):
            x = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(cuda_device).to(torch.bfloat16)
            codes, scales, offs = _planar(N, x, stream)
            want = torch.empty((M, Nout), dtype=torch.bfloat16, device=cuda_device)
            N.check(L.tn_q4_0_linear_q8_tp(P(codes.data_ptr()), K, P(scales.data_ptr()), P(offs.data_ptr()),
                                           P(w.data_ptr()), None, P(want.data_ptr()), N.TN_BF16, M, Nout, K,
                                           N.TN_WEIGHTS_STATIC, None, stream))
            # every slot once per step (the counters are compared with the epoch)
            for slot, buf in ((0, 0), (1, 1), (200, 0)):
                got = torch.full((M, Nout), float("nan"), dtype=torch.bfloat16, device=cuda_device)
                link.slot, link.dst_offset = slot, buf * ((part_bytes + 255) // 256 * 256)
                N.check(L.tn_q4_0_linear_q8_tp(P(codes.data_ptr()), K, P(scales.data_ptr()), P(offs.data_ptr()),
                                               P(w.data_ptr()), None, P(got.data_ptr()), N.TN_BF16, M, Nout, K,
                                               N.TN_WEIGHTS_STATIC, ctypes.addressof(link), stream))
                torch.cuda.synchronize()
                assert torch.equal(got, want), f"step {step} slot {slot}"
            N.check(L.tn_tp_step_end(base, stream))
        torch.cuda.synchronize()
        N.device_status(reset=False)  # no wait gave up
    finally:
        torch.cuda.synchronize()
        L.tn_tp_region_free(base)
    N.device_status(reset=True)


def test_reduce_link_refusals(N, cuda_device):
    L = N.lib()
    link = N.TpLink()
    link.world, link.rank, link.reduce, link.wait_slot = 1, 0, 1, -1
    link.bases[0] = 16
    link.dst_row_stride = 64
    for slot, wait, stride, flags, why in ((256, -1, 64, 0, "slot"), (0, 3, 64, 0, "slot"),
                                           (0, -1, 32, 0, "row stride"),
                                           (0, -1, 128, N.TN_EPILOGUE_SILU_MUL_PAIRS, "pair epilogue")):
        link.slot, link.wait_slot, link.dst_row_stride = slot, wait, stride
        codes = torch.zeros((1, 64), dtype=torch.int8, device=cuda_device)
        sc = torch.zeros((1, 2), device=cuda_device)
        with pytest.raises((RuntimeError, NotImplementedError), match=why):
            N.check(L.tn_q4_0_linear_q8_tp(P(codes.data_ptr()), 64, P(sc.data_ptr()), P(sc.data_ptr()), P(16), None,
                                           P(16), N.TN_BF16, 1, 64 if flags == 0 else 128, 64, flags,
                                           ctypes.addressof(link), None))
    N.device_status(reset=True)
