"""A bounded device wait that runs out, on one GPU, without a fault.

The peer all-gather (tn_tp_allgather) of a two-rank group whose second rank
never runs: rank 0 stores its slice into both ranks' exchange regions,
signals, and waits for rank 1's counter -- which nothing ever sets. With the
wait budget cut to ~1 ms (tn_set_wait_budget) the kernel must give up, record
TN_ERR_TIMEOUT for tn_device_status, make the next gather fail fast, and leave
the device usable: after the status is cleared, a Q4_0 linear still matches
the oracle. No rank, kernel or collective is left waiting on another.
"""

import ctypes
import time

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


def test_a_peer_that_never_signals_times_out_and_the_device_stays_usable(N, cuda_device):
    L = N.lib()
    N.device_status(reset=True)
    regions = []
    for _ in range(2):  # rank 0's region and the one rank 1 would own
        base, handle = ctypes.c_void_p(), (ctypes.c_uint8 * 64)()
        N.check(L.tn_tp_region_alloc(1 << 16, ctypes.byref(base), handle))
        regions.append(base)
    bases = (ctypes.c_void_p * 2)(regions[0].value, regions[1].value)
    local = torch.arange(64, device=cuda_device, dtype=torch.float32).to(torch.bfloat16).view(1, 64)
    stream = P(torch.cuda.current_stream().cuda_stream)
    prev = N.set_wait_budget(2_000_000)  # ~1 ms of GPU clock
    try:
        t0 = time.perf_counter()
        N.check(L.tn_tp_allgather(bases, 0, 2, P(local.data_ptr()), 64, 1, 64, 0, 128, 0, stream))
        torch.cuda.synchronize()
        first = time.perf_counter() - t0
        with pytest.raises(TimeoutError, match="bounded wait gave up"):
            N.device_status(reset=False)
        # rank 0's slice reached both regions before the wait
        off = int(L.tn_tp_region_data_offset())
        for base in regions:
            # read the region's first row back with the layout kernel (G = 1: a copy)
            tmp = torch.empty(64, dtype=torch.bfloat16, device=cuda_device)
            N.check(L.tn_tp_unshard(P(base.value + off), P(tmp.data_ptr()), 1, 1, 64, stream))
            torch.cuda.synchronize()
            assert torch.equal(tmp, local.view(64))
        # the next gather fails fast: the error word is already set
        t0 = time.perf_counter()
        N.check(L.tn_tp_allgather(bases, 0, 2, P(local.data_ptr()), 64, 1, 64, 0, 128, 1, stream))
        torch.cuda.synchronize()
        assert time.perf_counter() - t0 < 0.5
        assert first < 0.5, f"the first gather took {first:.3f} s with a ~1 ms budget"
        with pytest.raises(TimeoutError):
            N.device_status(reset=True)  # read and cleared
        N.device_status(reset=False)     # clean now
    finally:
        N.set_wait_budget(prev)
        torch.cuda.synchronize()
        for base in regions:
            L.tn_tp_region_free(base)
    # the context is intact: a Q4_0 linear still matches the oracle
    rng = np.random.default_rng(3)
    blob = q4_exact.random_q4_0_blob(rng, 256, 512)
    x = rng.standard_normal((2, 512)).astype(np.float32)
    from torchnative_b200 import quant

    w = quant._quantized_from_blob(blob, (256, 512), "q4_0", cuda_device)
    y = quant._quantized_linear(torch.from_numpy(x).to(cuda_device), w).cpu().numpy().astype(np.float64)
    exact, abs_sum, ref_err = q4_exact.exact_linear_q4_0(oracle.q8_0_quantize(x), blob, 2, 256, 512)
    assert float(np.max(np.abs(y - exact) / q4_exact.linear_bound(512, abs_sum, ref_err))) <= 1.0
    N.device_status(reset=True)
