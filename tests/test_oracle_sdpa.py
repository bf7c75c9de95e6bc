"""The SDPA oracle (sdpa_flash_cpu's default branch restated in C) against
upstream torch's CPU kernel on the reference's golden SDPA cases, with the
reference golden harness' per-dtype tolerances; plus strided (KV-cache view)
inputs and GQA against float64 math."""

import numpy as np
import pytest

from oracle import oracle
from tests import sdpa_ref


@pytest.mark.parametrize("case", sdpa_ref.golden_cases(), ids=lambda c: c["name"])
def test_oracle_matches_upstream_torch_on_golden_cases(case):
    dt = case["dtype"]
    q = sdpa_ref.to_storage(case["q"], case["q_shape"], dt)
    k = sdpa_ref.to_storage(case["k"], case["kv_shape"], dt)
    v = sdpa_ref.to_storage(case["v"], case["kv_shape"], dt)
    mask = None
    if case.get("mask") is not None:
        mask = sdpa_ref.to_storage(case["mask"], case["mask_shape"], dt)
    out, lse = oracle.sdpa(q, k, v, dtype=dt, is_causal=case["causal"], scale=case["scale"], attn_mask=mask)
    tol = sdpa_ref.TOL[dt]
    assert sdpa_ref.isclose_all(sdpa_ref.from_storage(out, dt), case["out"], tol)
    lse_tol = sdpa_ref.TOL["float64" if dt == "float64" else "float32"]
    assert sdpa_ref.isclose_all(lse, case["lse"], lse_tol)


def test_oracle_reads_a_kv_cache_view_in_place():
    """K/V narrowed out of a [B, Hkv, cap, D] buffer (kv_cache.py:92-114 of the
    reference): the oracle reads the strided view, same answer as contiguous."""
    rng = np.random.default_rng(3)
    B, Hq, Hkv, L, cap, S, D = 2, 8, 2, 1, 40, 23, 16
    q = rng.standard_normal((B, Hq, L, D)).astype(np.float32)
    kbuf = rng.standard_normal((B, Hkv, cap, D)).astype(np.float32)
    vbuf = rng.standard_normal((B, Hkv, cap, D)).astype(np.float32)
    k, v = kbuf[:, :, :S, :], vbuf[:, :, :S, :]
    o1, l1 = oracle.sdpa(q, k, v, threads=3)
    o2, l2 = oracle.sdpa(q, np.ascontiguousarray(k), np.ascontiguousarray(v))
    assert (o1 == o2).all() and (l1 == l2).all()
    ref, ref_lse = sdpa_ref.f64_reference(q.astype(np.float64), k.astype(np.float64), v.astype(np.float64),
                                          False, None)
    assert np.max(np.abs(o1 - ref)) < 1e-5 and np.max(np.abs(l1 - ref_lse)) < 1e-5
