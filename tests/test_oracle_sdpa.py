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


@pytest.mark.parametrize("dtype", ["float32", "bfloat16", "float16", "float64"])
def test_oracle_fully_masked_rows_answer_zeros_and_lse_zero(dtype):
    """A query row whose every key is masked (-inf) gets zeros and a
    logsumexp of 0: what upstream torch's CPU flash kernel returns, and what the
    reference's blocked kernel reproduces (torch_c/src/flash.rs:758-776). The
    other rows of the same call are untouched by the rule."""
    import torch

    tdt = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16,
           "float64": torch.float64}[dtype]
    g = torch.Generator().manual_seed(9)
    q = torch.randn((1, 4, 5, 64), generator=g).to(tdt)
    k = torch.randn((1, 2, 7, 64), generator=g).to(tdt)
    v = torch.randn((1, 2, 7, 64), generator=g).to(tdt)
    mask = torch.zeros((1, 4, 5, 7), dtype=tdt)
    mask[0, 1, 2, :] = float("-inf")
    mask[0, 3, :, :] = float("-inf")
    mask[0, 0, 4, 3] = float("-inf")
    kk, vv = k.repeat_interleave(2, 1), v.repeat_interleave(2, 1)
    want, want_lse = torch.ops.aten._scaled_dot_product_flash_attention_for_cpu(q, kk, vv, 0.0, False,
                                                                                attn_mask=mask)[:2]

    def st(t):
        return t.view(torch.int16).numpy().view(np.uint16) if dtype == "bfloat16" else t.numpy()

    out, lse = oracle.sdpa(st(q), st(k), st(v), dtype=dtype, attn_mask=st(mask), mask_dtype=dtype)
    out = sdpa_ref.from_storage(out, dtype)
    assert not np.isnan(out).any() and not np.isnan(lse).any()
    assert (out[0, 1, 2] == 0).all() and (out[0, 3] == 0).all()
    assert lse[0, 1, 2] == 0 and (lse[0, 3] == 0).all()
    assert (want.double().numpy()[0, 3] == 0).all() and (want_lse.double().numpy()[0, 3] == 0).all()
    tol = sdpa_ref.TOL[dtype]
    assert sdpa_ref.isclose_all(out, want.double().numpy(), tol)
    assert sdpa_ref.isclose_all(lse, want_lse.double().numpy(), sdpa_ref.TOL["float64" if dtype == "float64"
                                                                               else "float32"])
