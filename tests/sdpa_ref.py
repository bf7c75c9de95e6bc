"""Shared SDPA test helpers: golden cases, input packing, and the GPU bound.

Tolerances: the reference's golden harness compares against upstream torch
with math.isclose per dtype (tests/golden/dtypes.py:29-39 of the reference:
f64 1e-9, f32 1e-5, f16 5e-3, bf16 6e-2, rel and abs). A fused GPU kernel is
held to the reference's device rule (tests/devices/mps/test_mpsflash.py:150-154):
    max|dev - f64| <= max(4 * max|cpu_dtype - f64|, max(max|f64|, 1) * 2^-21)
where cpu_dtype is the reference's own CPU arithmetic in the input dtype (the
oracle here) and f64 is the float64 math answer on the dtype-rounded inputs.
"""

from __future__ import annotations

import json
import math
import os

import numpy as np

from oracle import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "sdpa_golden.json")

TOL = {"float64": 1e-9, "float32": 1e-5, "float16": 5e-3, "bfloat16": 6e-2}


def golden_cases():
    with open(GOLDEN) as fh:
        return json.load(fh)["cases"]


def to_storage(vals, shape, dtype):
    a = np.asarray(vals, dtype=np.float64).reshape(shape)
    if dtype == "bfloat16":
        return oracle.f32_to_bf16_bits(a.astype(np.float32))
    return a.astype({"float32": np.float32, "float16": np.float16, "float64": np.float64}[dtype])


def from_storage(a, dtype):
    if dtype == "bfloat16":
        return oracle.bf16_bits_to_f32(a).astype(np.float64)
    return np.asarray(a, dtype=np.float64)


def isclose_all(got, want, tol):
    got, want = np.asarray(got, np.float64).ravel(), np.asarray(want, np.float64).ravel()
    inf = np.isinf(want) | np.isinf(got)
    if not np.array_equal(got[inf], want[inf]):
        return False
    g, w = got[~inf], want[~inf]
    return bool(np.all(np.abs(g - w) <= np.maximum(tol * np.maximum(np.abs(g), np.abs(w)), tol)))


def f64_reference(q, k, v, causal, scale, mask=None):
    """float64 softmax(q k^T * scale [+ causal upper-left] [+ mask]) v and its
    logsumexp, GQA by h // (Hq/Hkv). Inputs float64 [B,H,T,D]."""
    B, Hq, L, D = q.shape
    Hkv, S = k.shape[1], k.shape[2]
    rep = Hq // Hkv
    k = np.repeat(k, rep, axis=1)
    v = np.repeat(v, rep, axis=1)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    s = np.einsum("bhld,bhsd->bhls", q, k) * scale
    if causal:
        keep = np.tril(np.ones((L, S), dtype=bool))
        s = np.where(keep, s, -np.inf)
    if mask is not None:
        s = s + mask
    m = s.max(axis=-1, keepdims=True)
    w = np.exp(s - m)
    z = w.sum(axis=-1, keepdims=True)
    out = np.einsum("bhls,bhsd->bhld", w / z, v)
    lse = (np.log(z) + m)[..., 0]
    return out, lse


def device_bound(cpu_dtype_out, f64_out):
    """test_mpsflash.py:150-154's rule: 4x the CPU dtype path's own distance
    to float64, floored at max(|f64|,1) * 2^-21."""
    worst_cpu = float(np.max(np.abs(np.asarray(cpu_dtype_out, np.float64) - f64_out))) if f64_out.size else 0.0
    floor = max(float(np.max(np.abs(f64_out))) if f64_out.size else 0.0, 1.0) * 2.0 ** -21
    return max(4.0 * worst_cpu, floor)
