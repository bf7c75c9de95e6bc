"""The exact value of a Q4_0 x Q8_0 linear and the counted float32 bound on it.

Restates the reference's scripts/q4quality/q4_gguf_ref.py:398-465 and 511:
every block term  d_x * d_w * sum(q_x * q_w)  is exact in float64 (11 + 11 + 15
bits), so the exact answer is a finite sum the tests can form, and a float32
implementation may differ from it by at most gamma_K * sum|t| with
K = K_in/32 + 3 (the accumulation depth the reference counted), plus the float64
summation error of the exact sum itself.

The GPU kernels' own accumulation is shallower than that K (a per-lane chain of
ceil(nb/32) fused multiply-adds over exact products, then a 5-level shuffle
tree), so the reference's bound covers them a fortiori.
"""

from __future__ import annotations

import math

import numpy as np

U32 = 2.0 ** -24
U64 = 2.0 ** -53


def gamma(k: int) -> float:
    return k * U32 / (1.0 - k * U32)


def accumulation_k(in_features: int) -> int:
    return in_features // 32 + 3


def q4_0_parts(blob: bytes, out_features: int, in_features: int):
    raw = np.frombuffer(blob, dtype=np.uint8).reshape(out_features, in_features // 32, 18)
    d = raw[:, :, 0:2].copy().view(np.float16).astype(np.float64)[..., 0]
    qs = raw[:, :, 2:]
    lo = (qs & 0x0F).astype(np.int64) - 8
    hi = (qs >> 4).astype(np.int64) - 8
    return d, np.concatenate([lo, hi], axis=2)


def q8_0_parts(blob: bytes, rows: int, in_features: int):
    raw = np.frombuffer(blob, dtype=np.uint8).reshape(rows, in_features // 32, 34)
    d = raw[:, :, 0:2].copy().view(np.float16).astype(np.float64)[..., 0]
    q = raw[:, :, 2:].copy().view(np.int8).astype(np.int64)
    return d, q


def _sum_terms(terms: np.ndarray):
    lead, n = terms.shape[:-1], terms.shape[-1]
    if int(np.prod(lead)) <= 4096:
        flat = terms.reshape(-1, n)
        return np.array([math.fsum(r) for r in flat]).reshape(lead), U64
    return terms.sum(axis=-1), n * U64 / (1.0 - n * U64)


def exact_linear_q4_0(xq_blob: bytes, w_blob: bytes, rows: int, out_features: int, in_features: int):
    """(value, abs_sum, ref_err), each (rows, out) float64."""
    dw, qw = q4_0_parts(w_blob, out_features, in_features)
    dx, qx = q8_0_parts(xq_blob, rows, in_features)
    ints = np.einsum("rbk,obk->rob", qx, qw)
    absints = np.einsum("rbk,obk->rob", np.abs(qx), np.abs(qw))
    scale = dx[:, None, :] * dw[None, :, :]
    value, rel = _sum_terms(ints.astype(np.float64) * scale)
    abs_sum = (absints.astype(np.float64) * np.abs(scale)).sum(axis=2)
    return value, abs_sum, rel * abs_sum


def linear_bound(in_features: int, abs_sum, ref_err):
    return gamma(accumulation_k(in_features)) * abs_sum + ref_err


def q8_0_ties(x: np.ndarray) -> int:
    """Elements whose scaled value sits exactly on .5 (half-even and
    half-away quantisers disagree there)."""
    b = x.astype(np.float32).reshape(-1, 32)
    amax = np.abs(b).max(axis=1, keepdims=True)
    d = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        idv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    v = (b * idv).astype(np.float32)
    return int(np.sum(np.abs(v - np.trunc(v)) == 0.5))


def signed_max_ties(x: np.ndarray, block: int = 32) -> int:
    b = x.astype(np.float32).reshape(-1, block)
    a = np.abs(b)
    m = a.max(axis=1, keepdims=True)
    hits = (a == m)
    pos = np.any(hits & (b > 0), axis=1)
    neg = np.any(hits & (b < 0), axis=1)
    return int(np.sum(pos & neg))


def tie_free_gauss(rows: int, cols: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((rows, cols)) * 1.7).astype(np.float32)
    assert q8_0_ties(x) == 0 and signed_max_ties(x) == 0
    return x


def q4_0_blob_from_codes(codes: np.ndarray, d: np.ndarray) -> bytes:
    """A Q4_0 blob from signed codes in [-8, 7] ([N, K]) and f16 scales
    ([N, K/32]); the element layout is k_quants.rs:219-239's."""
    n, k = codes.shape
    u = (codes + 8).astype(np.uint8).reshape(n, k // 32, 32)
    qs = (u[:, :, :16] | (u[:, :, 16:] << 4)).astype(np.uint8)
    out = np.empty((n, k // 32, 18), dtype=np.uint8)
    out[:, :, 0:2] = np.asarray(d, dtype=np.float16).reshape(n, k // 32, 1).view(np.uint8)
    out[:, :, 2:] = qs
    return out.tobytes()


def random_q4_0_blob(rng: np.random.Generator, n: int, k: int) -> bytes:
    """The benchmark's synthetic weight: codes uniform in [-8, 7], scales
    f16(|N(0,1)| * 0.01), built directly in the block layout."""
    codes = rng.integers(-8, 8, size=(n, k), dtype=np.int64)
    d = (np.abs(rng.standard_normal((n, k // 32))) * 0.01).astype(np.float16)
    return q4_0_blob_from_codes(codes, d)


def exact_linear_q8_0(xq_blob: bytes, w_blob: bytes, rows: int, out_features: int, in_features: int):
    """The same for a Q8_0 weight (BlockQ8_0::vec_dot_unopt, k_quants.rs:737-756):
    every term d_x * d_w * sum(q_x * q_w) is exact in float64 (11 + 11 + 20 bits)."""
    dw, qw = q8_0_parts(w_blob, out_features, in_features)
    dx, qx = q8_0_parts(xq_blob, rows, in_features)
    ints = np.einsum("rbk,obk->rob", qx, qw)
    absints = np.einsum("rbk,obk->rob", np.abs(qx), np.abs(qw))
    scale = dx[:, None, :] * dw[None, :, :]
    value, rel = _sum_terms(ints.astype(np.float64) * scale)
    abs_sum = (absints.astype(np.float64) * np.abs(scale)).sum(axis=2)
    return value, abs_sum, rel * abs_sum


def q8_0_blob_from_codes(codes: np.ndarray, d: np.ndarray) -> bytes:
    """A Q8_0 blob from signed codes in [-127, 127] ([N, K]) and f16 scales
    ([N, K/32]), in BlockQ8_0's layout (k_quants.rs:652-674)."""
    n, k = codes.shape
    out = np.empty((n, k // 32, 34), dtype=np.uint8)
    out[:, :, 0:2] = np.asarray(d, dtype=np.float16).reshape(n, k // 32, 1).view(np.uint8)
    out[:, :, 2:] = codes.astype(np.int8).reshape(n, k // 32, 32).view(np.uint8)
    return out.tobytes()


def random_q8_0_blob(rng: np.random.Generator, n: int, k: int) -> bytes:
    """Synthetic Q8_0 weight: codes uniform in [-127, 127], scales
    f16(|N(0,1)| * 0.001)."""
    codes = rng.integers(-127, 128, size=(n, k), dtype=np.int64)
    d = (np.abs(rng.standard_normal((n, k // 32))) * 0.001).astype(np.float16)
    return q8_0_blob_from_codes(codes, d)
