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


# ---- Q4_K weights, Q8_K activations (k_quants.rs:153-190, 1478-1544) --------

def q4_k_scale_min(sc12: np.ndarray):
    """6-bit sub-block scales and mins [..., 8] from the 12 packed bytes
    (get_scale_min_k4, quantized/utils.rs:50-60)."""
    q = sc12.astype(np.int64)
    sc = np.empty(q.shape[:-1] + (8,), np.int64)
    mn = np.empty_like(sc)
    sc[..., :4] = q[..., 0:4] & 63
    mn[..., :4] = q[..., 4:8] & 63
    sc[..., 4:] = (q[..., 8:12] & 0xF) | ((q[..., 0:4] >> 6) << 4)
    mn[..., 4:] = (q[..., 8:12] >> 4) | ((q[..., 4:8] >> 6) << 4)
    return sc, mn


def q4_k_parts(blob: bytes, rows: int, in_features: int):
    raw = np.frombuffer(blob, dtype=np.uint8).reshape(rows, in_features // 256, 144)
    d = raw[:, :, 0:2].copy().view(np.float16).astype(np.float64)[..., 0]
    dmin = raw[:, :, 2:4].copy().view(np.float16).astype(np.float64)[..., 0]
    sc, mn = q4_k_scale_min(raw[:, :, 4:16])
    qs = raw[:, :, 16:].reshape(rows, in_features // 256, 4, 32).astype(np.int64)
    q = np.stack([qs & 0xF, qs >> 4], axis=3).reshape(rows, in_features // 256, 256)  # element order
    return d, dmin, sc, mn, q


def q8_k_parts(blob: bytes, rows: int, in_features: int):
    raw = np.frombuffer(blob, dtype=np.uint8).reshape(rows, in_features // 256, 292)
    d = raw[:, :, 0:4].copy().view(np.float32).astype(np.float64)[..., 0]
    q = raw[:, :, 4:260].copy().view(np.int8).astype(np.int64)
    bs = raw[:, :, 260:292].copy().view(np.int16).astype(np.int64)
    return d, q, bs


def _split_exact(scale: np.ndarray, ints: np.ndarray):
    """scale * ints as two float64 pieces whose products are exact (|ints| < 2^26,
    scale a 35-bit product): ints = hi * 2^13 + lo."""
    hi = np.floor_divide(ints, 1 << 13)
    lo = ints - hi * (1 << 13)
    return scale * (hi.astype(np.float64) * (1 << 13)), scale * lo.astype(np.float64)


def exact_linear_q4_k(xq_blob: bytes, w_blob: bytes, rows: int, out_features: int, in_features: int):
    """(value, abs_sum, ref_err) of a Q4_K x Q8_K linear, each (rows, out): per
    super-block d_w d_x sum_s sc_s isum_s - dmin_w d_x sum_j m_(j/2) bsum_j, summed
    exactly (every term split so each piece is exact in float64, then fsum)."""
    dw, dm, sc, mn, qw = q4_k_parts(w_blob, out_features, in_features)
    dx, qx, bs = q8_k_parts(xq_blob, rows, in_features)
    nsb = in_features // 256
    isum = np.einsum("rbsk,obsk->robs", qx.reshape(rows, nsb, 8, 32), qw.reshape(out_features, nsb, 8, 32))
    iabs = np.einsum("rbsk,obsk->robs", np.abs(qx).reshape(rows, nsb, 8, 32), qw.reshape(out_features, nsb, 8, 32))
    S = np.einsum("robs,obs->rob", isum, sc)
    Sa = np.einsum("robs,obs->rob", iabs, sc)
    bs2 = bs.reshape(rows, nsb, 8, 2).sum(axis=3)
    Mt = np.einsum("rbs,obs->rob", bs2, mn)
    Ma = np.einsum("rbs,obs->rob", np.abs(bs.reshape(rows, nsb, 8, 2)).sum(axis=3), mn)
    s1 = dw[None, :, :] * dx[:, None, :]
    s2 = dm[None, :, :] * dx[:, None, :]
    p1, p2 = _split_exact(s1, S)
    p3, p4 = _split_exact(s2, Mt)
    terms = np.concatenate([p1, p2, -p3, -p4], axis=2)
    value, rel = _sum_terms(terms)
    abs_sum = (np.abs(s1) * Sa + np.abs(s2) * Ma).sum(axis=2)
    return value, abs_sum, rel * abs_sum


def linear_bound_q4_k(in_features: int, abs_sum, ref_err):
    """The counted bound for Q4_K: per super-block the reference rounds the
    scale product, the lane products and the min term, accumulates over the
    super-blocks and adds eight lanes and the min sum at the end; k = 2 *
    (K/256) + 12 covers that and the GPU's shallower order."""
    return gamma(2 * (in_features // 256) + 12) * abs_sum + ref_err


def q4_k_blob(rng: np.random.Generator, n: int, k: int, lossless: bool = False) -> bytes:
    """A Q4_K blob: random nibbles and 6-bit scales/mins, d and dmin
    f16(|N(0,1)| * 0.001); lossless: d = 1, every scale 1, every min 0."""
    nsb = k // 256
    out = np.empty((n, nsb, 144), dtype=np.uint8)
    if lossless:
        d = np.ones((n, nsb), np.float16)
        dm = np.zeros((n, nsb), np.float16)
        sc12 = np.zeros((n, nsb, 12), np.uint8)
        sc12[..., 0:4] = 1
        sc12[..., 8:12] = 1  # scales 4..7 = 1 (low nibble), mins 0
    else:
        d = (np.abs(rng.standard_normal((n, nsb))) * 0.001).astype(np.float16)
        dm = (np.abs(rng.standard_normal((n, nsb))) * 0.001).astype(np.float16)
        sc12 = rng.integers(0, 256, size=(n, nsb, 12), dtype=np.uint8)
    out[:, :, 0:2] = d.reshape(n, nsb, 1).view(np.uint8)
    out[:, :, 2:4] = dm.reshape(n, nsb, 1).view(np.uint8)
    out[:, :, 4:16] = sc12
    out[:, :, 16:] = rng.integers(0, 256, size=(n, nsb, 128), dtype=np.uint8)
    return out.tobytes()
