"""numpy front end of the CPU restatement in tn_oracle.c.

TEST INFRASTRUCTURE ONLY. This module is the parity checker and the CPU
baseline; only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
--impl reference arms import it. The product package (torchnative_b200) never
does, and fails loudly rather than fall back here.

Every function restates the reference file:line named in tn_oracle.h.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtn_oracle.so")

DTYPE_CODES = {"float32": 0, "float16": 1, "bfloat16": 2, "float64": 3}
Q4_0_BLOCK_BYTES = 18
Q8_0_BLOCK_BYTES = 34


def build(force: bool = False) -> str:
    """Compile tn_oracle.c with its Makefile (gcc only; seconds)."""
    src = os.path.join(HERE, "tn_oracle.c")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE, "-B" if force else "libtn_oracle.so"], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        p, i64, f32p = ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p
        L.tno_f32_to_f16.restype = ctypes.c_uint16
        L.tno_f32_to_f16.argtypes = [ctypes.c_float]
        L.tno_f16_to_f32.restype = ctypes.c_float
        L.tno_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.tno_f32_to_bf16.restype = ctypes.c_uint16
        L.tno_f32_to_bf16.argtypes = [ctypes.c_float]
        for name in ("tno_q4_0_quantize", "tno_q8_0_quantize"):
            getattr(L, name).argtypes = [p, p, i64]
            getattr(L, name).restype = None
        for name in ("tno_q4_0_dequantize", "tno_q8_0_dequantize"):
            getattr(L, name).argtypes = [p, p, i64]
            getattr(L, name).restype = None
        L.tno_q4_0_q8_0_dot.argtypes = [p, p, i64]
        L.tno_q4_0_q8_0_dot.restype = ctypes.c_float
        L.tno_q4_0_linear.argtypes = [p, p, p, f32p, i64, i64, i64, ctypes.c_int]
        L.tno_q4_0_linear.restype = None
        L.tno_q8_0_q8_0_dot.argtypes = [p, p, i64]
        L.tno_q8_0_q8_0_dot.restype = ctypes.c_float
        L.tno_q8_0_linear.argtypes = [p, p, p, f32p, i64, i64, i64, ctypes.c_int]
        L.tno_q8_0_linear.restype = None
        for name in ("tno_q4_k_dequantize", "tno_q8_k_quantize"):
            getattr(L, name).argtypes = [p, p, i64]
            getattr(L, name).restype = None
        L.tno_q4_k_q8_k_dot.argtypes = [p, p, i64]
        L.tno_q4_k_q8_k_dot.restype = ctypes.c_float
        L.tno_q4_k_linear.argtypes = [p, p, p, f32p, i64, i64, i64, ctypes.c_int]
        L.tno_q4_k_linear.restype = None
        L.tno_sdpa.argtypes = [p, p, p, p, ctypes.c_int, p, p, p, ctypes.c_int, i64, i64, i64, i64,
                               i64, i64, p, p, p, ctypes.c_int, ctypes.c_double, ctypes.c_int]
        L.tno_sdpa.restype = None
        _lib = L
    return _lib


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# ---- Q4_0 / Q8_0 codecs ------------------------------------------------------


def q4_0_quantize(x: np.ndarray) -> bytes:
    """BlockQ4_0::from_float (k_quants.rs:241-277). x: float32, size % 32 == 0."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    assert x.size % 32 == 0
    out = np.empty(x.size // 32 * Q4_0_BLOCK_BYTES, dtype=np.uint8)
    lib().tno_q4_0_quantize(_ptr(x), _ptr(out), x.size)
    return out.tobytes()


def q4_0_dequantize(blob: bytes, n: int) -> np.ndarray:
    """BlockQ4_0::to_float (k_quants.rs:219-239)."""
    b = np.frombuffer(blob, dtype=np.uint8)
    assert b.size == n // 32 * Q4_0_BLOCK_BYTES
    out = np.empty(n, dtype=np.float32)
    lib().tno_q4_0_dequantize(_ptr(np.ascontiguousarray(b)), _ptr(out), n)
    return out


def q8_0_quantize(x: np.ndarray) -> bytes:
    """BlockQ8_0::from_float (k_quants.rs:676-706)."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    assert x.size % 32 == 0
    out = np.empty(x.size // 32 * Q8_0_BLOCK_BYTES, dtype=np.uint8)
    lib().tno_q8_0_quantize(_ptr(x), _ptr(out), x.size)
    return out.tobytes()


def q8_0_dequantize(blob: bytes, n: int) -> np.ndarray:
    b = np.frombuffer(blob, dtype=np.uint8)
    out = np.empty(n, dtype=np.float32)
    lib().tno_q8_0_dequantize(_ptr(np.ascontiguousarray(b)), _ptr(out), n)
    return out


def q4_0_linear(x: np.ndarray, w_blob: bytes | np.ndarray, n_out: int, bias: np.ndarray | None = None,
                threads: int = 1) -> np.ndarray:
    """torch._C._quantized_linear on the CPU (quant.rs:286-369 -> k_quants.rs:2430-2580)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    lead, k = x.shape[:-1], x.shape[-1]
    m = int(np.prod(lead)) if lead else 1
    w = np.frombuffer(w_blob, dtype=np.uint8) if isinstance(w_blob, (bytes, bytearray)) else w_blob
    w = np.ascontiguousarray(w, dtype=np.uint8)
    assert w.size == n_out * (k // 32) * Q4_0_BLOCK_BYTES
    y = np.empty((m, n_out), dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    lib().tno_q4_0_linear(_ptr(x), _ptr(w), _ptr(b), _ptr(y), m, n_out, k, int(threads))
    return y.reshape(*lead, n_out)


def q8_0_linear(x: np.ndarray, w_blob: bytes | np.ndarray, n_out: int, bias: np.ndarray | None = None,
                threads: int = 1) -> np.ndarray:
    """torch._C._quantized_linear for a Q8_0 weight on the CPU (quant.rs:286-369 ->
    k_quants.rs:2430-2580 with BlockQ8_0::vec_dot_unopt, :737-756)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    lead, k = x.shape[:-1], x.shape[-1]
    m = int(np.prod(lead)) if lead else 1
    w = np.frombuffer(w_blob, dtype=np.uint8) if isinstance(w_blob, (bytes, bytearray)) else w_blob
    w = np.ascontiguousarray(w, dtype=np.uint8)
    assert w.size == n_out * (k // 32) * Q8_0_BLOCK_BYTES
    y = np.empty((m, n_out), dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    lib().tno_q8_0_linear(_ptr(x), _ptr(w), _ptr(b), _ptr(y), m, n_out, k, int(threads))
    return y.reshape(*lead, n_out)


Q4_K_BLOCK_BYTES = 144
Q8_K_BLOCK_BYTES = 292


def q4_k_dequantize(blob: bytes, n: int) -> np.ndarray:
    """BlockQ4K::to_float (k_quants.rs:1722-1748): n elements (a multiple of 256)."""
    b = np.frombuffer(blob, dtype=np.uint8)
    assert b.size == n // 256 * Q4_K_BLOCK_BYTES
    y = np.empty(n, dtype=np.float32)
    lib().tno_q4_k_dequantize(_ptr(np.ascontiguousarray(b)), _ptr(y), n)
    return y


def q8_k_quantize(x: np.ndarray) -> bytes:
    """BlockQ8K::from_float (k_quants.rs:2376-2410): rows of x -> 292-byte blocks."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    assert x.size % 256 == 0
    out = np.empty(x.size // 256 * Q8_K_BLOCK_BYTES, dtype=np.uint8)
    lib().tno_q8_k_quantize(_ptr(x), _ptr(out), x.size)
    return out.tobytes()


def q4_k_linear(x: np.ndarray, w_blob: bytes | np.ndarray, n_out: int, bias: np.ndarray | None = None,
                threads: int = 1) -> np.ndarray:
    """torch._C._quantized_linear for a Q4_K weight on the CPU (quant.rs:286-369 ->
    k_quants.rs:2430-2580 with BlockQ4K::vec_dot_unopt, :1478-1544)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    lead, k = x.shape[:-1], x.shape[-1]
    m = int(np.prod(lead)) if lead else 1
    w = np.frombuffer(w_blob, dtype=np.uint8) if isinstance(w_blob, (bytes, bytearray)) else w_blob
    w = np.ascontiguousarray(w, dtype=np.uint8)
    assert w.size == n_out * (k // 256) * Q4_K_BLOCK_BYTES
    y = np.empty((m, n_out), dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    lib().tno_q4_k_linear(_ptr(x), _ptr(w), _ptr(b), _ptr(y), m, n_out, k, int(threads))
    return y.reshape(*lead, n_out)


# ---- SDPA --------------------------------------------------------------------


def _as_storage(a: np.ndarray, dtype: str) -> np.ndarray:
    """bfloat16 travels as uint16 bit patterns; everything else as itself."""
    if dtype == "bfloat16":
        assert a.dtype == np.uint16, "pass bfloat16 as uint16 bit patterns"
        return a
    return a.astype({"float32": np.float32, "float16": np.float16, "float64": np.float64}[dtype], copy=False)


def sdpa(q: np.ndarray, k: np.ndarray, v: np.ndarray, dtype: str = "float32", is_causal: bool = False,
         scale: float | None = None, attn_mask: np.ndarray | None = None, mask_dtype: str | None = None,
         threads: int = 1):
    """aten._scaled_dot_product_flash_attention_for_cpu's default branch
    (aten.rs:10327-10420). Arrays are [B, H, T, D] in `dtype` (bf16 as uint16
    bits), any strides. Returns (out [B,Hq,L,D] in dtype storage, lse f32/f64)."""
    q, k, v = (_as_storage(t, dtype) for t in (q, k, v))
    B, Hq, L, D = q.shape
    Hkv, S = k.shape[1], k.shape[2]
    assert Hq % Hkv == 0
    if scale is None:
        scale = 1.0 / float(np.sqrt(D))
    es = q.dtype.itemsize
    qs = np.array([s // es for s in q.strides], dtype=np.int64)
    ks = np.array([s // es for s in k.strides], dtype=np.int64)
    vs = np.array([s // es for s in v.strides], dtype=np.int64)
    out = np.empty((B, Hq, L, D), dtype=q.dtype)
    lse = np.empty((B, Hq, L), dtype=np.float64 if dtype == "float64" else np.float32)
    mptr, mcode, mstr = None, 0, None
    if attn_mask is not None:
        md = mask_dtype or dtype
        m = _as_storage(attn_mask, md)
        m = np.broadcast_to(m, (B, Hq, L, S))
        mstr = np.array([s // m.dtype.itemsize for s in m.strides], dtype=np.int64)
        mptr, mcode = m, DTYPE_CODES[md]
    lib().tno_sdpa(_ptr(q), _ptr(k), _ptr(v), None if mptr is None else mptr.ctypes.data_as(ctypes.c_void_p),
                   mcode, _ptr(mstr), _ptr(out), _ptr(lse), DTYPE_CODES[dtype], B, Hq, Hkv, L, S, D,
                   _ptr(qs), _ptr(ks), _ptr(vs), int(bool(is_causal)), float(scale), int(threads))
    return out, lse


# ---- bfloat16 helpers (numpy has no bfloat16) ---------------------------------


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round to nearest even, NaN kept quiet (the `half` crate's bf16::from_f32)."""
    x = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (x & 0x7FFFFFFF) > 0x7F800000
    r = ((x + 0x7FFF + ((x >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((x[nan] >> 16) | 0x40).astype(np.uint16)
    return r.reshape(np.shape(a))


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32).reshape(np.shape(b))
