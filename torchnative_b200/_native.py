"""ctypes binding of libtorchnative_b200.so (the C ABI in include/torchnative_b200.h).

There is no fallback: if the library is missing or does not load, every
operator raises. Build it with ``python -m torchnative_b200.build``.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libtorchnative_b200.so")

TN_OK = 0
TN_ERR_NOT_IMPLEMENTED = 1
TN_ERR_SHAPE = 2
TN_ERR_INVALID = 3
TN_ERR_CUDA = 4
TN_ERR_OOM = 5
TN_ERR_TIMEOUT = 6

TN_F32, TN_F16, TN_BF16, TN_F64 = 0, 1, 2, 3
TN_ACT_Q8_0, TN_ACT_FLOAT = 0, 1
TN_WEIGHTS_STATIC = 1
TN_EPILOGUE_SILU_MUL_PAIRS = 2
TN_X_BF16, TN_X_RMSNORM, TN_X_SILU_MUL = 1, 2, 3

# Every entry point declared in include/torchnative_b200.h, with its ctypes signature.
_P, _I, _I64, _SZ, _D = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t, ctypes.c_double


class TpLink(ctypes.Structure):
    """tn_tp_link (include/torchnative_b200.h): a GEMV's place in a
    tensor-parallel gather, as producer (slot) and/or consumer (wait_slot), or
    (reduce = 1) a row-parallel linear with its all-reduce fused in."""
    _fields_ = [("world", ctypes.c_int), ("rank", ctypes.c_int), ("bases", ctypes.c_void_p * 8),
                ("dst_offset", ctypes.c_int64), ("dst_row_stride", ctypes.c_int64), ("slot", ctypes.c_int),
                ("wait_slot", ctypes.c_int), ("reduce", ctypes.c_int), ("reserved", ctypes.c_int)]
_PI64 = ctypes.POINTER(ctypes.c_int64)


class Counters(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in (
        "q4_linear_calls", "q4_gemv_launches", "q4_gemv_generic", "q4_gemm_launches", "q8_quant_launches",
        "q4_codec_launches", "sdpa_calls", "sdpa_decode_launches", "sdpa_prefill_launches", "bytes_allocated",
        "q4_skinny_launches", "decode_token_launches", "refusals", "resolves")] + [("reserved", ctypes.c_uint64 * 2)]


class LlamaQ4Model(ctypes.Structure):
    """tn_llama_q4_model (include/torchnative_b200.h): the persistent decode
    kernel's view of a Llama-shaped Q4_0 model (per-layer fields are host
    arrays of device pointers)."""
    _fields_ = [(n, ctypes.c_int32) for n in ("layers", "hidden", "inter", "heads", "kv_heads", "head_dim",
                                              "vocab")] + [
        ("eps", ctypes.c_float), ("embed", ctypes.c_void_p), ("final_norm", ctypes.c_void_p),
        ("lm_head", ctypes.c_void_p)] + [
        (n, ctypes.POINTER(ctypes.c_void_p)) for n in ("attn_norm", "qkv", "o", "mlp_norm", "gate_up", "down",
                                                       "k_cache", "v_cache")] + [
        ("capacity", ctypes.c_int64), ("inv_freq", ctypes.c_void_p)]


class DecodeLayout(ctypes.Structure):
    """tn_llama_decode_layout: byte offsets of the persistent kernel's workspace."""
    _fields_ = [(n, ctypes.c_int64) for n in ("total", "layers", "h", "qkv", "attn", "act", "o_out", "down_out",
                                              "aq", "ad", "ac", "gq", "gd", "gc", "part_o", "part_ml", "amax",
                                              "sync")]


SIGNATURES = {
    "tn_abi_version": (_I, []),
    "tn_last_error": (ctypes.c_char_p, []),
    "tn_status_name": (ctypes.c_char_p, [_I]),
    "tn_device_info": (_I, [_I, ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_I), _PI64, _PI64]),
    "tn_device_status": (_I, [_I]),
    "tn_set_wait_budget": (_I, [_I64, _PI64]),
    "tn_stream_set": (_I, [_I, _P]),
    "tn_stream_get": (_I, [_I, ctypes.POINTER(_P)]),
    "tn_alloc": (_I, [ctypes.POINTER(_P), _SZ, _P]),
    "tn_free": (_I, [_P, _P]),
    "tn_empty_cache": (_I, []),
    "tn_memory_stats": (_I, [ctypes.POINTER(_SZ), ctypes.POINTER(_SZ)]),
    "tn_get_counters": (_I, [ctypes.POINTER(Counters)]),
    "tn_reset_counters": (_I, []),
    "tn_q4_0_quantize": (_I, [_P, _P, _I64, _I64, _P]),
    "tn_q4_0_dequantize": (_I, [_P, _P, _I64, _I64, _P]),
    "tn_q8_0_dequantize": (_I, [_P, _P, _I64, _I64, _P]),
    "tn_q8_0_quantize": (_I, [_P, _I, _I64, _P, _I64, _I64, _P]),
    "tn_q4_0_linear": (_I, [_P, _I, _I64, _P, _P, _P, _I, _I64, _I64, _I64, _I, _P]),
    "tn_q8_0_linear": (_I, [_P, _I, _I64, _P, _P, _P, _I, _I64, _I64, _I64, _I, _P]),
    "tn_q4_k_linear": (_I, [_P, _I, _I64, _P, _P, _P, _I, _I64, _I64, _I64, _I, _P]),
    "tn_q4_k_dequantize": (_I, [_P, _P, _I64, _I64, _P]),
    "tn_q8_0_quantize_planar": (_I, [_P, _I, _I64, _P, _I64, _P, _P, _I64, _I64, _P]),
    "tn_q4_0_linear_q8": (_I, [_P, _I64, _P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _I, _P]),
    "tn_q4_0_linear_fused": (_I, [_I, _P, _I64, _P, _P, _P, ctypes.c_float, _P, _P, _P, _I, _I64, _I64, _I64, _I,
                                  _P]),
    "tn_q4_0_linear_fused_q8out": (_I, [_I, _P, _I64, _P, _P, _P, ctypes.c_float, _P, _P, _P, _I, _I64, _I64, _I64,
                                        _I, _P, _I64, _P, _P, _P]),
    "tn_q4_0_linear_noalloc": (_I, [_P, _I, _I64, _P, _P, _P, _I, _I64, _I64, _I64, _P]),
    "tn_sdpa_flash_attention": (_I, [_P, _P, _P, _P, _I, _PI64, _P, _P, _I, _I64, _I64, _I64, _I64, _I64, _I64,
                                     _PI64, _PI64, _PI64, _I, _D, _P]),
    "tn_sdpa_decode_cache": (_I, [_P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _I64, _I64, _PI64, _PI64, _PI64, _P,
                                  _I64, _D, _P]),
    "tn_sdpa_decode_step": (_I, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _PI64, _PI64, _P, _D, _P]),
    "tn_sdpa_decode_step_q8": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _PI64, _PI64, _P,
                                    _D, _P]),
    "tn_llama_add_rmsnorm_q8": (_I, [_P, _P, _P, _P, ctypes.c_float, _I64, _I64, _P, _P, _P, _P]),
    "tn_llama_silu_mul_q8": (_I, [_P, _I64, _I64, _P, _P, _P, _P]),
    "tn_llama_rope_append": (_I, [_P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P, _P, _P, _I64, _I64, _P]),
    "tn_llama_argmax_embed": (_I, [_P, _I64, _I64, _P, _P, _I64, _P, _P, _P]),
    "tn_llama_embed": (_I, [_P, _I64, _P, _I64, _P, _P]),
    "tn_llama_decode_layout_of": (_I, [_P, _P]),
    "tn_llama_decode_plan": (_I, [_P, _P, _I64, ctypes.POINTER(_P)]),
    "tn_llama_decode_token": (_I, [_P, _P, _P, _P, _P, _I, _P]),
    "tn_llama_decode_trace_bytes": (_I64, [_P]),
    "tn_llama_decode_token_timeline": (_I, [_P, _P, _P, _P, _P, _P]),
    "tn_llama_decode_reset": (_I, [_P, _P]),
    "tn_llama_decode_plan_free": (_I, [_P]),
    "tn_tp_unshard": (_I, [_P, _P, _I64, _I64, _I64, _P]),
    "tn_tp_region_alloc": (_I, [ctypes.c_size_t, _P, _P]),
    "tn_tp_region_open": (_I, [_P, _P]),
    "tn_tp_region_close": (_I, [_P]),
    "tn_tp_region_free": (_I, [_P]),
    "tn_tp_region_data_offset": (_I64, []),
    "tn_tp_allgather": (_I, [_P, _I, _I, _P, _I64, _I64, _I64, _I64, _I64, _I, _P]),
    "tn_tp_step_end": (_I, [_P, _P]),
    "tn_q4_0_linear_q8_tp": (_I, [_P, _I64, _P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _I, _P, _P]),
    "tn_q4_0_linear_fused_tp": (_I, [_I, _P, _I64, _P, _P, _P, ctypes.c_float, _P, _P, _P, _I, _I64, _I64, _I64, _I,
                                     _P, _P]),
}

_lib = None
_lock = threading.Lock()


class NativeLibraryMissing(RuntimeError):
    pass


def lib() -> ctypes.CDLL:
    """The loaded library; raises if it is not built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise NativeLibraryMissing(
                        f"torchnative_b200: {LIB_PATH} is not built; run `python -m torchnative_b200.build`. "
                        "There is no CPU fallback.")
                L = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = L
    return _lib


def last_error() -> str:
    msg = lib().tn_last_error()
    return msg.decode() if msg else ""


def check(status: int) -> None:
    """Raise the exception the reference raises for this status
    (torch_c/src/err.rs: not_implemented -> NotImplementedError, the rest
    RuntimeError naming the op)."""
    if status == TN_OK:
        return
    msg = last_error() or f"torchnative_b200 call failed with status {status}"
    if status == TN_ERR_NOT_IMPLEMENTED:
        raise NotImplementedError(msg)
    if status == TN_ERR_TIMEOUT:
        raise TimeoutError(msg)
    raise RuntimeError(msg)


def counters() -> dict:
    c = Counters()
    check(lib().tn_get_counters(ctypes.byref(c)))
    return {n: int(getattr(c, n)) for n, _ in Counters._fields_ if n != "reserved"}


def reset_counters() -> None:
    check(lib().tn_reset_counters())


_DISPATCH_KEYS = ("q4_linear_calls", "sdpa_calls", "q4_codec_launches", "q8_quant_launches", "decode_token_launches")


def cuda_counters(index: int = 0) -> dict:
    """The reference's `_C._cuda_counters()` shape (torch_c/src/device.rs:1671-1700):
    resolves, dispatches, refusals and the per-op counts ("ops"), plus the
    device's free and total bytes. Opens no device that is not already in use
    (None for the memory figures then)."""
    c = counters()
    out = {"resolves": c["resolves"], "dispatches": sum(c[k] for k in _DISPATCH_KEYS),
           "readback_refusals": 0, "refusals": c["refusals"],
           "ops": {k: v for k, v in c.items() if k not in ("resolves", "refusals", "bytes_allocated")}}
    free = total = None
    try:
        import torch

        if torch.cuda.is_available() and torch.cuda.is_initialized():
            free, total = torch.cuda.mem_get_info(index)
    except Exception:  # noqa: BLE001 -- absence is a value here, as in the reference
        pass
    out["device_free_bytes"], out["device_total_bytes"] = free, total
    return out


def device_status(reset: bool = True) -> None:
    check(lib().tn_device_status(1 if reset else 0))


def set_wait_budget(cycles: int) -> int:
    """Set the current device's bounded-wait budget (cycles; <= 0 restores the
    default); returns the previous one."""
    prev = ctypes.c_int64(0)
    check(lib().tn_set_wait_budget(int(cycles), ctypes.byref(prev)))
    return int(prev.value)
