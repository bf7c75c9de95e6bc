"""scaled_dot_product_attention on a B200, mirroring the reference's CUDA arm of
`aten._scaled_dot_product_flash_attention_for_cpu.default` (reached through
`torch._C._aten_dispatch`, torchnative/rust/torch_c/src/aten.rs:1524 -> 2687 ->
routed 2771 -> CUDA arm 2861-2865 -> sdpa_flash_cpu 10092-10460).

Same signature, result pair and refusals as the reference; the compute is the
C ABI's tn_sdpa_flash_attention. No CPU path: a CPU tensor is refused by name.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _native as N

OP = "aten._scaled_dot_product_flash_attention_for_cpu.default"
_CODE = {torch.float32: N.TN_F32, torch.bfloat16: N.TN_BF16, torch.float16: N.TN_F16, torch.float64: N.TN_F64}


def _strides(t: torch.Tensor):
    """Element strides in [b, h, t, d] order; a size-1 dimension is never
    stepped through, so its stride is passed as 0."""
    return (ctypes.c_int64 * 4)(*[0 if t.shape[i] == 1 and i < 3 else t.stride(i) for i in range(4)])


def _needs_copy(t: torch.Tensor) -> bool:
    """The kernel reads K/V rows with 16-byte copies: unit d stride, 16-byte
    aligned base and 16-byte multiple strides (true of a KV-cache view)."""
    es = t.element_size()
    if t.stride(-1) != 1 or t.data_ptr() % 16 != 0:
        return True
    return any(t.shape[i] > 1 and (t.stride(i) * es) % 16 != 0 for i in range(3))


def scaled_dot_product_flash_attention_for_cpu(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                                               dropout_p: float = 0.0, is_causal: bool = False, *,
                                               attn_mask: torch.Tensor | None = None,
                                               scale: float | None = None):
    """(out, logsumexp). GQA when key/value have fewer heads than the query
    (query head h reads kv head h // (Hq/Hkv)); is_causal is upper-left aligned;
    attn_mask is additive and composes with is_causal (aten.rs:10038-10060)."""
    if query.dtype != key.dtype or query.dtype != value.dtype:
        raise RuntimeError(f"{OP}: Expected query, key, and value to have the same dtype, but got query.dtype: "
                           f"{query.dtype} key.dtype: {key.dtype} and value.dtype: {value.dtype} instead.")
    if not query.dtype.is_floating_point:
        raise RuntimeError("scaled_dot_product_attention_flash_attention: Expected data type in FP32, FP64, BF16, "
                           f"FP16, but got {query.dtype} instead.")
    if dropout_p > 0.0:
        raise RuntimeError("scaled_dot_product_attention_flash_attention: Currently do not support dropout > 0")
    for t in (query, key, value):
        if t.dim() != 4:
            raise RuntimeError("scaled_dot_product_attention_flash_attention: Accept only 4 dims inputs shape of "
                               "{B, H, T, K}")
    if attn_mask is not None and attn_mask.dtype not in (query.dtype, torch.float32):
        raise RuntimeError("scaled_dot_product_attention_flash_attention: Attention mask is the same data type as "
                           "query")
    for t in (query, key, value) + ((attn_mask,) if attn_mask is not None else ()):
        if t.device.type != "cuda":
            raise NotImplementedError(f"{OP}: this is the CUDA arm (sm_100a); a {t.device.type} tensor belongs to "
                                      "torchnative's CPU path")
        if t.device != query.device:
            raise RuntimeError(f"{OP}: Expected all tensors to be on the same device")
    if query.dtype == torch.float64:
        raise NotImplementedError(f"{OP}: torch.float64 attention is not implemented on CUDA")
    B, Hq, L, D = query.shape
    Bk, Hkv, S, Dk = key.shape
    for name, t in (("key", key), ("value", value)):
        if t.shape[0] != B or t.shape[2] != S or t.shape[3] != D or t.shape[1] != Hkv:
            raise RuntimeError(f"{OP}: query {list(query.shape)} and {name} {list(t.shape)} do not describe one "
                               "attention -- batch, key length and head dimension all have to agree")
    out = torch.empty((B, Hq, L, D), dtype=query.dtype, device=query.device)
    lse = torch.empty((B, Hq, L), dtype=torch.float32, device=query.device)
    if B == 0 or Hq == 0 or L == 0:
        return out, lse
    if query.stride(-1) != 1:
        query = query.contiguous()
    if _needs_copy(key):
        key = key.contiguous()
    if _needs_copy(value):
        value = value.contiguous()
    mptr, mcode, mstr = None, 0, None
    if attn_mask is not None:
        m = attn_mask.expand(B, Hq, L, S)
        mptr, mcode = ctypes.c_void_p(m.data_ptr()), _CODE[m.dtype]
        mstr = (ctypes.c_int64 * 4)(*[0 if m.shape[i] == 1 else m.stride(i) for i in range(4)])
        attn_mask = m
    sc = -1.0 if scale is None else float(scale)
    stream = ctypes.c_void_p(torch.cuda.current_stream(query.device).cuda_stream)
    N.check(N.lib().tn_sdpa_flash_attention(
        ctypes.c_void_p(query.data_ptr()), ctypes.c_void_p(key.data_ptr()), ctypes.c_void_p(value.data_ptr()),
        mptr, mcode, mstr, ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(lse.data_ptr()), _CODE[query.dtype],
        B, Hq, Hkv, L, S, D, _strides(query), _strides(key), _strides(value), int(bool(is_causal)), sc, stream))
    return out, lse


def aten_dispatch(op: str, *args, **kwargs):
    """The slice of `_C._aten_dispatch` this backend implements: the flash SDPA op."""
    if op != OP:
        raise NotImplementedError(f"{op} is not implemented by torchnative_b200 (only {OP})")
    return scaled_dot_product_flash_attention_for_cpu(*args, **kwargs)


def smoke_check(dev: torch.device) -> None:
    """One decode-shaped call checked against a float64 reference."""
    g = torch.Generator(device="cpu").manual_seed(0)
    q = torch.randn(1, 8, 1, 128, generator=g)
    k = torch.randn(1, 2, 77, 128, generator=g)
    v = torch.randn(1, 2, 77, 128, generator=g)
    out, lse = scaled_dot_product_flash_attention_for_cpu(q.to(dev), k.to(dev), v.to(dev))
    kk, vv = k.double().repeat_interleave(4, 1), v.double().repeat_interleave(4, 1)
    s = q.double() @ kk.transpose(-1, -2) / math.sqrt(128)
    ref = torch.softmax(s, -1) @ vv
    err = (out.double().cpu() - ref).abs().max().item()
    assert err < 1e-5, f"SDPA smoke: max error {err}"
    assert (lse.double().cpu() - torch.logsumexp(s, -1)).abs().max().item() < 1e-5
