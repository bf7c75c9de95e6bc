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


def sdpa_validate(query, key, value, attn_mask=None) -> None:
    """The argument checks of aten::scaled_dot_product_attention before any
    backend is chosen (torch_c/src/bootstrap.py:12850-12870): three tensors of
    rank >= 2, a mask that is bool, float32 or the query's dtype."""
    if query.dim() < 2 or key.dim() < 2 or value.dim() < 2:
        raise RuntimeError("Expected query, key, and value to all be  at least 2 dimensional, but got "
                           f"query.dim: {query.dim()} key.dim: {key.dim()} and value.dim: {value.dim()} instead.")
    if attn_mask is not None and attn_mask.dtype not in (torch.bool, torch.float32, query.dtype):
        raise RuntimeError("Expected attn_mask dtype to be bool or float or to match query dtype, but got "
                           f"attn_mask.dtype: {attn_mask.dtype} and  query.dtype: {query.dtype} instead.")


def sdpa_takes_flash(query, key, value, attn_mask=None, dropout_p: float = 0.0, enable_gqa: bool = False) -> bool:
    """Whether aten::scaled_dot_product_attention picks the flash op (the
    reference's _cia_sdpa_flash_ok, bootstrap.py:12873-12918, upstream's
    use_flash_attention_cpp): no dropout; all three 4-D with one batch size;
    equal head counts, or under enable_gqa equal key/value heads that divide
    the query's; a 2-D or 4-D mask broadcastable to (B, Hq, L, S) that needs no
    grad; one head dimension; unit last-dim strides; a float dtype. Anything
    else is upstream's math op. Host logic only: no tensor is read."""
    if dropout_p > 0.0:
        return False
    if not (query.dim() == 4 and key.dim() == 4 and value.dim() == 4):
        return False
    if not (query.shape[0] == key.shape[0] == value.shape[0]):
        return False
    hq, hk, hv = query.shape[1], key.shape[1], value.shape[1]
    if enable_gqa:
        if not (hk == hv and hk > 0 and hq % hk == 0):
            return False
    elif not (hq == hk == hv):
        return False
    if attn_mask is not None:
        if attn_mask.requires_grad:
            return False
        if attn_mask.dim() == 1:
            raise IndexError("Dimension out of range (expected to be in range of [-1, 0], but got -2)")
        if attn_mask.dim() not in (2, 4):
            return False
        ms = list(attn_mask.shape)
        if ms[-2] not in (1, query.shape[2]) or ms[-1] not in (1, key.shape[2]):
            return False
        if attn_mask.dim() == 4 and (ms[0] not in (1, query.shape[0]) or ms[1] not in (1, hq)):
            return False
    if not (query.shape[-1] == key.shape[-1] == value.shape[-1]):
        return False
    if not (query.stride(-1) == 1 and key.stride(-1) == 1 and value.stride(-1) == 1):
        return False
    return query.dtype in (torch.float32, torch.float64, torch.float16, torch.bfloat16)


def additive_mask(mask: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """A bool mask as the additive one the flash op reads: 0 where True (the
    key attends), -inf where False (bootstrap.py:12921-12929,
    convert_boolean_attn_mask)."""
    zero = torch.zeros((), dtype=dtype, device=mask.device)
    return torch.where(mask, zero, torch.tensor(float("-inf"), dtype=dtype, device=mask.device))


MATH_OP = "aten._scaled_dot_product_attention_math.default"


def scaled_dot_product_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                                 attn_mask: torch.Tensor | None = None, dropout_p: float = 0.0,
                                 is_causal: bool = False, *, scale: float | None = None, enable_gqa: bool = False):
    """aten::scaled_dot_product_attention as the reference composes it
    (_cia_sdpa, bootstrap.py:13028-13080): validate; an empty input gives
    zeros of shape q[:-1] + [Ev]; choose the flash op (sdpa_takes_flash); turn
    a bool mask additive in the query's dtype; then the flash op's output.
    Calls the flash op cannot take (upstream's math op) are refused by name:
    that op is not on this backend. This is what transformers'
    sdpa_attention_forward reaches through torch.nn.functional on the
    reference, whose torch._C it replaces."""
    sdpa_validate(query, key, value, attn_mask)
    if query.numel() == 0 or key.numel() == 0 or value.numel() == 0:
        return torch.zeros(list(query.shape[:-1]) + [value.shape[-1]], dtype=query.dtype, device=query.device)
    flash = sdpa_takes_flash(query, key, value, attn_mask, dropout_p, enable_gqa)
    if attn_mask is not None and attn_mask.dtype == torch.bool:
        attn_mask = additive_mask(attn_mask, query.dtype)
    if not flash:
        raise NotImplementedError(f"{MATH_OP}: the math attention path is not implemented on this backend (the "
                                  "call has dropout, a 3-D/5-D mask, unequal heads without enable_gqa, or another "
                                  "shape the flash op does not take)")
    if attn_mask is not None and attn_mask.dim() == 2:
        attn_mask = attn_mask[None, None]
    return scaled_dot_product_flash_attention_for_cpu(query, key, value, dropout_p, is_causal, attn_mask=attn_mask,
                                                      scale=scale)[0]


def transformers_attention_forward(module, query, key, value, attention_mask, dropout: float = 0.0,
                                   scaling: float | None = None, is_causal: bool | None = None, **kwargs):
    """transformers' attention-function contract (the `sdpa` entry of
    ALL_ATTENTION_FUNCTIONS, integrations/sdpa_attention.py) with its calls
    landing on `scaled_dot_product_attention` above instead of
    torch.nn.functional's: GQA through enable_gqa when there is no mask
    (repeat_kv otherwise), is_causal only for more than one query row without
    a mask, output transposed to [B, L, H, D]."""
    kw = {}
    n_rep = getattr(module, "num_key_value_groups", 1)
    if n_rep > 1 or hasattr(module, "num_key_value_groups"):
        if attention_mask is None:
            kw["enable_gqa"] = True
        elif n_rep > 1:
            b, hkv, s, d = key.shape
            key = key[:, :, None].expand(b, hkv, n_rep, s, d).reshape(b, hkv * n_rep, s, d)
            value = value[:, :, None].expand(b, hkv, n_rep, s, d).reshape(b, hkv * n_rep, s, d)
    causal = is_causal if is_causal is not None else getattr(module, "is_causal", True)
    causal = bool(query.shape[2] > 1 and attention_mask is None and causal)
    out = scaled_dot_product_attention(query, key, value, attn_mask=attention_mask, dropout_p=dropout,
                                       is_causal=causal, scale=scaling, **kw)
    return out.transpose(1, 2).contiguous(), None


TRANSFORMERS_NAME = "torchnative_b200"


def register_transformers(name: str = TRANSFORMERS_NAME) -> str:
    """Register `transformers_attention_forward` with transformers'
    AttentionInterface; load a model with `attn_implementation=name`."""
    from transformers import AttentionInterface

    AttentionInterface.register(name, transformers_attention_forward)
    return name


def aten_dispatch(op: str, *args, **kwargs):
    """The slice of `_C._aten_dispatch` this backend implements: the flash SDPA
    op, and aten::scaled_dot_product_attention composed onto it as _cia_sdpa
    does."""
    if op == OP:
        return scaled_dot_product_flash_attention_for_cpu(*args, **kwargs)
    if op == "aten.scaled_dot_product_attention.default":
        return scaled_dot_product_attention(*args, **kwargs)
    raise NotImplementedError(f"{op} is not implemented by torchnative_b200 (only {OP} and "
                              "aten.scaled_dot_product_attention.default)")


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
