"""SDPA on the GPU against the oracle (the reference's default CPU arithmetic,
restated) and float64, under the reference's own device rule
(tests/devices/mps/test_mpsflash.py:150-154 of the reference):

    max|gpu - f64| <= max(4 * max|cpu_dtype - f64|, max(max|f64|, 1) * 2^-21)

where cpu_dtype is the oracle in the call's dtype. Shapes follow the reference's
fused-kernel cases (SmolLM2-like 9/3 heads D=64, Qwen3-like 16/8 D=128, MHA
L=5 S=40, decode L=1) plus the BASELINE decode shape family (32/8 heads,
D=128, a KV cache read in place), an additive mask, and the upper-left causal
alignment with L != S.
"""

import math

import numpy as np
import pytest
import torch

from oracle import oracle
from tests import sdpa_ref

pytestmark = pytest.mark.gpu

DT = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


@pytest.fixture(scope="module")
def att(cuda_device):
    from torchnative_b200 import _native, attention, build

    build.build()
    _native.lib()
    return attention


def _inputs(seed, b, hq, hkv, l, s, d, dtype):
    g = torch.Generator().manual_seed(seed)
    q = (torch.rand((b, hq, l, d), generator=g) * 2 - 1).to(DT[dtype])
    k = (torch.rand((b, hkv, s, d), generator=g) * 2 - 1).to(DT[dtype])
    v = (torch.rand((b, hkv, s, d), generator=g) * 2 - 1).to(DT[dtype])
    return q, k, v


def _np_storage(t: torch.Tensor, dtype):
    if dtype == "bfloat16":
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def _check(att, dev, q, k, v, dtype, causal, mask=None, scale=None, label=""):
    out, lse = att.scaled_dot_product_flash_attention_for_cpu(q.to(dev), k.to(dev), v.to(dev), 0.0, causal,
                                                              attn_mask=None if mask is None else mask.to(dev),
                                                              scale=scale)
    assert out.dtype == q.dtype and lse.dtype == torch.float32
    got = out.float().cpu().numpy().astype(np.float64)
    got_lse = lse.cpu().numpy().astype(np.float64)
    f64, f64_lse = sdpa_ref.f64_reference(q.double().numpy(), k.double().numpy(), v.double().numpy(), causal, scale,
                                          None if mask is None else mask.double().numpy())
    mask_np = None if mask is None else (_np_storage(mask, dtype) if mask.dtype == q.dtype else mask.numpy())
    mdt = None if mask is None else ("float32" if mask.dtype == torch.float32 else dtype)
    cpu, cpu_lse = oracle.sdpa(_np_storage(q, dtype), _np_storage(k, dtype), _np_storage(v, dtype), dtype=dtype,
                               is_causal=causal, scale=scale, attn_mask=mask_np, mask_dtype=mdt, threads=8)
    cpu = sdpa_ref.from_storage(cpu, dtype)
    bound = sdpa_ref.device_bound(cpu, f64)
    worst = float(np.max(np.abs(got - f64)))
    assert worst <= bound, f"{label}: max|gpu - f64| = {worst:.3e} > bound {bound:.3e}"
    lse_bound = sdpa_ref.device_bound(cpu_lse.astype(np.float64), f64_lse)
    lworst = float(np.max(np.abs(got_lse - f64_lse)))
    assert lworst <= lse_bound, f"{label}: lse {lworst:.3e} > {lse_bound:.3e}"
    return worst, bound


# (label, b, hq, hkv, l, s, d, causal)
CASES = [
    ("smollm2-like causal prefill L=S=37", 1, 9, 3, 37, 37, 64, True),
    ("smollm2-like causal prefill L=S=64", 2, 9, 3, 64, 64, 64, True),
    ("qwen3-like causal prefill L=S=37", 1, 16, 8, 37, 37, 128, True),
    ("mha non-causal L=5 S=40", 1, 4, 4, 5, 40, 64, False),
    ("qwen3-like decode L=1 S=37", 1, 16, 8, 1, 37, 128, False),
    ("smollm2-like decode L=1 S=37", 2, 9, 3, 1, 37, 64, False),
    ("llama3-like decode L=1 S=1024", 2, 32, 8, 1, 1024, 128, False),
    ("causal L=3 S=9 (upper-left)", 1, 4, 2, 3, 9, 64, True),
    ("causal L > S", 1, 4, 2, 9, 3, 64, True),
    ("llama3-like decode long S=5000", 1, 32, 8, 1, 5000, 128, False),
    # prefill shapes (bf16/f16 here run the tcgen05 kernel: D = 128, many query rows)
    ("llama3-like causal prefill L=S=300", 1, 32, 8, 300, 300, 128, True),
    ("llama3-like causal prefill L=S=513 B=2", 2, 8, 2, 513, 513, 128, True),
    ("non-causal L=200 S=700", 1, 4, 1, 200, 700, 128, False),
    ("causal L=260 S=100 (rows past the last key)", 1, 2, 2, 260, 100, 128, True),
    ("causal L=130 S=400 (upper-left with S > L)", 1, 4, 4, 130, 400, 128, True),
    ("smollm2-like causal prefill L=S=700", 1, 9, 3, 700, 700, 64, True),
    ("qwen3-like causal prefill L=S=1100", 1, 16, 8, 1100, 1100, 128, True),
]


@pytest.mark.parametrize("dtype", ["float32", "bfloat16", "float16"])
@pytest.mark.parametrize("case", CASES, ids=lambda c: c[0])
def test_sdpa_within_the_reference_device_rule(att, cuda_device, case, dtype):
    label, b, hq, hkv, l, s, d, causal = case
    q, k, v = _inputs(178 + len(label), b, hq, hkv, l, s, d, dtype)
    _check(att, cuda_device, q, k, v, dtype, causal, label=f"{dtype} {label}")


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_additive_mask_and_explicit_scale(att, cuda_device, dtype):
    q, k, v = _inputs(1781, 1, 4, 2, 6, 6, 64, dtype)
    g = torch.Generator().manual_seed(5)
    mask = (torch.rand((1, 1, 6, 6), generator=g) * 2 - 1)
    mask[..., 2] = float("-inf")
    _check(att, cuda_device, q, k, v, dtype, False, mask=mask.to(torch.float32), label="mask f32")
    _check(att, cuda_device, q, k, v, dtype, True, mask=mask.to(DT[dtype]), scale=0.1, label="mask + causal")


@pytest.mark.parametrize("dtype", ["float32", "bfloat16", "float16"])
def test_masked_prefill_per_head_mask(att, cuda_device, dtype):
    """Many query rows with an additive [B, Hq, L, S] mask: the FP32-pipe flash
    kernel (the tcgen05 kernel takes no mask)."""
    q, k, v = _inputs(1790, 2, 8, 2, 200, 300, 128, dtype)
    g = torch.Generator().manual_seed(7)
    mask = torch.rand((2, 8, 200, 300), generator=g) * 4 - 2
    mask[:, :, :, 250:] = float("-inf")
    _check(att, cuda_device, q, k, v, dtype, False, mask=mask.to(torch.float32), label="per-head mask f32")
    _check(att, cuda_device, q, k, v, dtype, True, mask=mask.to(DT[dtype]), label="per-head mask + causal")


def test_unaligned_query_view_matches_the_contiguous_call(att, cuda_device):
    """q sliced out of a wider buffer (row stride 129 elements: no TMA
    descriptor can describe it) runs on the FP32-pipe kernel and agrees with
    the tcgen05 kernel on the contiguous copy within the device rule."""
    g = torch.Generator().manual_seed(11)
    B, Hq, Hkv, L, D = 1, 8, 2, 320, 128
    buf = (torch.rand((B, Hq, L, D + 1), generator=g) * 2 - 1).to(torch.bfloat16).to(cuda_device)
    qv = buf[..., 1:]
    assert qv.stride(2) == D + 1
    k = (torch.rand((B, Hkv, L, D), generator=g) * 2 - 1).to(torch.bfloat16).to(cuda_device)
    v = (torch.rand((B, Hkv, L, D), generator=g) * 2 - 1).to(torch.bfloat16).to(cuda_device)
    o1, l1 = att.scaled_dot_product_flash_attention_for_cpu(qv, k, v, 0.0, True)
    q = qv.contiguous()
    o2, l2 = att.scaled_dot_product_flash_attention_for_cpu(q, k, v, 0.0, True)
    f64, f64_lse = sdpa_ref.f64_reference(q.double().cpu().numpy(), k.double().cpu().numpy(),
                                          v.double().cpu().numpy(), True, None)
    cpu, _ = oracle.sdpa(_np_storage(q.cpu(), "bfloat16"), _np_storage(k.cpu(), "bfloat16"),
                         _np_storage(v.cpu(), "bfloat16"), dtype="bfloat16", is_causal=True, threads=8)
    bound = sdpa_ref.device_bound(sdpa_ref.from_storage(cpu, "bfloat16"), f64)
    for o in (o1, o2):
        assert float(np.max(np.abs(o.double().cpu().numpy() - f64))) <= bound
    assert float((l1 - l2).abs().max()) <= 1e-4


@pytest.mark.parametrize("dtype,d", [("float32", 64), ("float16", 64), ("float32", 128)])
def test_long_prefill_rows_sampled(att, cuda_device, dtype, d):
    """L = S = 16448 with 32 query heads: more 8-row groups than a grid's y
    dimension holds (the split-KV kernel's layout), one FP32-pipe launch here.
    Sampled rows are checked against the oracle run on that row alone (row i of
    an upper-left causal call equals a one-row call over keys 0..i)."""
    B, Hq, Hkv, L = 1, 32, 8, 16448
    g = torch.Generator().manual_seed(23)
    q = (torch.rand((B, Hq, L, d), generator=g) * 2 - 1).to(DT[dtype])
    k = (torch.rand((B, Hkv, L, d), generator=g) * 2 - 1).to(DT[dtype])
    v = (torch.rand((B, Hkv, L, d), generator=g) * 2 - 1).to(DT[dtype])
    out, lse = att.scaled_dot_product_flash_attention_for_cpu(q.to(cuda_device), k.to(cuda_device),
                                                              v.to(cuda_device), 0.0, True)
    out, lse = out.float().cpu(), lse.cpu()
    for h, i in [(0, 0), (5, 63), (31, 64), (12, 4097), (17, 9999), (31, L - 1)]:
        hk = h // (Hq // Hkv)
        qi, ki, vi = q[:, h:h + 1, i:i + 1], k[:, hk:hk + 1, :i + 1], v[:, hk:hk + 1, :i + 1]
        f64, f64_lse = sdpa_ref.f64_reference(qi.double().numpy(), ki.double().numpy(), vi.double().numpy(),
                                              False, None)
        cpu, cpu_lse = oracle.sdpa(_np_storage(qi.contiguous(), dtype), _np_storage(ki.contiguous(), dtype),
                                   _np_storage(vi.contiguous(), dtype), dtype=dtype, is_causal=False, threads=1)
        bound = sdpa_ref.device_bound(sdpa_ref.from_storage(cpu, dtype), f64)
        got = out[:, h:h + 1, i:i + 1].double().numpy()
        assert float(np.max(np.abs(got - f64))) <= bound, (h, i)
        lb = sdpa_ref.device_bound(cpu_lse.astype(np.float64), f64_lse)
        assert abs(float(lse[0, h, i]) - float(f64_lse[0, 0, 0])) <= lb, (h, i)


def test_kv_cache_view_is_read_in_place(att, cuda_device):
    """K/V narrowed out of a preallocated [B, Hkv, cap, D] buffer
    (PreallocatedLayer, kv_cache.py:92-114 of the reference): same answer as
    the contiguous copy, bit for bit."""
    g = torch.Generator().manual_seed(3)
    B, Hq, Hkv, cap, S, D = 2, 32, 8, 300, 217, 128
    kbuf = torch.randn((B, Hkv, cap, D), generator=g).to(torch.bfloat16).to(cuda_device)
    vbuf = torch.randn((B, Hkv, cap, D), generator=g).to(torch.bfloat16).to(cuda_device)
    q = torch.randn((B, Hq, 1, D), generator=g).to(torch.bfloat16).to(cuda_device)
    k, v = kbuf[:, :, :S], vbuf[:, :, :S]
    assert not k.is_contiguous()
    o1, l1 = att.scaled_dot_product_flash_attention_for_cpu(q, k, v)
    o2, l2 = att.scaled_dot_product_flash_attention_for_cpu(q, k.contiguous(), v.contiguous())
    assert torch.equal(o1, o2) and torch.equal(l1, l2)


def test_refusals_in_the_reference_wording(att, cuda_device):
    q = torch.zeros(1, 4, 3, 64, device=cuda_device)
    with pytest.raises(RuntimeError, match="Currently do not support dropout > 0"):
        att.scaled_dot_product_flash_attention_for_cpu(q, q, q, 0.5)
    with pytest.raises(RuntimeError, match="Accept only 4 dims inputs"):
        att.scaled_dot_product_flash_attention_for_cpu(q[0], q[0], q[0])
    with pytest.raises(NotImplementedError, match="head counts do not divide"):
        att.scaled_dot_product_flash_attention_for_cpu(torch.zeros(1, 5, 3, 64, device=cuda_device), q, q)
    with pytest.raises(NotImplementedError, match="head dimension 4"):
        z = torch.zeros(1, 2, 3, 4, device=cuda_device)
        att.scaled_dot_product_flash_attention_for_cpu(z, z, z)
    with pytest.raises(RuntimeError, match="Attention mask is the same data type as query"):
        att.scaled_dot_product_flash_attention_for_cpu(q, q, q, attn_mask=torch.zeros(3, 3, dtype=torch.int64,
                                                                                      device=cuda_device))
    with pytest.raises(NotImplementedError, match="CUDA arm"):
        att.scaled_dot_product_flash_attention_for_cpu(q.cpu(), q.cpu(), q.cpu())
    out, lse = att.scaled_dot_product_flash_attention_for_cpu(q[:, :, :0], q, q)
    assert out.shape == (1, 4, 0, 64) and lse.shape == (1, 4, 0)


def test_prefill_runs_the_tcgen05_kernel(att, cuda_device):
    from torchnative_b200 import _native

    q = torch.randn(1, 32, 512, 128, device=cuda_device, dtype=torch.bfloat16)
    k = torch.randn(1, 8, 512, 128, device=cuda_device, dtype=torch.bfloat16)
    before = _native.counters()
    att.scaled_dot_product_flash_attention_for_cpu(q, k, k, 0.0, True)
    after = _native.counters()
    assert after["sdpa_prefill_launches"] == before["sdpa_prefill_launches"] + 1
    _native.device_status(reset=True)


def test_counters_show_the_fused_kernel_ran(att, cuda_device):
    from torchnative_b200 import _native

    q = torch.randn(1, 32, 1, 128, device=cuda_device, dtype=torch.bfloat16)
    k = torch.randn(1, 8, 333, 128, device=cuda_device, dtype=torch.bfloat16)
    before = _native.counters()
    att.scaled_dot_product_flash_attention_for_cpu(q, k, k)
    after = _native.counters()
    assert after["sdpa_calls"] == before["sdpa_calls"] + 1
    assert after["sdpa_decode_launches"] == before["sdpa_decode_launches"] + 1
    _native.device_status(reset=True)
