"""The `_cia_sdpa` mirror (torchnative_b200.attention.scaled_dot_product_attention):
aten::scaled_dot_product_attention as the reference composes it
(torch_c/src/bootstrap.py:13028-13080, flash-vs-math choice 12873-12918, bool
mask conversion 12921-12929).

The routing decisions are host logic (shapes and strides only) and run on the
CPU; the GPU tests check that the conversions reach the flash op intact: a
bool mask gives the bits of its additive twin, enable_gqa the result of the
expanded heads, a 2-D mask the result of its 4-D broadcast."""

import math

import numpy as np
import pytest
import torch

from torchnative_b200 import attention as A


def _qkv(b=1, hq=4, hk=4, lq=8, s=8, d=16, dtype=torch.float32, device="cpu", seed=0):
    g = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn((b, hq, lq, d), generator=g, device=device).to(dtype)
    k = torch.randn((b, hk, s, d), generator=g, device=device).to(dtype)
    v = torch.randn((b, hk, s, d), generator=g, device=device).to(dtype)
    return q, k, v


def test_flash_is_taken_for_the_plain_4d_call():
    q, k, v = _qkv()
    assert A.sdpa_takes_flash(q, k, v)
    assert A.sdpa_takes_flash(q, k, v, torch.zeros(8, 8))  # 2-D mask
    assert A.sdpa_takes_flash(q, k, v, torch.zeros(1, 4, 8, 8))
    assert A.sdpa_takes_flash(q, k, v, torch.zeros(1, 1, 1, 8))  # broadcast over rows


def test_math_cases_leave_the_flash_op():
    q, k, v = _qkv()
    assert not A.sdpa_takes_flash(q, k, v, dropout_p=0.1)
    assert not A.sdpa_takes_flash(q[0], k[0], v[0])  # 3-D
    assert not A.sdpa_takes_flash(q, k, v, torch.zeros(4, 8, 8))  # 3-D mask
    assert not A.sdpa_takes_flash(q, k, v, torch.zeros(8, 8, requires_grad=True))
    assert not A.sdpa_takes_flash(q, k, v, torch.zeros(1, 4, 3, 8))  # rows neither 1 nor L
    assert not A.sdpa_takes_flash(q, k.transpose(2, 3).contiguous().transpose(2, 3), v)  # d stride != 1
    assert not A.sdpa_takes_flash(q.to(torch.int32), k.to(torch.int32), v.to(torch.int32))
    with pytest.raises(IndexError, match="Dimension out of range"):
        A.sdpa_takes_flash(q, k, v, torch.zeros(8))


def test_gqa_needs_enable_gqa_and_a_dividing_head_count():
    q, k, v = _qkv(hq=8, hk=2)
    assert not A.sdpa_takes_flash(q, k, v)
    assert A.sdpa_takes_flash(q, k, v, enable_gqa=True)
    q3, k3, v3 = _qkv(hq=8, hk=3)
    assert not A.sdpa_takes_flash(q3, k3, v3, enable_gqa=True)


def test_bool_mask_becomes_zero_or_minus_inf_in_the_query_dtype():
    m = torch.tensor([[True, False], [False, True]])
    a = A.additive_mask(m, torch.bfloat16)
    assert a.dtype == torch.bfloat16
    assert a[0, 0] == 0 and a[1, 1] == 0 and torch.isneginf(a[0, 1].float()) and torch.isneginf(a[1, 0].float())


def test_validation_and_refusals_by_name():
    q, k, v = _qkv()
    with pytest.raises(RuntimeError, match="at least 2 dimensional"):
        A.scaled_dot_product_attention(q[0, 0, 0], k, v)
    with pytest.raises(RuntimeError, match="Expected attn_mask dtype to be bool or float"):
        A.scaled_dot_product_attention(q, k, v, torch.zeros(8, 8, dtype=torch.int64))
    with pytest.raises(NotImplementedError, match="_scaled_dot_product_attention_math"):
        A.scaled_dot_product_attention(q, k, v, dropout_p=0.5)
    # an empty input is answered before any backend: zeros of q[:-1] + [Ev]
    e = A.scaled_dot_product_attention(q[:, :, :0], k, v)
    assert e.shape == (1, 4, 0, 16)
    # the flash op itself is the CUDA arm: a CPU call is refused by name
    with pytest.raises(NotImplementedError, match="CUDA arm"):
        A.scaled_dot_product_attention(q, k, v)


@pytest.mark.gpu
def test_bool_mask_gives_the_bits_of_its_additive_twin(cuda_device):
    from torchnative_b200 import build

    build.build()
    q, k, v = _qkv(b=2, hq=4, hk=4, lq=40, s=72, d=64, dtype=torch.bfloat16, device=cuda_device, seed=3)
    g = torch.Generator(device=cuda_device).manual_seed(9)
    keep = torch.rand((2, 1, 40, 72), generator=g, device=cuda_device) > 0.3
    keep[..., 0] = True  # every row sees a key
    got = A.scaled_dot_product_attention(q, k, v, keep)
    add = torch.where(keep, 0.0, float("-inf")).to(torch.bfloat16)
    want = A.scaled_dot_product_flash_attention_for_cpu(q, k, v, attn_mask=add.expand(2, 4, 40, 72))[0]
    assert torch.equal(got, want)


@pytest.mark.gpu
def test_enable_gqa_and_a_2d_mask_reach_the_flash_op(cuda_device):
    from tests import sdpa_ref

    q, k, v = _qkv(b=1, hq=8, hk=2, lq=24, s=24, d=64, device=cuda_device, seed=5)
    got = A.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
    ke = k.repeat_interleave(4, dim=1)
    ve = v.repeat_interleave(4, dim=1)
    ref, _ = sdpa_ref.f64_reference(q.double().cpu().numpy(), ke.double().cpu().numpy(), ve.double().cpu().numpy(),
                                    True, None)
    assert float(np.max(np.abs(got.double().cpu().numpy() - ref))) <= 1e-5
    m2 = torch.randn((24, 24), device=cuda_device)
    got2 = A.scaled_dot_product_attention(q[:, :2], k, v, m2, scale=0.5 / math.sqrt(64))
    want2 = A.scaled_dot_product_flash_attention_for_cpu(q[:, :2], k, v, attn_mask=m2.expand(1, 2, 24, 24),
                                                          scale=0.5 / math.sqrt(64))[0]
    assert torch.equal(got2, want2)
