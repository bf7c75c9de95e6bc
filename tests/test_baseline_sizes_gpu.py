"""Parity at the sizes the benchmark times (BASELINE configs[1] and [2]).

Every kernel whose throughput bench.py reports is checked here at that size,
against the oracle (the reference's CPU arithmetic restated) and float64
under the reference's own rules:

- tcgen05 prefill attention, bf16 and f16, 32/8 heads, D 128, causal, B 1 and
  4 at S 4096 and 16384: sampled rows (first and last rows of query tiles and
  of the two-tile CTAs, the middle, the last row, and random ones, over
  several heads and batches), each row against a one-row oracle call over its
  causal keys (row i of an upper-left causal call is a one-row call over keys
  0..i), under the device rule of tests/devices/mps/test_mpsflash.py:150-154;
- split-KV decode, bf16 and f32, S 8192 and 32768, B 1, 8 and 32, through
  tn_sdpa_flash_attention (a KV-cache view), tn_sdpa_decode_cache (length on
  the device) and, for bf16, tn_sdpa_decode_step (RoPE + append + attention):
  sampled (batch, KV head) groups against the oracle over the whole cache;
- the prefill Q4_0 GEMM (tcgen05) at M 128 and 2048 on the three BASELINE
  (N, K) shapes: sampled rows and columns against the exact value of the
  quantised operands under the counted bound (q4_gguf_ref.py:398-465);
- rows whose every key is masked, on the FP32-pipe prefill kernel and the
  split-KV decode kernel (the tcgen05 kernel takes no mask and upper-left
  causal rows always see key 0): zeros and logsumexp 0, as upstream and
  torch_c/src/flash.rs:758-776 answer.
"""

import ctypes
import math

import numpy as np
import pytest
import torch

from oracle import oracle
from tests import q4_exact, sdpa_ref

pytestmark = pytest.mark.gpu
P = ctypes.c_void_p
DT = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}
HQ, HKV, D = 32, 8, 128


@pytest.fixture(scope="module")
def tn(cuda_device):
    from torchnative_b200 import _native, attention, build

    build.build()
    _native.lib()
    return _native, attention


def _st(t: torch.Tensor, dtype: str):
    t = t.contiguous().cpu()
    if dtype == "bfloat16":
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def _check_row(q_row, k_rows, v_rows, got_row, got_lse, dtype, label):
    """One query row (1 head) against its keys: oracle in the call's dtype and
    float64 on the dtype-rounded inputs; the device rule for out and lse."""
    f64, f64_lse = sdpa_ref.f64_reference(q_row.double().numpy(), k_rows.double().numpy(),
                                          v_rows.double().numpy(), False, None)
    cpu, cpu_lse = oracle.sdpa(_st(q_row, dtype), _st(k_rows, dtype), _st(v_rows, dtype), dtype=dtype,
                               is_causal=False, threads=1)
    bound = sdpa_ref.device_bound(sdpa_ref.from_storage(cpu, dtype), f64)
    worst = float(np.max(np.abs(got_row - f64)))
    assert worst <= bound, f"{label}: max|gpu - f64| {worst:.3e} > {bound:.3e}"
    lb = sdpa_ref.device_bound(cpu_lse.astype(np.float64), f64_lse)
    lw = float(np.max(np.abs(got_lse - f64_lse)))
    assert lw <= lb, f"{label}: lse {lw:.3e} > {lb:.3e}"


def _sample_rows(S, rng):
    rows = {0, 1, 127, 128, 255, 256, 257, 383, 384, S // 2 - 1, S // 2, S - 257, S - 256, S - 129, S - 128,
            S - 2, S - 1}
    rows |= set(int(r) for r in rng.integers(0, S, size=6))
    return sorted(r for r in rows if 0 <= r < S)


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("B,S", [(1, 4096), (4, 4096), (1, 16384), (4, 16384)])
def test_tcgen05_prefill_at_baseline_sizes(tn, cuda_device, B, S, dtype):
    N, att = tn
    g = torch.Generator(device=cuda_device).manual_seed(S + B)
    q = torch.randn((B, HQ, S, D), device=cuda_device, generator=g).to(DT[dtype])
    k = torch.randn((B, HKV, S, D), device=cuda_device, generator=g).to(DT[dtype])
    v = torch.randn((B, HKV, S, D), device=cuda_device, generator=g).to(DT[dtype])
    before = N.counters()
    out, lse = att.scaled_dot_product_flash_attention_for_cpu(q, k, v, 0.0, True)
    torch.cuda.synchronize()
    assert N.counters()["sdpa_prefill_launches"] == before["sdpa_prefill_launches"] + 1
    rng = np.random.default_rng(S * 3 + B)
    rows = _sample_rows(S, rng)
    groups = [(0, 0), (0, 3), (0, 4), (0, 17), (0, 31)] + ([(B - 1, 1), (B - 1, 30), (B // 2, 12)] if B > 1 else [])
    for b, h in groups:
        hk = h // (HQ // HKV)
        kc, vc = k[b, hk].float().cpu(), v[b, hk].float().cpu()
        qc = q[b, h].float().cpu()
        oc, lc = out[b, h].float().cpu().numpy().astype(np.float64), lse[b, h].cpu().numpy().astype(np.float64)
        for i in rows:
            # the dtype-rounded values: the f32 copies are exact widenings
            qi = qc[i:i + 1].to(DT[dtype]).view(1, 1, 1, D)
            ki = kc[:i + 1].to(DT[dtype]).view(1, 1, i + 1, D)
            vi = vc[:i + 1].to(DT[dtype]).view(1, 1, i + 1, D)
            _check_row(qi, ki, vi, oc[i:i + 1].reshape(1, 1, 1, D), lc[i:i + 1].reshape(1, 1, 1), dtype,
                       f"B{B} S{S} b{b} h{h} row {i}")
    N.device_status(reset=True)


def _decode_inputs(cuda_device, B, S, dtype, cap, hq=HQ):
    g = torch.Generator(device=cuda_device).manual_seed(S * 7 + B)
    kbuf = torch.randn((B, HKV, cap, D), device=cuda_device, generator=g).to(DT[dtype])
    vbuf = torch.randn((B, HKV, cap, D), device=cuda_device, generator=g).to(DT[dtype])
    q = torch.randn((B, hq, 1, D), device=cuda_device, generator=g).to(DT[dtype])
    return q, kbuf, vbuf


def _decode_groups(B):
    return sorted({(0, 0), (0, 7), (B // 2, 3), (B - 1, 5), (B - 1, 0)})


def _check_decode_groups(q, k, v, out, lse, S, dtype, label):
    """q [B, Hq, 1, D] (rounded), k/v [B, Hkv, >= S, D]: the first S keys."""
    B = q.shape[0]
    rep = q.shape[1] // HKV
    for b, hk in _decode_groups(B):
        qg = q[b:b + 1, hk * rep:(hk + 1) * rep].cpu()
        kg = k[b:b + 1, hk:hk + 1, :S].cpu()
        vg = v[b:b + 1, hk:hk + 1, :S].cpu()
        f64, f64_lse = sdpa_ref.f64_reference(qg.double().numpy(), kg.double().numpy(), vg.double().numpy(), False,
                                              None)
        cpu, cpu_lse = oracle.sdpa(_st(qg, dtype), _st(kg, dtype), _st(vg, dtype), dtype=dtype, threads=4)
        bound = sdpa_ref.device_bound(sdpa_ref.from_storage(cpu, dtype), f64)
        got = out[b:b + 1, hk * rep:(hk + 1) * rep].float().cpu().numpy().astype(np.float64).reshape(f64.shape)
        worst = float(np.max(np.abs(got - f64)))
        assert worst <= bound, f"{label} b{b} kv{hk}: {worst:.3e} > {bound:.3e}"
        if lse is not None:
            gl = lse[b:b + 1, hk * rep:(hk + 1) * rep].cpu().numpy().astype(np.float64).reshape(f64_lse.shape)
            lb = sdpa_ref.device_bound(cpu_lse.astype(np.float64), f64_lse)
            assert float(np.max(np.abs(gl - f64_lse))) <= lb, f"{label} b{b} kv{hk}: lse"


@pytest.mark.parametrize("dtype", ["bfloat16", "float32"])
@pytest.mark.parametrize("S", [8192, 32768])
@pytest.mark.parametrize("B", [1, 8, 32])
def test_split_kv_decode_at_baseline_sizes(tn, cuda_device, B, S, dtype):
    N, att = tn
    cap = S + 8
    q, kbuf, vbuf = _decode_inputs(cuda_device, B, S, dtype, cap)
    k, v = kbuf[:, :, :S], vbuf[:, :, :S]
    # 1) the flash op on a KV-cache view (L = 1: the split-KV kernel)
    before = N.counters()
    out, lse = att.scaled_dot_product_flash_attention_for_cpu(q, k, v)
    torch.cuda.synchronize()
    assert N.counters()["sdpa_decode_launches"] == before["sdpa_decode_launches"] + 1
    _check_decode_groups(q, kbuf, vbuf, out, lse, S, dtype, f"flash op B{B} S{S}")
    # 2) tn_sdpa_decode_cache: the length on the device (S - 1 cached + 1 added)
    out2 = torch.empty_like(q)
    lse2 = torch.empty((B, HQ, 1), device=cuda_device)
    ln = torch.tensor([S - 1], dtype=torch.int32, device=cuda_device)
    qs = (ctypes.c_int64 * 4)(q.stride(0), q.stride(1), 0, 1)
    ks = (ctypes.c_int64 * 4)(*kbuf.stride())
    code = {"bfloat16": N.TN_BF16, "float32": N.TN_F32}[dtype]
    N.check(N.lib().tn_sdpa_decode_cache(P(q.data_ptr()), P(kbuf.data_ptr()), P(vbuf.data_ptr()), P(out2.data_ptr()),
                                         P(lse2.data_ptr()), code, B, HQ, HKV, D, cap, qs, ks, ks, P(ln.data_ptr()), 1,
                                         1.0 / math.sqrt(D), P(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    _check_decode_groups(q, kbuf, vbuf, out2, lse2, S, dtype, f"decode_cache B{B} S{S}")
    N.device_status(reset=True)


def test_split_kv_decode_at_the_70b_shape(tn, cuda_device):
    """BASELINE configs[4]'s attention: 64 query / 8 KV heads (a GQA group of
    8 rows per KV head), batch 32, an 8192-slot cache, bf16, through
    tn_sdpa_decode_cache with the length on the device."""
    N, _ = tn
    B, S, hq, dtype = 32, 8192, 64, "bfloat16"
    cap = S
    q, kbuf, vbuf = _decode_inputs(cuda_device, B, S, dtype, cap, hq=hq)
    out = torch.empty_like(q)
    lse = torch.empty((B, hq, 1), device=cuda_device)
    ln = torch.tensor([S - 1], dtype=torch.int32, device=cuda_device)
    qs = (ctypes.c_int64 * 4)(q.stride(0), q.stride(1), 0, 1)
    ks = (ctypes.c_int64 * 4)(*kbuf.stride())
    N.check(N.lib().tn_sdpa_decode_cache(P(q.data_ptr()), P(kbuf.data_ptr()), P(vbuf.data_ptr()), P(out.data_ptr()),
                                         P(lse.data_ptr()), N.TN_BF16, B, hq, HKV, D, cap, qs, ks, ks,
                                         P(ln.data_ptr()), 1, 1.0 / math.sqrt(D),
                                         P(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    _check_decode_groups(q, kbuf, vbuf, out, lse, S, dtype, "70B shape B32 S8192")
    N.device_status(reset=True)


@pytest.mark.parametrize("S", [8192, 32768])
@pytest.mark.parametrize("B", [1, 8, 32])
def test_decode_step_at_baseline_sizes(tn, cuda_device, B, S):
    """tn_sdpa_decode_step (bf16): RoPE of q and the new k (transformers'
    apply_rotary_pos_emb), k and v appended at slot S - 1, attention over
    keys 0..S-1; checked against the oracle on the rotated rows."""
    from transformers.models.llama import modeling_llama as ml

    from torchnative_b200.llama_decode import rope_inv_freq

    N, _ = tn
    cap, pos = S + 8, S - 1
    _, kbuf, vbuf = _decode_inputs(cuda_device, B, S, "bfloat16", cap)
    g = torch.Generator(device=cuda_device).manual_seed(B + S)
    qkv = torch.randn((B, (HQ + 2 * HKV) * D), device=cuda_device, generator=g).to(torch.bfloat16)
    inv = rope_inv_freq(D, 500000.0).to(cuda_device)
    out = torch.empty((B, HQ, D), device=cuda_device, dtype=torch.bfloat16)
    lse = torch.empty((B, HQ), device=cuda_device)
    pos_dev = torch.tensor([pos], dtype=torch.int32, device=cuda_device)
    ks = (ctypes.c_int64 * 4)(*kbuf.stride())
    N.check(N.lib().tn_sdpa_decode_step(P(qkv.data_ptr()), P(inv.data_ptr()), P(kbuf.data_ptr()), P(vbuf.data_ptr()),
                                        P(out.data_ptr()), P(lse.data_ptr()), B, HQ, HKV, D, cap, ks, ks,
                                        P(pos_dev.data_ptr()), 1.0 / math.sqrt(D),
                                        P(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    freqs = inv[None, :] * torch.tensor([[float(pos)]], device=cuda_device)
    emb = torch.cat((freqs, freqs), dim=-1)
    cos, sin = emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)
    qh = qkv[:, :HQ * D].view(B, HQ, 1, D)
    kh = qkv[:, HQ * D:(HQ + HKV) * D].view(B, HKV, 1, D)
    vh = qkv[:, (HQ + HKV) * D:].view(B, HKV, 1, D)
    qe, ke = ml.apply_rotary_pos_emb(qh, kh, cos[None], sin[None])
    assert torch.equal(kbuf[:, :, pos], ke[:, :, 0]) and torch.equal(vbuf[:, :, pos], vh[:, :, 0])
    _check_decode_groups(qe, kbuf, vbuf, out.view(B, HQ, 1, D), lse.view(B, HQ, 1), S, "bfloat16",
                         f"decode_step B{B} S{S}")
    N.device_status(reset=True)


Q4_SHAPES = [(14336, 4096), (4096, 14336), (6144, 4096)]


@pytest.mark.parametrize("N_,K", Q4_SHAPES)
@pytest.mark.parametrize("M", [128, 2048])
def test_q4_gemm_at_baseline_shapes(tn, cuda_device, M, N_, K):
    N, _ = tn
    from torchnative_b200 import quant

    rng = np.random.default_rng(M + N_ + K)
    blob = q4_exact.random_q4_0_blob(rng, N_, K)
    w = quant._quantized_from_blob(blob, (N_, K), "q4_0", cuda_device)
    g = torch.Generator(device=cuda_device).manual_seed(M * 3 + N_)
    x = torch.randn((M, K), device=cuda_device, generator=g).to(torch.bfloat16)
    before = N.counters()
    y = torch.empty((M, N_), device=cuda_device)
    N.check(N.lib().tn_q4_0_linear(P(x.data_ptr()), N.TN_BF16, K, P(w.blob.data_ptr()), None, P(y.data_ptr()), N.TN_F32,
                                   M, N_, K, N.TN_ACT_Q8_0, P(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    assert N.counters()["q4_gemm_launches"] == before["q4_gemm_launches"] + 1
    rows = sorted({0, 1, 63, 64, 127, M - 1} | set(int(r) for r in rng.integers(0, M, 10)))
    cols = sorted({0, 1, 127, 128, 255, 256, N_ // 2, N_ - 129, N_ - 128, N_ - 1} |
                  set(int(c) for c in rng.integers(0, N_, 22)))
    x_np = x[rows].float().cpu().numpy()
    raw = np.frombuffer(blob, np.uint8).reshape(N_, -1)
    sub = raw[cols].tobytes()
    exact, abs_sum, ref_err = q4_exact.exact_linear_q4_0(oracle.q8_0_quantize(x_np), sub, len(rows), len(cols), K)
    bound = q4_exact.linear_bound(K, abs_sum, ref_err)
    got = y.cpu().numpy()[np.ix_(rows, cols)].astype(np.float64)
    worst = float(np.max(np.abs(got - exact) / bound))
    assert worst <= 1.0, f"M{M} ({N_}, {K}): |gpu - exact| reaches {worst:.3g}x the counted bound"
    N.device_status(reset=True)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16", "float16"])
def test_fully_masked_rows_on_the_fp32_pipe_prefill_kernel(tn, cuda_device, dtype):
    N, att = tn
    g = torch.Generator().manual_seed(41)
    B, hq, hkv, L, S = 1, 8, 2, 200, 300
    q = (torch.rand((B, hq, L, D), generator=g) * 2 - 1).to(DT[dtype])
    k = (torch.rand((B, hkv, S, D), generator=g) * 2 - 1).to(DT[dtype])
    v = (torch.rand((B, hkv, S, D), generator=g) * 2 - 1).to(DT[dtype])
    mask = torch.rand((B, hq, L, S), generator=g) * 2 - 1
    mask[0, 2, 7, :] = float("-inf")
    mask[0, 5] = float("-inf")
    mask[0, 1, 100:, 17:] = float("-inf")
    for causal in (False, True):
        out, lse = att.scaled_dot_product_flash_attention_for_cpu(q.to(cuda_device), k.to(cuda_device),
                                                                  v.to(cuda_device), 0.0, causal,
                                                                  attn_mask=mask.to(cuda_device))
        o, l = out.float().cpu(), lse.cpu()
        assert not torch.isnan(o).any() and not torch.isnan(l).any()
        assert (o[0, 2, 7] == 0).all() and l[0, 2, 7] == 0
        assert (o[0, 5] == 0).all() and (l[0, 5] == 0).all()
        cpu, cpu_lse = oracle.sdpa(_st(q, dtype), _st(k, dtype), _st(v, dtype), dtype=dtype, is_causal=causal,
                                   attn_mask=mask.numpy(), mask_dtype="float32", threads=8)
        cpu = sdpa_ref.from_storage(cpu, dtype)
        live = np.ones((B, hq, L), dtype=bool)
        live[0, 2, 7] = False
        live[0, 5] = False
        f64, f64_lse = sdpa_ref.f64_reference(q.double().numpy(), k.double().numpy(), v.double().numpy(), causal,
                                              None, mask.double().numpy())
        bound = sdpa_ref.device_bound(cpu[live], f64[live])
        assert float(np.max(np.abs(o.double().numpy()[live] - f64[live]))) <= bound
        assert (cpu[~live] == 0).all() and (cpu_lse[~live] == 0).all()
    N.device_status(reset=True)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_fully_masked_rows_on_the_split_kv_decode_kernel(tn, cuda_device, dtype):
    """L = 1 with a mask and 3000 keys: the SIMT split-KV kernel with several
    key splits, all of one head's splits masked, merged by the last CTA."""
    N, att = tn
    g = torch.Generator().manual_seed(43)
    B, S = 2, 3000
    q = (torch.rand((B, HQ, 1, D), generator=g) * 2 - 1).to(DT[dtype])
    k = (torch.rand((B, HKV, S, D), generator=g) * 2 - 1).to(DT[dtype])
    v = (torch.rand((B, HKV, S, D), generator=g) * 2 - 1).to(DT[dtype])
    mask = torch.zeros((B, HQ, 1, S))
    mask[0, 4] = float("-inf")
    mask[1, 31] = float("-inf")
    mask[1, 0, 0, :2990] = float("-inf")  # only the last split's keys live
    out, lse = att.scaled_dot_product_flash_attention_for_cpu(q.to(cuda_device), k.to(cuda_device),
                                                              v.to(cuda_device), attn_mask=mask.to(cuda_device))
    o, l = out.float().cpu(), lse.cpu()
    assert not torch.isnan(o).any() and not torch.isnan(l).any()
    assert (o[0, 4] == 0).all() and l[0, 4] == 0 and (o[1, 31] == 0).all() and l[1, 31] == 0
    f64, f64_lse = sdpa_ref.f64_reference(q.double().numpy(), k.double().numpy(), v.double().numpy(), False, None,
                                          mask.double().numpy())
    cpu, _ = oracle.sdpa(_st(q, dtype), _st(k, dtype), _st(v, dtype), dtype=dtype, attn_mask=mask.numpy(),
                         mask_dtype="float32", threads=8)
    cpu = sdpa_ref.from_storage(cpu, dtype)
    live = np.ones((B, HQ, 1), dtype=bool)
    live[0, 4] = live[1, 31] = False
    bound = sdpa_ref.device_bound(cpu[live], f64[live])
    assert float(np.max(np.abs(o.double().numpy()[live] - f64[live]))) <= bound
    lb = sdpa_ref.device_bound(oracle.sdpa(_st(q, dtype), _st(k, dtype), _st(v, dtype), dtype=dtype,
                                           attn_mask=mask.numpy(), mask_dtype="float32")[1][live].astype(np.float64),
                               f64_lse[live])
    assert float(np.max(np.abs(l.double().numpy()[live] - f64_lse[live]))) <= lb
    N.device_status(reset=True)
