"""The persistent whole-token decode kernel (tn_llama_decode_token) at the real
Llama-3-8B width, checked operator by operator on its own inputs.

One token of a two-layer model of full width (hidden 4096, 32/8 heads, MLP
14336, vocabulary 128256) with a 257-token cache; the kernel copies the exact
Q8_0 input tiles of the traced layer's q/k/v and gate/up linears and of
lm_head, and its workspace holds the layer's other intermediates. Then:

- every Q4_0 linear (q/k/v, o_proj, gate/up, down_proj, sampled lm_head rows)
  lies within the reference's counted bound (q4_gguf_ref.py:398-465: K/32 + 3
  accumulations) of the exact value of its own Q8_0 input and weight, plus
  half a bf16 ulp for the rounding of its bf16 output;
- each planar Q8_0 the kernel writes (attention output, SiLU*up) is byte for
  byte BlockQ8_0::from_float (k_quants.rs:676-706) of the bf16 values it
  quantised, and the layer-0 q/k/v input is transformers' RMSNorm of the
  embedding quantised the same way (up to a bf16 ulp of the norm in a block);
- attention (RoPE'd q against the cache with the new RoPE'd key appended at
  slot pos) is within the reference's device rule of the oracle
  (test_mpsflash.py:150-154);
- the token is the first index of the maximum of its own bf16 logits.

A second test runs a whole 32-layer model for several tokens and requires the
same token stream as the launch-per-operator step."""

import math

import numpy as np
import pytest
import torch

from oracle import oracle
from tests import q4_exact, sdpa_ref

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def N(cuda_device):
    from torchnative_b200 import _native, build

    build.build()
    _native.lib()
    return _native


def _blob_of(codes: np.ndarray, scales: np.ndarray) -> bytes:
    """Planar Q8_0 (codes int8 [K], f32 scales [K/32]) back to GGML blocks."""
    nb = scales.size
    out = np.empty((nb, 34), dtype=np.uint8)
    out[:, 0:2] = scales.astype(np.float16).reshape(nb, 1).view(np.uint8)
    out[:, 2:] = codes.reshape(nb, 32).view(np.uint8)
    return out.tobytes()


def _tile(trace: np.ndarray, t: int, K: int):
    """Trace tile t: codes [K] int8, scales [K/32] f32, offsets [K/32] f32."""
    base = t * (K + K // 4)
    codes = trace[base:base + K].view(np.int8)
    f = trace[base + K:base + K + K // 4].view(np.float32)
    return codes, f[:K // 32], f[K // 32:]


def _check_linear(xq_blob, w_blob: bytes, rows_idx, n_full: int, K: int, got_bf16: np.ndarray, label: str):
    raw = np.frombuffer(w_blob, np.uint8).reshape(n_full, -1)
    sub = raw[rows_idx].tobytes()
    exact, abs_sum, ref_err = q4_exact.exact_linear_q4_0(xq_blob, sub, 1, len(rows_idx), K)
    exact, abs_sum, ref_err = exact[0], abs_sum[0], ref_err[0]
    bound = q4_exact.linear_bound(K, abs_sum, ref_err) + np.abs(exact) * 2.0 ** -8
    worst = float(np.max(np.abs(got_bf16.astype(np.float64) - exact) / bound))
    assert worst <= 1.0, f"{label}: |gpu - exact| reaches {worst:.3g}x the counted bound"


def _q8_same(values_f32: np.ndarray, codes: np.ndarray, scales: np.ndarray, offsets: np.ndarray, label: str):
    want = np.frombuffer(oracle.q8_0_quantize(values_f32), np.uint8).reshape(-1, 34)
    got = np.frombuffer(_blob_of(codes, scales), np.uint8).reshape(-1, 34)
    assert (want == got).all(), f"{label}: planar Q8_0 differs from BlockQ8_0::from_float"
    s = codes.reshape(-1, 32).astype(np.int64).sum(axis=1)
    assert np.array_equal(offsets, (12582912.0 + 8.0 * s).astype(np.float32)), f"{label}: offsets"


def _bf16_np(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


def test_one_token_at_full_width_each_operator_on_its_own_inputs(N, cuda_device):
    from transformers.models.llama import modeling_llama as ml

    from torchnative_b200.llama_decode import LLAMA3_8B, Q4LlamaDecoder

    s = LLAMA3_8B
    pos0, cap = 257, 320
    dec = Q4LlamaDecoder(s, batch=1, capacity=cap, device=cuda_device, seed=5, layers=2, mega=True)
    assert dec.mega and dec.kernels_per_step == 1
    dec.fill_prompt_cache(pos0)
    tok0 = 1234
    dec.start(torch.tensor([tok0], device=cuda_device))
    trace = torch.zeros(dec.mega_trace_bytes(), dtype=torch.uint8, device=cuda_device)
    H, I, HD, D = s.hidden, s.inter, s.heads * s.head_dim, s.head_dim

    # token 1, trace layer 0: the q/k/v input is RMSNorm(embedding) quantised
    before = N.counters()
    dec._step_mega(dec._stream(), trace, 0)
    torch.cuda.synchronize()
    N.device_status(reset=False)
    after = N.counters()
    assert after["decode_token_launches"] == before["decode_token_launches"] + 1
    assert after["q4_gemv_launches"] == before["q4_gemv_launches"]
    tr = trace.cpu().numpy()
    codes, sc, off = _tile(tr, 0, H)
    h0 = dec.embed[tok0].float()
    w = dec.layers[0]["attn_norm"]
    var = h0.pow(2).mean(-1, keepdim=True)
    xn = (w * (h0 * torch.rsqrt(var + s.eps)).to(torch.bfloat16)).float().cpu().numpy()
    want = np.frombuffer(oracle.q8_0_quantize(xn), np.uint8).reshape(-1, 34)
    got = np.frombuffer(_blob_of(codes, sc), np.uint8).reshape(-1, 34)
    assert (want == got).all(axis=1).mean() >= 0.97
    assert int(dec.pos.item()) == pos0 + 1

    # token 2, trace layer 1 (the last): every operator of that layer
    pos = int(dec.pos.item())
    tok1 = int(dec.tokens.item())
    dec._step_mega(dec._stream(), trace, 1)
    torch.cuda.synchronize()
    N.device_status(reset=False)
    tr = trace.cpu().numpy()
    v = dec.mega_views()
    lw = dec.layers[1]
    blob = {k: lw[k].cpu().numpy().tobytes() for k in ("qkv", "o", "gate_up", "down")}
    rng = np.random.default_rng(0)

    # q/k/v
    codes, sc, off = _tile(tr, 0, H)
    assert np.array_equal(off, (12582912.0 + 8.0 * codes.reshape(-1, 32).astype(np.int64).sum(1)).astype(np.float32))
    xq = _blob_of(codes, sc)
    qkv = _bf16_np(v["qkv"])
    _check_linear(xq, blob["qkv"], np.arange(s.qkv), s.qkv, H, qkv, "q/k/v")

    # attention: RoPE'd q and k at `pos`, k and v appended at slot pos, SDPA over 0..pos
    inv = dec.inv_freq
    freqs = inv[None, :] * torch.tensor([[float(pos)]], device=cuda_device)
    emb = torch.cat((freqs, freqs), dim=-1)
    cos, sin = emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)
    qkv_t = v["qkv"].view(1, -1)
    qh = qkv_t[:, :HD].view(1, s.heads, 1, D)
    kh = qkv_t[:, HD:HD + s.kv_heads * D].view(1, s.kv_heads, 1, D)
    vh = qkv_t[:, HD + s.kv_heads * D:].view(1, s.kv_heads, 1, D)
    qe, ke = ml.apply_rotary_pos_emb(qh, kh, cos[None], sin[None])
    kc, vc = dec.k_cache[1], dec.v_cache[1]
    assert torch.equal(kc[:, :, pos], ke[:, :, 0]) and torch.equal(vc[:, :, pos], vh[:, :, 0])
    kk, vv = kc[:, :, :pos + 1].contiguous().cpu(), vc[:, :, :pos + 1].contiguous().cpu()
    qn = qe.cpu()

    def st(t):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)

    f64, _ = sdpa_ref.f64_reference(qn.double().numpy(), kk.double().numpy(), vv.double().numpy(), False, None)
    cpu, _ = oracle.sdpa(st(qn), st(kk), st(vv), dtype="bfloat16", threads=8)
    bound = sdpa_ref.device_bound(sdpa_ref.from_storage(cpu, "bfloat16"), f64)
    attn = _bf16_np(v["attn"]).astype(np.float64).reshape(f64.shape)
    worst = float(np.max(np.abs(attn - f64)))
    assert worst <= bound, f"attention: {worst:.3e} > {bound:.3e}"
    # its planar Q8_0, then o_proj
    _q8_same(_bf16_np(v["attn"]), v["aq"].cpu().numpy(), v["ad"].cpu().numpy(), v["ac"].cpu().numpy(), "attn Q8")
    xq = _blob_of(v["aq"].cpu().numpy(), v["ad"].cpu().numpy())
    _check_linear(xq, blob["o"], np.arange(H), H, HD, _bf16_np(v["o_out"]), "o_proj")

    # gate/up on its traced input, SiLU*up, its planar Q8_0, down_proj
    codes, sc, off = _tile(tr, 1, H)
    xq = _blob_of(codes, sc)
    raw = np.frombuffer(blob["gate_up"], np.uint8).reshape(2 * I, -1)
    exact, abs_sum, ref_err = q4_exact.exact_linear_q4_0(xq, raw.tobytes(), 1, 2 * I, H)
    g, u = exact[0, 0::2], exact[0, 1::2]
    bnd = q4_exact.linear_bound(H, abs_sum[0], ref_err[0])
    gb = torch.from_numpy(g).float().to(torch.bfloat16).float()
    ub = torch.from_numpy(u).float().to(torch.bfloat16).float()
    act_ref = (torch.nn.functional.silu(gb).to(torch.bfloat16).float() * ub).to(torch.bfloat16).double().numpy()
    act = _bf16_np(v["act"]).astype(np.float64)
    # g and u may sit on either side of a bf16 rounding boundary within their
    # bound, so act may differ from the reference by a few bf16 ulps
    scale_ok = np.abs(act - act_ref) <= 2.0 ** -6 * np.abs(act_ref) + 4 * np.maximum(bnd[0::2], bnd[1::2])
    assert scale_ok.mean() == 1.0, f"act: {np.argwhere(~scale_ok)[:5]}"
    _q8_same(_bf16_np(v["act"]), v["gq"].cpu().numpy(), v["gd"].cpu().numpy(), v["gc"].cpu().numpy(), "act Q8")
    xq = _blob_of(v["gq"].cpu().numpy(), v["gd"].cpu().numpy())
    _check_linear(xq, blob["down"], np.arange(H), H, I, _bf16_np(v["down_out"]), "down_proj")

    # lm_head on its traced input (sampled rows + the argmax), and the token
    codes, sc, off = _tile(tr, 2, H)
    xq = _blob_of(codes, sc)
    logits = _bf16_np(dec.logits[0])
    tok2 = int(dec.tokens.item())
    assert tok2 == int(np.argmax(logits))
    rows = np.unique(np.concatenate([rng.integers(0, s.vocab, 3000), [0, s.vocab - 1, tok2]]))
    _check_linear(xq, dec.lm_head.cpu().numpy().tobytes(), rows, s.vocab, H, logits[rows], "lm_head")
    assert tok1 >= 0
    dec.close()
    N.device_status(reset=True)


def test_token_stream_equals_the_launch_per_operator_step(N, cuda_device):
    """A whole Llama-3-8B-shaped model (32 layers), 6 greedy tokens from a
    2048-token cache: the persistent kernel and the 5-launch-per-layer step
    give the same tokens, and bf16 logits within 4 bf16 ulps of the largest
    logit of each other (the two sum the same exact block terms in different
    orders; through 32 layers a last-bit difference can move a Q8_0 activation
    code by one step). The operator-level bounds are the test above."""
    from torchnative_b200.llama_decode import LLAMA3_8B, Q4LlamaDecoder

    runs = {}
    for mega in (True, False):
        dec = Q4LlamaDecoder(LLAMA3_8B, batch=1, capacity=2100, device=cuda_device, seed=77, mega=mega)
        assert dec.mega == mega
        dec.fill_prompt_cache(2048)
        dec.start(torch.tensor([4321], device=cuda_device))
        toks, logits = [], []
        for _ in range(6):
            dec.step()
            toks.append(int(dec.tokens.item()))
            logits.append(dec.logits[0].float().cpu())
        runs[mega] = (toks, torch.stack(logits))
        dec.close()
        del dec
        torch.cuda.empty_cache()
    N.device_status(reset=True)
    assert runs[True][0] == runs[False][0], f"{runs[True][0]} vs {runs[False][0]}"
    diff = float((runs[True][1] - runs[False][1]).abs().max())
    top = float(runs[False][1].abs().max())
    assert diff <= 4 * 2.0 ** (math.floor(math.log2(top)) - 7), (diff, top)
