"""The decode-step glue on the GPU against transformers' Llama modules (the
caller of the two hot operators), and one full decode step of a small
Q4_0 Llama against a host reference assembled from the same definitions."""

import ctypes
import math

import numpy as np
import pytest
import torch

from oracle import oracle
from tests import q4_exact

pytestmark = pytest.mark.gpu
P = ctypes.c_void_p


@pytest.fixture(scope="module")
def N(cuda_device):
    from torchnative_b200 import _native, build

    build.build()
    _native.lib()
    return _native


def _stream():
    return P(torch.cuda.current_stream().cuda_stream)


def _planar_to_blob(codes, scales, rows, cols):
    """Planar Q8_0 (codes, f32 scales) back to GGML Q8_0 bytes, for comparing
    with the oracle's quantiser."""
    nb = cols // 32
    out = np.empty((rows, nb, 34), dtype=np.uint8)
    out[:, :, 0:2] = scales.reshape(rows, nb, 1).astype(np.float16).view(np.uint8)
    out[:, :, 2:] = codes.reshape(rows, nb, 32).view(np.uint8)
    return out.tobytes()


def _ref_rmsnorm(h, w, eps):
    x = h.float()
    var = x.pow(2).mean(-1, keepdim=True)
    return w * (x * torch.rsqrt(var + eps)).to(torch.bfloat16)


def test_add_rmsnorm_q8_matches_llama_rmsnorm(N, cuda_device):
    B, H, eps = 3, 4096, 1e-5
    g = torch.Generator(device=cuda_device).manual_seed(1)
    h = torch.randn((B, H), device=cuda_device, generator=g).to(torch.bfloat16)
    d = torch.randn((B, H), device=cuda_device, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(H, device=cuda_device, generator=g)).to(torch.bfloat16)
    h_out = torch.empty_like(h)
    codes = torch.empty((B, H), dtype=torch.int8, device=cuda_device)
    sc = torch.empty((B, H // 32), device=cuda_device)
    of = torch.empty((B, H // 32), device=cuda_device)
    N.check(N.lib().tn_llama_add_rmsnorm_q8(P(h.data_ptr()), P(d.data_ptr()), P(h_out.data_ptr()), P(w.data_ptr()),
                                            eps, B, H, P(codes.data_ptr()), P(sc.data_ptr()), P(of.data_ptr()),
                                            _stream()))
    want_h = (h + d)
    assert torch.equal(h_out, want_h)
    y = _ref_rmsnorm(want_h, w, eps)
    want = np.frombuffer(oracle.q8_0_quantize(y.float().cpu().numpy()), np.uint8).reshape(B, H // 32, 34)
    got = np.frombuffer(_planar_to_blob(codes.cpu().numpy(), sc.cpu().numpy(), B, H), np.uint8).reshape(B, H // 32, 34)
    # the norm's f32 reduction order differs from torch's: a block may see one bf16 ulp of difference
    same = (got == want).all(axis=2).mean()
    assert same >= 0.97, same
    deq_g = oracle.q8_0_dequantize(got.tobytes(), B * H)
    deq_w = oracle.q8_0_dequantize(want.tobytes(), B * H)
    assert np.max(np.abs(deq_g - deq_w)) <= 0.02 * np.max(np.abs(deq_w))
    # the offsets are 12582912 + 8 * sum(codes)
    assert torch.equal(of.cpu(), 12582912.0 + 8.0 * codes.cpu().view(B, H // 32, 32).sum(-1).float())


def test_silu_mul_q8_matches_llama_mlp(N, cuda_device):
    B, I = 2, 14336
    g = torch.Generator(device=cuda_device).manual_seed(2)
    gu = torch.randn((B, 2 * I), device=cuda_device, generator=g).to(torch.bfloat16)
    codes = torch.empty((B, I), dtype=torch.int8, device=cuda_device)
    sc = torch.empty((B, I // 32), device=cuda_device)
    of = torch.empty((B, I // 32), device=cuda_device)
    N.check(N.lib().tn_llama_silu_mul_q8(P(gu.data_ptr()), B, I, P(codes.data_ptr()), P(sc.data_ptr()),
                                         P(of.data_ptr()), _stream()))
    act = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
    want = oracle.q8_0_quantize(act.float().cpu().numpy())
    got = _planar_to_blob(codes.cpu().numpy(), sc.cpu().numpy(), B, I)
    g8 = np.frombuffer(got, np.uint8).reshape(-1, 34)
    w8 = np.frombuffer(want, np.uint8).reshape(-1, 34)
    assert (g8 == w8).all(axis=1).mean() >= 0.99


def test_rope_append_matches_apply_rotary_pos_emb(N, cuda_device):
    from transformers.models.llama import modeling_llama as ml

    from torchnative_b200.llama_decode import rope_inv_freq

    B, Hq, Hkv, D, cap, pos, theta = 2, 8, 2, 128, 64, 37, 500000.0
    g = torch.Generator(device=cuda_device).manual_seed(3)
    qkv = torch.randn((B, (Hq + 2 * Hkv) * D), device=cuda_device, generator=g).to(torch.bfloat16)
    inv = rope_inv_freq(D, theta).to(cuda_device)
    q_out = torch.empty((B, Hq, D), device=cuda_device, dtype=torch.bfloat16)
    kc = torch.zeros((B, Hkv, cap, D), device=cuda_device, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    N.check(N.lib().tn_llama_rope_append(P(qkv.data_ptr()), P(inv.data_ptr()), None, pos, B, Hq, Hkv, D,
                                         P(q_out.data_ptr()), P(kc.data_ptr()), P(vc.data_ptr()), kc.stride(0),
                                         kc.stride(1), _stream()))
    # transformers: freqs = inv_freq x pos (float32), cos/sin -> bf16, q*cos + rotate_half(q)*sin in bf16
    freqs = inv[None, :] * torch.tensor([[float(pos)]], device=cuda_device)
    emb = torch.cat((freqs, freqs), dim=-1)
    cos, sin = emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)
    q = qkv[:, :Hq * D].view(B, Hq, 1, D)
    k = qkv[:, Hq * D:(Hq + Hkv) * D].view(B, Hkv, 1, D)
    v = qkv[:, (Hq + Hkv) * D:].view(B, Hkv, 1, D)
    qe, ke = ml.apply_rotary_pos_emb(q, k, cos[None], sin[None])
    assert torch.equal(q_out, qe[:, :, 0])
    assert torch.equal(kc[:, :, pos], ke[:, :, 0])
    assert torch.equal(vc[:, :, pos], v[:, :, 0])
    assert kc[:, :, :pos].abs().sum() == 0 and kc[:, :, pos + 1:].abs().sum() == 0


@pytest.mark.parametrize("V", [1000, 1003, 128256])
def test_argmax_embed_picks_the_first_maximum(N, cuda_device, V):
    B, H = 3, 64
    logits = torch.randn((B, V), device=cuda_device).to(torch.bfloat16)
    logits[1, 10] = 50.0
    logits[1, 700] = 50.0  # tie: the first index wins, as torch.argmax
    logits[2, V - 2] = 60.0
    logits[2, 17] = 60.0  # tie across the row: 17 (inside a 16-byte load with 16) wins
    logits[2, 16] = 59.0
    embed = torch.randn((V, H), device=cuda_device).to(torch.bfloat16)
    tokens = torch.zeros(B, dtype=torch.int32, device=cuda_device)
    h = torch.empty((B, H), device=cuda_device, dtype=torch.bfloat16)
    pos = torch.tensor([5], dtype=torch.int32, device=cuda_device)
    N.check(N.lib().tn_llama_argmax_embed(P(logits.data_ptr()), B, V, P(tokens.data_ptr()), P(embed.data_ptr()), H,
                                          P(h.data_ptr()), P(pos.data_ptr()), _stream()))
    want = torch.argmax(logits.float(), dim=-1)
    assert torch.equal(tokens.long(), want) and int(tokens[1]) == 10
    assert torch.equal(h, embed[want])
    assert int(pos.item()) == 6


def _host_reference_step(dec, tok, pos):
    """One decode token from the same weights, assembled on the host: glue in
    torch bf16 (transformers' definitions), every Q4_0 linear as the exact
    value of (Q8_0(x), W) rounded to bf16, SDPA in float64. Returns logits (f64)."""
    from transformers.models.llama import modeling_llama as ml

    s, dev = dec.s, "cpu"
    bf = torch.bfloat16

    def linear(x_bf, blob, n, k):
        x = x_bf.float().numpy()
        xq = oracle.q8_0_quantize(x)
        exact, _, _ = q4_exact.exact_linear_q4_0(xq, blob.cpu().numpy().tobytes(), x.shape[0], n, k)
        return torch.from_numpy(exact).to(bf)

    def norm(h, w):
        return _ref_rmsnorm(h, w.cpu(), s.eps)

    h = dec.embed.cpu()[tok]
    inv = dec.inv_freq.cpu()
    freqs = inv[None, :] * torch.tensor([[float(pos)]])
    emb = torch.cat((freqs, freqs), dim=-1)
    cos, sin = emb.cos().to(bf), emb.sin().to(bf)
    B, D, Hq, Hkv = tok.shape[0], s.head_dim, s.heads, s.kv_heads
    for li, lw in enumerate(dec.layers):
        x = norm(h, lw["attn_norm"])
        qkv = linear(x, lw["qkv"], s.qkv, s.hidden)
        q = qkv[:, :Hq * D].view(B, Hq, 1, D)
        k = qkv[:, Hq * D:(Hq + Hkv) * D].view(B, Hkv, 1, D)
        v = qkv[:, (Hq + Hkv) * D:].view(B, Hkv, 1, D)
        qe, ke = ml.apply_rotary_pos_emb(q, k, cos[None], sin[None])
        kc = dec.k_cache[li].cpu()[:, :, :pos + 1].clone()
        vc = dec.v_cache[li].cpu()[:, :, :pos + 1].clone()
        kc[:, :, pos], vc[:, :, pos] = ke[:, :, 0], v[:, :, 0]
        kk = kc.double().repeat_interleave(Hq // Hkv, 1)
        vv = vc.double().repeat_interleave(Hq // Hkv, 1)
        att = torch.softmax(qe.double() @ kk.transpose(-1, -2) / math.sqrt(D), -1) @ vv
        o = linear(att.to(bf).reshape(B, Hq * D), lw["o"], s.hidden, Hq * D)
        h = h + o
        x = norm(h, lw["mlp_norm"])
        gu = linear(x, lw["gate_up"], 2 * s.inter, s.hidden)  # rows interleaved: gate_i, up_i
        act = torch.nn.functional.silu(gu[:, 0::2]) * gu[:, 1::2]
        h = h + linear(act, lw["down"], s.hidden, s.inter)
    x = norm(h, dec.final_norm)
    xq = oracle.q8_0_quantize(x.float().numpy())
    exact, _, _ = q4_exact.exact_linear_q4_0(xq, dec.lm_head.cpu().numpy().tobytes(), B, s.vocab, s.hidden)
    return exact


@pytest.mark.parametrize("fused,B", [(True, 2), (False, 2), (False, 16)],
                         ids=["fused-5-kernels", "separate-11-kernels", "separate-11-kernels-batch16"])
def test_one_decode_step_of_a_small_q4_llama_against_the_host_reference(N, cuda_device, fused, B):
    from torchnative_b200.llama_decode import LlamaShape, Q4LlamaDecoder

    shape = LlamaShape(hidden=512, inter=1024, heads=8, kv_heads=2, head_dim=64, vocab=2048, layers=2,
                       rope_theta=10000.0)
    prompt = 40
    dec = Q4LlamaDecoder(shape, batch=B, capacity=64, device=cuda_device, seed=11)
    assert dec.fused == (B <= 4)
    dec.fused = fused
    dec.fill_prompt_cache(prompt)
    tok = torch.tensor([5, 1234] + [(97 * i + 11) % 2048 for i in range(B - 2)], dtype=torch.int32)
    ref = _host_reference_step(dec, tok.long(), prompt)
    dec.start(tok.to(cuda_device))
    dec.step()
    torch.cuda.synchronize()
    got = dec.logits.float().cpu().numpy().astype(np.float64)
    scale = np.max(np.abs(ref))
    assert np.max(np.abs(got - ref)) <= 0.05 * scale, np.max(np.abs(got - ref)) / scale
    top2 = np.sort(ref, axis=1)[:, -2:]
    for b in range(B):
        if top2[b, 1] - top2[b, 0] > 0.05 * scale:  # a clear winner must be the engine's token
            assert int(dec.tokens[b]) == int(np.argmax(ref[b]))
    assert int(dec.pos.item()) == prompt + 1
    N.device_status(reset=True)


@pytest.mark.parametrize("fused,B", [(True, 1), (False, 1), (False, 16)],
                         ids=["fused-5-kernels", "separate-11-kernels", "separate-11-kernels-batch16"])
def test_decode_step_replays_as_one_graph(N, cuda_device, fused, B):
    from torchnative_b200.llama_decode import LlamaShape, Q4LlamaDecoder

    shape = LlamaShape(hidden=512, inter=1024, heads=8, kv_heads=2, head_dim=64, vocab=2048, layers=2,
                       rope_theta=10000.0)
    dec = Q4LlamaDecoder(shape, batch=B, capacity=80, device=cuda_device, seed=12)
    dec.fused = fused
    first = (torch.arange(B, dtype=torch.int32, device=cuda_device) * 131 + 7) % 2048
    dec.fill_prompt_cache(30)
    dec.start(first)
    eager = []
    for _ in range(4):
        dec.step()
        eager.append(dec.tokens.tolist())
    dec.fill_prompt_cache(30)
    dec.start(first)
    g = dec.capture()
    dec.fill_prompt_cache(30)
    dec.start(first)
    replay = []
    for _ in range(4):
        g.replay()
        replay.append(dec.tokens.tolist())
    assert replay == eager
    assert int(dec.pos.item()) == 34


def test_decode_attention_writes_the_planar_q8_of_its_output(N, cuda_device):
    """tn_sdpa_decode_step_q8: the same bf16 output as tn_sdpa_decode_step,
    and codes / scales / offsets byte-identical to tn_q8_0_quantize_planar
    of that output (the o_proj GEMV then stages them directly)."""
    from torchnative_b200.llama_decode import rope_inv_freq

    g = torch.Generator().manual_seed(21)
    B, Hq, Hkv, D, cap = 2, 32, 8, 128, 300
    pos0 = 217
    dev = cuda_device
    qkv = torch.randn((B, (Hq + 2 * Hkv) * D), generator=g).to(torch.bfloat16).to(dev)
    kc = torch.randn((B, Hkv, cap, D), generator=g).to(torch.bfloat16).to(dev)
    vc = torch.randn((B, Hkv, cap, D), generator=g).to(torch.bfloat16).to(dev)
    inv = rope_inv_freq(D, 500000.0).to(dev)
    st = (ctypes.c_int64 * 4)(*kc.stride())
    outs = []
    for q8 in (False, True):
        k2, v2 = kc.clone(), vc.clone()
        pos = torch.tensor([pos0], dtype=torch.int32, device=dev)
        out = torch.empty((B, Hq, D), device=dev, dtype=torch.bfloat16)
        if q8:
            codes = torch.zeros((B, Hq * D), device=dev, dtype=torch.int8)
            scales = torch.zeros((B, Hq * D // 32), device=dev)
            offs = torch.zeros((B, Hq * D // 32), device=dev)
            N.check(N.lib().tn_sdpa_decode_step_q8(P(qkv.data_ptr()), P(inv.data_ptr()), P(k2.data_ptr()),
                                                   P(v2.data_ptr()), P(out.data_ptr()), None, P(codes.data_ptr()),
                                                   P(scales.data_ptr()), P(offs.data_ptr()), B, Hq, Hkv, D, cap, st, st,
                                                   P(pos.data_ptr()), 1.0 / math.sqrt(D), _stream()))
        else:
            N.check(N.lib().tn_sdpa_decode_step(P(qkv.data_ptr()), P(inv.data_ptr()), P(k2.data_ptr()),
                                                P(v2.data_ptr()), P(out.data_ptr()), None, B, Hq, Hkv, D, cap, st, st,
                                                P(pos.data_ptr()), 1.0 / math.sqrt(D), _stream()))
        outs.append(out)
    assert torch.equal(outs[0], outs[1])
    rc = torch.zeros_like(codes)
    rs, ro = torch.zeros_like(scales), torch.zeros_like(offs)
    K = Hq * D
    N.check(N.lib().tn_q8_0_quantize_planar(P(outs[1].data_ptr()), N.TN_BF16, K, P(rc.data_ptr()), K,
                                            P(rs.data_ptr()), P(ro.data_ptr()), B, K, _stream()))
    torch.cuda.synchronize()
    assert torch.equal(codes, rc) and torch.equal(scales, rs) and torch.equal(offs, ro)
    N.device_status(reset=True)


@pytest.mark.parametrize("mode,pairs,M,Nout,K", [
    ("rmsnorm", True, 1, 2 * 2048, 4096),   # LlamaMLP's gate/up, decode batch 1
    ("rmsnorm", True, 3, 2 * 1024, 512),
    ("rmsnorm", True, 2, 2 * 32 * 5, 256),  # 5 blocks: CTAs with and without a block
    ("bf16", False, 2, 4096, 1024),
    ("bf16", False, 4, 96, 256),
])
def test_gemv_writes_the_planar_q8_of_its_output(N, cuda_device, mode, pairs, M, Nout, K):
    """tn_q4_0_linear_fused_q8out: the same bf16 y as tn_q4_0_linear_fused, and
    codes / scales / offsets byte-identical to tn_q8_0_quantize_planar of that
    y (the down_proj GEMV stages them; the quantiser launch disappears)."""
    rng = np.random.default_rng(M * 131 + Nout + K)
    dev = cuda_device
    blob = q4_exact.random_q4_0_blob(rng, Nout, K)
    w = torch.frombuffer(bytearray(blob), dtype=torch.uint8).to(dev)
    x = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(torch.bfloat16).to(dev)
    delta = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32) * 0.5).to(torch.bfloat16).to(dev)
    nw = torch.from_numpy(1.0 + 0.1 * rng.standard_normal(K).astype(np.float32)).to(torch.bfloat16).to(dev)
    xm = N.TN_X_RMSNORM if mode == "rmsnorm" else N.TN_X_BF16
    flags = N.TN_WEIGHTS_STATIC | (N.TN_EPILOGUE_SILU_MUL_PAIRS if pairs else 0)
    cols = Nout // 2 if pairs else Nout
    ys = [torch.full((M, cols), float("nan"), device=dev, dtype=torch.bfloat16) for _ in range(2)]
    hs = [torch.zeros((M, K), device=dev, dtype=torch.bfloat16) for _ in range(2)]
    codes = torch.full((M, cols), 99, device=dev, dtype=torch.int8)
    scales = torch.full((M, cols // 32), -1.0, device=dev)
    offs = torch.full((M, cols // 32), -1.0, device=dev)
    common = lambda h, y: [xm, P(x.data_ptr()), K, P(delta.data_ptr()) if xm == N.TN_X_RMSNORM else None,  # noqa: E731
                           P(h.data_ptr()) if xm == N.TN_X_RMSNORM else None,
                           P(nw.data_ptr()) if xm == N.TN_X_RMSNORM else None, 1e-5, P(w.data_ptr()), None,
                           P(y.data_ptr()), N.TN_BF16, M, Nout, K, flags]
    N.check(N.lib().tn_q4_0_linear_fused(*common(hs[0], ys[0]), _stream()))
    N.check(N.lib().tn_q4_0_linear_fused_q8out(*common(hs[1], ys[1]), P(codes.data_ptr()), cols,
                                               P(scales.data_ptr()), P(offs.data_ptr()), _stream()))
    rc = torch.zeros_like(codes)
    rs, ro = torch.zeros_like(scales), torch.zeros_like(offs)
    N.check(N.lib().tn_q8_0_quantize_planar(P(ys[1].data_ptr()), N.TN_BF16, cols, P(rc.data_ptr()), cols,
                                            P(rs.data_ptr()), P(ro.data_ptr()), M, cols, _stream()))
    torch.cuda.synchronize()
    assert torch.equal(ys[0], ys[1]) and torch.equal(hs[0], hs[1])
    assert torch.equal(codes, rc) and torch.equal(scales, rs) and torch.equal(offs, ro)
    N.device_status(reset=True)


def test_gemv_planar_q8_output_refuses_what_it_cannot_quantise(N, cuda_device):
    """A float32 y, or y columns that are not whole 32-element blocks, are
    refused by name before anything is launched."""
    dev = cuda_device
    w = torch.zeros(64 * 8 * 18, device=dev, dtype=torch.uint8)
    x = torch.zeros((1, 256), device=dev, dtype=torch.bfloat16)
    y = torch.zeros((1, 64), device=dev)
    q = torch.zeros(64, device=dev, dtype=torch.int8)
    sc = torch.zeros(2, device=dev)

    def call(y_dtype, nout, flags):
        return N.lib().tn_q4_0_linear_fused_q8out(N.TN_X_BF16, P(x.data_ptr()), 256, None, None, None, 1e-5,
                                                  P(w.data_ptr()), None, P(y.data_ptr()), y_dtype, 1, nout, 256,
                                                  flags, P(q.data_ptr()), 64, P(sc.data_ptr()), P(sc.data_ptr()),
                                                  _stream())

    assert call(N.TN_F32, 64, 0) == N.TN_ERR_NOT_IMPLEMENTED
    assert "bf16" in N.last_error()
    assert call(N.TN_BF16, 48, 0) == N.TN_ERR_SHAPE
    assert call(N.TN_BF16, 32, N.TN_EPILOGUE_SILU_MUL_PAIRS) == N.TN_ERR_SHAPE  # 16 columns of act


@pytest.mark.parametrize("M,K", [(1, 4096), (3, 4096), (4, 4096), (2, 8192)])
@pytest.mark.parametrize("with_delta", [True, False])
def test_fused_rmsnorm_prologue_equals_the_separate_kernels(N, cuda_device, with_delta, M, K):
    """The q/k/v and gate/up GEMVs' fused RMSNorm + Q8_0 prologue (packed bf16
    arithmetic with all rows' loads in flight at once up to K = 4096, the
    per-element loop above) against tn_llama_add_rmsnorm_q8 + the planar GEMV
    (float arithmetic), bit for bit. Activations are multiples of 0.5, so the
    sum of squares is exact in any reduction order and both sides see the
    same rsqrt; every other rounding must then agree."""
    dev, Nout, eps = cuda_device, 512, 1e-5
    g = torch.Generator(device=dev).manual_seed(5 + M)
    x = (torch.randint(-4, 5, (M, K), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    d = (torch.randint(-2, 3, (M, K), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(K, generator=g, device=dev)).to(torch.bfloat16)
    blob = torch.frombuffer(bytearray(q4_exact.random_q4_0_blob(np.random.default_rng(6), Nout, K)),
                            dtype=torch.uint8).to(dev)
    delta = P(d.data_ptr()) if with_delta else None
    h1, h2 = torch.zeros_like(x), torch.zeros_like(x)
    y1 = torch.full((M, Nout), float("nan"), device=dev, dtype=torch.bfloat16)
    y2 = torch.full_like(y1, float("nan"))
    N.check(N.lib().tn_q4_0_linear_fused(N.TN_X_RMSNORM, P(x.data_ptr()), K, delta, P(h1.data_ptr()),
                                         P(w.data_ptr()), eps, P(blob.data_ptr()), None, P(y1.data_ptr()), N.TN_BF16,
                                         M, Nout, K, N.TN_WEIGHTS_STATIC, _stream()))
    codes = torch.empty((M, K), dtype=torch.int8, device=dev)
    sc, of = torch.empty((M, K // 32), device=dev), torch.empty((M, K // 32), device=dev)
    N.check(N.lib().tn_llama_add_rmsnorm_q8(P(x.data_ptr()), delta, P(h2.data_ptr()), P(w.data_ptr()), eps, M, K,
                                            P(codes.data_ptr()), P(sc.data_ptr()), P(of.data_ptr()), _stream()))
    N.check(N.lib().tn_q4_0_linear_q8(P(codes.data_ptr()), K, P(sc.data_ptr()), P(of.data_ptr()),
                                      P(blob.data_ptr()), None, P(y2.data_ptr()), N.TN_BF16, M, Nout, K,
                                      N.TN_WEIGHTS_STATIC, _stream()))
    torch.cuda.synchronize()
    assert torch.equal(h1, h2) and torch.equal(h1, x + d if with_delta else x)
    assert torch.equal(y1, y2)
    N.device_status(reset=True)


def test_fused_rmsnorm_refuses_a_misaligned_h_out(N, cuda_device):
    """h_out is written 16 bytes at a time: an unaligned one is refused before
    anything is launched."""
    dev, K = cuda_device, 256
    x = torch.zeros((1, K), device=dev, dtype=torch.bfloat16)
    h = torch.zeros(K + 1, device=dev, dtype=torch.bfloat16)
    w = torch.zeros(K, device=dev, dtype=torch.bfloat16)
    blob = torch.zeros(64 * K // 32 * 18, device=dev, dtype=torch.uint8)
    y = torch.zeros((1, 64), device=dev, dtype=torch.bfloat16)
    rc = N.lib().tn_q4_0_linear_fused(N.TN_X_RMSNORM, P(x.data_ptr()), K, None, P(h.data_ptr() + 2),
                                      P(w.data_ptr()), 1e-5, P(blob.data_ptr()), None, P(y.data_ptr()), N.TN_BF16,
                                      1, 64, K, 0, _stream())
    assert rc == N.TN_ERR_INVALID
    assert "16-byte aligned" in N.last_error()
