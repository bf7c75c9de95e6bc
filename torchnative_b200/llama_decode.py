"""One greedy decode token of a Llama-shaped model with Q4_0 linears, on the
device, as a single replayable CUDA graph.

This is the caller the two hot operators sit in (transformers'
LlamaForCausalLM driven by `generate`, with torchnative's QuantizedLinear in
every linear): per layer RMSNorm -> q/k/v (one fused Q4_0 linear) -> RoPE and
KV append -> SDPA against the cache -> o_proj -> residual -> RMSNorm ->
gate/up (one fused Q4_0 linear) -> SiLU*up -> down_proj -> residual; then the
final norm, lm_head and argmax. The KV cache is the reference's
PreallocatedCache layout (torchnative/python/torchnative/kernels/kv_cache.py:
51-185): one [B, Hkv, capacity, D] buffer per layer, read in place.

Weights are random (synthetic, seeded): Q4_0 blobs built directly in the
block layout (codes uniform in [-8, 7], scales f16(|N(0,1)| * 0.01)), bf16
norms and embeddings. The position counter lives on the device, so one
captured graph serves every step while the cache grows.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch

from . import _native as N

P = ctypes.c_void_p


@dataclass(frozen=True)
class LlamaShape:
    hidden: int
    inter: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    layers: int
    rope_theta: float
    eps: float = 1e-5

    @property
    def qkv(self) -> int:
        return (self.heads + 2 * self.kv_heads) * self.head_dim


LLAMA3_8B = LlamaShape(4096, 14336, 32, 8, 128, 128256, 32, 500000.0)
LLAMA3_70B = LlamaShape(8192, 28672, 64, 8, 128, 128256, 80, 500000.0)
SMOLLM2_135M = LlamaShape(576, 1536, 9, 3, 64, 49152, 30, 10000.0)


def q4_bytes(n: int, k: int) -> int:
    return n * k // 32 * 18


def random_q4_blob(n: int, k: int, gen: torch.Generator, dev) -> torch.Tensor:
    nb = k // 32
    qs = torch.randint(0, 256, (n, nb, 16), dtype=torch.uint8, device=dev, generator=gen)
    d = (torch.randn((n, nb, 1), device=dev, generator=gen).abs() * 0.01).to(torch.float16).view(torch.uint8)
    return torch.cat([d, qs], dim=2).reshape(-1).contiguous()


def rope_inv_freq(head_dim: int, theta: float) -> torch.Tensor:
    """transformers' default rotary inv_freq: 1 / theta^(arange(0, D, 2) / D), in float32."""
    return 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))


class Q4LlamaDecoder:
    """The decode step on one GPU, or on rank `tp.rank` of a tensor-parallel
    group (`tp` a torchnative_b200.tp.TPGroup): then q/k/v, gate/up and
    lm_head hold their column shards, attention its KV-head group, and o_proj
    and down_proj either their K-slices with the all-reduce fused into the
    GEMV (tp_plan "rowwise") or their column shards with an all-gather after
    each sharded output ("colwise"). The weights are generated in full from
    the seed and sliced, so every group size runs the same model."""

    def __init__(self, shape: LlamaShape, batch: int, capacity: int, device, seed: int = 0,
                 layers: int | None = None, tp=None, exchange: str = "p2p", weights: dict | None = None,
                 mega: bool | None = None, tp_plan: str = "rowwise"):
        """`weights` (from `from_gguf`): the full model's tensors on `device`
        -- per layer attn_norm, qkv, o, mlp_norm, gate_up, down as below, plus
        final_norm, lm_head, embed -- used instead of the seeded random ones.
        `mega`: run each token as the one persistent kernel
        (tn_llama_decode_token) -- True insists (one GPU, batch 1, a shape it
        supports); None and False keep the launch-per-operator step, which
        measures faster today. `tp_plan` (tensor parallel only): "rowwise"
        makes o_proj and down_proj row-parallel with their all-reduce fused
        into the GEMV (peer-memory exchange, batch <= 4; otherwise it falls
        back to "colwise"), "colwise" column-shards every linear with an
        all-gather after each (the one-GPU token stream bit for bit)."""
        from . import tp as tpm

        self.s = shape
        self.B, self.cap = batch, capacity
        self.dev = torch.device(device)
        self.n_layers = shape.layers if layers is None else layers
        self.tp = tp if tp is not None and tp.world > 1 else None
        G, r = (self.tp.world, self.tp.rank) if self.tp else (1, 0)
        self.G = G
        if tp_plan not in ("rowwise", "colwise"):
            raise ValueError(f"unknown tp_plan {tp_plan!r} (rowwise or colwise)")
        # rowwise at batch <= 4 (the fused five-launch step), and up to 16 rows
        # while the row-parallel K-slices still fit the GEMV's one-launch tile
        # (o_proj and down_proj carry the fused reduction; 16 rows of at most
        # 7168 columns)
        self.rowwise = (self.tp is not None and tp_plan == "rowwise" and exchange == "p2p" and
                        (batch <= 4 or (batch <= 16 and shape.inter // G <= 7168 and
                                        shape.heads // G * shape.head_dim <= 7168)))
        s, dev = shape, self.dev
        for n, what in ((s.heads, "query heads"), (s.kv_heads, "key/value heads"), (s.hidden, "hidden size"),
                        (s.inter, "intermediate size"), (s.vocab, "vocabulary")):
            if n % G != 0:
                raise ValueError(f"{what} ({n}) does not divide by the tensor-parallel size {G}")
        self.hq, self.hkv = s.heads // G, s.kv_heads // G   # local heads
        self.h_l, self.i_l, self.v_l = s.hidden // G, s.inter // G, s.vocab // G
        self.qkv_l = (self.hq + 2 * self.hkv) * s.head_dim
        # rowwise: SiLU*up's planar Q8_0 from gate/up's own epilogue needs whole
        # 32-column blocks per CTA, so gate/up runs on at most i_l / 32 CTAs.
        # Below half an SM's worth of blocks (Llama-3-8B on 8 ranks: 56)
        # down_proj quantises act in its own prologue instead. On 4 ranks (112
        # blocks) both ways measured alike: gate/up 10.1 -> 8.0 us, down 4.2 ->
        # 7.6 us, 679 -> 672 tok/s, so the epilogue keeps it there.
        self.rowwise_q8out = self.i_l // 32 >= 74
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed)
        bf = torch.bfloat16
        self.layers = []
        for li in range(self.n_layers):
            lw = dict(weights["layers"][li]) if weights is not None else {
                "attn_norm": (1.0 + 0.1 * torch.randn(s.hidden, device=dev, generator=gen)).to(bf),
                "qkv": random_q4_blob(s.qkv, s.hidden, gen, dev),
                "o": random_q4_blob(s.hidden, s.heads * s.head_dim, gen, dev),
                "mlp_norm": (1.0 + 0.1 * torch.randn(s.hidden, device=dev, generator=gen)).to(bf),
                # gate_proj and up_proj interleaved row by row (row 2i = gate_i,
                # row 2i+1 = up_i), so one GEMV writes SiLU(gate) * up directly
                "gate_up": random_q4_blob(2 * s.inter, s.hidden, gen, dev),
                "down": random_q4_blob(s.hidden, s.inter, gen, dev),
            }
            if G > 1:
                lw["qkv"] = tpm.shard_qkv(lw["qkv"], s.heads, s.kv_heads, s.head_dim, s.hidden, r, G)
                lw["gate_up"] = tpm.shard_gate_up_pairs(lw["gate_up"], s.inter, s.hidden, r, G)
                shard = tpm.shard_cols if self.rowwise else tpm.shard_rows
                lw["o"] = shard(lw["o"], s.hidden, s.heads * s.head_dim, r, G)
                lw["down"] = shard(lw["down"], s.hidden, s.inter, r, G)
            self.layers.append(lw)
        if weights is not None:
            self.final_norm, self.lm_head = weights["final_norm"], weights["lm_head"]
        else:
            self.final_norm = (1.0 + 0.1 * torch.randn(s.hidden, device=dev, generator=gen)).to(bf)
            self.lm_head = random_q4_blob(s.vocab, s.hidden, gen, dev)
        if G > 1:
            self.lm_head = tpm.shard_rows(self.lm_head, s.vocab, s.hidden, r, G)
        if weights is not None:
            self.embed = weights["embed"]
        else:
            self.embed = (0.02 * torch.randn((s.vocab, s.hidden), device=dev, generator=gen)).to(bf)
        self.k_cache = [torch.zeros((batch, self.hkv, capacity, s.head_dim), device=dev, dtype=bf)
                        for _ in range(self.n_layers)]
        self.v_cache = [torch.zeros_like(self.k_cache[0]) for _ in range(self.n_layers)]
        self.inv_freq = rope_inv_freq(s.head_dim, s.rope_theta).to(dev)
        B, H, I = batch, s.hidden, s.inter
        kmax = max(H, I, s.heads * s.head_dim)
        self.h = torch.zeros((B, H), device=dev, dtype=bf)
        self.h2 = torch.zeros((B, H), device=dev, dtype=bf)  # the residual's other half (ping-pong)
        # Gather destinations: with the peer-memory exchange they live in this
        # rank's IPC region, where every rank writes its slice directly.
        self.xchg = None
        if self.tp is not None and exchange == "p2p":
            nbytes = 2 * B * (s.heads * s.head_dim + H + I + s.vocab) + 4 * 256
            if self.rowwise:  # two partial buffers [B][G * H] of tagged 8-byte words, alternating
                nbytes += 2 * (B * G * H * 8 + 256)
            self.xchg = tpm.PeerExchange(self.tp, nbytes, dev)
            attn2d, self._off_attn = self.xchg.buffer(B, s.heads * s.head_dim)
            self.attn = attn2d.view(B, s.heads, 1, s.head_dim)
            self.delta, self._off_delta = self.xchg.buffer(B, H)
            self.act, self._off_act = self.xchg.buffer(B, I)
            self.logits, self._off_logits = self.xchg.buffer(B, s.vocab)
            for t in (self.attn, self.delta, self.act, self.logits):
                t.zero_()
            if self.rowwise:
                self._off_part = [self.xchg.reserve(B * G * H * 8) for _ in range(2)]
        elif self.tp is not None and exchange != "nccl":
            raise ValueError(f"unknown exchange {exchange!r} (p2p or nccl)")
        else:
            self.delta = torch.zeros((B, H), device=dev, dtype=bf)
        self.codes = torch.zeros((B, kmax), device=dev, dtype=torch.int8)
        self.scales = torch.zeros((B, kmax // 32), device=dev, dtype=torch.float32)
        self.offsets = torch.zeros((B, kmax // 32), device=dev, dtype=torch.float32)
        self.qkv_out = torch.zeros((B, self.qkv_l), device=dev, dtype=bf)
        self.q_rot = torch.zeros((B, self.hq, 1, s.head_dim), device=dev, dtype=bf)
        if self.xchg is None:
            self.attn = torch.zeros((B, s.heads, 1, s.head_dim), device=dev, dtype=bf)
            self.act = torch.zeros((B, I), device=dev, dtype=bf)
            self.logits = torch.zeros((B, s.vocab), device=dev, dtype=bf)
        if G > 1:  # each rank's slice of the sharded outputs, gathered into the full buffers above
            self.attn_l = torch.zeros((B, self.hq, 1, s.head_dim), device=dev, dtype=bf)
            self.delta_l = torch.zeros((B, self.h_l), device=dev, dtype=bf)
            self.act_l = torch.zeros((B, self.i_l), device=dev, dtype=bf)
            self.logits_l = torch.zeros((B, self.v_l), device=dev, dtype=bf)
            self.gather_scratch = torch.zeros(G * B * max(self.h_l, self.i_l, self.v_l, self.hq * s.head_dim),
                                              device=dev, dtype=bf)
        else:
            self.attn_l, self.delta_l, self.act_l, self.logits_l = self.attn, self.delta, self.act, self.logits
            self.gather_scratch = None
        self.tokens = torch.zeros(B, device=dev, dtype=torch.int32)
        self.pos = torch.zeros(1, device=dev, dtype=torch.int32)
        st = lambda t: (ctypes.c_int64 * 4)(*[0 if t.shape[i] == 1 and i < 3 else t.stride(i) for i in range(4)])  # noqa: E731
        self._qstr = st(self.q_rot)
        self._kstr = st(self.k_cache[0])
        self._graph = None
        # Up to 4 rows, RMSNorm and the activation quantisation run inside the
        # Q4_0 GEMVs, SiLU*up in the gate/up GEMV's epilogue, and RoPE/append/
        # split-merge inside the SDPA launch: 6 kernels a layer. Larger batches
        # use the separate kernels.
        self.fused = batch <= 4
        # With the peer-memory exchange, the o_proj and down_proj gathers run
        # inside those GEMVs (rows scattered to every rank, the next RMSNorm GEMV
        # waits); the attention, SiLU*up and logits gathers stay separate launches.
        self.fused_gather = self.fused and self.xchg is not None
        self._links = self._build_links()
        self._mega = None
        if mega and self.tp is None and batch == 1:
            self._mega_plan()
        elif mega:
            raise NotImplementedError("the persistent decode kernel runs batch 1 on one GPU")

    # ---- the persistent whole-token kernel (batch 1, one GPU)

    def _mega_plan(self) -> None:
        s, n = self.s, self.n_layers
        lib = N.lib()
        keep = []

        def arr(ts):
            a = (ctypes.c_void_p * n)(*[t.data_ptr() for t in ts])
            keep.append(a)
            return ctypes.cast(a, ctypes.POINTER(ctypes.c_void_p))

        L = self.layers
        m = N.LlamaQ4Model(layers=n, hidden=s.hidden, inter=s.inter, heads=s.heads, kv_heads=s.kv_heads,
                           head_dim=s.head_dim, vocab=s.vocab, eps=s.eps, embed=self.embed.data_ptr(),
                           final_norm=self.final_norm.data_ptr(), lm_head=self.lm_head.data_ptr(),
                           attn_norm=arr([lw["attn_norm"] for lw in L]), qkv=arr([lw["qkv"] for lw in L]),
                           o=arr([lw["o"] for lw in L]), mlp_norm=arr([lw["mlp_norm"] for lw in L]),
                           gate_up=arr([lw["gate_up"] for lw in L]), down=arr([lw["down"] for lw in L]),
                           k_cache=arr(self.k_cache), v_cache=arr(self.v_cache), capacity=self.cap,
                           inv_freq=self.inv_freq.data_ptr())
        lo = N.DecodeLayout()
        N.check(lib.tn_llama_decode_layout_of(ctypes.byref(m), ctypes.byref(lo)))
        self.mega_ws = torch.zeros(lo.total, dtype=torch.uint8, device=self.dev)
        plan = ctypes.c_void_p()
        N.check(lib.tn_llama_decode_plan(ctypes.byref(m), P(self.mega_ws.data_ptr()), lo.total, ctypes.byref(plan)))
        self._mega, self._mega_layout, self._mega_keep = plan, lo, (m, keep)

    @property
    def mega(self) -> bool:
        return self._mega is not None

    def mega_views(self) -> dict:
        """The persistent kernel's intermediates after a token (views of its
        workspace): h, qkv, attn, o_out, act, down_out (bf16) and the planar
        Q8_0 of attn (aq, ad, ac) and act (gq, gd, gc) -- the last layer's."""
        lo, s, ws = self._mega_layout, self.s, self.mega_ws
        HD, QKV = s.heads * s.head_dim, s.qkv

        def v(off, n, dt):
            return ws[off:off + n * torch.empty((), dtype=dt).element_size()].view(dt)

        bf = torch.bfloat16
        return {"h": v(lo.h, s.hidden, bf), "qkv": v(lo.qkv, QKV, bf), "attn": v(lo.attn, HD, bf),
                "o_out": v(lo.o_out, s.hidden, bf), "act": v(lo.act, s.inter, bf),
                "down_out": v(lo.down_out, s.hidden, bf), "aq": v(lo.aq, HD, torch.int8),
                "ad": v(lo.ad, HD // 32, torch.float32), "ac": v(lo.ac, HD // 32, torch.float32),
                "gq": v(lo.gq, s.inter, torch.int8), "gd": v(lo.gd, s.inter // 32, torch.float32),
                "gc": v(lo.gc, s.inter // 32, torch.float32)}

    def mega_trace_bytes(self) -> int:
        return int(N.lib().tn_llama_decode_trace_bytes(self._mega))

    def mega_reset(self) -> None:
        """Zero the kernel's barrier counter, epoch and merge tickets (after a
        launch that recorded a timeout)."""
        N.check(N.lib().tn_llama_decode_reset(self._mega, self._stream()))

    def _step_mega(self, stream, trace=None, trace_layer: int = -1) -> None:
        N.check(N.lib().tn_llama_decode_token(self._mega, P(self.tokens.data_ptr()), P(self.pos.data_ptr()),
                                              P(self.logits.data_ptr()), None if trace is None else
                                              P(trace.data_ptr()), trace_layer, stream))

    def _off(self, full: torch.Tensor) -> int:
        return {self.attn.data_ptr(): self._off_attn, self.delta.data_ptr(): self._off_delta,
                self.act.data_ptr(): self._off_act, self.logits.data_ptr(): self._off_logits}[full.data_ptr()]

    def _gather(self, local: torch.Tensor, full: torch.Tensor, slot: int, stream) -> None:
        """The all-gather after a sharded output (nothing on one GPU). Slots
        number the gathers of a step: 4 per layer (attention, o_proj, SiLU*up,
        down_proj), then the logits."""
        if self.tp is None:
            return
        local2d, full2d = local.reshape(self.B, -1), full.view(self.B, -1)
        if self.xchg is not None:
            self.xchg.allgather(local2d, self._off(full), full2d.shape[1], slot, stream)
            return
        from . import tp as tpm

        tpm.gather_rows(self.tp, local2d, full2d, self.gather_scratch, stream)

    def _link(self, slot: int = -1, full: torch.Tensor | None = None, wait_slot: int = -1):
        """tn_tp_link for a GEMV whose output feeds gather `slot` (written into
        `full` on every rank) and/or that reads gather `wait_slot`; None when
        the gathers are not fused (one GPU, or NCCL)."""
        if self.xchg is None or not self.fused_gather:
            return None
        if slot >= 0:
            return self.xchg.link(slot, self._off(full), full.view(self.B, -1).shape[1], wait_slot)
        return self.xchg.link(wait_slot=wait_slot)

    def _step_end(self, stream) -> None:
        if self.xchg is not None:
            self.xchg.step_end(stream)

    def close(self) -> None:
        """Release the peer-memory exchange (call on every rank after a
        barrier, with no step in flight and no graph left that uses it) and
        the persistent kernel's plan."""
        self._graph = None
        if self._mega is not None:
            N.lib().tn_llama_decode_plan_free(self._mega)
            self._mega = None
        if self.xchg is not None:
            self.xchg.close()
            self.xchg = None

    # ---- bookkeeping

    @property
    def weight_bytes(self) -> int:
        """HBM bytes of this rank's weights read per step (its shards, plus the
        replicated norms)."""
        s, G = self.s, self.G
        per_layer = (q4_bytes(self.qkv_l, s.hidden) + q4_bytes(self.h_l, s.heads * s.head_dim) +
                     q4_bytes(2 * self.i_l, s.hidden) + q4_bytes(self.h_l, s.inter) + 2 * 2 * s.hidden)
        return per_layer * self.n_layers + q4_bytes(self.v_l, s.hidden) + 2 * s.hidden

    def kv_bytes(self, length: int) -> int:
        s = self.s
        return 2 * self.n_layers * self.B * self.hkv * length * s.head_dim * 2

    @property
    def kernels_per_layer(self) -> int:
        """Our kernels per layer: the peer-memory all-gathers are ours, NCCL's
        are not (they add the layout step at batch > 1)."""
        if self.xchg is not None:
            extra = 2 if self.fused_gather else 4
        else:
            extra = 4 if (self.tp is not None and self.B > 1) else 0
        if self._mega is not None:
            return 0  # the whole token is one launch (kernels_per_step)
        if self.rowwise:  # both reductions inside the GEMVs
            return 5 if self.fused else 10
        if self.fused:
            # one GPU: gate/up also writes the planar Q8_0 of act (no quantiser launch)
            return (5 if self.tp is None else 6) + extra
        return 11 + extra

    @property
    def kernels_per_step(self) -> int:
        if self._mega is not None:
            return 1
        if self.xchg is not None:
            extra = 2  # the logits gather and the epoch step
        else:
            extra = 1 if (self.tp is not None and self.B > 1) else 0
        return self.kernels_per_layer * self.n_layers + (2 if self.fused else 3) + extra

    @classmethod
    def from_gguf(cls, path, batch: int, capacity: int, device, layers: int | None = None, tp=None,
                  exchange: str = "p2p") -> "Q4LlamaDecoder":
        """A decoder whose weights are a llama GGUF file's own tensors
        (transformers' GGUF tensor map for llama: blk.N.attn_q / attn_k /
        attn_v / attn_output / ffn_gate / ffn_up / ffn_down / attn_norm /
        ffn_norm, token_embd, output_norm, output). Every linear must be Q4_0;
        its blocks reach HBM byte for byte (torchnative_b200.gguf), q and k with
        llama.cpp's rotary row order undone by rows, then q/k/v rows are
        concatenated and gate/up rows interleaved as the fused kernels read
        them. Norms are held in bf16 (transformers' dtype=bfloat16 load) and the
        embedding is dequantised to bf16. A missing `output` ties lm_head to
        token_embd, as transformers does."""
        from . import gguf as G

        dev = torch.device(device)
        bf = torch.bfloat16
        with G.GGUFContainer(path) as f:
            md = f.metadata
            if md.get("general.architecture") != "llama":
                raise G.GGUFUnsupported(f"{f.path}: architecture {md.get('general.architecture')!r}; the decode "
                                        "engine runs llama")

            def need(key):
                if key not in md:
                    raise G.GGUFMalformed(f"{f.path}: metadata {key!r} is missing")
                return md[key]

            H, I = int(need("llama.embedding_length")), int(need("llama.feed_forward_length"))
            heads = int(need("llama.attention.head_count"))
            kv = int(md.get("llama.attention.head_count_kv", heads))
            n_layers = int(need("llama.block_count"))
            vocab = f.slot("token_embd.weight").shape[0]
            shape = LlamaShape(H, I, heads, kv, int(md.get("llama.attention.key_length", H // heads)), vocab, n_layers,
                               float(md.get("llama.rope.freq_base", 10000.0)),
                               float(md.get("llama.attention.layer_norm_rms_epsilon", 1e-5)))

            def q4(name, heads_perm=None):
                info = f.slot(name)
                if info.block_format != "q4_0":
                    raise G.GGUFUnsupported(f"{f.path}: {name} is {info.type_name}; the decode engine's linears "
                                            "are Q4_0")
                return G.load_tensor(f, name, keep_blocks=True, permute_heads=heads_perm, device=dev).blob

            def dense_bf16(name):
                t = G.load_tensor(f, name, keep_blocks=False, device=dev)
                return t.to(bf).contiguous()

            lw_all = []
            for li in range(n_layers if layers is None else layers):
                b = f"blk.{li}."
                gate, up = q4(b + "ffn_gate.weight"), q4(b + "ffn_up.weight")
                row = len(gate) // I
                lw_all.append({
                    "attn_norm": dense_bf16(b + "attn_norm.weight"),
                    "qkv": torch.cat([q4(b + "attn_q.weight", heads), q4(b + "attn_k.weight", kv),
                                      q4(b + "attn_v.weight")]),
                    "o": q4(b + "attn_output.weight"),
                    "mlp_norm": dense_bf16(b + "ffn_norm.weight"),
                    "gate_up": torch.stack([gate.view(I, row), up.view(I, row)], dim=1).reshape(-1).contiguous(),
                    "down": q4(b + "ffn_down.weight"),
                })
            lm = "output.weight" if "output.weight" in f.tensors else "token_embd.weight"
            weights = {"layers": lw_all, "final_norm": dense_bf16("output_norm.weight"), "lm_head": q4(lm),
                       "embed": dense_bf16("token_embd.weight")}
        return cls(shape, batch, capacity, dev, layers=layers, tp=tp, exchange=exchange, weights=weights)

    def fill_prompt_cache(self, length: int, seed: int = 1) -> None:
        """The prompt's K/V: synthetic N(0,1) values in slots [0, length), and
        the position set to `length` (the decode loop continues from there)."""
        g = torch.Generator(device=self.dev)
        g.manual_seed(seed)
        s = self.s
        h0 = (self.tp.rank if self.tp else 0) * self.hkv  # this rank's KV heads of the full cache
        for kc, vc in zip(self.k_cache, self.v_cache):
            for c in (kc, vc):
                full = torch.empty((self.B, s.kv_heads, length, s.head_dim), device=self.dev, dtype=c.dtype)
                full.normal_(generator=g)
                c[:, :, :length].copy_(full[:, h0:h0 + self.hkv])
        self.pos.fill_(length)

    def start(self, tokens: torch.Tensor) -> None:
        """Embed the first tokens (one per sequence)."""
        self.tokens.copy_(tokens.to(torch.int32))
        N.check(N.lib().tn_llama_embed(P(self.tokens.data_ptr()), self.B, P(self.embed.data_ptr()), self.s.hidden,
                                       P(self.h.data_ptr()), self._stream()))

    # ---- the step

    @staticmethod
    def _stream():
        return P(torch.cuda.current_stream().cuda_stream)

    def _linear(self, w, y, n, k, stream, flags=0, link=None):
        N.check(N.lib().tn_q4_0_linear_q8_tp(P(self.codes.data_ptr()), k, P(self.scales.data_ptr()),
                                             P(self.offsets.data_ptr()), P(w.data_ptr()), None, P(y.data_ptr()),
                                             N.TN_BF16, self.B, n, k, N.TN_WEIGHTS_STATIC | flags,
                                             None if link is None else ctypes.addressof(link), stream))

    def _norm(self, delta, weight, stream):
        N.check(N.lib().tn_llama_add_rmsnorm_q8(P(self.h.data_ptr()), None if delta is None else P(delta.data_ptr()),
                                                P(self.h.data_ptr()), P(weight.data_ptr()), self.s.eps, self.B,
                                                self.s.hidden, P(self.codes.data_ptr()), P(self.scales.data_ptr()),
                                                P(self.offsets.data_ptr()), stream))

    def step(self, stream=None) -> None:
        """One token for every sequence: reads tokens' embeddings in self.h and
        the position self.pos; leaves the next tokens in self.tokens, their
        embeddings in self.h, and self.pos advanced by one."""
        if self._mega is not None:
            return self._step_mega(stream or self._stream())
        if self.fused:
            return self._step_fused(stream or self._stream())
        if self.rowwise:
            return self._step_rowwise_rows(stream or self._stream())
        L, s, B = N.lib(), self.s, self.B
        stream = stream or self._stream()
        D, Hq, Hkv = s.head_dim, self.hq, self.hkv  # local heads
        for li, lw in enumerate(self.layers):
            self._norm(None if li == 0 else self.delta, lw["attn_norm"], stream)
            self._linear(lw["qkv"], self.qkv_out, self.qkv_l, s.hidden, stream)
            kc, vc = self.k_cache[li], self.v_cache[li]
            N.check(L.tn_llama_rope_append(P(self.qkv_out.data_ptr()), P(self.inv_freq.data_ptr()),
                                           P(self.pos.data_ptr()), 0, B, Hq, Hkv, D, P(self.q_rot.data_ptr()),
                                           P(kc.data_ptr()), P(vc.data_ptr()), kc.stride(0), kc.stride(1), stream))
            N.check(L.tn_sdpa_decode_cache(P(self.q_rot.data_ptr()), P(kc.data_ptr()), P(vc.data_ptr()),
                                           P(self.attn_l.data_ptr()), None, N.TN_BF16, B, Hq, Hkv, D, self.cap,
                                           self._qstr, self._kstr, self._kstr, P(self.pos.data_ptr()), 1,
                                           1.0 / math.sqrt(D), stream))
            self._gather(self.attn_l, self.attn, 4 * li, stream)
            HD = s.heads * D
            N.check(L.tn_q8_0_quantize_planar(P(self.attn.data_ptr()), N.TN_BF16, HD, P(self.codes.data_ptr()),
                                              HD, P(self.scales.data_ptr()), P(self.offsets.data_ptr()), B, HD,
                                              stream))
            self._linear(lw["o"], self.delta_l, self.h_l, HD, stream)
            self._gather(self.delta_l, self.delta, 4 * li + 1, stream)
            self._norm(self.delta, lw["mlp_norm"], stream)
            self._linear(lw["gate_up"], self.act_l, 2 * self.i_l, s.hidden, stream, N.TN_EPILOGUE_SILU_MUL_PAIRS)
            self._gather(self.act_l, self.act, 4 * li + 2, stream)
            N.check(L.tn_q8_0_quantize_planar(P(self.act.data_ptr()), N.TN_BF16, s.inter, P(self.codes.data_ptr()),
                                              s.inter, P(self.scales.data_ptr()), P(self.offsets.data_ptr()), B,
                                              s.inter, stream))
            self._linear(lw["down"], self.delta_l, self.h_l, s.inter, stream)
            self._gather(self.delta_l, self.delta, 4 * li + 3, stream)
        self._norm(self.delta, self.final_norm, stream)
        self._linear(self.lm_head, self.logits_l, self.v_l, s.hidden, stream)
        self._gather(self.logits_l, self.logits, 4 * self.n_layers, stream)
        N.check(L.tn_llama_argmax_embed(P(self.logits.data_ptr()), B, s.vocab, P(self.tokens.data_ptr()),
                                        P(self.embed.data_ptr()), s.hidden, P(self.h.data_ptr()),
                                        P(self.pos.data_ptr()), stream))
        self._step_end(stream)

    def _fused_linear(self, mode, x, x_stride, delta, h_out, norm_w, w, y, n, k, stream, flags=0, link=None,
                      q8=False):
        if q8:
            # also the planar Q8_0 of y (the next linear's activations) from the same launch
            cols = n // 2 if flags & N.TN_EPILOGUE_SILU_MUL_PAIRS else n
            N.check(N.lib().tn_q4_0_linear_fused_q8out(
                mode, P(x.data_ptr()), x_stride, None if delta is None else P(delta.data_ptr()),
                None if h_out is None else P(h_out.data_ptr()), None if norm_w is None else P(norm_w.data_ptr()),
                self.s.eps, P(w.data_ptr()), None, P(y.data_ptr()), N.TN_BF16, self.B, n, k,
                N.TN_WEIGHTS_STATIC | flags, P(self.codes.data_ptr()), cols, P(self.scales.data_ptr()),
                P(self.offsets.data_ptr()), stream))
            return
        N.check(N.lib().tn_q4_0_linear_fused_tp(mode, P(x.data_ptr()), x_stride,
                                                None if delta is None else P(delta.data_ptr()),
                                                None if h_out is None else P(h_out.data_ptr()),
                                                None if norm_w is None else P(norm_w.data_ptr()), self.s.eps,
                                                P(w.data_ptr()), None, P(y.data_ptr()), N.TN_BF16, self.B, n, k,
                                                N.TN_WEIGHTS_STATIC | flags,
                                                None if link is None else ctypes.addressof(link), stream))

    def _step_rowwise(self, stream) -> None:
        """The tensor-parallel step under the rowwise plan, the one-GPU fused
        step's five launches a layer on this rank's shards: q/k/v and gate/up
        column-sharded, attention on the local heads writing their planar
        Q8_0 (o_proj's K-slice), SiLU*up's planar Q8_0 local (down_proj's
        K-slice), o_proj and down_proj each ending in the all-reduce fused
        into the GEMV, so the replicated residual stream reads `delta` in
        stream order. Only the logits are gathered."""
        L, s, B = N.lib(), self.s, self.B
        D, Hq, Hkv, H = s.head_dim, self.hq, self.hkv, s.hidden
        ha, hb = self.h, self.h2
        links = self._links
        q8out = self.rowwise_q8out
        for li, lw in enumerate(self.layers):
            self._fused_linear(N.TN_X_RMSNORM, ha, H, None if li == 0 else self.delta, hb, lw["attn_norm"],
                               lw["qkv"], self.qkv_out, self.qkv_l, H, stream)
            kc, vc = self.k_cache[li], self.v_cache[li]
            N.check(L.tn_sdpa_decode_step_q8(P(self.qkv_out.data_ptr()), P(self.inv_freq.data_ptr()),
                                             P(kc.data_ptr()), P(vc.data_ptr()), P(self.attn_l.data_ptr()), None,
                                             P(self.codes.data_ptr()), P(self.scales.data_ptr()),
                                             P(self.offsets.data_ptr()), B, Hq, Hkv, D, self.cap, self._kstr,
                                             self._kstr, P(self.pos.data_ptr()), 1.0 / math.sqrt(D), stream))
            self._linear(lw["o"], self.delta, H, Hq * D, stream, link=links[("o", li)])
            self._fused_linear(N.TN_X_RMSNORM, hb, H, self.delta, ha, lw["mlp_norm"], lw["gate_up"], self.act_l,
                               2 * self.i_l, H, stream, N.TN_EPILOGUE_SILU_MUL_PAIRS, q8=q8out)
            if q8out:
                self._linear(lw["down"], self.delta, H, self.i_l, stream, link=links[("down", li)])
            else:
                self._fused_linear(N.TN_X_BF16, self.act_l, self.i_l, None, None, None, lw["down"], self.delta, H,
                                   self.i_l, stream, link=links[("down", li)])
        self._fused_linear(N.TN_X_RMSNORM, ha, H, self.delta, hb, self.final_norm, self.lm_head, self.logits_l,
                           self.v_l, H, stream)
        self._gather(self.logits_l, self.logits, 0, stream)
        N.check(L.tn_llama_argmax_embed(P(self.logits.data_ptr()), B, s.vocab, P(self.tokens.data_ptr()),
                                        P(self.embed.data_ptr()), s.hidden, P(ha.data_ptr()),
                                        P(self.pos.data_ptr()), stream))
        self._step_end(stream)

    def _step_rowwise_rows(self, stream) -> None:
        """The rowwise plan for 5 to 16 rows: the separate-kernel step (RMSNorm
        + Q8_0 launches, the tensor-core skinny kernel for q/k/v and gate/up on
        this rank's columns, RoPE + append, split-KV attention on the local
        heads), with o_proj and down_proj row-parallel GEMVs whose reduction
        is fused in (their K-slices are the local heads' attention output and
        the local SiLU*up columns, each quantised once). 10 launches a layer,
        2 exchanges, where the colwise step has 15 launches and 4 gathers."""
        L, s, B = N.lib(), self.s, self.B
        D, Hq, Hkv, H = s.head_dim, self.hq, self.hkv, s.hidden
        HD = Hq * D
        links = self._links
        for li, lw in enumerate(self.layers):
            self._norm(None if li == 0 else self.delta, lw["attn_norm"], stream)
            self._linear(lw["qkv"], self.qkv_out, self.qkv_l, H, stream)
            kc, vc = self.k_cache[li], self.v_cache[li]
            N.check(L.tn_llama_rope_append(P(self.qkv_out.data_ptr()), P(self.inv_freq.data_ptr()),
                                           P(self.pos.data_ptr()), 0, B, Hq, Hkv, D, P(self.q_rot.data_ptr()),
                                           P(kc.data_ptr()), P(vc.data_ptr()), kc.stride(0), kc.stride(1), stream))
            N.check(L.tn_sdpa_decode_cache(P(self.q_rot.data_ptr()), P(kc.data_ptr()), P(vc.data_ptr()),
                                           P(self.attn_l.data_ptr()), None, N.TN_BF16, B, Hq, Hkv, D, self.cap,
                                           self._qstr, self._kstr, self._kstr, P(self.pos.data_ptr()), 1,
                                           1.0 / math.sqrt(D), stream))
            N.check(L.tn_q8_0_quantize_planar(P(self.attn_l.data_ptr()), N.TN_BF16, HD, P(self.codes.data_ptr()), HD,
                                              P(self.scales.data_ptr()), P(self.offsets.data_ptr()), B, HD, stream))
            self._linear(lw["o"], self.delta, H, HD, stream, link=links[("o", li)])
            self._norm(self.delta, lw["mlp_norm"], stream)
            self._linear(lw["gate_up"], self.act_l, 2 * self.i_l, H, stream, N.TN_EPILOGUE_SILU_MUL_PAIRS)
            N.check(L.tn_q8_0_quantize_planar(P(self.act_l.data_ptr()), N.TN_BF16, self.i_l,
                                              P(self.codes.data_ptr()), self.i_l, P(self.scales.data_ptr()),
                                              P(self.offsets.data_ptr()), B, self.i_l, stream))
            self._linear(lw["down"], self.delta, H, self.i_l, stream, link=links[("down", li)])
        self._norm(self.delta, self.final_norm, stream)
        self._linear(self.lm_head, self.logits_l, self.v_l, H, stream)
        self._gather(self.logits_l, self.logits, 0, stream)
        N.check(L.tn_llama_argmax_embed(P(self.logits.data_ptr()), B, s.vocab, P(self.tokens.data_ptr()),
                                        P(self.embed.data_ptr()), s.hidden, P(self.h.data_ptr()),
                                        P(self.pos.data_ptr()), stream))
        self._step_end(stream)

    def _step_fused(self, stream) -> None:
        if self.rowwise:
            return self._step_rowwise(stream)
        L, s, B = N.lib(), self.s, self.B
        D, Hq, Hkv, H, I = s.head_dim, self.hq, self.hkv, s.hidden, s.inter  # local heads
        HD = s.heads * D
        ha, hb = self.h, self.h2
        fg = self.xchg is not None and self.fused_gather
        links = self._links  # built once per (decoder); ctypes structs must outlive the launches
        for li, lw in enumerate(self.layers):
            # residual: hb = ha + (previous layer's down_proj); qkv = Q4(RMSNorm(hb))
            self._fused_linear(N.TN_X_RMSNORM, ha, H, None if li == 0 else self.delta, hb, lw["attn_norm"],
                               lw["qkv"], self.qkv_out, self.qkv_l, H, stream,
                               link=links[("qkv", li)] if fg and li > 0 else None)
            kc, vc = self.k_cache[li], self.v_cache[li]
            if self.tp is None:
                # one GPU: the attention's merging CTAs also write its planar Q8_0,
                # and o_proj stages those codes (no per-CTA bf16 -> Q8 prologue)
                N.check(L.tn_sdpa_decode_step_q8(P(self.qkv_out.data_ptr()), P(self.inv_freq.data_ptr()),
                                                 P(kc.data_ptr()), P(vc.data_ptr()), P(self.attn.data_ptr()), None,
                                                 P(self.codes.data_ptr()), P(self.scales.data_ptr()),
                                                 P(self.offsets.data_ptr()), B, Hq, Hkv, D, self.cap, self._kstr,
                                                 self._kstr, P(self.pos.data_ptr()), 1.0 / math.sqrt(D), stream))
                self._linear(lw["o"], self.delta, H, HD, stream)
            else:
                N.check(L.tn_sdpa_decode_step(P(self.qkv_out.data_ptr()), P(self.inv_freq.data_ptr()),
                                              P(kc.data_ptr()), P(vc.data_ptr()), P(self.attn_l.data_ptr()), None, B,
                                              Hq, Hkv, D, self.cap, self._kstr, self._kstr, P(self.pos.data_ptr()),
                                              1.0 / math.sqrt(D), stream))
                self._gather(self.attn_l, self.attn, 4 * li, stream)
                self._fused_linear(N.TN_X_BF16, self.attn, HD, None, None, None, lw["o"], self.delta_l, self.h_l, HD,
                                   stream, link=links[("o", li)] if fg else None)
            if not fg:
                self._gather(self.delta_l, self.delta, 4 * li + 1, stream)
            # residual: ha = hb + o_proj; act = SiLU(gate) * up of Q4(RMSNorm(ha))
            if self.tp is None:
                # one GPU: the same launch writes act's planar Q8_0 block by block
                # (each CTA owns whole 32-column blocks), which down_proj stages
                self._fused_linear(N.TN_X_RMSNORM, hb, H, self.delta, ha, lw["mlp_norm"], lw["gate_up"], self.act,
                                   2 * I, H, stream, N.TN_EPILOGUE_SILU_MUL_PAIRS, q8=True)
            else:
                self._fused_linear(N.TN_X_RMSNORM, hb, H, self.delta, ha, lw["mlp_norm"], lw["gate_up"], self.act_l,
                                   2 * self.i_l, H, stream, N.TN_EPILOGUE_SILU_MUL_PAIRS,
                                   link=links[("gate_up", li)] if fg else None)
                self._gather(self.act_l, self.act, 4 * li + 2, stream)
                # the activation quantiser once (not in each of the down GEMV's
                # CTAs: 448 blocks per CTA cost more than a launch)
                N.check(L.tn_q8_0_quantize_planar(P(self.act.data_ptr()), N.TN_BF16, I, P(self.codes.data_ptr()), I,
                                                  P(self.scales.data_ptr()), P(self.offsets.data_ptr()), B, I,
                                                  stream))
            self._linear(lw["down"], self.delta_l, self.h_l, I, stream, link=links[("down", li)] if fg else None)
            if not fg:
                self._gather(self.delta_l, self.delta, 4 * li + 3, stream)
        self._fused_linear(N.TN_X_RMSNORM, ha, H, self.delta, hb, self.final_norm, self.lm_head, self.logits_l,
                           self.v_l, H, stream, link=links[("lm_head", 0)] if fg else None)
        self._gather(self.logits_l, self.logits, 4 * self.n_layers, stream)
        N.check(L.tn_llama_argmax_embed(P(self.logits.data_ptr()), B, s.vocab, P(self.tokens.data_ptr()),
                                        P(self.embed.data_ptr()), s.hidden, P(ha.data_ptr()),
                                        P(self.pos.data_ptr()), stream))
        self._step_end(stream)

    def _build_links(self) -> dict:
        """Under the rowwise plan, the reduce links of o_proj and down_proj.
        Otherwise the fused gathers' links: o_proj and down_proj scatter their
        rows into every rank's `delta` (slots 4l + 1, 4l + 3); the next RMSNorm
        GEMV (gate/up, the next layer's q/k/v, lm_head) waits for them."""
        if self.rowwise:  # reductions 2l (o_proj) and 2l + 1 (down_proj), alternating partial buffers
            links = {}
            for li in range(self.n_layers):
                links[("o", li)] = self.xchg.reduce_link(2 * li, self._off_part[0], self.s.hidden)
                links[("down", li)] = self.xchg.reduce_link(2 * li + 1, self._off_part[1], self.s.hidden)
            return links
        if self.xchg is None or not self.fused_gather:
            return {}
        links = {}
        for li in range(self.n_layers):
            links[("o", li)] = self._link(slot=4 * li + 1, full=self.delta)
            links[("gate_up", li)] = self._link(wait_slot=4 * li + 1)
            links[("down", li)] = self._link(slot=4 * li + 3, full=self.delta)
            if li > 0:
                links[("qkv", li)] = self._link(wait_slot=4 * (li - 1) + 3)
        links[("lm_head", 0)] = self._link(wait_slot=4 * (self.n_layers - 1) + 3)
        return links

    def kernel_graphs(self) -> dict:
        """For timing the step's parts: one CUDA graph per kind of launch in
        the fused step, each running that launch once per layer with the
        step's own arguments (so 32 back-to-back launches over 32 layers'
        weights). Reads and writes the step's buffers; re-seed afterwards.
        Under the rowwise tensor-parallel plan the same launches on this
        rank's shards without their reductions (o_proj and down_proj write
        their local partial as `delta`): the step's time beyond these is the
        exchange and its waits."""
        if not self.fused or (self.tp is not None and not self.rowwise) or self._mega is not None:
            return {}
        L, s, B = N.lib(), self.s, self.B
        D, Hq, Hkv, H = s.head_dim, self.hq, self.hkv, s.hidden  # this rank's heads
        ha, hb = self.h, self.h2
        q8out = self.rowwise_q8out
        side = torch.cuda.Stream(self.dev)
        side.wait_stream(torch.cuda.current_stream(self.dev))
        parts = {
            "qkv_rmsnorm_gemv": lambda lw, li, st: self._fused_linear(
                N.TN_X_RMSNORM, ha, H, self.delta, hb, lw["attn_norm"], lw["qkv"], self.qkv_out, self.qkv_l, H, st),
            "sdpa_decode_step_q8": lambda lw, li, st: N.check(L.tn_sdpa_decode_step_q8(
                P(self.qkv_out.data_ptr()), P(self.inv_freq.data_ptr()), P(self.k_cache[li].data_ptr()),
                P(self.v_cache[li].data_ptr()), P(self.attn_l.data_ptr()), None, P(self.codes.data_ptr()),
                P(self.scales.data_ptr()), P(self.offsets.data_ptr()), B, Hq, Hkv, D, self.cap, self._kstr,
                self._kstr, P(self.pos.data_ptr()), 1.0 / math.sqrt(D), st)),
            "o_gemv": lambda lw, li, st: self._linear(lw["o"], self.delta, H, Hq * D, st),
            "gate_up_rmsnorm_gemv_silu_q8": lambda lw, li, st: self._fused_linear(
                N.TN_X_RMSNORM, hb, H, self.delta, ha, lw["mlp_norm"], lw["gate_up"], self.act_l, 2 * self.i_l, H,
                st, N.TN_EPILOGUE_SILU_MUL_PAIRS, q8=q8out),
            "down_gemv": (lambda lw, li, st: self._linear(lw["down"], self.delta, H, self.i_l, st)) if q8out else
                         (lambda lw, li, st: self._fused_linear(N.TN_X_BF16, self.act_l, self.i_l, None, None, None,
                                                                lw["down"], self.delta, H, self.i_l, st)),
        }
        graphs = {}
        for name, fn in parts.items():
            with torch.cuda.stream(side):
                fn(self.layers[0], 0, self._stream())
            side.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                for li, lw in enumerate(self.layers):
                    fn(lw, li, self._stream())
            graphs[name] = g
        torch.cuda.current_stream(self.dev).wait_stream(side)
        return graphs

    def capture(self):
        """One eager step first, on the stream the capture will use (the
        library's workspaces are per stream, and are sized by that step;
        nothing may allocate while capturing), then the step captured as a
        CUDA graph on that stream. The eager step advances the state, so
        callers re-seed (fill_prompt_cache / start) afterwards. With the
        persistent kernel a token is one launch already: the returned object's
        replay() launches it directly (no graph to build)."""
        if self._mega is not None:
            self.step()
            torch.cuda.current_stream(self.dev).synchronize()
            dec = self

            class _Direct:
                def replay(self):
                    dec.step()

            self._graph = _Direct()
            return self._graph
        side = torch.cuda.Stream(self.dev)
        side.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(side):
            self.step()
        side.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            self.step()
        torch.cuda.current_stream(self.dev).wait_stream(side)
        self._graph = g
        self._capture_stream = side
        return g
