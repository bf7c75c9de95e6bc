"""bench.py -- the driver's benchmark contract.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--batch B]

Workload (Llama-3-8B-shaped, batch 1 by default): one
step is one greedy decode token, the whole of it -- for each of 32 layers:
RMSNorm (+ the Q8_0 activation quantiser the reference runs before every Q4_0
linear), the fused q/k/v Q4_0 linear (6144 x 4096), RoPE + KV-cache append,
SDPA against the cache (32 query / 8 KV heads, D = 128), o_proj (4096 x 4096),
residual + RMSNorm, the fused gate/up Q4_0 linear (28672 x 4096), SiLU*up,
down_proj (4096 x 14336), residual; then final norm, lm_head (128256 x 4096),
argmax and the next token's embedding. The KV cache holds a 2048-token prompt
(synthetic values) and grows by one slot per step. Weights are random Q4_0
blobs (codes uniform in [-8, 7], scales f16(|N(0,1)| * 0.01)), bf16
activations. 4.2 GB of weights per token, far beyond L2 (126 MB). The step is
one CUDA graph, replayed.

Prints one JSON line (rank 0). `value` is device-resident tokens/s; `e2e`
adds, every step, the pinned host->device copy of the input token ids, their
embedding, and the device->host copy of the next token ids. The same line
carries, at every N (tensor-parallel over the same group when N > 1), the
batch-16 step (`decode_batch16`) and the Llama-3-70B-shaped batch-32 step over
an 8192-slot cache (`llama3_70b_b32`); on one GPU also
the op-level figures (`op_level`).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s + Q4-linear/SDPA %HBM-roofline at 1/2/4/8 B200 vs host CPU"

HIDDEN, INTER, HEADS, KV_HEADS, HEAD_DIM, VOCAB, LAYERS = 4096, 14336, 32, 8, 128, 128256, 32
QKV_N = (HEADS + 2 * KV_HEADS) * HEAD_DIM  # 6144
# (name, N, K) of the Q4_0 linears of one layer, in execution order
LAYER_LINEARS = [("qkv", QKV_N, HIDDEN), ("o", HIDDEN, HIDDEN), ("gate_up", 2 * INTER, HIDDEN),
                 ("down", HIDDEN, INTER)]


def q4_bytes(n: int, k: int) -> int:
    return n * k // 32 * 18


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ops", action="store_true", help="skip the op-level BASELINE figures (configs[1], [2])")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the batch-16 and Llama-3-70B batch-32 decode lines (BASELINE configs[3] at batch 16, "
                         "configs[4])")
    ap.add_argument("--mega", action="store_true", help="run the step as the one persistent kernel per token "
                                                        "(tn_llama_decode_token) instead of the launch-per-operator graph")
    ap.add_argument("--case", default=None, choices=["gemv", "gemm", "sdpa_decode", "sdpa_prefill"],
                    help="kernel-level case instead of the decode step: 'gemv' times the decode GEMV alone on the "
                         "BASELINE (N, K) shapes over rotating weights (~0.3-0.6 GB on the device; the ncu case)")
    ap.add_argument("--rows", type=int, default=1, help="activation rows M for --case gemv")
    ap.add_argument("--fused", action="store_true",
                    help="--case gemv: the launch as the decode step runs gate/up -- RMSNorm prologue on bf16 h + "
                         "delta, SiLU*up pair epilogue, act's planar Q8_0 written by the same launch "
                         "(tn_q4_0_linear_fused_q8out; N is the interleaved gate/up rows, M <= 4)")
    ap.add_argument("--shape", default=None, help="one N,K for --case gemv (default: BASELINE's four shapes)")
    ap.add_argument("--format", default="q4_0", choices=["q4_0", "q8_0", "q4_k"],
                    help="weight format for --case gemv (q8_0 / q4_k time tn_q8_0_linear / tn_q4_k_linear: "
                         "activation quantiser + GEMV)")
    ap.add_argument("--batch", type=int, default=1, help="sequences decoded together (BASELINE: 1 and 16)")
    ap.add_argument("--seqs", default="512,4096,16384", help="sequence lengths for --case sdpa_prefill")
    ap.add_argument("--exchange", default="p2p", choices=["p2p", "nccl"],
                    help="tensor-parallel all-gather: peer-memory kernel or NCCL")
    ap.add_argument("--tp-plan", default="rowwise", choices=["rowwise", "colwise"],
                    help="tensor-parallel plan with the peer-memory exchange up to 16 rows: o_proj/down_proj "
                         "row-parallel with the all-reduce fused into the GEMV (rowwise), or every linear "
                         "column-sharded with an all-gather after each (colwise; always beyond 16 rows)")
    return ap.parse_args()


# --------------------------------------------------------------------------- clocks


class ClockSampler:
    """SM clock and throttle reasons sampled during the timed region: NVML
    polled every 5 ms from a thread (nvidia-smi's own loop is too coarse for a
    timed region of tens of milliseconds), nvidia-smi as a fallback."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4}

    def __init__(self, index: int):
        self.index = index
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))

            def poll():
                while not self._stop.is_set():
                    try:
                        mhz = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                        rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.samples.append((float(mhz), int(rs)))
                    except Exception:
                        pass
                    self._stop.wait(0.005)

            self._t = threading.Thread(target=poll, daemon=True)
            self._t.start()
        except Exception:
            self._t = None
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t is not None:
            self._t.join(timeout=2)

    def summary(self):
        if not self.samples:
            return None
        reasons = sorted({n for _, r in self.samples for n, bit in self.REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples), "source": "nvml"}


# --------------------------------------------------------------------------- workload


def random_q4_blob(n: int, k: int, gen, dev):
    from torchnative_b200.llama_decode import random_q4_blob as r

    return r(n, k, gen, dev)


def random_q8_blob(n: int, k: int, gen, dev):
    """A synthetic Q8_0 weight on the device: random code bytes, scales
    f16(|N(0,1)| * 0.001), in BlockQ8_0's 34-byte layout."""
    import torch

    nb = n * (k // 32)
    blob = torch.randint(0, 256, (nb * 34,), device=dev, dtype=torch.uint8, generator=gen)
    d = (torch.randn(nb, device=dev, generator=gen).abs() * 0.001).to(torch.float16)
    blob.view(nb, 34)[:, 0:2] = d.view(torch.uint8).view(nb, 2)
    return blob


def random_q4k_blob(n: int, k: int, gen, dev):
    """A synthetic Q4_K weight on the device: random scale/min and nibble
    bytes, d and dmin f16(|N(0,1)| * 0.001), in BlockQ4K's 144-byte layout."""
    import torch

    nb = n * (k // 256)
    blob = torch.randint(0, 256, (nb * 144,), device=dev, dtype=torch.uint8, generator=gen)
    d = (torch.randn(nb, 2, device=dev, generator=gen).abs() * 0.001).to(torch.float16)
    blob.view(nb, 144)[:, 0:4] = d.view(torch.uint8).view(nb, 4)
    return blob


PROMPT = 2048


# --------------------------------------------------------------------------- CPU side


def cpu_step_seconds(layer_blobs: dict, lm_head_blob, threads: int, reps: int = 1, context: int = PROMPT) -> float:
    """The reference's CPU arithmetic (oracle/tn_oracle.c) for the two hot
    operators of one token: per layer the four Q4_0 linears (Q8_0 activations,
    vec_dot_unopt, 4-column quads over `threads` workers; the same layer's
    weights each time) and SDPA over a `context`-token cache (sdpa_flash_cpu's
    default arithmetic, f32), then lm_head. Returns seconds per token (min over
    reps). The glue between them (norms, RoPE, SiLU) is not timed."""
    import numpy as np

    from oracle import oracle

    rng = np.random.default_rng(1)
    xs = {k: rng.standard_normal((1, k)).astype(np.float32) for k in (HIDDEN, INTER)}
    q = rng.standard_normal((1, HEADS, 1, HEAD_DIM)).astype(np.float32)
    kc = rng.standard_normal((1, KV_HEADS, context, HEAD_DIM)).astype(np.float32)
    vc = rng.standard_normal((1, KV_HEADS, context, HEAD_DIM)).astype(np.float32)
    best = float("inf")
    for _ in range(reps):
        t0 = time.perf_counter()
        for _layer in range(LAYERS):
            for name, n, k in LAYER_LINEARS:
                oracle.q4_0_linear(xs[k], layer_blobs[name], n, threads=threads)
            oracle.sdpa(q, kc, vc, threads=threads)
        oracle.q4_0_linear(xs[HIDDEN], lm_head_blob, VOCAB, threads=threads)
        best = min(best, time.perf_counter() - t0)
    return best


def upstream_cpu_step_seconds(layer_blobs: dict, lm_head_blob, threads: int, reps: int = 1,
                              context: int = PROMPT) -> float:
    """The labelled "upstream CPU" comparator: the same token's two hot
    operators in upstream torch on the host -- each Q4_0 weight dequantised to
    f32 once, outside the timing (the dequantised values are exact), then per
    layer four f32 `x @ W.T` and torch's own CPU scaled_dot_product_attention
    over a `context`-token f32 cache with GQA, and lm_head. Not the
    reference's arithmetic (no Q8_0 activations): a yardstick beside it.
    Seconds per token (min over reps)."""
    import numpy as np
    import torch

    from oracle import oracle

    torch.set_num_threads(threads)
    ws = {name: torch.from_numpy(oracle.q4_0_dequantize(layer_blobs[name], n * k).reshape(n, k))
          for name, n, k in LAYER_LINEARS}
    lm = torch.from_numpy(oracle.q4_0_dequantize(lm_head_blob, VOCAB * HIDDEN).reshape(VOCAB, HIDDEN))
    g = torch.Generator().manual_seed(2)
    xs = {k: torch.randn((1, k), generator=g) for k in (HIDDEN, INTER)}
    q = torch.randn((1, HEADS, 1, HEAD_DIM), generator=g)
    kc = torch.randn((1, KV_HEADS, context, HEAD_DIM), generator=g)
    vc = torch.randn((1, KV_HEADS, context, HEAD_DIM), generator=g)
    best = float("inf")
    with torch.no_grad():
        for _ in range(reps):
            t0 = time.perf_counter()
            for _layer in range(LAYERS):
                for name, _n, k in LAYER_LINEARS:
                    xs[k] @ ws[name].T
                torch.nn.functional.scaled_dot_product_attention(q, kc, vc, enable_gqa=True)
            xs[HIDDEN] @ lm.T
            best = min(best, time.perf_counter() - t0)
    return best


def cpu_model() -> str:
    """The host CPU's model name (/proc/cpuinfo), for the baseline's label."""
    try:
        with open("/proc/cpuinfo") as fh:
            for line in fh:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or "unknown"


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as fh:
            d = json.load(fh)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def committed_traffic(name: str = "q4_gemv_traffic.json"):
    """dram__bytes_read.sum + dram__bytes_write.sum per launch of the dominant
    kernel, from the committed ncu summary under profiles/ (None without one)."""
    p = os.path.join(ROOT, "profiles", name)
    if os.path.exists(p):
        with open(p) as fh:
            return json.load(fh).get("bytes_per_launch")
    return None


def scaled_traffic(n_rows: int):
    """The committed per-launch DRAM traffic of the 28672-row gate/up launch
    as the step runs it (RMSNorm prologue, SiLU*up epilogue, planar Q8_0 out),
    scaled to a rank's shard of n_rows rows (traffic grows with the rows
    streamed); None without a committed capture."""
    t = committed_traffic("q4_gemv_gate_up_fused_traffic.json")
    return None if t is None else int(t * n_rows / (2 * INTER))


# --------------------------------------------------------------------------- arms


def dist_setup(args):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_ours(args, rank, world, local):
    import ctypes

    import torch

    from torchnative_b200 import _native, build
    from torchnative_b200.llama_decode import LLAMA3_8B, Q4LlamaDecoder

    build.build()
    dev = torch.device("cuda", local)
    B = args.batch
    cap = PROMPT + args.warmup + args.steps + 8
    tp = None
    if world > 1:  # tensor parallelism over the group (--tp-plan: rowwise by default)
        import torch.distributed as dist

        from torchnative_b200.tp import TPGroup

        tp = TPGroup(rank, world, dist.group.WORLD)
    dec = Q4LlamaDecoder(LLAMA3_8B, batch=B, capacity=cap, device=dev, seed=1234, tp=tp, exchange=args.exchange,
                         mega=True if (args.mega and world == 1 and B == 1) else None, tp_plan=args.tp_plan)
    P = ctypes.c_void_p
    cur = lambda: P(torch.cuda.current_stream().cuda_stream)  # noqa: E731
    first = torch.randint(0, LLAMA3_8B.vocab, (B,), device=dev, dtype=torch.int32)

    dec.fill_prompt_cache(PROMPT)
    dec.start(first)
    g = dec.capture()  # runs one eager step, then captures
    _native.device_status(reset=True)
    dec.fill_prompt_cache(PROMPT)
    dec.start(first)

    # the dominant kernel alone: 32 back-to-back gate/up linears over the 32
    # layers' weights (run once on the capture stream first: the library's
    # workspaces are per stream, and nothing may allocate while capturing)
    def gate_up_layers():
        for lw in dec.layers:
            _native.check(_native.lib().tn_q4_0_linear_q8(
                P(dec.codes.data_ptr()), HIDDEN, P(dec.scales.data_ptr()), P(dec.offsets.data_ptr()),
                P(lw["gate_up"].data_ptr()), None, P(dec.act_l.data_ptr()), _native.TN_BF16, B, 2 * dec.i_l, HIDDEN,
                _native.TN_WEIGHTS_STATIC | _native.TN_EPILOGUE_SILU_MUL_PAIRS, cur()))

    gd = None
    if not dec.mega:
        gs = torch.cuda.Stream(dev)
        gs.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(gs):
            gate_up_layers()
        gs.synchronize()
        gd = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gd, stream=gs):
            gate_up_layers()
        torch.cuda.current_stream(dev).wait_stream(gs)

    for _ in range(args.warmup):
        g.replay()
    torch.cuda.synchronize()
    barrier(world)
    pos0 = int(dec.pos.item())
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        start.record()
        for _ in range(args.steps):
            g.replay()
        end.record()
        torch.cuda.synchronize()
    ms = start.elapsed_time(end) / args.steps
    assert int(dec.pos.item()) == pos0 + args.steps, "the step did not advance the cache"
    barrier(world)
    ms = max_over_ranks(ms, world)
    mean_ctx = pos0 + (args.steps + 1) / 2.0

    # end to end: pinned H2D of the token ids, their embedding, the step, D2H of the next ids
    torch.manual_seed(4321)  # the same token ids on every rank of a tensor-parallel group
    tok_host = torch.randint(0, LLAMA3_8B.vocab, (B,), dtype=torch.int32).pin_memory()
    out_host = torch.empty((B,), dtype=torch.int32).pin_memory()
    dec.fill_prompt_cache(PROMPT)

    def e2e_step():
        dec.tokens.copy_(tok_host, non_blocking=True)
        _native.check(_native.lib().tn_llama_embed(P(dec.tokens.data_ptr()), B, P(dec.embed.data_ptr()), HIDDEN,
                                                   P(dec.h.data_ptr()), cur()))
        g.replay()
        out_host.copy_(dec.tokens, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    dec.fill_prompt_cache(PROMPT)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)

    dom_us = ms * 1e3
    if gd is not None:
        for _ in range(3):
            gd.replay()
        torch.cuda.synchronize()
        d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 10
        d0.record()
        for _ in range(reps):
            gd.replay()
        d1.record()
        torch.cuda.synchronize()
        dom_us = d0.elapsed_time(d1) * 1e3 / (reps * LAYERS)
    # the step's parts, each as 32 back-to-back launches (one per layer)
    kernel_us = {}
    for name, kg in dec.kernel_graphs().items():
        kg.replay()
        torch.cuda.synchronize()
        k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        k0.record()
        for _ in range(5):
            kg.replay()
        k1.record()
        torch.cuda.synchronize()
        kernel_us[name] = round(k0.elapsed_time(k1) * 1e3 / (5 * LAYERS), 2)
    _native.device_status(reset=True)

    peak, peak_kind = measured_peaks()
    n, k = 2 * dec.i_l, HIDDEN
    # the dominant launch as the step runs it: on one GPU at batch <= 4 the
    # RMSNorm-prologue gate/up GEMV with the SiLU*up epilogue writing act's
    # planar Q8_0 (bf16 h and delta in, norm weight, weights, act + its Q8 out)
    step_bytes = dec.weight_bytes + dec.kv_bytes(int(mean_ctx))
    if dec.mega:
        # the whole token is one launch: its algorithmic bytes are the step's
        # (every weight byte once, the K/V of the mean context, the small
        # activations and logits), its time the step's
        dom_name = "decode_mega_kernel (the whole token: 32 layers + lm_head + argmax, one persistent launch)"
        algo = step_bytes
    elif "gate_up_rmsnorm_gemv_silu_q8" in kernel_us:
        dom_us = kernel_us["gate_up_rmsnorm_gemv_silu_q8"]
        dom_name = "q4_gemv_q8_kernel<X_NORM> (gate/up as the step runs it: RMSNorm prologue, SiLU*up epilogue, planar Q8_0 out)"
        algo = q4_bytes(n, k) + B * k * 2 * 3 + k * 2 + B * (n // 2) * (2 + 1) + B * (n // 64) * 8
    else:
        dom_name = f"{'q4_skinny_kernel' if 9 <= B <= 32 else 'q4_gemv_q8_kernel'} (gate/up {n}x{k} on this rank, SiLU*up epilogue)"
        algo = q4_bytes(n, k) + B * (k + k // 32 * 8) + B * (n // 2) * 2
    achieved = algo / (dom_us * 1e-6) / 1e9
    per_kernel = {}
    if kernel_us:
        ctx = int(mean_ctx)
        kv = 2 * B * dec.hkv * ctx * HEAD_DIM * 2
        hd_l = dec.hq * HEAD_DIM  # this rank's heads (all of them on one GPU)
        kbytes = {"qkv_rmsnorm_gemv": q4_bytes(dec.qkv_l, HIDDEN) + B * HIDDEN * 4 + HIDDEN * 2 + B * dec.qkv_l * 2,
                  "sdpa_decode_step_q8": kv + B * dec.qkv_l * 2 + B * hd_l * 3,
                  "o_gemv": q4_bytes(HIDDEN, hd_l) + B * hd_l * 5 // 4 + B * HIDDEN * 2,
                  "gate_up_rmsnorm_gemv_silu_q8": algo,
                  "down_gemv": q4_bytes(HIDDEN, dec.i_l) + B * dec.i_l * 5 // 4 + B * HIDDEN * 2}
        for name, us in kernel_us.items():
            b = kbytes.get(name)
            per_kernel[name] = {"us": us, "bytes": b,
                                "frac": None if b is None else round(b / (us * 1e-6) / 1e9 / peak, 3)}
        layer_us = sum(kernel_us.values())
        per_kernel["per_layer_total"] = {"us": round(layer_us, 2), "bytes": sum(kbytes.values()),
                                         "frac": round(sum(kbytes.values()) / (layer_us * 1e-6) / 1e9 / peak, 3)}
        if world > 1:
            # the same launches on this rank's shards without their reductions,
            # against the step: what remains is the exchanges, their waits and
            # the lm_head / logits gather / argmax tail
            step_us = ms * 1e3
            per_kernel["tp_breakdown"] = {
                "step_us": round(step_us, 2), "local_kernels_us_per_layer": round(layer_us, 2),
                "layers_x_local_us": round(LAYERS * layer_us, 2),
                "exchange_wait_and_tail_share": round(max(0.0, 1.0 - LAYERS * layer_us / step_us), 3)}
    result = {
        "metric": METRIC,
        "value": B * 1000.0 / ms,  # one model, tensor-parallel over the group: B tokens per step
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None,
        "dtype": "bf16 activations; Q4_0 x Q8_0 linears (int dot, f32 scale/accumulate); f32 attention math",
        "data": "synthetic: random Q4_0 weights (codes U[-8,7], scales f16(|N(0,1)|*0.01)), bf16 norms/embeddings, "
                "N(0,1) prompt KV cache",
        "config": {"workload": f"Llama-3-8B-shaped Q4_0 greedy decode step, batch {B}, {PROMPT}-token prompt cache "
                               "growing one slot per step",
                   "model": "Llama-3-8B-shaped (32 layers, 4096 hidden, 32/8 heads, D 128, MLP 14336, vocab 128256)",
                   "global_batch": B, "seq_len": PROMPT,
                   "parallelism": (f"tp{world} (rowwise: q/k/v, gate/up and lm_head column-sharded, "
                                   "KV-head-group attention, o_proj/down_proj row-parallel with the all-reduce "
                                   "fused into the GEMV over peer memory; logits all-gathered)" if dec.rowwise else
                                   f"tp{world} (column-sharded Q4_0 linears, KV-head-group attention, "
                                   f"{'peer-memory' if args.exchange == 'p2p' else 'NCCL'} all-gather after each "
                                   "sharded output)") if world > 1 else "tp1",
                   "l2": "inputs larger than L2 (4.22 GB of weights per step)",
                   "mean_context": mean_ctx, "bytes_per_step": step_bytes,
                   "hbm_roofline_tok_s": B * peak * 1e9 / step_bytes},
        "roofline": {"bound": "hbm", "kernel": dom_name,
                     "achieved": achieved,
                     "peak": peak, "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": (committed_traffic("decode_mega_traffic.json") if dec.mega else scaled_traffic(n)),
                     "algorithmic_bytes": algo, "avg_launch_us": dom_us},
        "step_hbm_frac": (step_bytes / (ms * 1e-3) / 1e9) / peak,
        "kernel_us_back_to_back": kernel_us,
        "per_kernel": per_kernel,
        "e2e": {"value": B * 1000.0 / e2e_ms, "unit": "tok/s", "h2d_bytes_per_step": 4 * B,
                "d2h_bytes_per_step": 4 * B},
        "gpu_launches": dec.kernels_per_step * args.steps,
        "clocks": clocks.summary(),
    }
    result["config"]["step_kernel"] = ("one persistent kernel per token (tn_llama_decode_token)" if dec.mega else
                                       f"{dec.kernels_per_step} launches per token in one CUDA graph")
    # graphs holding NCCL calls go before the process group does; no rank frees
    # its exchange region while a peer may still write it
    dec._graph = None
    del g, gd
    torch.cuda.synchronize()
    barrier(world)
    dec.close()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        blobs = {"qkv": dec.layers[0]["qkv"].cpu().numpy(), "o": dec.layers[0]["o"].cpu().numpy(),
                 "gate_up": dec.layers[0]["gate_up"].cpu().numpy(), "down": dec.layers[0]["down"].cpu().numpy()}
        lm = dec.lm_head.cpu().numpy()
        th = host_threads()
        sec = cpu_step_seconds(blobs, lm, th, reps=2)
        result["cpu_baseline"] = {"value": 1.0 / sec, "unit": "tok/s", "cores": th, "kind": "port",
                                  "host": cpu_model(), "nproc": os.cpu_count(),
                                  "sample": f"one token at batch 1: layer 0's four Q4_0 linears and SDPA over a "
                                            f"{PROMPT}-token f32 cache, 32 times, + lm_head; oracle/tn_oracle.c "
                                            "restatement of the reference CPU arithmetic; min of 2"}
        try:  # a comparator only: it must never cost the line
            usec = upstream_cpu_step_seconds(blobs, lm, th, reps=2)
            result["upstream_cpu"] = {"value": 1.0 / usec, "unit": "tok/s", "cores": th, "host": cpu_model(),
                                      "sample": "the same token in upstream torch " + torch.__version__ +
                                                " on the host: f32 weights dequantised once (untimed), four f32 "
                                                "x @ W.T and torch's CPU scaled_dot_product_attention (GQA) per "
                                                "layer, 32 times, + lm_head; min of 2. A yardstick, not the "
                                                "reference's arithmetic"}
        except Exception as e:  # noqa: BLE001
            result["upstream_cpu"] = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
    return result


def _time_graph(launches, warmup: int, reps: int) -> float:
    """Microseconds per launch of `launches` (a list of zero-argument calls,
    each one launch), captured once as a CUDA graph on a side stream after
    one eager pass there (the library's workspaces are per stream and nothing
    may allocate while capturing), timed with CUDA events on that stream."""
    import torch

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for fn in launches:
            fn()
    side.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        for fn in launches:
            fn()
    with torch.cuda.stream(side):
        for _ in range(warmup):
            g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(side)
        for _ in range(reps):
            g.replay()
        e1.record(side)
    side.synchronize()
    del g
    return e0.elapsed_time(e1) * 1e3 / (reps * len(launches))


def op_level(dev) -> dict:
    """BASELINE configs[1] and [2] at op level, each through the C ABI with
    device-resident inputs, CUDA events over CUDA-graph replays:
    - Q4_0 linear tn_q4_0_linear, bf16 activations (quantiser + linear), M in
      {1, 4, 16, 128, 2048} on the three BASELINE (N, K) shapes; M <= 16 over
      rotating weight copies (> L2) against HBM, M >= 128 against dense bf16;
    - SDPA decode, the flash op at L = 1 on a KV-cache view, bf16, S in {1024,
      8192, 32768} x B in {1, 8, 32}, against HBM (K/V bytes);
    - SDPA prefill, causal bf16, B in {1, 4} x S in {512, 4096, 16384}, against
      dense bf16 (causal flops)."""
    import ctypes
    import math

    import torch

    from torchnative_b200 import _native as N
    from torchnative_b200.llama_decode import random_q4_blob as rq4

    hbm, _ = measured_peaks()
    tf = _measured_tflops()
    P = ctypes.c_void_p
    L = N.lib()
    cur = lambda: P(torch.cuda.current_stream().cuda_stream)  # noqa: E731
    gen = torch.Generator(device=dev).manual_seed(11)
    res = {"q4_linear": [], "sdpa_decode": [], "sdpa_prefill": []}
    for (n, k) in ((14336, 4096), (4096, 14336), (6144, 4096)):
        wb = q4_bytes(n, k)
        copies = max(2, -(-300_000_000 // wb))
        ws = [rq4(n, k, gen, dev) for _ in range(copies)]
        for M in (1, 4, 16, 128, 2048):
            x = torch.randn((M, k), device=dev, generator=gen).to(torch.bfloat16)
            y = torch.empty((M, n), device=dev, dtype=torch.bfloat16)
            use = ws if M <= 16 else ws[:1]
            fns = [lambda w=w: N.check(L.tn_q4_0_linear(P(x.data_ptr()), N.TN_BF16, k, P(w.data_ptr()), None,
                                                         P(y.data_ptr()), N.TN_BF16, M, n, k, N.TN_ACT_Q8_0, cur()))
                   for w in use]
            us = _time_graph(fns, 3, 10 if M <= 128 else 5)
            kern = ("q4_gemv_q8_kernel" if M <= 8 else "q4_skinny_kernel" if M <= 32 else "q4_gemm_kernel")
            algo = wb + M * k * 2 + M * n * 2
            ent = {"M": M, "N": n, "K": k, "kernel": kern + " (+ Q8_0 activation quantiser)", "us": round(us, 2)}
            if M <= 16:
                ent.update({"GBps": round(algo / us / 1e3, 1), "frac_hbm": round(algo / us / 1e3 / hbm, 3)})
            else:
                tfl = 2.0 * M * n * k / us / 1e6
                ent.update({"TFLOPs": round(tfl, 1), "frac_bf16": round(tfl / tf, 3)})
            res["q4_linear"].append(ent)
            del x, y
        del ws
        torch.cuda.empty_cache()
    for S in (1024, 8192, 32768):
        for B in (1, 8, 32):
            cap = S + 64
            kb = torch.randn((B, KV_HEADS, cap, HEAD_DIM), device=dev, generator=gen).to(torch.bfloat16)
            vb = torch.randn((B, KV_HEADS, cap, HEAD_DIM), device=dev, generator=gen).to(torch.bfloat16)
            q = torch.randn((B, HEADS, 1, HEAD_DIM), device=dev, generator=gen).to(torch.bfloat16)
            out = torch.empty_like(q)
            lse = torch.empty((B, HEADS, 1), device=dev)
            qs = (ctypes.c_int64 * 4)(HEADS * HEAD_DIM, HEAD_DIM, 0, 1)
            ks = (ctypes.c_int64 * 4)(*kb.stride())
            fns = [lambda: N.check(L.tn_sdpa_flash_attention(P(q.data_ptr()), P(kb.data_ptr()), P(vb.data_ptr()), None,
                                                             0, None, P(out.data_ptr()), P(lse.data_ptr()), N.TN_BF16,
                                                             B, HEADS, KV_HEADS, 1, S, HEAD_DIM, qs, ks, ks, 0,
                                                             1.0 / math.sqrt(HEAD_DIM), cur()))]
            us = _time_graph(fns, 3, 20)
            algo = 2 * B * KV_HEADS * S * HEAD_DIM * 2 + 2 * B * HEADS * HEAD_DIM * 2 + 4 * B * HEADS
            res["sdpa_decode"].append({"B": B, "S": S, "kernel": "sdpa_decode_mma_kernel (split-KV + merge)",
                                       "us": round(us, 2), "GBps": round(algo / us / 1e3, 1),
                                       "frac_hbm": round(algo / us / 1e3 / hbm, 3)})
            del kb, vb, q, out, lse
        torch.cuda.empty_cache()
    for B in (1, 4):
        for S in (512, 4096, 16384):
            q = torch.randn((B, HEADS, S, HEAD_DIM), device=dev, generator=gen).to(torch.bfloat16)
            kk = torch.randn((B, KV_HEADS, S, HEAD_DIM), device=dev, generator=gen).to(torch.bfloat16)
            vv = torch.randn((B, KV_HEADS, S, HEAD_DIM), device=dev, generator=gen).to(torch.bfloat16)
            out = torch.empty_like(q)
            lse = torch.empty((B, HEADS, S), device=dev)
            qs = (ctypes.c_int64 * 4)(*q.stride())
            ks = (ctypes.c_int64 * 4)(*kk.stride())
            fns = [lambda: N.check(L.tn_sdpa_flash_attention(P(q.data_ptr()), P(kk.data_ptr()), P(vv.data_ptr()), None,
                                                             0, None, P(out.data_ptr()), P(lse.data_ptr()), N.TN_BF16,
                                                             B, HEADS, KV_HEADS, S, S, HEAD_DIM, qs, ks, ks, 1,
                                                             1.0 / math.sqrt(HEAD_DIM), cur()))]
            us = _time_graph(fns, 3, 10)
            fl = 4.0 * B * HEADS * HEAD_DIM * S * (S + 1) / 2
            tfl = fl / us / 1e6
            res["sdpa_prefill"].append({"B": B, "S": S, "kernel": "sdpa_prefill2_kernel" if S > 128 else
                                        "sdpa_prefill_kernel", "us": round(us, 2), "TFLOPs": round(tfl, 1),
                                        "frac_bf16": round(tfl / tf, 3)})
            del q, kk, vv, out, lse
        torch.cuda.empty_cache()
    N.device_status(reset=True)
    return res


def decode_config(dev, shape, B: int, cache: int, steps: int, warmup: int, rank: int = 0, world: int = 1,
                  exchange: str = "p2p", seed: int = 99, tp_plan: str = "rowwise") -> dict:
    """One BASELINE decode configuration on this rank's GPU (tensor-parallel
    over the process group when world > 1): `shape` (Llama-3-8B or -70B),
    batch B, every sequence's KV cache `cache` slots long with the prompt
    filling all but the slots the timed steps append. The step replayed as
    one CUDA graph; CUDA events on the replay stream between barriers, max
    over ranks. tok/s counts the B tokens of a step; the HBM fraction is this
    rank's bytes (its weight shards, its KV heads of the cache) over its time,
    against the measured copy peak."""
    import torch

    from torchnative_b200.llama_decode import Q4LlamaDecoder

    tp = None
    if world > 1:
        import torch.distributed as dist

        from torchnative_b200.tp import TPGroup

        tp = TPGroup(rank, world, dist.group.WORLD)
    prompt = cache - (warmup + steps + 2)
    torch.cuda.empty_cache()
    dec = Q4LlamaDecoder(shape, batch=B, capacity=cache, device=dev, seed=seed, tp=tp, exchange=exchange,
                         tp_plan=tp_plan)
    gen = torch.Generator(device=dev).manual_seed(seed)  # the same first tokens on every rank
    first = torch.randint(0, shape.vocab, (B,), device=dev, dtype=torch.int32, generator=gen)
    dec.fill_prompt_cache(prompt)
    dec.start(first)
    g = dec.capture()
    dec.fill_prompt_cache(prompt)
    dec.start(first)
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    barrier(world)
    pos0 = int(dec.pos.item())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    assert int(dec.pos.item()) == pos0 + steps, "the step did not advance the cache"
    hbm, _ = measured_peaks()
    step_bytes = dec.weight_bytes + dec.kv_bytes(int(pos0 + (steps + 1) / 2))
    out = {"model": f"{shape.layers} layers, hidden {shape.hidden}, {shape.heads}/{shape.kv_heads} heads, "
                    f"MLP {shape.inter}, vocab {shape.vocab}",
           "batch": B, "kv_cache_slots": cache, "mean_context": pos0 + (steps + 1) / 2.0, "n_gpus": world,
           "parallelism": f"tp{world}" + (" rowwise" if dec.rowwise else " colwise" if world > 1 else ""),
           "steps": steps, "warmup": warmup,
           "tok_s": round(B * 1000.0 / ms, 1), "ms_per_step": round(ms, 4),
           "step_hbm_frac": round(step_bytes / (ms * 1e-3) / 1e9 / hbm, 3), "bytes_per_step_per_gpu": step_bytes,
           "kernels_per_step": dec.kernels_per_step}
    dec._graph = None
    del g
    torch.cuda.synchronize()
    barrier(world)
    dec.close()
    del dec
    torch.cuda.empty_cache()
    return out


def batched_decode(dev, B: int, steps: int = 10, warmup: int = 3, rank: int = 0, world: int = 1,
                   exchange: str = "p2p") -> dict:
    """BASELINE configs[3] at batch B: the Llama-3-8B-shaped decode step of B
    sequences over a PROMPT-token cache (from 9 rows the batched path: the
    tcgen05 skinny Q4_0 kernel)."""
    from torchnative_b200.llama_decode import LLAMA3_8B

    return decode_config(dev, LLAMA3_8B, B, PROMPT + warmup + steps + 2, steps, warmup, rank, world, exchange)


def llama70b_decode(dev, steps: int = 6, warmup: int = 3, rank: int = 0, world: int = 1,
                    exchange: str = "p2p") -> dict:
    """the Llama-3-70B-shaped decoder (80 layers, hidden
    8192, 64/8 heads, MLP 28672; ~39 GB of Q4_0 weights), batch 32, an
    8192-slot KV cache per sequence (~86 GB in bf16 on one GPU)."""
    from torchnative_b200.llama_decode import LLAMA3_70B

    return decode_config(dev, LLAMA3_70B, 32, 8192, steps, warmup, rank, world, exchange, seed=70)


def _measured_tflops() -> float:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as fh:
            return float(json.load(fh)["bf16_tflops"])
    return 1590.0


def run_reference(args, rank, world):
    """The reference's CPU arithmetic (the oracle port; the reference is a
    Rust crate that cannot be built here) on the same workload, all host
    threads; each step one token (a bounded sample, see cpu_step_seconds)."""
    import numpy as np

    if rank != 0:
        return None
    rng = np.random.default_rng(7)

    def blob(n, k):
        nb = k // 32
        out = np.empty((n, nb, 18), dtype=np.uint8)
        out[:, :, 2:] = rng.integers(0, 256, size=(n, nb, 16), dtype=np.uint8)
        out[:, :, 0:2] = (np.abs(rng.standard_normal((n, nb, 1))) * 0.01).astype(np.float16).view(np.uint8)
        return out.reshape(-1)

    blobs = {name: blob(n, k) for name, n, k in LAYER_LINEARS}
    lm = blob(VOCAB, HIDDEN)
    th = host_threads()
    for _ in range(min(args.warmup, 1)):
        cpu_step_seconds(blobs, lm, th)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_step_seconds(blobs, lm, th)
    sec = (time.perf_counter() - t0) / args.steps
    v = 1.0 / sec
    return {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "q4_0 x q8_0 -> f32 accumulate", "data": "synthetic",
        "config": {"workload": f"Llama-3-8B-shaped Q4_0 greedy decode step, batch 1, {PROMPT}-token cache: the "
                               "two hot operators on the host CPU (layer weights reused per layer)",
                   "global_batch": 1, "seq_len": PROMPT, "parallelism": "host CPU"},
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": th, "kind": "port",
                         "sample": "one token per step: one layer's four Q4_0 linears and SDPA over a "
                                   f"{PROMPT}-token cache, 32 times, + lm_head"},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    args = parse()
    if args.case == "gemv":
        run_case_gemv(args)
        return
    if args.case == "gemm":
        return run_case_gemm(args)
    if args.case == "sdpa_decode":
        run_case_sdpa_decode(args)
        return
    if args.case == "sdpa_prefill":
        run_case_sdpa_prefill(args)
        return
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        res = run_reference(args, rank, world)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    rank, world, local = dist_setup(args)
    res = run_ours(args, rank, world, local)
    import torch

    dev = torch.device("cuda", local)
    if rank == 0 and world == 1 and not args.no_ops:
        res["op_level"] = op_level(dev)
    if not args.no_configs:
        # BASELINE configs[3] at batch 16 and configs[4] (70B, batch 32, 8192-slot
        # cache), tensor-parallel over the same group at N > 1: every rank runs them
        res["decode_batch16"] = batched_decode(dev, 16, rank=rank, world=world, exchange=args.exchange)
        res["llama3_70b_b32"] = llama70b_decode(dev, rank=rank, world=world, exchange=args.exchange)
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()



def run_case_sdpa_decode(args):
    """Kernel-level timing of the fused decode-step attention
    (tn_sdpa_decode_step: RoPE + KV append + split-KV SDPA + merge) on the
    Llama-3-8B shape, 32 layers' caches of PROMPT tokens (~270 MB, beyond L2)
    rotated, batch --batch. One JSON line: us per launch and the HBM fraction
    of its K/V bytes."""
    import ctypes
    import math

    import torch

    from torchnative_b200 import _native as N, build
    from torchnative_b200.llama_decode import rope_inv_freq

    build.build()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, Hq, Hkv, D, cap = args.batch, HEADS, KV_HEADS, HEAD_DIM, PROMPT + 64
    g = torch.Generator(device=dev).manual_seed(3)
    ks = [torch.randn((B, Hkv, cap, D), device=dev, generator=g).to(torch.bfloat16) for _ in range(LAYERS)]
    vs = [torch.randn((B, Hkv, cap, D), device=dev, generator=g).to(torch.bfloat16) for _ in range(LAYERS)]
    qkv = torch.randn((B, (Hq + 2 * Hkv) * D), device=dev, generator=g).to(torch.bfloat16)
    out = torch.empty((B, Hq, D), device=dev, dtype=torch.bfloat16)
    inv = rope_inv_freq(D, 500000.0).to(dev)
    pos = torch.tensor([PROMPT], dtype=torch.int32, device=dev)
    P = ctypes.c_void_p
    st = (ctypes.c_int64 * 4)(*ks[0].stride())
    s = lambda: P(torch.cuda.current_stream().cuda_stream)  # noqa: E731

    def launch(li):
        N.check(N.lib().tn_sdpa_decode_step(P(qkv.data_ptr()), P(inv.data_ptr()), P(ks[li].data_ptr()),
                                            P(vs[li].data_ptr()), P(out.data_ptr()), None, B, Hq, Hkv, D, cap, st, st,
                                            P(pos.data_ptr()), 1.0 / math.sqrt(D), s()))

    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        launch(0)
    side.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr, stream=side):
        for li in range(LAYERS):
            launch(li)
    for _ in range(args.warmup):
        gr.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        gr.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (args.steps * LAYERS)
    kv = 2 * B * Hkv * (PROMPT + 1) * D * 2
    peak, kind = measured_peaks()
    print(json.dumps({"case": "sdpa_decode", "B": B, "S": PROMPT + 1, "us_per_launch": us, "kv_bytes": kv,
                      "GBps": kv / us / 1e3, "frac": kv / us / 1e3 / peak, "peak_kind": kind}), flush=True)
    N.device_status(reset=True)


def run_case_sdpa_prefill(args):
    """Kernel-level timing of causal prefill SDPA (32
    query / 8 KV heads, D = 128, bf16) at batch --batch and the sequence
    lengths of --seqs. One JSON line per length: TFLOP/s of the causal work
    (4 * B * Hq * D * S(S+1)/2) against the measured dense bf16 peak."""
    import ctypes

    import torch

    from torchnative_b200 import _native as N, attention, build

    build.build()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peak = 1590.0
    kind = "fallback"
    pp = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pp):
        with open(pp) as fh:
            peak, kind = float(json.load(fh)["bf16_tflops"]), "measured"
    B = args.batch
    for S in [int(x) for x in args.seqs.split(",")]:
        g = torch.Generator(device=dev).manual_seed(S)
        q = torch.randn((B, HEADS, S, HEAD_DIM), device=dev, generator=g).to(torch.bfloat16)
        k = torch.randn((B, KV_HEADS, S, HEAD_DIM), device=dev, generator=g).to(torch.bfloat16)
        v = torch.randn((B, KV_HEADS, S, HEAD_DIM), device=dev, generator=g).to(torch.bfloat16)
        for _ in range(args.warmup):
            attention.scaled_dot_product_flash_attention_for_cpu(q, k, v, 0.0, True)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            attention.scaled_dot_product_flash_attention_for_cpu(q, k, v, 0.0, True)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        flops = 4.0 * B * HEADS * HEAD_DIM * S * (S + 1) / 2
        print(json.dumps({"case": "sdpa_prefill", "B": B, "S": S, "ms": ms, "TFLOPs": flops / ms / 1e9,
                          "frac": flops / ms / 1e9 / peak, "peak": peak, "peak_kind": kind}), flush=True)
        del q, k, v
    N.device_status(reset=True)


def run_case_gemv(args):
    """Kernel-level timing of the decode GEMV (planar Q8_0 activations already
    on the device) on BASELINE's (N, K) shapes, rotating over enough weight
    copies that the weights never sit in L2. Prints one JSON line per shape."""
    import ctypes

    import torch

    from torchnative_b200 import _native as N, build

    build.build()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(5)
    M = args.rows
    peak, peak_kind = measured_peaks()
    P = ctypes.c_void_p
    L = N.lib()
    shapes = ((14336, 4096), (4096, 14336), (6144, 4096), (28672, 4096))
    if args.shape:
        shapes = (tuple(int(x) for x in args.shape.split(",")),)
    q8w, q4k = args.format == "q8_0", args.format == "q4_k"
    for n, k in shapes:
        wbytes = n * (k // 32) * 34 if q8w else (n * (k // 256) * 144 if q4k else q4_bytes(n, k))
        copies = max(2, -(-300_000_000 // wbytes))
        mk = random_q8_blob if q8w else (random_q4k_blob if q4k else random_q4_blob)
        ws = [mk(n, k, gen, dev) for _ in range(copies)]
        x = torch.randn((M, k), device=dev, generator=gen).to(torch.bfloat16)
        codes = torch.empty((M, k), device=dev, dtype=torch.int8)
        scales = torch.empty((M, k // 32), device=dev)
        offs = torch.empty((M, k // 32), device=dev)
        y = torch.empty((M, n), device=dev, dtype=torch.bfloat16)
        s = lambda: P(torch.cuda.current_stream().cuda_stream)  # noqa: E731
        N.check(L.tn_q8_0_quantize_planar(P(x.data_ptr()), N.TN_BF16, k, P(codes.data_ptr()), k,
                                          P(scales.data_ptr()), P(offs.data_ptr()), M, k, s()))

        if args.fused:
            h = torch.randn((M, k), device=dev, generator=gen).to(torch.bfloat16)
            delta = (0.1 * torch.randn((M, k), device=dev, generator=gen)).to(torch.bfloat16)
            h_out = torch.empty_like(h)
            norm_w = (1.0 + 0.1 * torch.randn(k, device=dev, generator=gen)).to(torch.bfloat16)
            y = torch.empty((M, n // 2), device=dev, dtype=torch.bfloat16)
            oq = torch.empty((M, n // 2), device=dev, dtype=torch.int8)
            od = torch.empty((M, n // 64), device=dev)
            oc = torch.empty((M, n // 64), device=dev)

        def launch(w):
            if args.fused:
                N.check(L.tn_q4_0_linear_fused_q8out(
                    N.TN_X_RMSNORM, P(h.data_ptr()), k, P(delta.data_ptr()), P(h_out.data_ptr()),
                    P(norm_w.data_ptr()), 1e-5, P(w.data_ptr()), None, P(y.data_ptr()), N.TN_BF16, M, n, k,
                    N.TN_WEIGHTS_STATIC | N.TN_EPILOGUE_SILU_MUL_PAIRS, P(oq.data_ptr()), n // 2, P(od.data_ptr()),
                    P(oc.data_ptr()), s()))
                return
            if q8w or q4k:  # the bf16 activation's quantiser launch, then the GEMV of that weight format
                fn = L.tn_q8_0_linear if q8w else L.tn_q4_k_linear
                N.check(fn(P(x.data_ptr()), N.TN_BF16, k, P(w.data_ptr()), None, P(y.data_ptr()), N.TN_BF16, M, n, k,
                           N.TN_ACT_Q8_0, s()))
                return
            N.check(L.tn_q4_0_linear_q8(P(codes.data_ptr()), k, P(scales.data_ptr()), P(offs.data_ptr()),
                                        P(w.data_ptr()), None, P(y.data_ptr()), N.TN_BF16, M, n, k,
                                        N.TN_WEIGHTS_STATIC, s()))

        # warm on the capture stream: the workspace is per stream and must
        # exist before the capture (nothing may allocate while capturing)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            launch(ws[0])
        side.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            for w in ws:
                launch(w)
        torch.cuda.current_stream().wait_stream(side)
        for _ in range(args.warmup):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (args.steps * copies)
        algo = wbytes + M * (k + k // 32 * 8) + M * n * 2
        kernel = "q4_skinny_kernel" if args.format == "q4_0" and 9 <= M <= 32 and k % 256 == 0 else "q4_gemv_q8_kernel"
        if args.fused:  # bf16 h, delta and h_out, the norm weight; bf16 act + its planar Q8_0 out
            algo = wbytes + M * k * 2 * 3 + k * 2 + M * (n // 2) * (2 + 1) + M * (n // 64) * 8
            kernel = "q4_gemv_q8_kernel<X_NORM> (RMSNorm prologue, SiLU*up epilogue, planar Q8_0 out)"
        print(json.dumps({"case": "gemv", "format": args.format, "kernel": kernel, "M": M, "N": n, "K": k,
                          "us_per_launch": us,
                          "GBps": algo / us / 1e3, "frac": algo / us / 1e3 / peak, "peak": peak,
                          "peak_kind": peak_kind, "copies": copies}), flush=True)
        del ws
        torch.cuda.empty_cache()
    N.device_status(reset=True)


def run_case_gemm(args):
    """Kernel-level timing of the prefill Q4_0 linear (tn_q4_0_linear with bf16
    activations: the f16-code Q8_0 quantiser plus the tcgen05 GEMM) on
    BASELINE's (N, K) shapes at --rows M (default 2048). One JSON line per
    shape: TFLOP/s of 2*M*N*K against the measured dense bf16 peak."""
    import ctypes

    import torch

    from torchnative_b200 import _native as N_, build

    build.build()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(6)
    M = args.rows if args.rows > 16 else 2048
    peak = 1590.0
    kind = "fallback"
    pp = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pp):
        with open(pp) as fh:
            peak, kind = float(json.load(fh)["bf16_tflops"]), "measured"
    P = ctypes.c_void_p
    shapes = ((14336, 4096), (4096, 14336), (6144, 4096))
    if args.shape:
        shapes = (tuple(int(x) for x in args.shape.split(",")),)
    for n, k in shapes:
        w = random_q4_blob(n, k, gen, dev)
        x = torch.randn((M, k), device=dev, generator=gen).to(torch.bfloat16)
        y = torch.empty((M, n), device=dev, dtype=torch.bfloat16)
        s = lambda: P(torch.cuda.current_stream().cuda_stream)  # noqa: E731

        def launch():
            N_.check(N_.lib().tn_q4_0_linear(P(x.data_ptr()), N_.TN_BF16, k, P(w.data_ptr()), None,
                                             P(y.data_ptr()), N_.TN_BF16, M, n, k, N_.TN_ACT_Q8_0, s()))

        for _ in range(args.warmup):
            launch()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            launch()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        fl = 2.0 * M * n * k
        print(json.dumps({"case": "gemm", "M": M, "N": n, "K": k, "ms": ms, "TFLOPs": fl / ms / 1e9,
                          "frac": fl / ms / 1e9 / peak, "peak": peak, "peak_kind": kind}), flush=True)
        del w, x, y
    N_.device_status(reset=True)


if __name__ == "__main__":
    main()
