"""bench.py -- the driver's benchmark contract.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (Llama-3-8B-shaped, batch 1): one step is
the Q4_0 part of one greedy decode token -- for each of the 32 layers the
fused q/k/v projection (6144 x 4096), o_proj (4096 x 4096), the fused
gate/up projection (28672 x 4096) and down_proj (4096 x 14336), each preceded
by the Q8_0 activation quantiser the reference runs, then lm_head
(128256 x 4096): 4.22 GB of Q4_0 weights, all random (codes uniform in
[-8, 7], scales f16(|N(0,1)| * 0.01)), bf16 activations. The weights (4.2 GB)
are far larger than L2 (126 MB), so nothing is re-read from L2 between steps.
The step is captured once in a CUDA graph and replayed.

Prints one JSON line (rank 0). `value` is device-resident tokens/s; `e2e`
adds, every step, the pinned host->device copy of the token's hidden state
and the device->host copy of the logits.
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
    ap.add_argument("--case", default=None, choices=["gemv"],
                    help="kernel-level case instead of the decode step: 'gemv' times the decode GEMV alone on the "
                         "BASELINE (N, K) shapes over rotating weights (~0.3-0.6 GB on the device; the ncu case)")
    ap.add_argument("--rows", type=int, default=1, help="activation rows M for --case gemv")
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
    """Q4_0 blob built directly in the block layout on the device: two nibbles
    of uniform random bytes (codes uniform in [-8, 7]) and f16 scales
    |N(0,1)| * 0.01."""
    import torch

    nb = k // 32
    qs = torch.randint(0, 256, (n, nb, 16), dtype=torch.uint8, device=dev, generator=gen)
    d = (torch.randn((n, nb, 1), device=dev, generator=gen).abs() * 0.01).to(torch.float16).view(torch.uint8)
    return torch.cat([d, qs], dim=2).reshape(-1).contiguous()


class Q4DecodeStack:
    """The Q4_0 linears of a Llama-3-8B-shaped decode step at batch M, through
    the C ABI (planar Q8_0 quantiser + decode GEMV per linear)."""

    def __init__(self, dev, M=1, seed=0):
        import torch

        from torchnative_b200 import _native as N

        self.N = N
        self.dev, self.M = dev, M
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed)
        self.layers = [{name: random_q4_blob(n, k, gen, dev) for name, n, k in LAYER_LINEARS} for _ in range(LAYERS)]
        self.lm_head = random_q4_blob(VOCAB, HIDDEN, gen, dev)
        bf = torch.bfloat16
        self.h = torch.randn((M, HIDDEN), device=dev, generator=gen).to(bf)
        self.attn = torch.randn((M, HIDDEN), device=dev, generator=gen).to(bf)
        self.act = torch.randn((M, INTER), device=dev, generator=gen).to(bf)
        self.qkv = torch.empty((M, QKV_N), device=dev, dtype=bf)
        self.o = torch.empty((M, HIDDEN), device=dev, dtype=bf)
        self.gu = torch.empty((M, 2 * INTER), device=dev, dtype=bf)
        self.down = torch.empty((M, HIDDEN), device=dev, dtype=bf)
        self.logits = torch.empty((M, VOCAB), device=dev, dtype=bf)
        kmax = INTER
        self.codes = torch.empty((M, kmax), device=dev, dtype=torch.int8)
        self.scales = torch.empty((M, kmax // 32), device=dev, dtype=torch.float32)
        self.offsets = torch.empty((M, kmax // 32), device=dev, dtype=torch.float32)
        self.weight_bytes = sum(q4_bytes(n, k) for _, n, k in LAYER_LINEARS) * LAYERS + q4_bytes(VOCAB, HIDDEN)

    def _linear(self, x, w, y, n, k, stream):
        import ctypes

        L = self.N.lib()
        P = ctypes.c_void_p
        self.N.check(L.tn_q8_0_quantize_planar(P(x.data_ptr()), self.N.TN_BF16, k, P(self.codes.data_ptr()), k,
                                               P(self.scales.data_ptr()), P(self.offsets.data_ptr()), self.M, k,
                                               stream))
        self.N.check(L.tn_q4_0_linear_q8(P(self.codes.data_ptr()), k, P(self.scales.data_ptr()),
                                         P(self.offsets.data_ptr()), P(w.data_ptr()), None, P(y.data_ptr()),
                                         self.N.TN_BF16, self.M, n, k, self.N.TN_WEIGHTS_STATIC, stream))

    def step(self, stream):
        """One decode token's Q4_0 work: 4 linears x 32 layers + lm_head."""
        for lw in self.layers:
            self._linear(self.h, lw["qkv"], self.qkv, QKV_N, HIDDEN, stream)
            self._linear(self.attn, lw["o"], self.o, HIDDEN, HIDDEN, stream)
            self._linear(self.h, lw["gate_up"], self.gu, 2 * INTER, HIDDEN, stream)
            self._linear(self.act, lw["down"], self.down, HIDDEN, INTER, stream)
        self._linear(self.h, self.lm_head, self.logits, VOCAB, HIDDEN, stream)

    kernels_per_step = 2 * (4 * LAYERS + 1)

    def dominant_launch(self, stream, layer):
        """The gate/up GEMV alone (the largest Q4_0 kernel of a layer)."""
        import ctypes

        L = self.N.lib()
        P = ctypes.c_void_p
        self.N.check(L.tn_q4_0_linear_q8(P(self.codes.data_ptr()), HIDDEN, P(self.scales.data_ptr()),
                                         P(self.offsets.data_ptr()), P(self.layers[layer]["gate_up"].data_ptr()),
                                         None, P(self.gu.data_ptr()), self.N.TN_BF16, self.M, 2 * INTER, HIDDEN,
                                         self.N.TN_WEIGHTS_STATIC, stream))

    def dominant_algorithmic_bytes(self):
        n, k = 2 * INTER, HIDDEN
        # weights + planar Q8_0 activations (codes + scale + offset per block) + bf16 output
        return q4_bytes(n, k) + self.M * (k + k // 32 * 8) + self.M * n * 2


# --------------------------------------------------------------------------- CPU side


def cpu_step_seconds(layer_blobs: dict, lm_head_blob, threads: int, reps: int = 1) -> float:
    """The reference's CPU arithmetic (oracle/tn_oracle.c: Q8_0 activations,
    vec_dot_unopt, 4-column quads over `threads` workers) over one token:
    the four linears of a layer 32 times (the same layer's weights each time)
    and lm_head. Returns seconds per token (min over reps)."""
    import numpy as np

    from oracle import oracle

    rng = np.random.default_rng(1)
    xs = {k: rng.standard_normal((1, k)).astype(np.float32) for k in (HIDDEN, INTER)}
    best = float("inf")
    for _ in range(reps):
        t0 = time.perf_counter()
        for _layer in range(LAYERS):
            for name, n, k in LAYER_LINEARS:
                oracle.q4_0_linear(xs[k], layer_blobs[name], n, threads=threads)
        oracle.q4_0_linear(xs[HIDDEN], lm_head_blob, VOCAB, threads=threads)
        best = min(best, time.perf_counter() - t0)
    return best


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


def committed_traffic():
    """dram__bytes_read.sum + dram__bytes_write.sum per launch of the dominant
    kernel, from the committed ncu summary (profiles/q4_gemv_traffic.json)."""
    p = os.path.join(ROOT, "profiles", "q4_gemv_traffic.json")
    if os.path.exists(p):
        with open(p) as fh:
            return json.load(fh).get("bytes_per_launch")
    return None


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

    build.build()
    dev = torch.device("cuda", local)
    stack = Q4DecodeStack(dev, M=1, seed=1234 + rank)
    cur = lambda: ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)  # noqa: E731

    # eager warm-up: sets kernel attributes, checks the path runs
    stack.step(cur())
    torch.cuda.synchronize()
    _native.device_status(reset=True)

    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        stack.step(cur())
    gd = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gd):
        for layer in range(LAYERS):
            stack.dominant_launch(cur(), layer)

    for _ in range(args.warmup):
        g.replay()
    torch.cuda.synchronize()
    barrier(world)

    _native.reset_counters()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        start.record()
        for _ in range(args.steps):
            g.replay()
        end.record()
        torch.cuda.synchronize()
    ms = start.elapsed_time(end) / args.steps
    barrier(world)
    ms = max_over_ranks(ms, world)

    # end to end: pinned H2D of the hidden state + step + D2H of the logits, every step
    h_host = torch.randn((1, HIDDEN)).to(torch.bfloat16).pin_memory()
    logits_host = torch.empty((1, VOCAB), dtype=torch.bfloat16).pin_memory()
    for _ in range(2):
        stack.h.copy_(h_host, non_blocking=True)
        g.replay()
        logits_host.copy_(stack.logits, non_blocking=True)
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        stack.h.copy_(h_host, non_blocking=True)
        g.replay()
        logits_host.copy_(stack.logits, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)

    # dominant kernel: 32 back-to-back gate/up GEMVs over the 32 layers' weights
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
    _native.device_status(reset=True)

    peak, peak_kind = measured_peaks()
    algo = stack.dominant_algorithmic_bytes()
    achieved = algo / (dom_us * 1e-6) / 1e9
    launches = stack.kernels_per_step * args.steps

    result = {
        "metric": METRIC,
        "value": world * 1000.0 / ms,
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "q4_0 x q8_0 -> f32 accumulate (bf16 activations)",
        "data": "synthetic: random Q4_0 weights (codes U[-8,7], scales f16(|N(0,1)|*0.01)), N(0,1) activations",
        "config": {"workload": "Llama-3-8B-shaped Q4_0 decode, batch 1: the Q4_0 linears of one token "
                               "(32 x [qkv 6144x4096, o 4096x4096, gate_up 28672x4096, down 4096x14336] + "
                               "lm_head 128256x4096), each after the Q8_0 activation quantiser; CUDA graph",
                   "global_batch": world, "parallelism": f"replicas{world}",
                   "l2": "inputs larger than L2 (4.22 GB of weights per step)",
                   "weight_bytes_per_token": stack.weight_bytes,
                   "hbm_roofline_tok_s_per_gpu": peak * 1e9 / stack.weight_bytes},
        "roofline": {"bound": "hbm", "kernel": "q4_gemv_q8_kernel (gate_up 28672x4096, M=1)", "achieved": achieved,
                     "peak": peak, "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": committed_traffic(), "algorithmic_bytes": algo, "avg_launch_us": dom_us},
        "step_hbm_frac": (stack.weight_bytes / (ms * 1e-3) / 1e9) / peak,
        "e2e": {"value": world * 1000.0 / e2e_ms, "unit": "tok/s", "h2d_bytes_per_step": HIDDEN * 2,
                "d2h_bytes_per_step": VOCAB * 2},
        "gpu_launches": launches,
        "clocks": clocks.summary(),
        "counters": _native.counters(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        blobs = {name: stack.layers[0][name].cpu().numpy() for name, _, _ in LAYER_LINEARS}
        lm = stack.lm_head.cpu().numpy()
        th = host_threads()
        sec = cpu_step_seconds(blobs, lm, th, reps=3)
        result["cpu_baseline"] = {"value": 1.0 / sec, "unit": "tok/s", "cores": th, "kind": "port",
                                  "sample": "one token: layer 0's four Q4_0 linears run 32 times + lm_head, "
                                            "oracle/tn_oracle.c restatement of the reference CPU arithmetic, "
                                            "min of 3"}
    return result


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
    for _ in range(args.warmup):
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
        "config": {"workload": "Llama-3-8B-shaped Q4_0 decode, batch 1: the Q4_0 linears of one token "
                               "(layer weights reused per layer on the CPU)", "global_batch": 1,
                   "parallelism": "host CPU"},
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": th, "kind": "port",
                         "sample": "one token per step: one layer's four Q4_0 linears run 32 times + lm_head"},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    args = parse()
    if args.case == "gemv":
        run_case_gemv(args)
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
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()



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
    for n, k in ((14336, 4096), (4096, 14336), (6144, 4096), (28672, 4096)):
        wbytes = q4_bytes(n, k)
        copies = max(2, -(-300_000_000 // wbytes))
        ws = [random_q4_blob(n, k, gen, dev) for _ in range(copies)]
        x = torch.randn((M, k), device=dev, generator=gen).to(torch.bfloat16)
        codes = torch.empty((M, k), device=dev, dtype=torch.int8)
        scales = torch.empty((M, k // 32), device=dev)
        offs = torch.empty((M, k // 32), device=dev)
        y = torch.empty((M, n), device=dev, dtype=torch.bfloat16)
        s = lambda: P(torch.cuda.current_stream().cuda_stream)  # noqa: E731
        N.check(L.tn_q8_0_quantize_planar(P(x.data_ptr()), N.TN_BF16, k, P(codes.data_ptr()), k,
                                          P(scales.data_ptr()), P(offs.data_ptr()), M, k, s()))

        def launch(w):
            N.check(L.tn_q4_0_linear_q8(P(codes.data_ptr()), k, P(scales.data_ptr()), P(offs.data_ptr()),
                                        P(w.data_ptr()), None, P(y.data_ptr()), N.TN_BF16, M, n, k,
                                        N.TN_WEIGHTS_STATIC, s()))

        launch(ws[0])
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for w in ws:
                launch(w)
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
        print(json.dumps({"case": "gemv", "M": M, "N": n, "K": k, "us_per_launch": us,
                          "GBps": algo / us / 1e3, "frac": algo / us / 1e3 / peak, "peak": peak,
                          "peak_kind": peak_kind, "copies": copies}), flush=True)
        del ws
        torch.cuda.empty_cache()
    N.device_status(reset=True)


if __name__ == "__main__":
    main()
