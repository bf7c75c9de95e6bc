"""Phase timeline of the persistent decode kernel (tn_llama_decode_token_timeline).

    python -m torchnative_b200.mega_timeline [--layers N] [--context S] [--tokens T]

Builds a Llama-3-8B-shaped Q4_0 model (random weights, `--layers` of them,
default all 32) with a `--context`-token cache, runs `--tokens` tokens of the
persistent kernel, then one more with the timeline recorded, and prints, per
recorded event of layer 1, the minimum / median / maximum over CTAs in
microseconds from the earliest CTA's layer-1 start, plus the plain time per
token. A diagnostic of the kernel's schedule (which phase waits on what); the
token it runs is an ordinary one.
"""

from __future__ import annotations

import argparse
import ctypes
import json

import numpy as np
import torch

from . import _native as N, build
from .llama_decode import LLAMA3_8B, Q4LlamaDecoder

EVENTS = ["start", "Q wait", "Q done", "A wait", "A done", "O wait", "O done", "G wait", "G done", "D wait",
          "D done", "producer Q", "producer A", "producer O", "producer G", "producer D", "producer end", "end",
          "Q staged", "A staged", "A merged", "A posted"]
SLOTS = 64


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=LLAMA3_8B.layers)
    ap.add_argument("--context", type=int, default=2048)
    ap.add_argument("--tokens", type=int, default=10)
    ap.add_argument("--json", default=None, help="also write the summary here")
    args = ap.parse_args(argv)
    build.build()
    N.lib()
    dev = torch.device("cuda", 0)
    dec = Q4LlamaDecoder(LLAMA3_8B, batch=1, capacity=args.context + args.tokens + 16, device=dev, seed=5,
                         layers=args.layers, mega=True)
    dec.fill_prompt_cache(args.context)
    dec.start(torch.tensor([1234], device=dev))
    for _ in range(3):
        dec.step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.tokens):
        dec.step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.tokens
    G = torch.cuda.get_device_properties(dev).multi_processor_count
    stamps = torch.zeros((G, SLOTS), dtype=torch.int64, device=dev)
    P = ctypes.c_void_p
    N.check(N.lib().tn_llama_decode_token_timeline(dec._mega, P(dec.tokens.data_ptr()), P(dec.pos.data_ptr()),
                                                   P(dec.logits.data_ptr()), P(stamps.data_ptr()),
                                                   P(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    N.device_status(reset=True)
    s = stamps.cpu().numpy().astype(np.float64)
    t0 = s[:, 1][s[:, 1] > 0].min()
    out = {"ms_per_token": ms, "tok_s": 1000.0 / ms, "layers": args.layers, "context": args.context, "events": {}}
    print(f"{ms:.4f} ms per token ({1000.0 / ms:.1f} tok/s), {args.layers} layers, {args.context}-token cache")
    for i, name in enumerate(EVENTS):
        col = s[:, i]
        col = col[col > 0]
        if col.size == 0:
            continue
        rel = (col - t0) / 1000.0
        out["events"][name] = [round(float(rel.min()), 2), round(float(np.median(rel)), 2), round(float(rel.max()), 2)]
        print(f"{name:14s} min {rel.min():8.2f}  median {np.median(rel):8.2f}  max {rel.max():8.2f} us")
    d = s[:, 10][s[:, 10] > 0]
    if d.size:
        out["layer_us"] = float((d.max() - t0) / 1000.0)
        print(f"layer 1: {out['layer_us']:.2f} us")
    if args.json:
        with open(args.json, "w") as fh:
            json.dump(out, fh)
    dec.close()
    return out


if __name__ == "__main__":
    main()
