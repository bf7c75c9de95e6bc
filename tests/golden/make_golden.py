"""Regenerate the committed golden fixtures in this directory.

    python tests/golden/make_golden.py --reference /path/to/torchnative

Writes two files:

* ``q4_gguf_golden.json`` -- the Q4_0 and Q8_0 cases of the reference's
  ``scripts/q4quality/golden_gguf_py.json``: llama.cpp gguf-py's own bytes and
  dequantised bits for ten hand-built blocks (gauss, pos/neg extreme, zero,
  opposite signs, an f16-subnormal scale, two rows; Q8_0 gauss and exact .5
  ties) and its Q4_K case (three super-blocks written by llama.cpp, with
  gguf-py's dequantised bits). Copied value for value with its provenance, so
  the tests can pin the oracle's codec to them on a machine without the
  reference tree.

* ``sdpa_golden.json`` -- the reference's golden SDPA cases for
  ``aten._scaled_dot_product_flash_attention_for_cpu`` (tests/golden/cases.py
  :10976-11150 of the reference: plain / causal / explicit-scale (1,2,3,4) in
  four dtypes, an additive mask with a -inf column, causal q_len=2 kv_len=5,
  causal q_len > kv_len, a 9x9 causal block at scale 0.1), with inputs from the
  same linear congruential sequence the reference uses so both libraries see
  the same numbers, plus GQA cases. Each case stores upstream torch's CPU
  answer (out, logsumexp) and a float64 math answer.

Running it needs upstream torch (CPU) and, for the first file, the reference
tree; the tests only read the JSON.
"""

from __future__ import annotations

import argparse
import json
import math
import os

HERE = os.path.dirname(os.path.abspath(__file__))


def deterministic(n: int, seed: int = 1) -> list[float]:
    """n reproducible values in about [-1, 1]: the glibc-constant LCG the
    reference's golden harness feeds both libraries (tests/golden/cases.py
    :10231-10247 of the reference)."""
    out, state = [], seed
    for _ in range(n):
        state = (state * 1103515245 + 12345) % 2147483648
        out.append(round((state / 2147483648.0) * 2.0 - 1.0, 4))
    return out


def q4_fixture(reference: str) -> dict:
    src = os.path.join(reference, "scripts", "q4quality", "golden_gguf_py.json")
    with open(src) as fh:
        doc = json.load(fh)
    cases = [c for c in doc["cases"] if c["format"] in ("q4_0", "q8_0", "q4_k")]
    return {
        "what": "llama.cpp gguf-py bytes/bits for Q4_0, Q8_0 and Q4_K blocks, copied from the reference's "
        "scripts/q4quality/golden_gguf_py.json",
        "provenance": doc["provenance"],
        "cases": cases,
    }


def sdpa_cases() -> list[dict]:
    cases = []
    b, h, t, e = 1, 2, 3, 4
    n = b * h * t * e
    qf, kf, vf = deterministic(n, 1), deterministic(n, 2), deterministic(n, 3)
    for dt in ("float32", "float64", "float16", "bfloat16"):
        for causal, scale, note in ((False, None, "plain"), (True, None, "causal upper-left"),
                                    (False, 0.25, "explicit scale")):
            cases.append(dict(name=f"{note} {dt}", dtype=dt, q=qf, k=kf, v=vf, q_shape=[b, h, t, e],
                              kv_shape=[b, h, t, e], causal=causal, scale=scale, mask=None))
    mask = [0.0, 0.0, float("-inf")] * t
    for dt in ("float64", "float32"):
        for causal in (False, True):
            cases.append(dict(name=f"additive -inf column mask causal={causal} {dt}", dtype=dt, q=qf, k=kf, v=vf,
                              q_shape=[b, h, t, e], kv_shape=[b, h, t, e], causal=causal, scale=None,
                              mask=mask, mask_shape=[1, 1, t, t]))
    kv = 5
    for dt in ("float64", "float32"):
        cases.append(dict(name=f"causal q_len=2 kv_len=5 {dt}", dtype=dt, q=deterministic(2 * e, 4),
                          k=deterministic(kv * e, 5), v=deterministic(kv * e, 6), q_shape=[1, 1, 2, e],
                          kv_shape=[1, 1, kv, e], causal=True, scale=None, mask=None))
    for ql, kl in ((5, 2), (9, 3)):
        for dt in ("float64", "float32"):
            cases.append(dict(name=f"causal q_len={ql} kv_len={kl} {dt}", dtype=dt, q=deterministic(2 * ql * e, 7),
                              k=deterministic(2 * kl * e, 8), v=deterministic(2 * kl * e, 9), q_shape=[1, 2, ql, e],
                              kv_shape=[1, 2, kl, e], causal=True, scale=None, mask=None))
    for dt in ("float64", "float32"):
        cases.append(dict(name=f"9x9 causal scale=0.1 {dt}", dtype=dt, q=deterministic(2 * 9 * e, 10),
                          k=deterministic(2 * 9 * e, 11), v=deterministic(2 * 9 * e, 12), q_shape=[1, 2, 9, e],
                          kv_shape=[1, 2, 9, e], causal=True, scale=0.1, mask=None))
    # GQA (query head h reads kv head h // (Hq/Hkv)), decode and prefill shapes.
    for dt in ("float32", "bfloat16"):
        for (bb, hq, hk, ql, kl, d, causal) in ((1, 6, 3, 5, 5, 8, True), (2, 4, 2, 1, 9, 8, False),
                                               (1, 4, 1, 3, 7, 16, True)):
            seed = 100 + ql * 7 + kl
            cases.append(dict(name=f"gqa {hq}/{hk} L={ql} S={kl} D={d} causal={causal} {dt}", dtype=dt,
                              q=deterministic(bb * hq * ql * d, seed), k=deterministic(bb * hk * kl * d, seed + 1),
                              v=deterministic(bb * hk * kl * d, seed + 2), q_shape=[bb, hq, ql, d],
                              kv_shape=[bb, hk, kl, d], causal=causal, scale=None, mask=None))
    return cases


def run_upstream(case: dict) -> dict:
    import torch

    dt = getattr(torch, case["dtype"])
    q = torch.tensor(case["q"], dtype=torch.float64).reshape(case["q_shape"])
    k = torch.tensor(case["k"], dtype=torch.float64).reshape(case["kv_shape"])
    v = torch.tensor(case["v"], dtype=torch.float64).reshape(case["kv_shape"])
    mask = None
    if case.get("mask") is not None:
        mask = torch.tensor(case["mask"], dtype=torch.float64).reshape(case["mask_shape"])
    hq, hk = q.shape[1], k.shape[1]
    rep = hq // hk
    k_full, v_full = k.repeat_interleave(rep, dim=1), v.repeat_interleave(rep, dim=1)
    kw = {}
    if case["scale"] is not None:
        kw["scale"] = case["scale"]
    out, lse = torch.ops.aten._scaled_dot_product_flash_attention_for_cpu(
        q.to(dt), k_full.to(dt), v_full.to(dt), 0.0, case["causal"],
        attn_mask=None if mask is None else mask.to(dt), **kw)
    # float64 math answer, upper-left causal, from the float64 values of the dtype-rounded inputs
    qr, kr, vr = (t.to(dt).to(torch.float64) for t in (q, k_full, v_full))
    scale = case["scale"] if case["scale"] is not None else 1.0 / math.sqrt(q.shape[-1])
    s = qr @ kr.transpose(-1, -2) * scale
    if case["causal"]:
        L, S = s.shape[-2], s.shape[-1]
        keep = torch.ones(L, S, dtype=torch.bool).tril()
        s = s.masked_fill(~keep, float("-inf"))
    if mask is not None:
        s = s + mask.to(dt).to(torch.float64)
    ref = torch.softmax(s, dim=-1) @ vr
    ref_lse = torch.logsumexp(s, dim=-1)
    return dict(out=out.to(torch.float64).reshape(-1).tolist(), lse=lse.to(torch.float64).reshape(-1).tolist(),
                out_f64=ref.reshape(-1).tolist(), lse_f64=ref_lse.reshape(-1).tolist(), torch=torch.__version__)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None, help="root of the torchnative checkout")
    ap.add_argument("--q4-only", action="store_true", help="write only q4_gguf_golden.json")
    args = ap.parse_args()
    if args.reference:
        with open(os.path.join(HERE, "q4_gguf_golden.json"), "w") as fh:
            json.dump(q4_fixture(args.reference), fh, indent=1)
    if args.q4_only:
        return
    cases = sdpa_cases()
    for c in cases:
        c.update(run_upstream(c))
    with open(os.path.join(HERE, "sdpa_golden.json"), "w") as fh:
        json.dump({"what": "reference golden SDPA cases answered by upstream torch CPU "
                   "(_scaled_dot_product_flash_attention_for_cpu) and float64 math", "cases": cases}, fh)
    print(f"wrote {len(cases)} sdpa cases")


if __name__ == "__main__":
    main()
