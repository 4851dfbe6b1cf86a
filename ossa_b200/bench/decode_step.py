"""Decode step: one new token per (b, head) against a long routed context.

Workload: B = 1, 12 query / 2 kv heads, head_dim 128, a context of N positions
(default 32k and 128k), causal top-K in {64, 128}, random-init router (r = 64),
bf16 q/k/v ~ N(0, 1)/sqrt(128), seeded and synthetic.  The key and value caches
and the router's projected-key cache (``RouterKeyCache``) are preallocated at
capacity and filled with the first N - 1 positions; each step appends one
position (its key projected once), selects for the new query row among all
cached keys, and runs the gather for that row.  The reference has no decode
path (its patched forward is prefill-only).

    python -m ossa_b200.bench.decode_step [--seq 32768,131072] [--k 64,128] [--steps 20] [--warmup 3]

Prints one JSON line per (N, K): microseconds per decode step (device time,
CUDA events around the steps) and the selection's share of it.
"""

from __future__ import annotations

import argparse
import json
import math

import torch

from ..decode import RouterKeyCache
from ..router import ContentRouter, ContentRouterConfig
from ..topk_attention import topk_attention


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--seq", default="32768,131072")
    ap.add_argument("--k", default="64,128")
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, H, Hkv, D, r = 1, 12, 2, 128, 64
    for N in (int(x) for x in args.seq.split(",")):
        for K in (int(x) for x in args.k.split(",")):
            g = torch.Generator(device=dev).manual_seed(N + K)
            s = 1.0 / math.sqrt(D)
            steps = args.warmup + args.steps
            cap = N + steps
            k = (torch.randn(B, Hkv, cap, D, device=dev, generator=g) * s).bfloat16()
            v = (torch.randn(B, Hkv, cap, D, device=dev, generator=g) * s).bfloat16()
            q = (torch.randn(steps, B, H, 1, D, device=dev, generator=g) * s).bfloat16()
            router = ContentRouter(ContentRouterConfig(head_dim=D, n_heads=H, seq_len=cap, proj_dim=r)).to(dev)
            cache = RouterKeyCache(router, B, Hkv, capacity=cap)
            cache.append(k[:, :, :N - 1])
            ev = []
            with torch.inference_mode():
                for t in range(steps):
                    e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
                    pos = cache.length
                    e[0].record()
                    cache.append(k[:, :, pos:pos + 1])
                    idx = cache.topk(q[t], K)
                    e[1].record()
                    out = topk_attention(q[t], k, v, topk_indices=idx, q_start=pos)
                    e[2].record()
                    if t >= args.warmup:
                        ev.append(e)
                torch.cuda.synchronize()
            sel = sum(e[0].elapsed_time(e[1]) for e in ev) / len(ev) * 1e3
            gat = sum(e[1].elapsed_time(e[2]) for e in ev) / len(ev) * 1e3
            print(json.dumps({
                "metric": "decode step latency (append key, select, gather)", "value": sel + gat, "unit": "us",
                "select_us": sel, "gather_us": gat, "higher_is_better": False, "steps": args.steps,
                "warmup": args.warmup, "dtype": "bf16", "data": "synthetic",
                "output_finite": bool(torch.isfinite(out).all()),
                "config": {"workload": "decode, B=1, 12/2 heads, head_dim 128, random-init router (r=64)",
                           "context": N, "top_k": K},
            }), flush=True)
            del k, v, q, cache, router
            torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
