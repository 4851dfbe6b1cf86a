"""Oracle top-K attention: exact q.k selection, then the sparse gather.

The workload of the reference's oracle runs (ossa/bench/sparse_forward.py:194-202
selects the top-K keys of q k^T / sqrt(D) per query, then attends over them):
bf16, B = 4, 12 query / 2 kv heads, head_dim 128, N = 8192, causal, K in {32, 128}.
q and k are unit-normal plus a rank-8 component shared by all heads (each query
and key mixes the same 8 directions with its own N(0, 1) weights), so a query's
best keys stand out; v is unit-normal.  All tensors are seeded and synthetic.

Each step runs the selection (``oracle_topk``: the tensor-core selector at
head_dim 128, or with ``--exact`` the CUDA-core exact selector) and the gather
(``topk_attention``) on device-resident inputs.  W warm-up steps, then K steps
timed with CUDA events on the current stream (inputs are larger than L2).
``--check`` also compares the tensor-core indices with the exact selector's on
the full input.

    python -m ossa_b200.bench.oracle_select [--batch 4] [--seq 8192] [--k 32] [--steps 5] [--warmup 3]

Prints one JSON line: milliseconds per step for selection and gather, and
query tokens per second through both.
"""

from __future__ import annotations

import argparse
import json
import math
import os

import torch

from ..select import oracle_topk, oracle_topk_with_status
from ..topk_attention import topk_attention


def make_inputs(B, H, Hkv, N, D, device, seed=3, rank=8):
    g = torch.Generator(device=device).manual_seed(seed)
    basis = torch.linalg.qr(torch.randn(D, rank, device=device, generator=g))[0].T * math.sqrt(D / rank)
    q = torch.randn(B, H, N, D, device=device, generator=g) + \
        torch.randn(B, H, N, rank, device=device, generator=g) @ basis
    k = torch.randn(B, Hkv, N, D, device=device, generator=g) + \
        torch.randn(B, Hkv, N, rank, device=device, generator=g) @ basis
    v = torch.randn(B, Hkv, N, D, device=device, generator=g)
    return q.bfloat16(), k.bfloat16(), v.bfloat16()


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--heads", type=int, default=12)
    ap.add_argument("--kv-heads", type=int, default=2)
    ap.add_argument("--seq", type=int, default=8192)
    ap.add_argument("--k", type=int, default=32)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--exact", action="store_true", help="CUDA-core exact selector instead of the tensor-core one")
    ap.add_argument("--check", action="store_true", help="compare with the exact selector on the full input")
    args = ap.parse_args(argv)
    if args.exact:
        os.environ["OSSA_ORACLE_SELECT"] = "exact"
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    B, H, Hkv, N, D, K = args.batch, args.heads, args.kv_heads, args.seq, 128, args.k
    q, k, v = make_inputs(B, H, Hkv, N, D, dev)
    stream = torch.cuda.current_stream()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    with torch.inference_mode():
        for _ in range(max(1, args.warmup)):
            idx = oracle_topk(q, k, K)
            out = topk_attention(q, k, v, topk_indices=idx)
        _, fallback_rows, status = oracle_topk_with_status(q, k, K)
        torch.cuda.synchronize()
        for e in ev:
            e[0].record(stream)
            idx = oracle_topk(q, k, K)
            e[1].record(stream)
            out = topk_attention(q, k, v, topk_indices=idx)
            e[2].record(stream)
        torch.cuda.synchronize()
        sel = sum(e[0].elapsed_time(e[1]) for e in ev) / len(ev)
        gat = sum(e[1].elapsed_time(e[2]) for e in ev) / len(ev)
        equal = None
        if args.check:
            os.environ["OSSA_ORACLE_SELECT"] = "exact"
            try:
                equal = bool(torch.equal(oracle_topk(q, k, K), idx))
            finally:
                if not args.exact:
                    del os.environ["OSSA_ORACLE_SELECT"]
    print(json.dumps({
        "metric": "oracle top-K attention query tokens/s (selection + gather)",
        "value": B * N / ((sel + gat) / 1e3), "unit": "tokens/s",
        "select_ms": sel, "gather_ms": gat, "steps": args.steps, "warmup": args.warmup,
        "selector": "exact CUDA-core" if args.exact else "tensor-core (exact indices)",
        "equal_to_exact": equal, "output_finite": bool(torch.isfinite(out).all()),
        "fallback_rows": fallback_rows, "status": status,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "oracle top-K attention, unit-normal q/k plus a shared rank-8 component",
                   "batch": B, "heads": H, "kv_heads": Hkv, "seq_len": N, "head_dim": D, "top_k": K},
    }), flush=True)


if __name__ == "__main__":
    main()
