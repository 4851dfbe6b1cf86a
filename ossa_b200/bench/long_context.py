"""Long-context routed sparse attention, query blocks sharded over the GPUs.

The long-context workload: B = 1, 12 query / 2 kv heads, head_dim 128,
N in {32k, 64k, 128k}, causal top-K = 128, random-init router (r = 64,
Xavier-uniform projections, N(0, 1) position bias), q/k/v ~ N(0, 1)/sqrt(128) in
bf16, all seeded and synthetic.  One process per GPU (torchrun sets RANK /
WORLD_SIZE); every rank builds the same inputs, keeps its two zig-zag query
blocks, and each step runs ``sharded_routed_attention``: an NCCL all-gather of
K and V, then selection and the gather for the rank's rows.  On one process
the same call runs the whole sequence.

Timing: W warm-up steps, then K steps between a barrier and a device
synchronisation, CUDA events on the current stream, the maximum over ranks.

    python -m ossa_b200.bench.long_context [--seq 32768,65536,131072] [--k 128] [--steps 3] [--warmup 2]
    torchrun --nproc-per-node N -m ossa_b200.bench.long_context ...

Prints one JSON line per sequence length (rank 0): query tokens/s for the
whole job and milliseconds per step.
"""

from __future__ import annotations

import argparse
import json
import math
import os

import torch
import torch.distributed as dist

from ..sequence_shard import local_rows, sharded_routed_attention


def make_inputs(N, device, seed=0, B=1, H=12, Hkv=2, D=128, r=64):
    g = torch.Generator(device=device).manual_seed(seed)
    s = 1.0 / math.sqrt(D)
    q = (torch.randn(B, H, N, D, device=device, generator=g) * s).bfloat16()
    k = (torch.randn(B, Hkv, N, D, device=device, generator=g) * s).bfloat16()
    v = (torch.randn(B, Hkv, N, D, device=device, generator=g) * s).bfloat16()
    bound = math.sqrt(6.0 / (r + D))
    wq = (torch.rand(r, D, device=device, generator=g) * 2 - 1) * bound
    wk = (torch.rand(r, D, device=device, generator=g) * 2 - 1) * bound
    pb = torch.randn(2 * N, 1, device=device, generator=g)
    return q, k, v, wq, wk, pb


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--seq", default="32768,65536,131072")
    ap.add_argument("--k", type=int, default=128)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=2)
    args = ap.parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    for N in (int(x) for x in args.seq.split(",")):
        q, k, v, wq, wk, pb = make_inputs(N, dev)
        ql, kl, vl = local_rows(q, world, rank), local_rows(k, world, rank), local_rows(v, world, rank)
        del q, k, v

        def step():
            return sharded_routed_attention(ql, kl, vl, wq, wk, pb, N, args.k)

        with torch.inference_mode():
            for _ in range(max(1, args.warmup)):
                out = step()
            torch.cuda.synchronize()
            barrier()
            torch.cuda.synchronize()
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record()
            for _ in range(args.steps):
                out = step()
            t1.record()
            torch.cuda.synchronize()
            barrier()
        ms = torch.tensor([t0.elapsed_time(t1) / args.steps], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        ms = float(ms.item())
        finite = bool(torch.isfinite(out).all())
        if rank == 0:
            print(json.dumps({
                "metric": "long-context routed sparse attention query tokens/s (sequence-sharded)",
                "value": N / (ms / 1e3), "unit": "tokens/s", "n_gpus": world, "ms_per_step": ms,
                "steps": args.steps, "warmup": args.warmup, "scaling": "strong", "dtype": "bf16",
                "data": "synthetic", "output_finite": finite,
                "config": {"workload": "single-layer routed sparse attention, B=1, 12/2 heads, head_dim 128, "
                                       f"causal top-K={args.k}, random-init router (r=64)", "seq_len": N,
                           "parallelism": f"sequence zig-zag x{world}"},
            }), flush=True)
        del ql, kl, vl, out
        torch.cuda.empty_cache()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
