"""Full-model prefill with every attention layer on the routed sparse path.

The workload of the reference's full-model runs (ossa/bench/sparse_forward.py:
the patched Qwen2 model, every layer routed): the Qwen2.5-1.5B architecture
(28 layers, hidden 1536, 12 query / 2 kv heads, head_dim 128, SwiGLU 8960, RoPE
theta 1e6, vocab 151936) with random weights, bf16, one random-init
ContentRouter (r = 64, Xavier-uniform projections, N(0, 1) position bias) per
layer, causal top-K = 64, prefill of uniform random token ids.  No checkpoint or
dataset is involved (none is available here); all tensors are seeded.

Data-parallel by batch: one process per GPU (torchrun sets RANK / WORLD_SIZE),
each rank runs global_batch / world sequences; no collective on the data path.
Timing: W warm-up forwards, then K forwards bracketed by a barrier and a
device synchronisation, measured with CUDA events on the current stream; the
maximum over ranks is reported.  Prefill computes the logits of the last
position only (logits_to_keep=1), as a serving prefill does.

    python -m ossa_b200.bench.full_model [--batch 16] [--seq 4096] [--steps 3] [--warmup 2]
    torchrun --nproc-per-node N -m ossa_b200.bench.full_model ...

Prints one JSON line (rank 0): tokens/s for the whole job and per GPU.
"""

from __future__ import annotations

import argparse
import json
import math
import os

import torch

from ..router import ContentRouter, ContentRouterConfig
from .sparse_forward import patch_all_layers


def qwen25_15b_config(seq_len: int):
    from transformers import Qwen2Config

    return Qwen2Config(hidden_size=1536, intermediate_size=8960, num_hidden_layers=28, num_attention_heads=12,
                       num_key_value_heads=2, vocab_size=151936, max_position_embeddings=max(seq_len, 32768),
                       rope_theta=1e6, tie_word_embeddings=True)


def build_model(cfg, device, seed: int = 0):
    """Random-init model in bf16 on `device` (initialised there directly)."""
    from transformers import Qwen2ForCausalLM

    torch.manual_seed(seed)
    with torch.device(device):
        model = Qwen2ForCausalLM(cfg)
    return model.to(torch.bfloat16).eval()


def build_routers(model, seq_len: int, device, seed: int = 0) -> dict[int, ContentRouter]:
    """One random-init router per decoder layer, fp32 parameters."""
    gen = torch.Generator().manual_seed(seed + 1)
    out = {}
    for li, layer in enumerate(model.model.layers):
        a = layer.self_attn
        r = ContentRouter(ContentRouterConfig(head_dim=a.head_dim, n_heads=model.config.num_attention_heads,
                                              seq_len=seq_len, proj_dim=64))
        with torch.no_grad():
            for w in (r.q_proj[0].weight, r.k_proj[0].weight):
                bound = math.sqrt(6.0 / (w.shape[0] + w.shape[1]))
                w.copy_((torch.rand(w.shape, generator=gen) * 2 - 1) * bound)
            r.pos_bias.weight.copy_(torch.randn(r.pos_bias.weight.shape, generator=gen))
        out[li] = r.to(device)
    return out


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=16, help="global batch (split over ranks)")
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--k", type=int, default=64)
    ap.add_argument("--layers", type=int, default=28)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=2)
    args = ap.parse_args(argv)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.batch % world:
        raise SystemExit(f"global batch {args.batch} is not a multiple of {world} ranks")
    if world > 1:
        from datetime import timedelta

        torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=120))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)

    cfg = qwen25_15b_config(args.seq)
    cfg.num_hidden_layers = args.layers
    model = build_model(cfg, dev)
    routers = build_routers(model, args.seq, dev)
    patch_all_layers(model, "router", args.k, routers=routers, impl="gather")

    b_local = args.batch // world
    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    ids = torch.randint(0, cfg.vocab_size, (b_local, args.seq), device=dev, generator=gen)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    def step():
        return model(input_ids=ids, use_cache=False, logits_to_keep=1).logits

    with torch.inference_mode():
        for _ in range(max(1, args.warmup)):
            out = step()
        torch.cuda.synchronize()
        finite = bool(torch.isfinite(out).all())
        barrier()
        torch.cuda.synchronize()
        stream = torch.cuda.current_stream()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(args.steps):
            out = step()
        t1.record(stream)
        torch.cuda.synchronize()
        barrier()
        ms = t0.elapsed_time(t1)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms = float(t.item())
    tokens = args.batch * args.seq * args.steps
    if rank == 0:
        print(json.dumps({
            "metric": "full-model prefill tokens/s (all layers routed)",
            "value": tokens / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
            "per_gpu_tokens_s": tokens / (ms / 1e3) / world, "ms_per_step": ms / args.steps,
            "steps": args.steps, "warmup": args.warmup, "dtype": "bf16", "data": "synthetic",
            "logits_finite": finite,
            "config": {"workload": "Qwen2.5-1.5B architecture, random init, every layer routed (top-K "
                                   f"{args.k}, r=64), prefill", "global_batch": args.batch, "seq_len": args.seq,
                       "layers": args.layers, "parallelism": f"dp{world}"},
        }), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
