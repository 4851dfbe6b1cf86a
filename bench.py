"""Routed sparse-attention benchmark (router score + causal top-K select + gather).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one pass of the hot path over one batch of the single-layer
workload: ContentRouter projection + fused causal top-K selection
(ossa_router_topk) + gathered sparse attention (ossa_topk_attention_fwd).
Default workload is the bf16 single-GPU configuration: B=8, 12 query / 2 kv
heads, head_dim 128, seq 4096, K=64, random-init router (r=64, seq_len 4096),
q/k/v ~ N(0,1)/sqrt(128), synthetic and seeded.

With N GPUs (torchrun, one process per GPU) every rank runs its own batch:
independent replicas, no collective on the data path (weak scaling).  The
timed region is bracketed by a barrier and synchronize on both sides, every
step is timed with CUDA events on the launching stream, L2 is flushed between
steps (outside the events), and the max over ranks is reported.

``--impl reference`` times the reference's PyTorch path (restated in
oracle/reference_port.py) on the host CPU cores with all threads, on a bounded
sample of the same workload; only rank 0 runs it.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
METRIC = "routed sparse-attn tokens/s/GPU (seq 4k–128k, K=64) + % HBM/tensor roofline"

WORKLOAD = dict(B=8, H=12, Hkv=2, N=4096, D=128, K=64, r=64, seq_len=4096)
WORKLOAD_NAME = ("single-layer routed sparse attention, bf16: B=8, 12/2 heads, head_dim 128, seq 4096, "
                 "random-init router (r=64), causal top-K=64")


def _peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def _traffic() -> dict:
    """Per-launch DRAM bytes from an ncu capture (profiles/ncu_traffic.json), if any."""
    p = ROOT / "profiles" / "ncu_traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except ValueError:
            return {}
    return {}


def gather_bytes(B, H, N, D, K) -> int:
    """Algorithmic bytes of one gather launch: per (b, q-head, query) the q row,
    K int32 indices, K key rows and K value rows (bf16), and the output row."""
    return B * H * N * (D * 2 + K * 4 + 2 * K * D * 2 + D * 2)


def select_flops(B, H, Hkv, N, D, r) -> int:
    """Algorithmic flops of router projection + causal scoring (selection adds
    compares only): q' and k' projections (GQA: k' once per kv head) and
    r-dimensional dot products over the causal triangle."""
    return B * H * N * 2 * D * r + B * Hkv * N * 2 * D * r + B * H * (N * (N + 1) // 2) * 2 * r


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region: sampling starts
    before the region (the first sample is awaited, so the region is covered from its
    start) and only samples taken inside the region are summarised."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, local_index: int):
        # nvidia-smi numbers GPUs physically; map through CUDA_VISIBLE_DEVICES
        vis = [x.strip() for x in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if x.strip()]
        self.gpu_index = vis[local_index] if local_index < len(vis) else str(local_index)
        self.proc = None
        self.lines = []
        self.samples = []

    def _reader(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line))

    def __enter__(self):
        import threading

        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return self
        self.thread = threading.Thread(target=self._reader, daemon=True)
        self.thread.start()
        t_wait = time.monotonic()
        while not self.lines and time.monotonic() - t_wait < 5.0 and self.proc.poll() is None:
            time.sleep(0.01)
        self.t0 = time.monotonic()
        return self

    def __exit__(self, *exc):
        self.samples = []
        if self.proc is None:
            return False
        t1 = time.monotonic()
        time.sleep(0.06)  # let the sample that covers the end of the region arrive
        self.proc.terminate()
        try:
            self.proc.wait(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            self.proc.wait()
        self.thread.join(timeout=5)
        inside = [ln for t, ln in self.lines if self.t0 <= t <= t1 + 0.06]
        for line in inside:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) == 9:
                self.samples.append(parts)
        return False

    def summary(self) -> dict:
        if not getattr(self, "samples", None):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


def _config(world: int) -> dict:
    """The workload description both arms print (same keys, so the two lines
    describe the same job)."""
    return {"workload": WORKLOAD_NAME, "global_batch": WORKLOAD["B"] * world, "seq_len": WORKLOAD["N"],
            **WORKLOAD,
            "l2": "flushed between steps (256 MB write, outside the timed events)",
            "parallelism": f"replicas x{world} (batch-sharded, no data-path collective)"}


# Long-context configurations reported beside the headline workload: B=1, 12/2
# heads, head_dim 128, random-init router; seq 32k at K=64 and 64k/128k at K=128.
LONG_CONTEXT = ((32768, 64), (65536, 128), (131072, 128))


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def make_inputs(device, seed: int, w=WORKLOAD):
    """Seeded synthetic inputs of the workload (generated on the device)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    s = 1.0 / math.sqrt(w["D"])
    q = (torch.randn(w["B"], w["H"], w["N"], w["D"], device=device, generator=g) * s).bfloat16()
    k = (torch.randn(w["B"], w["Hkv"], w["N"], w["D"], device=device, generator=g) * s).bfloat16()
    v = (torch.randn(w["B"], w["Hkv"], w["N"], w["D"], device=device, generator=g) * s).bfloat16()
    gc = torch.Generator()
    gc.manual_seed(seed + 1)
    wq = torch.empty(w["r"], w["D"])
    wk = torch.empty(w["r"], w["D"])
    torch.nn.init.xavier_uniform_(wq, generator=gc)
    torch.nn.init.xavier_uniform_(wk, generator=gc)
    pb = torch.randn(2 * w["seq_len"], 1, generator=gc)
    return q, k, v, wq.to(device), wk.to(device), pb.to(device)


def _max_over_ranks(vals, dev, world):
    t = torch.tensor(vals, dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return t.tolist()


def run_long_context(dev, world, rank, steps: int, warmup: int) -> list:
    """Selection and gather at long context (LONG_CONTEXT), every rank its two
    zig-zag query blocks of the sequence (one process: the whole sequence).  Per
    step: the NCCL all-gather of K and V (N > 1), router_topk and topk_attention
    on the rank's rows, each timed with CUDA events on the launching stream; the
    step time and each part are maxima over ranks.  Inputs are larger than L2 (q
    alone is 100-400 MB), so no flush is needed between steps."""
    from ossa_b200 import router_topk, topk_attention
    from ossa_b200.bench.long_context import make_inputs
    from ossa_b200.select import project_router_keys, router_topk_projected
    from ossa_b200.sequence_shard import gather_sequence, local_rows, zigzag_blocks

    peaks = _peaks()
    traffic = _traffic()
    stream = torch.cuda.current_stream(dev)
    out = []
    for N, K in LONG_CONTEXT:
        q, k, v, wq, wk, pb = make_inputs(N, dev, seed=7)
        ql, kl, vl = local_rows(q, world, rank), local_rows(k, world, rank), local_rows(v, world, rank)
        del q, k, v
        blk = ql.shape[2] // 2
        if world == 1:  # the whole sequence in one call
            blocks, qbs = [(0, N)], [ql]
        else:
            blocks = zigzag_blocks(N, world, rank)
            qbs = [ql[:, :, h * blk:(h + 1) * blk].contiguous() for h in range(2)]

        def step(evs=None):
            if evs:
                evs[0].record(stream)
            kf = gather_sequence(kl, world)
            vf = gather_sequence(vl, world)
            if evs:
                evs[1].record(stream)
            if world == 1:
                idxs = [router_topk(qbs[0], kf, wq, wk, pb, N, K, causal=True, q_start=0)]
            else:  # the keys projected once for the rank's two query blocks
                kp = project_router_keys(kf, wk)
                idxs = [router_topk_projected(qb, kp, wq, pb, N, K, causal=True, q_start=st)
                        for qb, (st, _) in zip(qbs, blocks)]
            if evs:
                evs[2].record(stream)
            outs = [topk_attention(qb, kf, vf, topk_indices=ix, causal=True, q_start=st)
                    for qb, ix, (st, _) in zip(qbs, idxs, blocks)]
            if evs:
                evs[3].record(stream)
            return outs

        with torch.inference_mode():
            for _ in range(max(1, warmup)):
                step()
            if world > 1:
                torch.distributed.barrier()
            torch.cuda.synchronize()
            evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(steps)]
            for e in evs:
                step(e)
            torch.cuda.synchronize()
            if world > 1:
                torch.distributed.barrier()
        ag = sum(e[0].elapsed_time(e[1]) for e in evs) / steps
        sel = sum(e[1].elapsed_time(e[2]) for e in evs) / steps
        gat = sum(e[2].elapsed_time(e[3]) for e in evs) / steps
        tot = sum(e[0].elapsed_time(e[3]) for e in evs) / steps
        tot, ag, sel, gat = _max_over_ranks([tot, ag, sel, gat], dev, world)
        rows_local = 2 * blk  # query rows of this rank per head
        # per-rank algorithmic work of the largest rank (zig-zag ranks are balanced)
        sflops = (12 * rows_local * 2 * 128 * 64 + 2 * N * 2 * 128 * 64 +
                  12 * sum(((e - 1) * e - (s - 1) * s) // 2 + (e - s) for s, e in blocks) * 2 * 64)
        gbytes = gather_bytes(1, 12, rows_local, 128, K)
        tkey = f"gather_attn_fwd_n{N}_k{K}"
        entry = {
            "seq_len": N, "K": K, "n_gpus": world, "ms_per_step": tot, "tokens_s": N / (tot / 1e3),
            "allgather_ms": ag if world > 1 else 0.0, "select_ms": sel, "gather_ms": gat,
            "select": {"bound": "tensor", "achieved": sflops / (sel / 1e3) / 1e12, "peak": peaks["bf16_tflops"],
                       "unit": "TFLOP/s", "algorithmic": f"{sflops} flop per rank per step"},
            "gather": {"bound": "hbm", "achieved": gbytes / (gat / 1e3) / 1e9, "peak": peaks["hbm_gbs"],
                       "unit": "GB/s", "algorithmic": f"{gbytes} B per rank per step",
                       "traffic": traffic.get(tkey) if world == 1 else None},
            "parallelism": "whole sequence on one GPU" if world == 1 else f"sequence zig-zag x{world}, "
                           "NCCL all_gather_into_tensor of K and V",
        }
        for part in ("select", "gather"):
            entry[part]["frac"] = entry[part]["achieved"] / entry[part]["peak"]
        out.append(entry)
        del ql, kl, vl, qbs
        torch.cuda.empty_cache()
    return out


def host_link(dev, tensors) -> dict:
    """Copy-only host->device bandwidth of the e2e step's inputs (pinned, one
    cudaMemcpyAsync per tensor), CUDA events on the copying stream: the ceiling
    the e2e figure is held against."""
    dst = [torch.empty(t.shape, dtype=t.dtype, device=dev) for t in tensors]
    nbytes = sum(t.numel() * t.element_size() for t in tensors)
    stream = torch.cuda.current_stream(dev)
    for _ in range(2):
        for d, t in zip(dst, tensors):
            d.copy_(t, non_blocking=True)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 5
    a.record(stream)
    for _ in range(reps):
        for d, t in zip(dst, tensors):
            d.copy_(t, non_blocking=True)
    b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / reps
    return {"h2d_gbs": nbytes / (ms / 1e3) / 1e9, "bytes": nbytes, "ms": ms}


def run_ours(args) -> None:
    world, rank, local = _dist()
    if args.gpus != world:
        raise SystemExit(f"bench.py: --gpus {args.gpus} but WORLD_SIZE is {world}; launch N > 1 GPUs with "
                         f"torchrun --nproc-per-node {args.gpus}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=dev)
    from ossa_b200 import _lib, router_topk, topk_attention
    from ossa_b200.host_pipeline import routed_attention_from_host
    from ossa_b200.select import router_topk_with_status

    w = WORKLOAD
    B, H, Hkv, N, D, K, r, L = (w[x] for x in ("B", "H", "Hkv", "N", "D", "K", "r", "seq_len"))
    q, k, v, wq, wk, pb = make_inputs(dev, seed=1234 + rank)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)  # > 126 MB L2

    def step():
        idx = router_topk(q, k, wq, wk, pb, L, K, causal=True)
        return topk_attention(q, k, v, topk_indices=idx, causal=True)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    barrier()

    # --- device-resident timed steps ------------------------------------------------
    stream = torch.cuda.current_stream(dev)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
            torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    launches0 = _lib.launch_count()
    barrier()
    with ClockSampler(local) as clk:
        for e0, e1, e2 in evs:
            flush.zero_()
            e0.record(stream)
            idx = router_topk(q, k, wq, wk, pb, L, K, causal=True)
            e1.record(stream)
            topk_attention(q, k, v, topk_indices=idx, causal=True)
            e2.record(stream)
        barrier()
    launches = _lib.launch_count() - launches0
    _, fb_rows, sel_status = router_topk_with_status(q, k, wq, wk, pb, L, K, causal=True)
    sel_ms = [a.elapsed_time(b) for a, b, _ in evs]
    gat_ms = [b.elapsed_time(c) for _, b, c in evs]
    step_ms = [s + g for s, g in zip(sel_ms, gat_ms)]
    total_ms = sum(step_ms)

    # --- end to end through the public API with pinned host buffers --------------------
    qh = q.cpu().pin_memory()
    kh = k.cpu().pin_memory()
    vh = v.cpu().pin_memory()
    oh = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    h2d = qh.numel() * 2 + kh.numel() * 2 + vh.numel() * 2
    d2h = oh.numel() * 2

    chunk, groups, edge = 2, 1, 1

    def e2e_step():
        # public host-buffer entry point: chunked H2D / kernels / D2H on three streams
        routed_attention_from_host(qh, kh, vh, wq, wk, pb, L, K, oh, causal=True, chunk=chunk, groups=groups,
                                   edge_groups=edge)

    # pipeline depth: batch elements per chunk (or GQA groups of one element),
    # chosen in the untimed warm-up
    options = [(1, 1, 1), (2, 1, 1), (4, 1, 1)]
    if w["Hkv"] > 1:
        options += [(1, 1, w["Hkv"]), (1, w["Hkv"], 1)]
    trial = {}
    for c in options:
        chunk, groups, edge = c
        e2e_step()
        a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(2):
            e2e_step()
        b_.record(stream)
        torch.cuda.synchronize()
        trial[c] = a.elapsed_time(b_)
    tt = torch.tensor([trial[c] for c in options], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)  # every rank picks the same
    chunk, groups, edge = options[int(torch.argmin(tt).item())]
    for _ in range(max(1, args.warmup)):
        e2e_step()
    barrier()
    e2e_evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
    for a, b in e2e_evs:
        flush.zero_()
        a.record(stream)
        e2e_step()
        b.record(stream)
    barrier()
    e2e_ms = sum(a.elapsed_time(b) for a, b in e2e_evs)
    link = host_link(dev, [qh, kh, vh])
    del qh, kh, vh, oh

    t = torch.tensor([total_ms, e2e_ms, sum(sel_ms), sum(gat_ms)], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    total_ms, e2e_ms, sel_tot, gat_tot = t.tolist()
    del q, k, v, flush
    torch.cuda.empty_cache()
    long_ctx = None if args.no_long_context else run_long_context(dev, world, rank, args.long_steps, 2)

    tokens = world * args.steps * B * N
    value = tokens / (total_ms / 1e3)
    peaks = _peaks()
    gat_avg_s = gat_tot / args.steps / 1e3
    sel_avg_s = sel_tot / args.steps / 1e3
    gbytes = gather_bytes(B, H, N, D, K)
    sflops = select_flops(B, H, Hkv, N, D, r)
    traffic = _traffic()
    gather_roof = {"bound": "hbm", "achieved": gbytes / gat_avg_s / 1e9, "peak": peaks["hbm_gbs"],
                   "unit": "GB/s", "traffic": traffic.get("gather_attn_fwd")}
    gather_roof["frac"] = gather_roof["achieved"] / gather_roof["peak"]
    select_roof = {"bound": "tensor", "achieved": sflops / sel_avg_s / 1e12, "peak": peaks["bf16_tflops"],
                   "unit": "TFLOP/s", "traffic": traffic.get("router_tc")}
    select_roof["frac"] = select_roof["achieved"] / select_roof["peak"]
    dominant = gather_roof if gat_tot >= sel_tot else select_roof
    roof = dict(dominant)
    roof["kernel"] = ("gather_attn_fwd" if dominant is gather_roof else
                      "router selection step (router_topk: k projection, key statistics, query operand "
                      "(qproj_umma_kernel), router_tc_kernel, fallback), "
                      "timed with events around the call")
    roof["peak_source"] = f"{peaks['source']} (MEASURED_PEAKS.json burst)" if peaks["source"] == "measured" \
        else "fallback"
    roof["algorithmic"] = (f"{gbytes} B per launch (33,536 B per query-head at K=64)"
                           if dominant is gather_roof else f"{sflops} flop per step")

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_sample(seconds_hint=args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": _config(world),
            "per_gpu_tokens_s": value / world,
            "roofline": roof,
            "kernels": {"select": {"ms": sel_avg_s * 1e3, **select_roof},
                        "gather": {"ms": gat_avg_s * 1e3, **gather_roof}},
            "cpu_baseline": cpu,
            "e2e": {"value": world * args.steps * B * N / (e2e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms / args.steps, "host_link_copy_only": link,
                    "pipeline_chunk": chunk, "pipeline_groups": groups, "pipeline_edge_groups": edge},
            "long_context": long_ctx,
            "gpu_launches": launches,
            "select_exact_fallback_rows": fb_rows, "select_status": sel_status,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def _reference_sample_inputs(seed: int = 1234):
    """One GQA group (6 query heads of one kv head) of one batch element of the
    workload, fp32 on the CPU: 1/16 of a step's work."""
    w = WORKLOAD
    G = w["H"] // w["Hkv"]
    g = torch.Generator()
    g.manual_seed(seed)
    s = 1.0 / math.sqrt(w["D"])
    q = torch.randn(1, G, w["N"], w["D"], generator=g) * s
    k = torch.randn(1, 1, w["N"], w["D"], generator=g) * s
    v = torch.randn(1, 1, w["N"], w["D"], generator=g) * s
    wq = torch.empty(w["r"], w["D"])
    wk = torch.empty(w["r"], w["D"])
    torch.nn.init.xavier_uniform_(wq, generator=g)
    torch.nn.init.xavier_uniform_(wk, generator=g)
    pb = torch.randn(2 * w["seq_len"], 1, generator=g)
    return q, k, v, wq, wk, pb, G


def _reference_step(inp):
    from oracle import reference_port as rp

    q, k, v, wq, wk, pb, G = inp
    with torch.no_grad():
        rp.reference_layer_path(q, k, v, wq, wk, pb, WORKLOAD["seq_len"], WORKLOAD["K"])


def cpu_baseline_sample(seconds_hint: float = 20.0) -> dict:
    """Times the reference PyTorch path (router.score -> causal topk -> chunked
    gather, fp32) on the host with all threads, on one GQA group of one batch
    element (tokens credited: N * 6/12)."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    inp = _reference_sample_inputs()
    G = inp[-1]
    t0 = time.perf_counter()
    _reference_step(inp)
    one = time.perf_counter() - t0
    reps = max(1, min(5, int(seconds_hint / max(one, 1e-3))))
    t0 = time.perf_counter()
    for _ in range(reps):
        _reference_step(inp)
    dt = (time.perf_counter() - t0) / reps
    tokens = WORKLOAD["N"] * G / WORKLOAD["H"]
    return {"value": tokens / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": (f"1 batch element x 1 GQA group (6 of 12 query heads), N={WORKLOAD['N']}, K={WORKLOAD['K']}, "
                       f"fp32, reference PyTorch path (oracle/reference_port.py), {reps} timed reps after 1 warm-up; "
                       f"credited {tokens:.0f} tokens per rep")}


def run_reference(args) -> None:
    world, rank, _ = _dist()
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    inp = _reference_sample_inputs()
    G = inp[-1]
    for _ in range(args.warmup):
        _reference_step(inp)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        _reference_step(inp)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    tokens = args.steps * WORKLOAD["N"] * G / WORKLOAD["H"]
    value = tokens / total
    sample = (f"each step: 1 batch element x 1 GQA group (6 of 12 query heads) of the workload, N={WORKLOAD['N']}, "
              f"K={WORKLOAD['K']}, fp32 CPU, credited {WORKLOAD['N'] * G / WORKLOAD['H']:.0f} tokens")
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": _config(world),
        "impl": "reference",
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-long-context", action="store_true",
                    help="skip the long-context (32k-128k) selection and gather figures")
    ap.add_argument("--long-steps", type=int, default=3, help="timed steps per long-context configuration")
    args = ap.parse_args()
    if args.warmup < 3:
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    sys.path.insert(0, str(ROOT))
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
