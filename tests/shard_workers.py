"""Per-rank bodies of the sequence-sharding tests (imported by the spawned
processes; not a test module)."""

import datetime
import math
import os

import numpy as np
import torch
import torch.distributed as dist

import cases


def shard_inputs(B, H, Hkv, N, D, r, L, seed):
    q, k, v = cases.qkv(B, H, Hkv, N, D, seed=seed, scale=1.0 / math.sqrt(D))
    wq, wk, pb = cases.router_weights(D, r, L, seed)
    return q, k, v, wq, wk, pb


def _init(rank, world, port, backend, device=None):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    kw = {"device_id": device} if device is not None else {}
    dist.init_process_group(backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60), **kw)


def cpu_worker(rank, world, port, shape, out_dir):
    """gloo ranks on the CPU: the oracle selection and fp64 attention oracle
    stand in for the CUDA kernels, so this checks the sharding plumbing (block
    ownership, the k/v all-gather and its reordering, output assembly)."""
    import oracle
    from oracle import reference_port as rp
    from ossa_b200.sequence_shard import local_rows, sharded_routed_attention

    B, H, Hkv, N, D, r, L, K = shape
    _init(rank, world, port, "gloo")
    try:
        q, k, v, wq, wk, pb = shard_inputs(B, H, Hkv, N, D, r, L, seed=3)

        def select(qb, k_full, wq_, wk_, pb_, seq_len, top_k, causal=True, q_start=0):
            nq = qb.shape[2]
            rows = np.array([bh * N + i for bh in range(B * H) for i in range(q_start, q_start + nq)])
            ref = oracle.router_topk_rows(q, k_full, wq_, wk_, pb_, seq_len, top_k, rows, causal=causal)
            return torch.from_numpy(ref.reshape(B, H, nq, top_k))

        def attend(qb, k_full, v_full, topk_indices, causal=True, q_start=0):
            pos = torch.arange(q_start, q_start + qb.shape[2])
            return rp.masked_index_attention(qb, k_full, v_full, topk_indices, causal=causal, positions=pos)

        out = sharded_routed_attention(local_rows(q, world, rank), local_rows(k, world, rank),
                                       local_rows(v, world, rank), wq, wk, pb, L, K,
                                       select_fn=select, attend_fn=attend)
        torch.save(out, os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


def gpu_worker(rank, world, port, shape, out_dir):
    """NCCL ranks, one GPU each: the sharded CUDA path must return exactly the
    rows of the unsharded CUDA path computed on the same GPU."""
    from ossa_b200 import router_topk, topk_attention
    from ossa_b200.sequence_shard import local_rows, sharded_routed_attention

    B, H, Hkv, N, D, r, L, K = shape
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    _init(rank, world, port, "nccl", device=dev)
    try:
        q, k, v, wq, wk, pb = (t.to(dev) for t in shard_inputs(B, H, Hkv, N, D, r, L, seed=4))
        q, k, v = q.bfloat16(), k.bfloat16(), v.bfloat16()
        out = sharded_routed_attention(local_rows(q, world, rank), local_rows(k, world, rank),
                                       local_rows(v, world, rank), wq, wk, pb, L, K)
        idx = router_topk(q, k, wq, wk, pb, L, K)
        ref = local_rows(topk_attention(q, k, v, topk_indices=idx), world, rank)
        torch.cuda.synchronize()
        same = bool(torch.equal(out, ref))
        torch.save({"same": same, "max_diff": float((out.float() - ref.float()).abs().max())},
                   os.path.join(out_dir, f"rank{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()
