"""Sequence sharding for long contexts (ossa_b200.sequence_shard): zig-zag block
ownership, and the sharded computation against the unsharded one, as gloo
ranks on the CPU (oracle arithmetic) and as NCCL ranks on two GPUs (CUDA path,
bit-exact rows)."""

import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle
from oracle import reference_port as rp
from ossa_b200.sequence_shard import gather_sequence, local_rows, zigzag_blocks
from shard_workers import cpu_worker, gpu_worker, shard_inputs


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_zigzag_blocks_cover_and_balance(world):
    n = 64 * world
    owned = []
    causal_work = []
    for r in range(world):
        blocks = zigzag_blocks(n, world, r)
        assert len(blocks) == 2
        owned += [i for s, e in blocks for i in range(s, e)]
        causal_work.append(sum(i + 1 for s, e in blocks for i in range(s, e)))
    assert sorted(owned) == list(range(n))
    assert len(set(causal_work)) == 1  # every rank has the same number of causal (row, key) pairs


def test_zigzag_rejects_ragged_lengths():
    with pytest.raises(ValueError):
        zigzag_blocks(100, 3, 0)
    with pytest.raises(ValueError):
        zigzag_blocks(64, 2, 2)


def test_local_rows_then_gather_is_identity_single_rank():
    x = torch.randn(2, 3, 16, 4)
    assert torch.equal(gather_sequence(local_rows(x, 1, 0), 1), x)


def test_sharded_matches_unsharded_gloo(tmp_path):
    world = 2
    shape = (1, 4, 2, 64, 32, 16, 64, 8)  # B, H, Hkv, N, D, r, seq_len, K
    mp.spawn(cpu_worker, args=(world, _free_port(), shape, str(tmp_path)), nprocs=world, join=True)
    B, H, Hkv, N, D, r, L, K = shape
    q, k, v, wq, wk, pb = shard_inputs(B, H, Hkv, N, D, r, L, seed=3)
    idx = torch.from_numpy(oracle.router_topk(q, k, wq, wk, pb, L, K))
    full = rp.masked_index_attention(q, k, v, idx, causal=True)
    for rank in range(world):
        got = torch.load(tmp_path / f"rank{rank}.pt")
        np.testing.assert_allclose(got.numpy(), local_rows(full, world, rank).numpy(), rtol=0, atol=0)


@pytest.mark.gpu
def test_sharded_matches_unsharded_two_gpus(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    shape = (1, 12, 2, 4096, 128, 64, 4096, 64)
    mp.spawn(gpu_worker, args=(world, _free_port(), shape, str(tmp_path)), nprocs=world, join=True)
    for rank in range(world):
        res = torch.load(tmp_path / f"rank{rank}.pt")
        assert res["same"], res


@pytest.mark.gpu
def test_sharded_single_process_matches_unsharded():
    """One process (world 1): its two blocks are the two halves of the sequence,
    selected against keys projected once (project_router_keys +
    router_topk_projected, the default selector of the sharded path); the result
    equals the unsharded CUDA path bit for bit."""
    from ossa_b200 import router_topk, topk_attention
    from ossa_b200.sequence_shard import sharded_routed_attention

    B, H, Hkv, N, D, r, L, K = 1, 12, 2, 2048, 128, 64, 2048, 64
    q, k, v, wq, wk, pb = (t.to("cuda:0") for t in shard_inputs(B, H, Hkv, N, D, r, L, seed=6))
    q, k, v = q.bfloat16(), k.bfloat16(), v.bfloat16()
    out = sharded_routed_attention(q, k, v, wq, wk, pb, L, K)
    ref = topk_attention(q, k, v, topk_indices=router_topk(q, k, wq, wk, pb, L, K))
    assert torch.equal(out, ref)
