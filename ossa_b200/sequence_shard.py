"""Long-context routed sparse attention sharded over the sequence (one process
per GPU).

The reference runs one process over the whole sequence
(ossa/bench/sparse_forward.py:157-229).  For long contexts the query rows are
split across ranks instead, zig-zag for causal balance: the sequence is cut
into 2P equal blocks and rank r owns blocks r and 2P-1-r (an early block with
few causal keys and a late one with many).  Each rank holds q, k and v for its
own two blocks.  One collective per tensor brings every rank the full k and v
(``all_gather_into_tensor`` over NCCL); selection and the gather then run on the
rank's query blocks against all keys with the query-row-range entry points
(``router_topk(..., q_start=)``, ``topk_attention(..., q_start=)``), so each
rank's output rows equal the matching rows of the unsharded computation.
Outputs stay sharded.  Every rank takes the same collective steps in the same
order; nothing waits on another rank inside a kernel.
"""

from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

from .select import project_router_keys, router_topk, router_topk_projected
from .topk_attention import topk_attention

__all__ = ["zigzag_blocks", "local_rows", "gather_sequence", "sharded_routed_attention"]


def zigzag_blocks(n: int, world: int, rank: int) -> list[tuple[int, int]]:
    """The two [start, end) query ranges rank ``rank`` of ``world`` owns."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if n % (2 * world) != 0:
        raise ValueError(f"sequence length {n} must be a multiple of 2 * world = {2 * world}")
    blk = n // (2 * world)
    a, b = rank, 2 * world - 1 - rank
    return [(a * blk, (a + 1) * blk), (b * blk, (b + 1) * blk)]


def local_rows(x: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    """This rank's two zig-zag blocks of a (B, heads, N, D) tensor, concatenated
    along the sequence dimension (early block first)."""
    blocks = zigzag_blocks(x.shape[2], world, rank)
    return torch.cat([x[:, :, s:e] for s, e in blocks], dim=2).contiguous()


def gather_sequence(x_local: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """Inverse of ``local_rows`` across ranks: every rank gets the full
    (B, heads, N, D) tensor from each rank's (B, heads, 2 * blk, D) blocks."""
    if world == 1:
        return x_local.contiguous()
    x_local = x_local.contiguous()
    B, Hx, two_blk, D = x_local.shape
    blk = two_blk // 2
    if dist.get_backend(group) == "nccl":
        g = torch.empty((world * B, Hx, two_blk, D), dtype=x_local.dtype, device=x_local.device)
        dist.all_gather_into_tensor(g, x_local, group=group)
    else:
        parts = [torch.empty_like(x_local) for _ in range(world)]
        dist.all_gather(parts, x_local, group=group)
        g = torch.cat(parts, dim=0)
    g = g.view(world, B, Hx, 2, blk, D).permute(1, 2, 3, 0, 4, 5)  # (B, Hx, half, rank, blk, D)
    # half 0 of rank r is sequence block r; half 1 of rank r is block 2P-1-r
    full = torch.cat([g[:, :, 0], g[:, :, 1].flip(2)], dim=2)      # (B, Hx, 2P, blk, D)
    return full.reshape(B, Hx, world * two_blk, D)


def sharded_routed_attention(q_local: torch.Tensor, k_local: torch.Tensor, v_local: torch.Tensor,
                             wq: torch.Tensor, wk: torch.Tensor, pos_bias: torch.Tensor, seq_len: int,
                             top_k: int, *, group=None, causal: bool = True,
                             select_fn: Optional[Callable] = None,
                             attend_fn: Optional[Callable] = None) -> torch.Tensor:
    """Router selection + gathered attention for this rank's zig-zag blocks.

    q_local (B, H, 2*blk, D), k_local / v_local (B, Hkv, 2*blk, D): the rank's
    blocks as ``local_rows`` cuts them.  Returns the attention output for those
    query rows, (B, H, 2*blk, D).  ``select_fn`` / ``attend_fn`` default to this
    package's CUDA kernels (``router_topk``, ``topk_attention``) and take the
    same arguments.
    """
    own_select = select_fn is None
    select_fn = select_fn or router_topk
    attend_fn = attend_fn or topk_attention
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    if q_local.shape[2] != k_local.shape[2] or k_local.shape != v_local.shape:
        raise ValueError("q_local, k_local and v_local must hold the same two blocks of the sequence")
    n = q_local.shape[2] * world
    k_full = gather_sequence(k_local, world, group)
    v_full = gather_sequence(v_local, world, group)
    blk = q_local.shape[2] // 2
    # the keys are projected once for both query blocks (the default selector)
    kp = project_router_keys(k_full, wk) if own_select else None
    outs = []
    for half, (start, _end) in enumerate(zigzag_blocks(n, world, rank)):
        qb = q_local[:, :, half * blk:(half + 1) * blk].contiguous()
        if own_select:
            idx = router_topk_projected(qb, kp, wq, pos_bias, seq_len, top_k, causal=causal, q_start=start)
        else:
            idx = select_fn(qb, k_full, wq, wk, pos_bias, seq_len, top_k, causal=causal, q_start=start)
        outs.append(attend_fn(qb, k_full, v_full, topk_indices=idx, causal=causal, q_start=start))
    return torch.cat(outs, dim=2)
