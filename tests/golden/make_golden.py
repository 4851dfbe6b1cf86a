"""Generates tests/golden/*.npz by running the reference implementation itself.

Run in a checkout that has the reference source tree (read-only is fine), giving
the reference project's root directory (the one holding ``src/ossa`` and
``checkpoints/``) as the one required argument:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py <reference-root>

It imports the reference's ``ossa`` package (router.py, sparse_attention.py) and
its trained router checkpoint (checkpoints/content_router_layer14.pt) and records
the reference's outputs on seeded inputs (tests/golden/cases.py).  The fixtures
store the reference's top-K index sets (sorted ascending, entries > i dropped
and -1 padded, which is the set the causal sparse forward actually uses), the
same indices in torch.topk's own order (descending score), boundary-score gaps,
a few rows of raw logits and sparse-forward outputs.
"""

from __future__ import annotations

import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import cases  # noqa: E402


def causal_sets(idx: torch.Tensor) -> np.ndarray:
    """(B,H,N,K) indices -> ascending sets restricted to j <= i, -1 padded."""
    B, H, N, K = idx.shape
    pos = torch.arange(N).view(1, 1, N, 1)
    big = torch.iinfo(torch.int64).max
    keep = idx.masked_fill(idx > pos, big)
    s = torch.sort(keep, dim=-1).values
    s = s.masked_fill(s == big, -1)
    return s.to(torch.int32).numpy()


def full_sets(idx: torch.Tensor) -> np.ndarray:
    return torch.sort(idx, dim=-1).values.to(torch.int32).numpy()


def boundary_gap(selector: torch.Tensor, K: int) -> np.ndarray:
    """Per row: (K-th best) - ((K+1)-th best) causal score, inf when <= K eligible."""
    N = selector.shape[-1]
    causal = torch.tril(torch.ones(N, N, dtype=torch.bool))
    m = selector.masked_fill(~causal, float("-inf"))
    top = torch.topk(m, k=min(K + 1, N), dim=-1).values
    gap = torch.full(m.shape[:-1], float("inf"))
    if N > K:
        gap = top[..., K - 1] - top[..., K]
        gap = torch.where(torch.isfinite(gap), gap, torch.full_like(gap, float("inf")))
    return gap.numpy().astype(np.float32)


def main(ref_root: str) -> None:
    ref_root = Path(ref_root)
    sys.path.insert(0, str(ref_root / "src"))
    from ossa.router import ContentRouter, ContentRouterConfig
    from ossa.sparse_attention import (
        dense_attention_reference,
        sparse_attention_forward,
        sparse_attention_forward_chunked,
    )

    torch.set_num_threads(8)

    # --- A: the small single-layer workload with the trained layer-14 router
    ck = torch.load(ref_root / "checkpoints" / "content_router_layer14.pt", map_location="cpu",
                    weights_only=False)
    q, k, v = cases.c1_inputs()
    B, H, N, D = q.shape
    Hkv = k.shape[1]
    rep = H // Hkv
    K = 64
    router = ContentRouter(ContentRouterConfig(head_dim=D, n_heads=H, seq_len=512, proj_dim=64))
    router.load_state_dict(ck["state_dict"])
    router.eval()
    kr = k.repeat_interleave(rep, dim=1)
    vr = v.repeat_interleave(rep, dim=1)
    with torch.no_grad():
        logits = router.score(q.float(), kr.float())
        causal = torch.tril(torch.ones(N, N, dtype=torch.bool))
        top = torch.topk(logits.masked_fill(~causal, float("-inf")), k=K, dim=-1).indices
        out = sparse_attention_forward_chunked(q, kr, vr, topk_indices=top, chunk_size=64, causal=True)
    rows = np.array([0, 1, 2, 62, 63, 64, 255, 511])
    np.savez_compressed(
        HERE / "router_ckpt_c1.npz",
        wq=ck["state_dict"]["q_proj.0.weight"].numpy(),
        wk=ck["state_dict"]["k_proj.0.weight"].numpy(),
        pos_bias=ck["state_dict"]["pos_bias.weight"].numpy(),
        seq_len=np.int64(512), K=np.int64(K),
        checksum=cases.checksum(q, k, v),
        ref_sets=causal_sets(top).astype(np.int16),
        ref_order=top.numpy().astype(np.int16),
        ref_gap=boundary_gap(logits, K),
        logit_rows=rows,
        ref_logits=logits[:, :, rows, :].numpy(),
        out_heads=np.array([0, 7]),
        ref_out=out[:, [0, 7]].numpy(),
    )

    # --- B: random-init router, ragged GQA, clamped pos_bias ----------------
    q, k, v = cases.gqa_small_inputs()
    B, H, N, D = q.shape
    Hkv = k.shape[1]
    rep = H // Hkv
    r, L, K = 32, 128, 16
    wq, wk, pb = cases.router_weights(D, r, L, seed=5)
    router = ContentRouter(ContentRouterConfig(head_dim=D, n_heads=H, seq_len=L, proj_dim=r))
    with torch.no_grad():
        router.q_proj[0].weight.copy_(wq)
        router.k_proj[0].weight.copy_(wk)
        router.pos_bias.weight.copy_(pb)
    kr = k.repeat_interleave(rep, dim=1)
    vr = v.repeat_interleave(rep, dim=1)
    with torch.no_grad():
        logits = router.score(q, kr)
        causal = torch.tril(torch.ones(N, N, dtype=torch.bool))
        top_c = torch.topk(logits.masked_fill(~causal, float("-inf")), k=K, dim=-1).indices
        top_full = router.topk(q, kr, K)  # router.py:202-203, no causal mask
        out = sparse_attention_forward_chunked(q, kr, vr, topk_indices=top_c, chunk_size=64, causal=True)
    np.savez_compressed(
        HERE / "router_random_gqa.npz",
        r=np.int64(r), seq_len=np.int64(L), K=np.int64(K), weight_seed=np.int64(5),
        checksum=cases.checksum(q, k, v, wq, wk, pb),
        ref_sets=causal_sets(top_c).astype(np.int16),
        ref_gap=boundary_gap(logits, K),
        ref_full_sets=full_sets(top_full).astype(np.int16),
        ref_full_order=top_full.numpy().astype(np.int16),
        logit_rows=np.array([0, 1, 15, 16, 127, 128, 199]),
        ref_logits=logits[:, :, [0, 1, 15, 16, 127, 128, 199], :].numpy(),
        ref_out=out.numpy(),
    )

    # --- C: the reference tests' own shapes (sparse forward known answers) --
    q, k, v = cases.reference_test_inputs()
    B, H, N, D = q.shape
    K = 16
    with torch.no_grad():
        scores = q @ k.transpose(-2, -1)
        causal = torch.triu(torch.ones(N, N, dtype=torch.bool), diagonal=1)
        top = scores.masked_fill(causal, float("-inf")).topk(K, dim=-1).indices
        out_full = sparse_attention_forward(q, k, v, topk_indices=top)
        out_chunk = sparse_attention_forward_chunked(q, k, v, topk_indices=top, chunk_size=16)
        all_idx = torch.arange(N).view(1, 1, 1, N).expand(B, H, N, N).contiguous()
        out_alln = sparse_attention_forward(q, k, v, topk_indices=all_idx)
        out_dense = dense_attention_reference(q, k, v)
    np.savez_compressed(
        HERE / "sparse_forward_ref.npz",
        checksum=cases.checksum(q, k, v), K=np.int64(K),
        topk=top.numpy().astype(np.int16),
        out_full=out_full.numpy(), out_chunked=out_chunk.numpy(),
        out_all_keys=out_alln.numpy(), out_dense=out_dense.numpy(),
    )

    # --- D: oracle (exact q.k) selector -------------------------------------
    q, k, v = cases.oracle_inputs()
    B, H, N, D = q.shape
    rep = H // k.shape[1]
    K = 32
    kr = k.repeat_interleave(rep, dim=1)
    vr = v.repeat_interleave(rep, dim=1)
    with torch.no_grad():
        sel = torch.matmul(q, kr.transpose(-2, -1)) * (1.0 / math.sqrt(D))  # sparse_forward.py:194-196
        causal = torch.tril(torch.ones(N, N, dtype=torch.bool))
        top = torch.topk(sel.masked_fill(~causal, float("-inf")), k=K, dim=-1).indices
        out = sparse_attention_forward_chunked(q, kr, vr, topk_indices=top, chunk_size=64, causal=True)
    np.savez_compressed(
        HERE / "oracle_select.npz",
        checksum=cases.checksum(q, k, v), K=np.int64(K),
        ref_sets=causal_sets(top).astype(np.int16),
        ref_gap=boundary_gap(sel, K),
        out_heads=np.array([0, 3]),
        ref_out=out[:, [0, 3]].numpy(),
    )
    # --- E: router training step (distillation loss and its gradients) --------
    from ossa.router import distillation_loss

    q, k, _ = cases.distill_inputs()
    B, H, N, D = q.shape
    rep = H // k.shape[1]
    r, L, K = 32, 64, 16
    wq, wk, pb = cases.router_weights(D, r, L, seed=41)
    router = ContentRouter(ContentRouterConfig(head_dim=D, n_heads=H, seq_len=L, proj_dim=r))
    with torch.no_grad():
        router.q_proj[0].weight.copy_(wq)
        router.k_proj[0].weight.copy_(wk)
        router.pos_bias.weight.copy_(pb)
    kr = k.repeat_interleave(rep, dim=1)
    with torch.no_grad():
        causal = torch.tril(torch.ones(N, N, dtype=torch.bool))
        dense = torch.softmax((q @ kr.transpose(-2, -1) / math.sqrt(D)).masked_fill(~causal, float("-inf")), dim=-1)
        target_idx = torch.topk(dense, k=K, dim=-1).indices  # the targets distillation_loss builds
    logits = router.score(q, kr)
    loss = distillation_loss(logits, dense, k=K)
    loss.backward()
    np.savez_compressed(
        HERE / "router_distill.npz",
        r=np.int64(r), seq_len=np.int64(L), K=np.int64(K), weight_seed=np.int64(41),
        checksum=cases.checksum(q, k, wq, wk, pb),
        target_idx=target_idx.numpy().astype(np.int16),
        loss=np.float64(loss.item()),
        dwq=router.q_proj[0].weight.grad.numpy(),
        dwk=router.k_proj[0].weight.grad.numpy(),
        dpos_bias=router.pos_bias.weight.grad.numpy(),
    )
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <reference-root>  (the directory holding src/ossa and checkpoints/)")
    main(sys.argv[1])
