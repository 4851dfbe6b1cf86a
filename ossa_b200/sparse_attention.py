"""Sparse attention forwards under the reference's names (ossa/sparse_attention.py).

``sparse_attention_forward`` (sparse_attention.py:29-79) and
``sparse_attention_forward_chunked`` (:87-137) compute the same O(N*K) gathered
attention; both run the sm_100a gather kernel here (``chunk_size`` is accepted
and ignored: the kernel tiles queries itself).  ``dense_attention_reference``
(:140-151) is the dense causal attention the reference exports for tests and
wall-clock comparisons; it is plain PyTorch on purpose (it is not the sparse
path) and accepts GQA k/v.
"""

from __future__ import annotations

import math

import torch

from .topk_attention import topk_attention


def sparse_attention_forward(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    topk_indices: torch.Tensor,
    causal: bool = True,
) -> torch.Tensor:
    """Attention over only ``topk_indices`` keys per query (see topk_attention)."""
    return topk_attention(q, k, v, topk_indices=topk_indices, causal=causal)


def sparse_attention_forward_chunked(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    topk_indices: torch.Tensor,
    chunk_size: int = 64,
    causal: bool = True,
) -> torch.Tensor:
    """Same result as :func:`sparse_attention_forward`; ``chunk_size`` is ignored."""
    del chunk_size
    return topk_attention(q, k, v, topk_indices=topk_indices, causal=causal)


def dense_attention_reference(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, causal: bool = True
) -> torch.Tensor:
    """Dense softmax attention (q k^T / sqrt(D), optional causal mask) times V."""
    H, Hkv = q.shape[1], k.shape[1]
    if Hkv != H:
        k = k.repeat_interleave(H // Hkv, dim=1)
        v = v.repeat_interleave(H // Hkv, dim=1)
    N = q.shape[2]
    scores = torch.matmul(q, k.transpose(-2, -1)) * (1.0 / math.sqrt(q.shape[-1]))
    if causal:
        mask = torch.triu(torch.ones(N, N, device=q.device, dtype=torch.bool), diagonal=1)
        scores = scores.masked_fill(mask, float("-inf"))
    return torch.matmul(torch.softmax(scores, dim=-1), v)
