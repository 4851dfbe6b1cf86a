"""ossa_b200 — OSSA's routed sparse-attention hot path on Blackwell (sm_100a).

Drop-in for the reference package's hot-path API (ossa/__init__.py:3-20):
``topk_attention``, ``sparse_attention_forward[_chunked]``,
``dense_attention_reference``, ``HAS_TRITON``, plus ``ContentRouter`` /
``ContentRouterConfig`` (ossa/router.py) and the patched Qwen2 attention in
``ossa_b200.bench.sparse_forward``.  All sparse work runs in hand-written CUDA
kernels (libossa_b200.so, C ABI in include/ossa_b200.h); CPU tensors are
rejected rather than served by a fallback.
"""

from .router import ContentRouter, ContentRouterConfig
from .select import oracle_topk, router_scores, router_topk, with_diagonal
from .sparse_attention import (
    dense_attention_reference,
    sparse_attention_forward,
    sparse_attention_forward_chunked,
)
from .topk_attention import HAS_TRITON, topk_attention

__all__ = [
    "ContentRouter",
    "ContentRouterConfig",
    "dense_attention_reference",
    "sparse_attention_forward",
    "sparse_attention_forward_chunked",
    "topk_attention",
    "HAS_TRITON",
    "router_topk",
    "router_scores",
    "oracle_topk",
    "with_diagonal",
]
__version__ = "0.1.0"
