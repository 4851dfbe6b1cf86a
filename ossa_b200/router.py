"""ContentRouter with fused sm_100a scoring and selection (ossa/router.py:136-203).

Same configuration dataclass, parameter names and shapes as the reference, so
``load_state_dict`` accepts the reference's checkpoints unchanged
(``q_proj.0.weight`` (r, D), ``k_proj.0.weight`` (r, D), ``pos_bias.weight``
(2*seq_len, 1)).  ``score``/``forward`` materialise the (B, H, N, N) fp32 logits
with a CUDA kernel; ``topk`` never materialises them.

Additive differences:
* ``k`` may carry Hkv < H heads (GQA); the reference needs repeated heads.
* ``topk(..., causal=True)`` masks keys j > i before selecting (the patched
  forward's behaviour, sparse_forward.py:200-202); the default ``causal=False``
  is the reference's unmasked ``topk`` (ossa/router.py:202-203).
* ``topk`` returns each row's keys in torch.topk's order (descending fp32
  score, ties toward the lower key index), padded with -1 where fewer than
  ``top_k`` keys are eligible under the causal mask.  ``order="index"`` gives
  ascending key order instead (the selectors' native layout, which the gather
  consumes).  ``index_dtype`` defaults to int64 like torch.topk; int32 avoids a
  conversion.
* Scores are defined by a fixed fp32 evaluation order (fmaf chains) so the
  selected sets are reproducible bit for bit.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn

from . import select


@dataclass
class ContentRouterConfig:
    head_dim: int
    n_heads: int
    seq_len: int
    proj_dim: int = 64        # router-internal projection size
    layers: int = 1           # unused, kept for config compatibility


class ContentRouter(nn.Module):
    """Content-based router: score(i, j) = (q_i Wq^T) . (k_j Wk^T) / sqrt(r)
    + pos_bias[clamp(i - j + seq_len, 0, 2*seq_len - 1)]."""

    def __init__(self, cfg: ContentRouterConfig) -> None:
        super().__init__()
        self.cfg = cfg
        self.q_proj = nn.Sequential(nn.Linear(cfg.head_dim, cfg.proj_dim, bias=False))
        self.k_proj = nn.Sequential(nn.Linear(cfg.head_dim, cfg.proj_dim, bias=False))
        self.pos_bias = nn.Embedding(2 * cfg.seq_len, 1)

    def _params(self):
        return self.q_proj[0].weight, self.k_proj[0].weight, self.pos_bias.weight

    def with_seq_len(self, seq_len: int) -> "ContentRouter":
        """A copy sized for ``seq_len`` that scores every (i, j) exactly as this
        router does.  Additive: the reference sizes pos_bias as 2*seq_len and
        leaves longer contexts to retraining (README "Long context").  This
        router already clamps offsets i - j beyond +-seq_len to the table's edge
        entries (ossa/router.py:183-188), so the copy's table holds entry
        clamp(o - seq_len + S, 0, 2S - 1) of this one (S = this router's
        seq_len) at index o: the edge entries repeat outward when growing, and
        offsets within +-min(S, seq_len) keep their entries when shrinking.
        Projection weights are shared values (copied)."""
        if seq_len <= 0:
            raise ValueError(f"seq_len must be positive, got {seq_len}")
        S = self.cfg.seq_len
        cfg = ContentRouterConfig(head_dim=self.cfg.head_dim, n_heads=self.cfg.n_heads, seq_len=seq_len,
                                  proj_dim=self.cfg.proj_dim, layers=self.cfg.layers)
        dev = self.pos_bias.weight.device
        out = ContentRouter(cfg).to(dev)
        with torch.no_grad():
            out.q_proj[0].weight.copy_(self.q_proj[0].weight)
            out.k_proj[0].weight.copy_(self.k_proj[0].weight)
            src = (torch.arange(2 * seq_len, device=dev) - seq_len + S).clamp_(0, 2 * S - 1)
            out.pos_bias.weight.copy_(self.pos_bias.weight[src])
        return out.train(self.training)

    def score(self, q: torch.Tensor, k: torch.Tensor) -> torch.Tensor:
        """q: (B, H, N, D), k: (B, H or Hkv, N, D) -> (B, H, N, N) fp32 logits."""
        wq, wk, pb = self._params()
        return select.router_scores(q, k, wq, wk, pb, self.cfg.seq_len)

    def forward(self, q: torch.Tensor, k: Optional[torch.Tensor] = None) -> torch.Tensor:
        if k is None:
            raise TypeError("ContentRouter needs both q and k tensors; call .score(q, k).")
        return self.score(q, k)

    def distillation_loss(self, q: torch.Tensor, k: torch.Tensor, top_k: int, *,
                          targets: Optional[torch.Tensor] = None) -> torch.Tensor:
        """The reference's training loss, distillation_loss(self.score(q, k), dense,
        k=top_k) (ossa/router.py:80-99), with autograd into this router's
        parameters and no N x N tensor (see ossa_b200.train)."""
        from .train import distillation_loss

        return distillation_loss(self, q, k, top_k, targets=targets)

    def topk(self, q: torch.Tensor, k: torch.Tensor, top_k: int, *, causal: bool = False,
             index_dtype: torch.dtype = torch.int64, order: str = "score") -> torch.Tensor:
        """Indices (B, H, N, top_k) of the top_k keys per query, by descending
        score like torch.topk (ossa/router.py:202-203); ``order="index"`` lists
        each row's keys in ascending order instead (see module doc)."""
        if order not in ("score", "index"):
            raise ValueError(f"order must be 'score' or 'index', got {order!r}")
        N = q.shape[2]
        if not causal and top_k > N:
            raise RuntimeError(f"selected index k out of range: top_k={top_k} > N={N}")
        wq, wk, pb = self._params()
        fn = select.router_topk_by_score if order == "score" else select.router_topk
        idx = fn(q, k, wq, wk, pb, self.cfg.seq_len, top_k, causal=causal)
        return idx if index_dtype == torch.int32 else idx.to(index_dtype)
