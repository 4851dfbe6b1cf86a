"""ContentRouter distillation without the (B, H, N, N) logits.

The reference trains the router by distilling the dense attention
(ossa/router.py:80-99, ossa/bench/content_train.py:141-148): the target marks
each query row's top-k keys of the dense attention probabilities, and the loss
is binary cross-entropy with logits between ``router.score(q, k)`` and that
target, averaged over all B*H*N*N entries.  Both the logits and the dense
attention are (B, H, N, N) tensors there.

Here neither exists:

* ``dense_topk_targets`` takes the target sets from q and k directly: softmax is
  monotone along a row, so the top-k of the causal dense attention is the top-k
  of the causal scores q.k/sqrt(D), which the exact oracle selector computes
  (``oracle_topk``: fp32 scores, ties to the lower key index).  Rows with fewer
  than k eligible keys list all of them (-1 padding); the reference's torch.topk
  there also marks some masked positions (probability 0 ties).
* ``distillation_loss`` evaluates the same mean BCE over every (i, j) and its
  gradient for ``q_proj``, ``k_proj`` and ``pos_bias`` with one fused pass
  (``ossa_router_distill_grad``: scores recomputed tile by tile on the GPU,
  memory linear in N), wrapped as an autograd function so that
  ``loss.backward()`` fills the router's ``.grad`` fields and any optimizer
  steps as in the reference loop.  q and k are inputs, not differentiated (the
  reference detaches the captured projections).
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from .select import _as_kernel_input, _check_qk, _common_dtype, oracle_topk

__all__ = ["dense_topk_targets", "distillation_loss"]


def dense_topk_targets(q: torch.Tensor, k: torch.Tensor, top_k: int) -> torch.Tensor:
    """Top-k keys of the causal dense attention softmax(q k^T / sqrt(D)) per
    query row: (B, H, N, top_k) int32, ascending, -1 padded.  k may carry Hkv
    heads (GQA)."""
    return oracle_topk(q, k, top_k, causal=True)


class _DistillFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, wq, wk, pos_bias, q, k, targets, seq_len):
        B, H, Hkv, N, D = _check_qk(q, k)
        dev = _lib.require_cuda(q, k, wq, wk, pos_bias, targets)
        r = wq.shape[0]
        if wq.shape != (r, D) or wk.shape != (r, D):
            raise ValueError(f"projection weights must be ({r}, {D}); got {tuple(wq.shape)}, {tuple(wk.shape)}")
        if pos_bias.numel() != 2 * seq_len:
            raise ValueError(f"pos_bias has {pos_bias.numel()} entries, expected 2*seq_len = {2 * seq_len}")
        if targets.dim() != 4 or tuple(targets.shape[:3]) != (B, H, N):
            raise ValueError(f"targets must be (B, H, N, K) = ({B}, {H}, {N}, K); got {tuple(targets.shape)}")
        dt = _common_dtype(q, k)
        qc = _as_kernel_input(q.detach(), dt)
        kc = _as_kernel_input(k.detach(), dt)
        wqc = wq.detach().float().contiguous()
        wkc = wk.detach().float().contiguous()
        pbc = pos_bias.detach().float().contiguous()
        tc = targets.to(torch.int32).contiguous()
        L = _lib.lib()
        ws_bytes = L.ossa_router_distill_workspace_size(B, H, Hkv, N, r)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        loss = torch.empty((), dtype=torch.float32, device=dev)
        dwq = torch.empty_like(wqc)
        dwk = torch.empty_like(wkc)
        dpb = torch.empty_like(pbc)
        with torch.cuda.device(dev):
            st = L.ossa_router_distill_grad(qc.data_ptr(), kc.data_ptr(), _lib.dtype_code(qc), wqc.data_ptr(),
                                            wkc.data_ptr(), pbc.data_ptr(), B, H, Hkv, N, D, r, int(seq_len),
                                            tc.data_ptr(), tc.shape[-1], loss.data_ptr(), dwq.data_ptr(),
                                            dwk.data_ptr(), dpb.data_ptr(), ws.data_ptr(), ws_bytes,
                                            _lib.stream_ptr(dev))
        _lib.check(st)
        ctx.save_for_backward(dwq.to(wq.dtype), dwk.to(wk.dtype), dpb.view_as(pos_bias).to(pos_bias.dtype))
        return loss

    @staticmethod
    def backward(ctx, grad_out):
        dwq, dwk, dpb = ctx.saved_tensors
        return grad_out * dwq, grad_out * dwk, grad_out * dpb, None, None, None, None


def distillation_loss(router, q: torch.Tensor, k: torch.Tensor, top_k: int, *,
                      targets: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Mean BCE-with-logits over every (i, j) between ``router``'s scores and the
    0/1 target of ``targets`` (default: ``dense_topk_targets(q, k, top_k)``), as
    ``distillation_loss(router.score(q, k), dense, k=top_k)`` computes it in the
    reference, without materialising either N x N tensor.  Returns a scalar with
    autograd history into ``router``'s parameters.

    q: (B, H, N, D); k: (B, Hkv, N, D) (GQA or repeated heads); CUDA tensors.
    ``targets``: (B, H, N, K) key indices per row, -1 padded, any order."""
    if targets is None:
        targets = dense_topk_targets(q, k, top_k)
    wq, wk, pb = router.q_proj[0].weight, router.k_proj[0].weight, router.pos_bias.weight
    return _DistillFn.apply(wq, wk, pb, q, k, targets, router.cfg.seq_len)
