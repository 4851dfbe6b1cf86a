"""Top-K sparse attention forward on sm_100a (the reference's ``topk_attention``).

Drop-in for ``ossa.triton_kernel.topk_attention`` (ossa/triton_kernel.py:41-70):
same signature and result.  The reference dispatches between a Triton kernel
(never launched on hardware) and a PyTorch fallback; here there is exactly one
implementation, ``ossa_topk_attention_fwd`` in libossa_b200.so, and CPU tensors
are rejected.  Differences, all additive:

* k and v may carry Hkv < H heads (GQA, query head h reads kv head h // (H/Hkv));
  the reference needs them repeated to H heads first (sparse_forward.py:175-178).
* indices may be int32 or int64; an index outside [0, N) (for example the -1
  padding of ossa_b200's selectors) is treated as masked.
* ``block_m`` and ``use_triton`` are accepted for signature compatibility and
  ignored (there is no Triton path to select).
* forward only: the output carries no autograd history.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from . import _lib

# Import-compatibility name: the reference exports whether its fused GPU kernel
# is usable.  Here the fused sm_100a kernel is the only implementation.
HAS_TRITON = True


def _check(q, k, v, idx, rows=False):
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("q, k and v must be 4-D (B, H, N, D)")
    B, H, N, D = q.shape
    if k.shape != v.shape:
        raise ValueError(f"k {tuple(k.shape)} and v {tuple(v.shape)} must have the same shape")
    Bk, Hkv, Nk, Dk = k.shape
    if (B, D) != (Bk, Dk) or (not rows and N != Nk):
        raise ValueError(f"q {tuple(q.shape)} and k/v {tuple(k.shape)} disagree on B, N or D")
    if Hkv <= 0 or H % Hkv != 0:
        raise ValueError(f"query heads {H} must be a multiple of key/value heads {Hkv}")
    if idx.dim() != 4 or tuple(idx.shape[:3]) != (B, H, N):
        raise ValueError(f"topk_indices must be (B, H, N, K) = ({B}, {H}, {N}, K); got {tuple(idx.shape)}")
    if idx.dtype not in (torch.int32, torch.int64):
        raise TypeError(f"topk_indices must be int32 or int64, got {idx.dtype}")
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError(f"q, k, v dtypes differ: {q.dtype}, {k.dtype}, {v.dtype}")
    return B, H, Hkv, N, D, idx.shape[-1]


def topk_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    topk_indices: torch.Tensor,
    causal: bool = True,
    block_m: int = 32,
    use_triton: Optional[bool] = None,
    q_start: Optional[int] = None,
) -> torch.Tensor:
    """Top-K sparse attention forward.

    q: (B, H, N, D); k, v: (B, Hkv, N, D); topk_indices: (B, H, N, K).
    Returns (B, H, N, D) in q's dtype: per query, softmax over the K listed keys
    of (q . k) / sqrt(D) (keys > i masked when ``causal``), times V; rows with
    no unmasked key are 0.

    ``q_start`` (additive, for sequence sharding): q and topk_indices then hold
    Nq query rows at positions q_start .. q_start + Nq - 1 of a sequence whose
    Nk keys k, v hold in full; row l is masked causally against q_start + l.
    """
    del block_m, use_triton
    if q_start is not None:
        return _topk_attention_rows(q, k, v, topk_indices, causal, int(q_start))
    B, H, Hkv, N, D, K = _check(q, k, v, topk_indices)
    dev = _lib.require_cuda(q, k, v, topk_indices)
    code = _lib.dtype_code(q)
    qc, kc, vc = q.contiguous(), k.contiguous(), v.contiguous()
    ic = topk_indices.contiguous()
    out = torch.empty_like(qc)
    if out.numel() == 0:
        return out
    with torch.cuda.device(dev):
        st = _lib.lib().ossa_topk_attention_fwd(
            qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), ic.data_ptr(),
            1 if ic.dtype == torch.int64 else 0, code, B, H, Hkv, N, D, K,
            float(1.0 / math.sqrt(D)), 1 if causal else 0, out.data_ptr(), _lib.stream_ptr(dev))
    _lib.check(st)
    return out


def _topk_attention_rows(q, k, v, topk_indices, causal, q_start):
    if q_start < 0:
        raise ValueError(f"q_start must be >= 0, got {q_start}")
    B, H, Hkv, Nq, D, K = _check(q, k, v, topk_indices, rows=True)
    Nk = k.shape[2]
    dev = _lib.require_cuda(q, k, v, topk_indices)
    code = _lib.dtype_code(q)
    qc, kc, vc = q.contiguous(), k.contiguous(), v.contiguous()
    ic = topk_indices.contiguous()
    out = torch.empty_like(qc)
    if out.numel() == 0:
        return out
    with torch.cuda.device(dev):
        st = _lib.lib().ossa_topk_attention_fwd_rows(
            qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), ic.data_ptr(),
            1 if ic.dtype == torch.int64 else 0, code, B, H, Hkv, Nq, Nk, D, K,
            float(1.0 / math.sqrt(D)), 1 if causal else 0, q_start, out.data_ptr(), _lib.stream_ptr(dev))
    _lib.check(st)
    return out
