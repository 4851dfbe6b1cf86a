"""RoPE fused with the head transpose of the patched layer.

The patched forward (ossa/bench/sparse_forward.py:166-178) views each q/k/v
projection (B, N, Hx*D) as (B, Hx, N, D), applies Qwen2's
``apply_rotary_pos_emb`` to q and k, and the selection and gather read
contiguous rows.  ``rope_to_heads`` does that in one kernel pass, with the same
rounding as the eager expression ``x*cos + rotate_half(x)*sin``; the result is
bit-identical to it.  Additive: the reference runs the eager ops.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib


def rope_to_heads(x: torch.Tensor, n_heads: int, cos: Optional[torch.Tensor] = None,
                  sin: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x: (B, N, n_heads * D) or (B, N, n_heads, D); cos, sin: (B or 1, N, D)
    (Qwen2's position embeddings) or both None (layout only).  Returns the
    contiguous (B, n_heads, N, D) tensor, rotated when cos/sin are given."""
    if (cos is None) != (sin is None):
        raise ValueError("pass both cos and sin, or neither")
    B, N = x.shape[0], x.shape[1]
    D = x.shape[-1] if x.dim() == 4 else x.shape[-1] // n_heads
    if x.dim() not in (3, 4) or x.shape[2:] not in ((n_heads * D,), (n_heads, D)):
        raise ValueError(f"x of shape {tuple(x.shape)} is not (B, N, {n_heads} heads x D)")
    ts = [x] if cos is None else [x, cos, sin]
    dev = _lib.require_cuda(*ts)
    xc = x.contiguous()
    code = _lib.dtype_code(xc)
    cs = None
    if cos is not None:
        cos = cos.to(xc.dtype)
        sin = sin.to(xc.dtype)
        if cos.dim() == 2:
            cos, sin = cos.unsqueeze(0), sin.unsqueeze(0)
        if cos.shape != sin.shape or cos.shape[0] not in (1, B) or tuple(cos.shape[1:]) != (N, D):
            raise ValueError(f"cos/sin of shape {tuple(cos.shape)} do not match (B or 1, {N}, {D})")
        cs = (cos.contiguous(), sin.contiguous())
    out = torch.empty((B, n_heads, N, D), dtype=xc.dtype, device=dev)
    if out.numel() == 0:
        return out
    with torch.cuda.device(dev):
        st = _lib.lib().ossa_rope_to_heads(xc.data_ptr(), _lib.ptr(cs[0] if cs else None),
                                           _lib.ptr(cs[1] if cs else None),
                                           1 if cs is not None and cs[0].shape[0] == B and B > 1 else 0, code,
                                           B, N, n_heads, D, out.data_ptr(), _lib.stream_ptr(dev))
    _lib.check(st)
    return out
