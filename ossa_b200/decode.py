"""Decode-step selection with a cache of projected keys.

The reference's patched forward is prefill-only (ossa/bench/sparse_forward.py:
157-160 ignores ``past_key_values``).  For decoding, each generated token adds
one key per kv head; ``router_topk`` would project every cached key again at
every step.  ``RouterKeyCache`` projects each key once, k' = k Wk^T (the fp32
chain of ossa/router.py:180 that every selector scores with), into a preallocated
(B, Hkv, capacity, r) fp32 cache, and selects the new query rows against the
cached rows with ``ossa_router_topk_rows_kp``.  The indices are identical to
``router_topk(q_new, k_all, ..., q_start=...)`` on the same keys.
"""

from __future__ import annotations

import torch

from . import _lib


class RouterKeyCache:
    """Projected keys of one router for up to ``capacity`` positions.

    ``router``: a ContentRouter (q_proj, k_proj, pos_bias, cfg.seq_len).
    ``append(k_new)`` takes (B, Hkv, T, D) keys for the next T positions;
    ``topk(q_new, top_k)`` selects for (B, H, Tq, D) query rows at positions
    ``q_start .. q_start + Tq - 1`` (default: the last Tq cached positions)
    among the cached keys, causal by default."""

    def __init__(self, router, batch: int, kv_heads: int, capacity: int, device=None):
        wq, wk, pb = router.q_proj[0].weight, router.k_proj[0].weight, router.pos_bias.weight
        self.seq_len = int(router.cfg.seq_len)
        dev = torch.device(device) if device is not None else wk.device
        self.wq = wq.detach().float().contiguous().to(dev)
        self.wk = wk.detach().float().contiguous().to(dev)
        self.pos_bias = pb.detach().float().contiguous().to(dev)
        self.r, self.D = self.wk.shape
        self.B, self.Hkv, self.capacity = batch, kv_heads, capacity
        self.kp = torch.zeros((batch, kv_heads, capacity, self.r), dtype=torch.float32, device=dev)
        self.length = 0

    def append(self, k_new: torch.Tensor) -> None:
        if k_new.dim() != 4 or tuple(k_new.shape[:2]) != (self.B, self.Hkv) or k_new.shape[3] != self.D:
            raise ValueError(f"k_new must be ({self.B}, {self.Hkv}, T, {self.D}); got {tuple(k_new.shape)}")
        T = k_new.shape[2]
        if self.length + T > self.capacity:
            raise ValueError(f"cache of {self.capacity} positions cannot take {self.length} + {T}")
        if T == 0:
            return
        dev = _lib.require_cuda(k_new, self.kp)
        kc = k_new if k_new.dtype in (torch.float32, torch.bfloat16) else k_new.float()
        kc = kc.contiguous()
        tmp = torch.empty((self.B, self.Hkv, T, self.r), dtype=torch.float32, device=dev)
        with torch.cuda.device(dev):
            st = _lib.lib().ossa_router_project_keys(kc.data_ptr(), _lib.dtype_code(kc), self.wk.data_ptr(),
                                                     self.B * self.Hkv * T, self.D, self.r, tmp.data_ptr(),
                                                     _lib.stream_ptr(dev))
        _lib.check(st)
        self.kp[:, :, self.length:self.length + T].copy_(tmp)
        self.length += T

    def topk(self, q_new: torch.Tensor, top_k: int, *, q_start: int | None = None,
             causal: bool = True) -> torch.Tensor:
        """int32 (B, H, Tq, top_k) indices into the cached positions, ascending,
        -1 padded (the router_topk convention)."""
        if q_new.dim() != 4 or q_new.shape[0] != self.B or q_new.shape[3] != self.D:
            raise ValueError(f"q_new must be ({self.B}, H, Tq, {self.D}); got {tuple(q_new.shape)}")
        B, H, Tq, D = q_new.shape
        if H % self.Hkv != 0:
            raise ValueError(f"query heads {H} must be a multiple of key heads {self.Hkv}")
        if top_k <= 0:
            raise ValueError(f"top_k must be positive, got {top_k}")
        Nk = self.length
        q0 = Nk - Tq if q_start is None else int(q_start)
        if Nk == 0 or q0 < 0:
            raise ValueError(f"query positions from {q0} need cached keys (cached {Nk})")
        dev = _lib.require_cuda(q_new, self.kp)
        qc = q_new if q_new.dtype in (torch.float32, torch.bfloat16) else q_new.float()
        qc = qc.contiguous()
        if causal and q0 + Tq <= Nk:
            # causal rows never see a key past their own position, so the whole
            # cache can be passed as is (rows past `length` are zeros and masked)
            kp, Nk = self.kp, self.capacity
        else:
            kp = self.kp if Nk == self.capacity else self.kp[:, :, :Nk].contiguous()
        out = torch.empty((B, H, Tq, top_k), dtype=torch.int32, device=dev)
        L = _lib.lib()
        ws_bytes = L.ossa_router_workspace_size_kp(B, H, self.Hkv, Tq, Nk, self.r, int(top_k))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        with torch.cuda.device(dev):
            st = L.ossa_router_topk_rows_kp(qc.data_ptr(), _lib.dtype_code(qc), self.wq.data_ptr(), kp.data_ptr(),
                                            self.pos_bias.data_ptr(), B, H, self.Hkv, Tq, Nk, D, self.r,
                                            self.seq_len, int(top_k), 1 if causal else 0, q0, out.data_ptr(),
                                            ws.data_ptr(), ws_bytes, _lib.stream_ptr(dev))
        _lib.check(st)
        return out
