"""Fused causal top-K key selection (router and exact-dot oracle selectors).

Functional entry points behind ``ContentRouter.topk`` and the patched
attention forward.  The reference materialises the full (B, H, N, N) selector
and calls ``torch.topk`` (ossa/router.py:171-203,
ossa/bench/sparse_forward.py:180-202); here one sm_100a kernel scores and
selects per query block, so the N x N matrix never reaches HBM.

Index convention (shared by every ossa_b200 selector and consumed by
``topk_attention``): int32, shape (B, H, N, K), each row's chosen keys in
ascending key order, padded with -1 when fewer than K keys are eligible
(rows i < K-1 under the causal mask).  The set is exactly the set torch.topk
returns on fp32 scores with ties broken toward the lower key index.
"""

from __future__ import annotations

import ctypes
import math

from typing import Optional

import torch

from . import _lib


def _check_qk(q: torch.Tensor, k: torch.Tensor, rows: bool = False):
    if q.dim() != 4 or k.dim() != 4:
        raise ValueError(f"q and k must be (B, H, N, D); got {tuple(q.shape)} and {tuple(k.shape)}")
    B, H, N, D = q.shape
    Bk, Hkv, Nk, Dk = k.shape
    if (B, D) != (Bk, Dk) or (not rows and N != Nk):
        raise ValueError(f"q {tuple(q.shape)} and k {tuple(k.shape)} disagree on B, N or D")
    if Hkv <= 0 or H % Hkv != 0:
        raise ValueError(f"query heads {H} must be a multiple of key heads {Hkv}")
    return B, H, Hkv, N, D


def _as_kernel_input(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    if t.dtype not in (torch.float32, torch.bfloat16):
        t = t.float()  # float16 and friends convert exactly to fp32
    return t.to(dtype).contiguous()


def _common_dtype(q: torch.Tensor, k: torch.Tensor) -> torch.dtype:
    return torch.bfloat16 if (q.dtype == torch.bfloat16 and k.dtype == torch.bfloat16) else torch.float32


def router_topk(q: torch.Tensor, k: torch.Tensor, wq: torch.Tensor, wk: torch.Tensor,
                pos_bias: torch.Tensor, seq_len: int, top_k: int, *,
                causal: bool = True, q_start: Optional[int] = None) -> torch.Tensor:
    """ContentRouter top-K (ossa/router.py:171-190 scores) -> int32 (B, H, N, top_k).

    q: (B, H, N, D); k: (B, Hkv, N, D) with Hkv dividing H (or the repeated H
    heads).  wq, wk: (r, D) projection weights; pos_bias: (2*seq_len, 1) or
    (2*seq_len,).  Scores and selection are fp32.

    ``q_start`` (additive, for sequence sharding): q then holds Nq query rows at
    positions q_start .. q_start + Nq - 1 against all Nk keys of k; positions
    enter the causal mask and the position bias.  The result is (B, H, Nq, top_k)
    and equals the matching rows of the unsharded call.
    """
    return _router_topk(q, k, wq, wk, pos_bias, seq_len, top_k, causal=causal, q_start=q_start)[0]


def project_router_keys(k: torch.Tensor, wk: torch.Tensor) -> torch.Tensor:
    """Router key projections k' = k Wk^T (the k_proj of ossa/router.py:182), fp32
    (B, Hkv, Nk, r): every value the canonical fmaf chain router_topk computes
    internally.  Pass the result to ``router_topk_projected`` to select several query
    blocks against the same keys without projecting them again."""
    if k.dim() != 4:
        raise ValueError(f"k must be (B, Hkv, Nk, D); got {tuple(k.shape)}")
    B, Hkv, Nk, D = k.shape
    dev = _lib.require_cuda(k, wk)
    r = wk.shape[0]
    if wk.shape != (r, D):
        raise ValueError(f"projection weights must be ({r}, {D}); got {tuple(wk.shape)}")
    kc = _as_kernel_input(k, k.dtype if k.dtype in (torch.float32, torch.bfloat16) else torch.float32)
    wkc = wk.detach().float().contiguous()
    kp = torch.empty((B, Hkv, Nk, r), dtype=torch.float32, device=dev)
    if kp.numel() == 0:
        return kp
    with torch.cuda.device(dev):
        st = _lib.lib().ossa_router_project_keys(kc.data_ptr(), _lib.dtype_code(kc), wkc.data_ptr(), B * Hkv * Nk, D,
                                                 r, kp.data_ptr(), _lib.stream_ptr(dev))
    _lib.check(st)
    return kp


def router_topk_projected(q: torch.Tensor, kp: torch.Tensor, wq: torch.Tensor, pos_bias: torch.Tensor,
                          seq_len: int, top_k: int, *, causal: bool = True,
                          q_start: Optional[int] = None) -> torch.Tensor:
    """``router_topk`` with the keys given as their projections ``kp`` (from
    ``project_router_keys``), identical indices.  q: (B, H, Nq, D) query rows at
    positions q_start .. q_start + Nq - 1 (``q_start`` may be omitted when Nq equals
    the number of keys); kp: (B, Hkv, Nk, r) fp32."""
    if q.dim() != 4 or kp.dim() != 4:
        raise ValueError(f"q must be (B, H, Nq, D) and kp (B, Hkv, Nk, r); got {tuple(q.shape)}, {tuple(kp.shape)}")
    B, H, Nq, D = q.shape
    Bk, Hkv, Nk, r = kp.shape
    if Bk != B or Hkv <= 0 or H % Hkv != 0:
        raise ValueError(f"q {tuple(q.shape)} and kp {tuple(kp.shape)} disagree on B or the head grouping")
    if q_start is None and Nq != Nk:
        raise ValueError("q_start is needed when q holds fewer rows than there are keys")
    q0 = 0 if q_start is None else int(q_start)
    if q0 < 0:
        raise ValueError(f"q_start must be >= 0, got {q0}")
    if kp.dtype != torch.float32:
        raise ValueError("kp must be float32 (project_router_keys)")
    dev = _lib.require_cuda(q, kp, wq, pos_bias)
    if wq.shape != (r, D):
        raise ValueError(f"projection weights must be ({r}, {D}); got {tuple(wq.shape)}")
    if pos_bias.numel() != 2 * seq_len:
        raise ValueError(f"pos_bias has {pos_bias.numel()} entries, expected 2*seq_len = {2 * seq_len}")
    if top_k < 0:
        raise ValueError(f"top_k must be >= 0, got {top_k}")
    out = torch.empty((B, H, Nq, top_k), dtype=torch.int32, device=dev)
    if out.numel() == 0:
        return out
    qc = _as_kernel_input(q, q.dtype if q.dtype in (torch.float32, torch.bfloat16) else torch.float32)
    kpc = kp.contiguous()
    wqc = wq.detach().float().contiguous()
    pbc = pos_bias.detach().float().contiguous()
    L = _lib.lib()
    ws_bytes = L.ossa_router_workspace_size_kp(B, H, Hkv, Nq, Nk, r, int(top_k))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        st = L.ossa_router_topk_rows_kp(qc.data_ptr(), _lib.dtype_code(qc), wqc.data_ptr(), kpc.data_ptr(),
                                        pbc.data_ptr(), B, H, Hkv, Nq, Nk, D, r, int(seq_len), int(top_k),
                                        1 if causal else 0, q0, out.data_ptr(), ws.data_ptr(), ws_bytes,
                                        _lib.stream_ptr(dev))
    _lib.check(st)
    return out


def router_topk_with_status(q, k, wq, wk, pos_bias, seq_len: int, top_k: int, *, causal: bool = True):
    """router_topk plus (rows sent to the exact fallback, device status word),
    read back synchronously; a nonzero status means a bounded device wait
    expired and the indices are not valid."""
    return _router_topk(q, k, wq, wk, pos_bias, seq_len, top_k, causal=causal, with_status=True)


def router_topk_by_score(q: torch.Tensor, k: torch.Tensor, wq: torch.Tensor, wk: torch.Tensor,
                         pos_bias: torch.Tensor, seq_len: int, top_k: int, *, causal: bool = True) -> torch.Tensor:
    """router_topk with each row in torch.topk's order: keys by descending fp32
    score, ties toward the lower key index, -1 padding last (the order of
    ``torch.topk(score, k).indices`` in ossa/router.py:202-203).  Same sets as
    router_topk."""
    return _router_topk(q, k, wq, wk, pos_bias, seq_len, top_k, causal=causal, by_score=True)[0]


def _router_topk(q, k, wq, wk, pos_bias, seq_len, top_k, *, causal=True, with_status=False, q_start=None,
                 by_score=False):
    B, H, Hkv, N, D = _check_qk(q, k, rows=q_start is not None)
    Nk = k.shape[2]
    q0 = 0 if q_start is None else int(q_start)
    if q0 < 0:
        raise ValueError(f"q_start must be >= 0, got {q0}")
    dev = _lib.require_cuda(q, k, wq, wk, pos_bias)
    r = wq.shape[0]
    if wq.shape != (r, D) or wk.shape != (r, D):
        raise ValueError(f"projection weights must be ({r}, {D}); got {tuple(wq.shape)}, {tuple(wk.shape)}")
    if pos_bias.numel() != 2 * seq_len:
        raise ValueError(f"pos_bias has {pos_bias.numel()} entries, expected 2*seq_len = {2 * seq_len}")
    if top_k < 0:
        raise ValueError(f"top_k must be >= 0, got {top_k}")
    out = torch.empty((B, H, N, top_k), dtype=torch.int32, device=dev)
    if out.numel() == 0:
        return out, 0, 0
    dt = _common_dtype(q, k)
    qc = _as_kernel_input(q, dt)
    kc = _as_kernel_input(k, dt)
    wqc = wq.detach().float().contiguous()
    wkc = wk.detach().float().contiguous()
    pbc = pos_bias.detach().float().contiguous()
    L = _lib.lib()
    ws_bytes = L.ossa_router_workspace_size_rows(B, H, Hkv, N, Nk, r, top_k)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        if by_score:
            st = L.ossa_router_topk_sorted(qc.data_ptr(), kc.data_ptr(), _lib.dtype_code(qc), wqc.data_ptr(),
                                           wkc.data_ptr(), pbc.data_ptr(), B, H, Hkv, N, D, r, int(seq_len),
                                           int(top_k), 1 if causal else 0, out.data_ptr(), ws.data_ptr(),
                                           ws_bytes, _lib.stream_ptr(dev))
        elif q_start is None:
            st = L.ossa_router_topk(qc.data_ptr(), kc.data_ptr(), _lib.dtype_code(qc), wqc.data_ptr(),
                                    wkc.data_ptr(), pbc.data_ptr(), B, H, Hkv, N, D, r, int(seq_len),
                                    int(top_k), 1 if causal else 0, out.data_ptr(), ws.data_ptr(),
                                    ws_bytes, _lib.stream_ptr(dev))
        else:
            st = L.ossa_router_topk_rows(qc.data_ptr(), kc.data_ptr(), _lib.dtype_code(qc), wqc.data_ptr(),
                                         wkc.data_ptr(), pbc.data_ptr(), B, H, Hkv, N, Nk, D, r, int(seq_len),
                                         int(top_k), 1 if causal else 0, q0, out.data_ptr(), ws.data_ptr(),
                                         ws_bytes, _lib.stream_ptr(dev))
    _lib.check(st)
    if not with_status:
        return out, None, None
    fb = ctypes.c_int(0)
    status = ctypes.c_int(0)
    with torch.cuda.device(dev):
        _lib.check(L.ossa_router_status(ws.data_ptr(), ctypes.byref(fb), ctypes.byref(status)))
    return out, fb.value, status.value


def router_scores(q: torch.Tensor, k: torch.Tensor, wq: torch.Tensor, wk: torch.Tensor,
                  pos_bias: torch.Tensor, seq_len: int) -> torch.Tensor:
    """Materialised router logits (B, H, N, N) fp32 (ContentRouter.score)."""
    B, H, Hkv, N, D = _check_qk(q, k)
    dev = _lib.require_cuda(q, k, wq, wk, pos_bias)
    r = wq.shape[0]
    if wq.shape != (r, D) or wk.shape != (r, D):
        raise ValueError(f"projection weights must be ({r}, {D}); got {tuple(wq.shape)}, {tuple(wk.shape)}")
    if pos_bias.numel() != 2 * seq_len:
        raise ValueError(f"pos_bias has {pos_bias.numel()} entries, expected 2*seq_len = {2 * seq_len}")
    out = torch.empty((B, H, N, N), dtype=torch.float32, device=dev)
    if out.numel() == 0:
        return out
    dt = _common_dtype(q, k)
    qc = _as_kernel_input(q, dt)
    kc = _as_kernel_input(k, dt)
    wqc = wq.detach().float().contiguous()
    wkc = wk.detach().float().contiguous()
    pbc = pos_bias.detach().float().contiguous()
    L = _lib.lib()
    ws_bytes = L.ossa_router_workspace_size(B, H, Hkv, N, r, 0)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        st = L.ossa_router_score(qc.data_ptr(), kc.data_ptr(), _lib.dtype_code(qc), wqc.data_ptr(),
                                 wkc.data_ptr(), pbc.data_ptr(), B, H, Hkv, N, D, r, int(seq_len),
                                 out.data_ptr(), ws.data_ptr(), ws_bytes, _lib.stream_ptr(dev))
    _lib.check(st)
    return out


def oracle_topk(q: torch.Tensor, k: torch.Tensor, top_k: int, *, scale: float | None = None,
                causal: bool = True, with_status: bool = False):
    """Exact-dot selector (sparse_forward.py:194-202): top-K of (q . k) * scale,
    fp32, no router.  Returns int32 (B, H, N, top_k).

    At head_dim 128 and top_k <= 128 the selection runs on the tensor-core
    selector (fp16 scores with a per-row error bound pick the candidates, fp32
    scores decide them); the indices are the exact selector's bit for bit.
    OSSA_ORACLE_SELECT=exact forces the CUDA-core exact selector."""
    B, H, Hkv, N, D = _check_qk(q, k)
    dev = _lib.require_cuda(q, k)
    if top_k < 0:
        raise ValueError(f"top_k must be >= 0, got {top_k}")
    out = torch.empty((B, H, N, top_k), dtype=torch.int32, device=dev)
    if out.numel() == 0:
        return (out, 0, 0) if with_status else out
    s = float(1.0 / math.sqrt(D)) if scale is None else float(scale)
    dt = _common_dtype(q, k)
    qc = _as_kernel_input(q, dt)
    kc = _as_kernel_input(k, dt)
    L = _lib.lib()
    code = _lib.dtype_code(qc)
    ws_bytes = L.ossa_oracle_workspace_size(B, H, Hkv, N, D, int(top_k), code)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        st = L.ossa_oracle_topk_ws(qc.data_ptr(), kc.data_ptr(), code, B, H, Hkv, N, D, s, int(top_k),
                                   1 if causal else 0, out.data_ptr(), ws.data_ptr(), ws_bytes,
                                   _lib.stream_ptr(dev))
    _lib.check(st)
    if with_status:
        fb, status = ctypes.c_int(0), ctypes.c_int(0)
        with torch.cuda.device(dev):
            _lib.check(L.ossa_router_status(ws.data_ptr(), ctypes.byref(fb), ctypes.byref(status)))
        return out, fb.value, status.value
    return out


def oracle_topk_with_status(q: torch.Tensor, k: torch.Tensor, top_k: int, *, scale: float | None = None,
                            causal: bool = True):
    """oracle_topk plus (rows sent to the full-row exact fallback, device status
    word), read back synchronously; a nonzero status means a bounded device wait
    expired and the indices are not valid."""
    return oracle_topk(q, k, top_k, scale=scale, causal=causal, with_status=True)


def with_diagonal(idx: torch.Tensor) -> torch.Tensor:
    """Appends the query's own position to every row that does not already list
    it (-1 where it does): the forced diagonal of the reference's "mask" path
    (ossa/bench/sparse_forward.py:216-218), expressed as an index set."""
    N = idx.shape[2]
    pos = torch.arange(N, device=idx.device, dtype=idx.dtype).view(1, 1, N, 1)
    has = (idx == pos).any(dim=-1, keepdim=True)
    diag = torch.where(has, torch.full_like(pos.expand_as(has), -1), pos.expand_as(has))
    return torch.cat([idx, diag], dim=-1).contiguous()
