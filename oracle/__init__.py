"""CPU oracle for the routed sparse-attention hot path.

TEST INFRASTRUCTURE.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline leg of ``bench.py`` may import this package, and only as the checker
(or, for the baseline, as the CPU implementation being timed).  The product
package ``ossa_b200`` never imports it.

Two parts:

* ``ossa_oracle.c`` (wrapped below): the canonical fp32 router projections,
  scores and total-order top-K selection, bit-exact by construction (see the
  C file's header for the pinned arithmetic).  Pinned against the reference's
  own outputs by ``tests/golden`` (generated from the reference implementation
  by ``tests/golden/make_golden.py``).
* ``reference_port.py``: the reference's PyTorch path restated with torch CPU
  ops (router.score, causal mask + topk, chunked gather forward, dense
  attention) — the attention-output oracle and the timed CPU baseline.
"""

from __future__ import annotations

import ctypes
import math

import numpy as np

from . import build as _build

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = _build.build()
        l = ctypes.CDLL(str(path))
        fp = ctypes.POINTER(ctypes.c_float)
        ip = ctypes.POINTER(ctypes.c_int32)
        i64 = ctypes.c_int64
        ci = ctypes.c_int
        cf = ctypes.c_float
        l.orc_project.argtypes = [fp, fp, i64, ci, ci, fp]
        l.orc_project.restype = None
        l.orc_scores.argtypes = [fp, fp, fp, ci, ci, ci, ci, ci, ci, cf, fp]
        l.orc_scores.restype = None
        l.orc_topk.argtypes = [fp, fp, fp, ci, ci, ci, ci, ci, ci, cf, ci, ci, ip, fp]
        l.orc_topk.restype = None
        l.orc_topk_rows.argtypes = [fp, fp, fp, ci, ci, ci, ci, ci, ci, cf, ci, ci,
                                    ctypes.POINTER(ctypes.c_int64), i64, ip]
        l.orc_topk_rows.restype = None
        _lib = l
    return _lib


def _f32(a) -> np.ndarray:
    if hasattr(a, "detach"):  # torch tensor (any float dtype converts exactly to fp32 here)
        a = a.detach().cpu().float().numpy()
    return np.ascontiguousarray(a, dtype=np.float32)


def _fp(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def project(x, w) -> np.ndarray:
    """x: (..., D), w: (R, D) -> (..., R) via the pinned fmaf chain."""
    x = _f32(x)
    w = _f32(w)
    D = x.shape[-1]
    R, D2 = w.shape
    assert D == D2
    rows = int(np.prod(x.shape[:-1]))
    out = np.empty(x.shape[:-1] + (R,), dtype=np.float32)
    lib().orc_project(_fp(x), _fp(w), rows, D, R, _fp(out))
    return out


def _shape4(q, k):
    B, H, N, _ = q.shape
    Bk, Hkv, Nk, _ = k.shape
    assert B == Bk and N == Nk and H % Hkv == 0
    return B, H, Hkv, N


def router_scores(q, k, wq, wk, pos_bias, seq_len: int) -> np.ndarray:
    """Dense (B, H, N, N) router logits (ContentRouter.score, router.py:171-190)."""
    B, H, Hkv, N = _shape4(q, k)
    qp = project(q, wq)
    kp = project(k, wk)
    R = qp.shape[-1]
    bias = _f32(pos_bias).reshape(-1)
    out = np.empty((B, H, N, N), dtype=np.float32)
    scale = np.float32(1.0 / math.sqrt(R))
    lib().orc_scores(_fp(qp), _fp(kp), _fp(bias), seq_len, B, H, Hkv, N, R, float(scale), _fp(out))
    return out


def _topk_rows(a, b, bias, L, scale, K, causal, with_scores):
    B, H, N, R = a.shape
    Hkv = b.shape[1]
    out = np.empty((B, H, N, K), dtype=np.int32)
    sc = np.empty((B, H, N, K), dtype=np.float32) if with_scores else None
    bias_p = _fp(bias) if bias is not None else None
    lib().orc_topk(_fp(a), _fp(b), bias_p, L, B, H, Hkv, N, R, float(scale), K, 1 if causal else 0,
                   out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                   _fp(sc) if sc is not None else None)
    return (out, sc) if with_scores else out


def router_topk(q, k, wq, wk, pos_bias, seq_len: int, K: int, causal: bool = True,
                with_scores: bool = False):
    """Canonical router top-K: (B, H, N, K) int32 ascending key order, -1 padded."""
    _shape4(q, k)
    qp = project(q, wq)
    kp = project(k, wk)
    R = qp.shape[-1]
    bias = _f32(pos_bias).reshape(-1)
    scale = np.float32(1.0 / math.sqrt(R))
    return _topk_rows(qp, kp, bias, seq_len, scale, K, causal, with_scores)


def oracle_topk(q, k, K: int, scale: float | None = None, causal: bool = True,
                with_scores: bool = False):
    """Exact-dot top-K (q k^T * scale in fp32), the oracle selector."""
    q = _f32(q)
    k = _f32(k)
    _shape4(q, k)
    D = q.shape[-1]
    s = np.float32(1.0 / math.sqrt(D) if scale is None else scale)
    return _topk_rows(q, k, None, 1, s, K, causal, with_scores)


def oracle_topk_rows(q, k, K: int, rows, scale: float | None = None, causal: bool = True) -> np.ndarray:
    """Exact-dot top-K for selected rows only (rows: flat ids (b*H + h)*N + i),
    (len(rows), K) int32: spot checks of full-size oracle selections."""
    B, H, Hkv, N = _shape4(q, k)
    rows = np.ascontiguousarray(rows, dtype=np.int64)
    D = q.shape[-1]
    qf = q.reshape(B * H * N, D)
    qsel = _f32(qf[torch_index(rows)] if hasattr(qf, "detach") else qf[rows])
    kf = _f32(k)
    s = np.float32(1.0 / math.sqrt(D) if scale is None else scale)
    out = np.empty((len(rows), K), dtype=np.int32)
    lib().orc_topk_rows(_fp(qsel), _fp(kf), None, 1, B, H, Hkv, N, D, float(s), K, 1 if causal else 0,
                        rows.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), len(rows),
                        out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)))
    return out


def router_topk_rows(q, k, wq, wk, pos_bias, seq_len: int, K: int, rows, causal: bool = True) -> np.ndarray:
    """Canonical router top-K for selected rows only.  rows: flat ids
    (b*H + h)*N + i.  Returns (len(rows), K) int32.  Only the listed query rows
    are projected, so full-size tensors can be spot-checked quickly."""
    B, H, Hkv, N = _shape4(q, k)
    rows = np.ascontiguousarray(rows, dtype=np.int64)
    qf = q.reshape(B * H * N, q.shape[-1])
    if hasattr(qf, "detach"):
        qsel = qf[torch_index(rows)]
    else:
        qsel = qf[rows]
    qp = project(qsel, wq)
    kp = project(k, wk)
    R = qp.shape[-1]
    bias = _f32(pos_bias).reshape(-1)
    scale = np.float32(1.0 / math.sqrt(R))
    out = np.empty((len(rows), K), dtype=np.int32)
    lib().orc_topk_rows(_fp(qp), _fp(kp), _fp(bias), seq_len, B, H, Hkv, N, R, float(scale), K,
                        1 if causal else 0, rows.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)),
                        len(rows), out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)))
    return out


def order_by_score(idx: np.ndarray, scores: np.ndarray) -> np.ndarray:
    """Reorders index rows (as router_topk(..., with_scores=True) returns them)
    to torch.topk's order: descending score (NaN first, as torch.topk ranks it),
    ties toward the lower key index, -1 padding last (ossa/router.py:202-203)."""
    bits = np.ascontiguousarray(scores, dtype=np.float32).view(np.uint32).astype(np.int64)
    bits = np.where(np.isnan(scores), 0x7FC00000, bits)
    okey = np.where(bits & 0x80000000, (~bits) & 0xFFFFFFFF, bits | 0x80000000)
    valid = idx >= 0
    primary = np.where(valid, -okey, 1)  # padding after every real score
    secondary = np.where(valid, idx, 0)
    perm = np.lexsort((secondary, primary), axis=-1)
    return np.take_along_axis(idx, perm, axis=-1)


def torch_index(rows: np.ndarray):
    import torch
    return torch.from_numpy(rows)
