"""The oracle selector (exact q.k * scale scores, ossa/bench/sparse_forward.py:194-202)
on the tensor-core kernel at head_dim 128.

fp16 tensor-core scores with a per-row error bound choose the candidates and
the fp32 canonical scores decide them, so every index row must equal the
CUDA-core exact selector's (OSSA_ORACLE_SELECT=exact) and the CPU oracle's.
"""

import ctypes
import math
import os

import numpy as np
import pytest
import torch

import cases
import oracle
from ossa_b200 import _lib, oracle_topk

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _assert_same(got: torch.Tensor, ref: np.ndarray):
    g = got.cpu().numpy()
    assert g.shape == ref.shape
    bad = (g != ref).any(-1)
    assert not bad.any(), f"{bad.sum()} rows differ; first at {np.argwhere(bad)[0]}"


def _oracle_ws(q, k, K, causal=True):
    """Tensor-core oracle selection through the C-ABI, with the fallback-row
    count and status word from the workspace counters."""
    B, H, N, D = q.shape
    Hkv = k.shape[1]
    L = _lib.lib()
    code = _lib.dtype_code(q)
    ws_bytes = L.ossa_oracle_workspace_size(B, H, Hkv, N, D, K, code)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
    out = torch.empty((B, H, N, K), dtype=torch.int32, device=DEV)
    st = L.ossa_oracle_topk_ws(q.data_ptr(), k.data_ptr(), code, B, H, Hkv, N, D, 1.0 / math.sqrt(D), K,
                               1 if causal else 0, out.data_ptr(), ws.data_ptr(), ws_bytes, _lib.stream_ptr(q.device))
    _lib.check(st)
    fb, status = ctypes.c_int(0), ctypes.c_int(0)
    _lib.check(L.ossa_router_status(ws.data_ptr(), ctypes.byref(fb), ctypes.byref(status)))
    return out, fb.value, status.value


def _exact(q, k, K, causal=True):
    os.environ["OSSA_ORACLE_SELECT"] = "exact"
    try:
        return oracle_topk(q, k, K, causal=causal)
    finally:
        del os.environ["OSSA_ORACLE_SELECT"]


def shared_component_qk(B, H, Hkv, N, D, seed, rank=8, strength=1.0):
    """q, k ~ N(0, 1) plus a rank-`rank` component shared by all heads (each
    query and key mixes the same `rank` directions with its own N(0, 1)
    weights), so a query's best keys stand out from the rest."""
    g = torch.Generator().manual_seed(seed)
    basis = torch.linalg.qr(torch.randn(D, rank, generator=g))[0].T * math.sqrt(D / rank)  # (rank, D)
    q = torch.randn(B, H, N, D, generator=g) + strength * torch.randn(B, H, N, rank, generator=g) @ basis
    k = torch.randn(B, Hkv, N, D, generator=g) + strength * torch.randn(B, Hkv, N, rank, generator=g) @ basis
    return q, k


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("N,K,causal", [
    (640, 32, True), (777, 64, True), (512, 100, True), (1024, 128, True),
    (640, 64, False), (600, 128, False), (300, 16, True),
])
def test_tensor_core_oracle_matches_exact_and_cpu(dtype, N, K, causal):
    B, H, Hkv, D = 1, 4, 2, 128
    q, k, _ = cases.qkv(B, H, Hkv, N, D, seed=N + K + int(causal), scale=1.0 / math.sqrt(D))
    q, k = q.to(dtype).to(DEV), k.to(dtype).to(DEV)
    tc, fb, status = _oracle_ws(q, k, K, causal)
    assert status == 0
    ex = _exact(q, k, K, causal)
    assert torch.equal(tc, ex), f"{(tc != ex).any(-1).sum().item()} rows differ"
    assert fb < 0.01 * B * H * N, f"{fb} rows fell back to the full-row exact selector"
    _assert_same(tc, oracle.oracle_topk(q.cpu(), k.cpu(), K, causal=causal))
    # the Python entry point takes the same path
    assert torch.equal(oracle_topk(q, k, K, causal=causal), tc)


@pytest.mark.parametrize("K", [32, 128])
def test_tensor_core_oracle_shared_component(K):
    """The oracle workload's distribution (unit-normal q, k plus a shared rank-8
    component) at 4096 keys: equal to the exact selector on every row and to the
    CPU oracle on sampled rows, with few rows on the full-row fallback."""
    B, H, Hkv, N, D = 1, 12, 2, 4096, 128
    q, k = shared_component_qk(B, H, Hkv, N, D, seed=7 + K)
    q, k = q.bfloat16().to(DEV), k.bfloat16().to(DEV)
    tc, fb, status = _oracle_ws(q, k, K)
    assert status == 0
    ex = _exact(q, k, K)
    assert torch.equal(tc, ex), f"{(tc != ex).any(-1).sum().item()} rows differ"
    assert fb < 0.01 * B * H * N, f"{fb} rows fell back to the full-row exact selector"
    rows = np.concatenate([np.arange(0, B * H * N, 509), np.array([N - 1, B * H * N - 1])]).astype(np.int64)
    ref = oracle.oracle_topk_rows(q.cpu(), k.cpu(), K, rows)
    _assert_same(tc.reshape(-1, K)[torch.from_numpy(rows).to(DEV)], ref)


def test_tensor_core_oracle_ties_and_non_finite():
    """Duplicate keys (exact score ties, lower index wins) and a NaN in one key
    row (its score ranks first for every query that sees it): the rows go to the
    exact fallback and the result is still the oracle's."""
    B, H, Hkv, N, D, K = 1, 2, 1, 512, 128, 64
    q, k, _ = cases.qkv(B, H, Hkv, N, D, seed=5, scale=1.0 / math.sqrt(D))
    k[0, 0, 200:260] = k[0, 0, 100]
    k[0, 0, 300, 5] = float("nan")
    q, k = q.to(DEV), k.to(DEV)
    tc, fb, status = _oracle_ws(q, k, K)
    assert status == 0
    _assert_same(tc, oracle.oracle_topk(q.cpu(), k.cpu(), K))
    assert torch.equal(tc, _exact(q, k, K))


@pytest.mark.parametrize("K", [1, 3, 65])
def test_tensor_core_oracle_small_and_odd_k(K):
    """K = 1 and 3 (the smallest lists for the K-th score search and the merge
    path) and K = 65 (the first wide K): equal to the exact selector and the CPU
    oracle."""
    B, H, Hkv, N, D = 1, 4, 2, 700, 128
    q, k, _ = cases.qkv(B, H, Hkv, N, D, seed=90 + K, scale=1.0 / math.sqrt(D))
    q, k = q.bfloat16().to(DEV), k.bfloat16().to(DEV)
    tc, fb, status = _oracle_ws(q, k, K)
    assert status == 0
    assert torch.equal(tc, _exact(q, k, K))
    _assert_same(tc, oracle.oracle_topk(q.cpu(), k.cpu(), K))


def test_tensor_core_oracle_infinite_key():
    """A key row holding +inf: every query that sees it scores it +inf or NaN
    (inf * 0 terms), and such rows go to the full-row exact selector; the result
    is still the oracle's."""
    B, H, Hkv, N, D, K = 1, 2, 1, 400, 128, 32
    q, k, _ = cases.qkv(B, H, Hkv, N, D, seed=17, scale=1.0 / math.sqrt(D))
    k[0, 0, 150, 7] = float("inf")
    q, k = q.to(DEV), k.to(DEV)
    tc, fb, status = _oracle_ws(q, k, K)
    assert status == 0
    _assert_same(tc, oracle.oracle_topk(q.cpu(), k.cpu(), K))
