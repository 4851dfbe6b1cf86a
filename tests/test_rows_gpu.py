"""Query-row ranges (q_start): a block of query rows at positions
q_start .. q_start + Nq - 1 against the full key sequence must give exactly the
matching rows of the unsharded call, for the tensor-core selector, the exact
selector and the gather; and the selection rows match the oracle."""

import math

import numpy as np
import pytest
import torch

import cases
import oracle
from ossa_b200 import router_topk, topk_attention

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _inputs(B, H, Hkv, N, D, r, L, seed):
    q, k, v = cases.qkv(B, H, Hkv, N, D, seed=seed, scale=1.0 / math.sqrt(D))
    wq, wk, pb = cases.router_weights(D, r, L, seed)
    return q.bfloat16(), k.bfloat16(), v.bfloat16(), wq, wk, pb


@pytest.mark.parametrize("r,K", [(64, 64), (64, 16), (32, 40), (64, 128)])
@pytest.mark.parametrize("q0,nq", [(0, 300), (300, 257), (129, 128), (640, 1), (511, 130)])
@pytest.mark.parametrize("causal", [True, False])
def test_router_rows_match_full(r, K, q0, nq, causal):
    B, H, Hkv, N, D, L = 1, 4, 2, 768, 128, 768
    q, k, _, wq, wk, pb = _inputs(B, H, Hkv, N, D, r, L, seed=r + K)
    qd, kd = q.to(DEV), k.to(DEV)
    args = (wq.to(DEV), wk.to(DEV), pb.to(DEV), L, K)
    full = router_topk(qd, kd, *args, causal=causal)
    part = router_topk(qd[:, :, q0:q0 + nq].contiguous(), kd, *args, causal=causal, q_start=q0)
    assert torch.equal(part, full[:, :, q0:q0 + nq])


def test_router_rows_match_oracle():
    B, H, Hkv, N, D, r, L, K = 2, 6, 2, 640, 128, 64, 512, 64
    q, k, _, wq, wk, pb = _inputs(B, H, Hkv, N, D, r, L, seed=5)
    q0, nq = 200, 333
    part = router_topk(q[:, :, q0:q0 + nq].contiguous().to(DEV), k.to(DEV), wq.to(DEV), wk.to(DEV),
                       pb.to(DEV), L, K, q_start=q0)
    rows = np.array([(bh * N + i) for bh in range(B * H) for i in range(q0, q0 + nq)])
    ref = oracle.router_topk_rows(q, k, wq, wk, pb, L, K, rows)
    np.testing.assert_array_equal(part.cpu().numpy().reshape(-1, K), ref)


@pytest.mark.parametrize("q0,nq", [(0, 100), (100, 155), (37, 1), (250, 5)])
@pytest.mark.parametrize("causal", [True, False])
def test_gather_rows_match_full(q0, nq, causal):
    B, H, Hkv, N, D, K = 2, 6, 2, 256, 128, 48
    q, k, v, _, _, _ = _inputs(B, H, Hkv, N, D, 64, 256, seed=q0 + nq)
    g = cases.gen(11)
    idx = torch.randint(-1, N, (B, H, N, K), generator=g).int()
    qd, kd, vd, idd = q.to(DEV), k.to(DEV), v.to(DEV), idx.to(DEV)
    full = topk_attention(qd, kd, vd, topk_indices=idd, causal=causal)
    part = topk_attention(qd[:, :, q0:q0 + nq].contiguous(), kd, vd,
                          topk_indices=idd[:, :, q0:q0 + nq].contiguous(), causal=causal, q_start=q0)
    assert torch.equal(part, full[:, :, q0:q0 + nq])


def test_rows_argument_checks():
    from ossa_b200._lib import OssaError

    q = torch.zeros(1, 2, 8, 128, device=DEV, dtype=torch.bfloat16)
    k = torch.zeros(1, 2, 16, 128, device=DEV, dtype=torch.bfloat16)
    idx = torch.zeros(1, 2, 8, 4, device=DEV, dtype=torch.int32)
    with pytest.raises(ValueError):
        topk_attention(q, k, k, topk_indices=idx, q_start=-1)
    with pytest.raises(ValueError):
        topk_attention(q, k, k, topk_indices=idx)  # row counts differ without q_start
    with pytest.raises(OssaError):
        topk_attention(q, k[:, :, :0], k[:, :, :0], topk_indices=idx, q_start=0)


@pytest.mark.parametrize("r,K", [(64, 64), (64, 128), (32, 100), (64, 160), (128, 16)])
@pytest.mark.parametrize("nq,where", [(1, "end"), (3, "end"), (1, "middle"), (2, "start")])
@pytest.mark.parametrize("causal", [True, False])
def test_decode_rows_split_selector(r, K, nq, where, causal):
    """Few query rows against a long key sequence (decode): the split selector
    (one warp per row and 1024-key range, then a merge over the ranges) gives
    exactly the oracle's rows and the CTA selector's."""
    import os

    B, H, Hkv, N, D, L = 2, 6, 2, 5000, 128, 4096
    q, k, _, wq, wk, pb = _inputs(B, H, Hkv, N, D, r, L, seed=r + K + nq)
    q0 = {"end": N - nq, "middle": 2047, "start": 0}[where]
    qd = q[:, :, q0:q0 + nq].contiguous().to(DEV)
    args = (k.to(DEV), wq.to(DEV), wk.to(DEV), pb.to(DEV), L, K)
    got = router_topk(qd, *args, causal=causal, q_start=q0)
    os.environ["OSSA_ROUTER_SELECT"] = "exact"
    try:
        cta = router_topk(qd, *args, causal=causal, q_start=q0)
    finally:
        del os.environ["OSSA_ROUTER_SELECT"]
    assert torch.equal(got, cta)
    rows = np.array([(bh * N + i) for bh in range(B * H) for i in range(q0, q0 + nq)])
    ref = oracle.router_topk_rows(q, k, wq, wk, pb, L, K, rows, causal=causal)
    np.testing.assert_array_equal(got.cpu().numpy().reshape(-1, K), ref)


def test_decode_split_selector_ties_across_ranges():
    """Equal keys on both sides of a 1024-key range boundary: the tie goes to the
    lower key index across ranges, as in the oracle."""
    B, H, Hkv, N, D, r, L, K = 1, 4, 1, 3000, 128, 64, 3000, 64
    q, k, _, wq, wk, pb = _inputs(B, H, Hkv, N, D, r, L, seed=3)
    pb = torch.zeros_like(pb)
    q0, nq = N - 2, 2
    # copies of the first row's best key, 81 equal scores straddling the boundary at 1024
    best = int(oracle.router_topk_rows(q, k, wq, wk, pb, L, 1, np.array([q0]))[0, 0])
    k[0, 0, 990:1070] = k[0, 0, best]
    got = router_topk(q[:, :, q0:].contiguous().to(DEV), k.to(DEV), wq.to(DEV), wk.to(DEV), pb.to(DEV), L, K,
                      q_start=q0)
    rows = np.array([(bh * N + i) for bh in range(B * H) for i in range(q0, q0 + nq)])
    ref = oracle.router_topk_rows(q, k, wq, wk, pb, L, K, rows)
    np.testing.assert_array_equal(got.cpu().numpy().reshape(-1, K), ref)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_router_key_cache_matches_router_topk(dtype):
    """Decoding with projected keys cached once per position gives the indices of
    router_topk on all keys so far, step after step (split selector for one new
    row; tensor-core selector for a 256-row prefill block)."""
    from ossa_b200 import ContentRouter, ContentRouterConfig
    from ossa_b200.decode import RouterKeyCache

    B, H, Hkv, N, D, r, L, K = 1, 12, 2, 2600, 128, 64, 4096, 64
    q, k, _, wq, wk, pb = _inputs(B, H, Hkv, N, D, r, L, seed=21)
    q, k = q.to(dtype).to(DEV), k.to(dtype).to(DEV)
    router = ContentRouter(ContentRouterConfig(head_dim=D, n_heads=H, seq_len=L, proj_dim=r))
    with torch.no_grad():
        router.q_proj[0].weight.copy_(wq)
        router.k_proj[0].weight.copy_(wk)
        router.pos_bias.weight.copy_(pb)
    router = router.to(DEV)
    args = (wq.to(DEV), wk.to(DEV), pb.to(DEV), L, K)
    cache = RouterKeyCache(router, B, Hkv, capacity=N)
    n0 = 2400
    cache.append(k[:, :, :n0 - 256])
    cache.append(k[:, :, n0 - 256:n0])
    blk = q[:, :, n0 - 256:n0].contiguous()
    assert torch.equal(cache.topk(blk, K), router_topk(blk, k[:, :, :n0].contiguous(), *args, q_start=n0 - 256))
    for pos in range(n0, N, 50):
        cache.append(k[:, :, cache.length:pos + 1])
        qn = q[:, :, pos:pos + 1].contiguous()
        got = cache.topk(qn, K)
        ref = router_topk(qn, k[:, :, :pos + 1].contiguous(), *args, q_start=pos)
        assert torch.equal(got, ref), f"position {pos}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("K", [64, 128])
def test_router_topk_projected_keys_match(dtype, K):
    """Keys projected once (project_router_keys) and two query blocks selected
    against them (router_topk_projected, what the sequence-sharded path does per
    rank) give exactly router_topk's rows; so does the whole sequence."""
    from ossa_b200.select import project_router_keys, router_topk_projected

    B, H, Hkv, N, D, r, L = 2, 12, 2, 1024, 128, 64, 1024
    q, k, _, wq, wk, pb = _inputs(B, H, Hkv, N, D, r, L, seed=71 + K)
    q, k = q.to(dtype).to(DEV), k.to(dtype).to(DEV)
    wq, wk, pb = wq.to(DEV), wk.to(DEV), pb.to(DEV)
    kp = project_router_keys(k, wk)
    assert kp.shape == (B, Hkv, N, r) and kp.dtype == torch.float32
    full = router_topk(q, k, wq, wk, pb, L, K)
    for q0, nq in ((0, 256), (256, 256), (768, 256)):
        blk = router_topk_projected(q[:, :, q0:q0 + nq].contiguous(), kp, wq, pb, L, K, q_start=q0)
        assert torch.equal(blk, full[:, :, q0:q0 + nq]), f"block at {q0}"
    assert torch.equal(router_topk_projected(q, kp, wq, pb, L, K), full)
