"""Bit-exact parity of the fused selection kernels against the CPU oracle.

ossa_router_topk / ossa_oracle_topk must return exactly the oracle's index
arrays (same sets, ascending order, -1 padding); ossa_router_score must return
exactly the oracle's fp32 logits.
"""

import math

import numpy as np
import pytest
import torch

import cases
import oracle
from ossa_b200 import ContentRouter, ContentRouterConfig, oracle_topk, router_scores, router_topk
from ossa_b200.select import router_topk_with_status

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _weights(D, r, L, seed, bias_scale=1.0):
    wq, wk, pb = cases.router_weights(D, r, L, seed)
    return wq, wk, pb * bias_scale


def _assert_same(got: torch.Tensor, ref: np.ndarray):
    g = got.cpu().numpy()
    assert g.shape == ref.shape
    bad = (g != ref).any(-1)
    assert not bad.any(), f"{bad.sum()} rows differ; first at {np.argwhere(bad)[0]}"


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B,H,Hkv,N,D,r,L,K", [
    (1, 12, 2, 512, 128, 64, 512, 64),     # the small single-layer shape
    (2, 6, 3, 200, 64, 32, 128, 16),       # ragged, clamped pos_bias
    (1, 4, 1, 1, 128, 64, 16, 8),          # single row
    (1, 2, 2, 65, 64, 16, 64, 64),         # K == N - 1
    (1, 4, 2, 300, 128, 128, 300, 100),    # K not a multiple of 32
    (1, 2, 1, 97, 32, 64, 40, 160),        # K > N: padded rows everywhere
    (2, 12, 2, 1000, 128, 64, 1000, 128),  # the long-context K
])
@pytest.mark.parametrize("causal", [True, False])
def test_router_topk_bit_exact(dtype, B, H, Hkv, N, D, r, L, K, causal):
    seed = B + H + N + D + r + K
    q, k, _ = cases.qkv(B, H, Hkv, N, D, seed=seed, scale=1.0 / math.sqrt(D))
    q, k = q.to(dtype), k.to(dtype)
    wq, wk, pb = _weights(D, r, L, seed)
    got = router_topk(q.to(DEV), k.to(DEV), wq.to(DEV), wk.to(DEV), pb.to(DEV), L, K, causal=causal)
    ref = oracle.router_topk(q, k, wq, wk, pb, L, K, causal=causal)
    _assert_same(got, ref)


@pytest.mark.parametrize("N,r", [(77, 64), (256, 32), (130, 128)])
def test_router_scores_bit_exact(N, r):
    B, H, Hkv, D, L = 2, 6, 2, 128, 96
    q, k, _ = cases.qkv(B, H, Hkv, N, D, seed=N + r)
    wq, wk, pb = _weights(D, r, L, seed=r)
    got = router_scores(q.to(DEV), k.to(DEV), wq.to(DEV), wk.to(DEV), pb.to(DEV), L)
    ref = oracle.router_scores(q, k, wq, wk, pb, L)
    np.testing.assert_array_equal(got.cpu().numpy(), ref)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("D,r", [(20, 64), (40, 16), (256, 64), (136, 32)])
def test_router_scores_head_dims(dtype, D, r):
    """Projection paths: D a multiple of the 16-byte vector and <= 128 (persistent
    kernel), and D that is not, or is > 128 (chunked kernel)."""
    B, H, Hkv, N, L = 1, 4, 2, 150, 80
    q, k, _ = cases.qkv(B, H, Hkv, N, D, seed=D + r)
    q, k = q.to(dtype), k.to(dtype)
    wq, wk, pb = _weights(D, r, L, seed=D)
    got = router_scores(q.to(DEV), k.to(DEV), wq.to(DEV), wk.to(DEV), pb.to(DEV), L)
    ref = oracle.router_scores(q, k, wq, wk, pb, L)
    np.testing.assert_array_equal(got.cpu().numpy(), ref)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B,H,Hkv,N,D,K", [
    (1, 4, 2, 256, 128, 32),
    (1, 12, 2, 700, 128, 128),
    (2, 2, 1, 50, 64, 8),
])
def test_oracle_topk_bit_exact(dtype, B, H, Hkv, N, D, K):
    q, k, _ = cases.qkv(B, H, Hkv, N, D, seed=N + K, scale=1.0 / math.sqrt(D))
    q, k = q.to(dtype), k.to(dtype)
    got = oracle_topk(q.to(DEV), k.to(DEV), K)
    ref = oracle.oracle_topk(q, k, K)
    _assert_same(got, ref)


def test_checkpoint_router_matches_reference(golden_dir):
    """The small single-layer workload (N=512) with the reference's trained router: the GPU selection equals the
    reference's own causal top-64 sets on all 6144 rows."""
    z = np.load(golden_dir / "router_ckpt_c1.npz")
    q, k, _ = cases.c1_inputs()
    router = ContentRouter(ContentRouterConfig(head_dim=128, n_heads=12, seq_len=512, proj_dim=64))
    router.load_state_dict({"q_proj.0.weight": torch.from_numpy(z["wq"]),
                            "k_proj.0.weight": torch.from_numpy(z["wk"]),
                            "pos_bias.weight": torch.from_numpy(z["pos_bias"])})
    router = router.to(DEV)
    got = router.topk(q.to(DEV), k.to(DEV), 64, causal=True, index_dtype=torch.int32, order="index")
    _assert_same(got, z["ref_sets"].astype(np.int32))
    logits = router.score(q.to(DEV), k.to(DEV))
    np.testing.assert_array_equal(logits[:, :, z["logit_rows"]].cpu().numpy(), z["ref_logits"])
    # torch.topk's order (descending score): row i's first min(64, i + 1) entries are
    # the reference's, element for element; the rest are -1 here and masked keys there
    ordered = router.topk(q.to(DEV), k.to(DEV), 64, causal=True).cpu().numpy()
    ref = z["ref_order"].astype(np.int64)
    n_valid = np.minimum(64, np.arange(512) + 1)
    lane = np.arange(64)
    prefix = lane[None, :] < n_valid[:, None]                 # (N, 64)
    np.testing.assert_array_equal(np.where(prefix, ordered, -1), np.where(prefix, ref, -1))
    assert (ordered[..., ~prefix] == -1).all()


def test_random_router_matches_reference_unmasked(golden_dir):
    """ContentRouter.topk without a causal mask (router.py:202-203) on the ragged
    GQA golden case: same sets as the reference's torch.topk."""
    z = np.load(golden_dir / "router_random_gqa.npz")
    q, k, _ = cases.gqa_small_inputs()
    D = q.shape[-1]
    r, L, K = int(z["r"]), int(z["seq_len"]), int(z["K"])
    wq, wk, pb = cases.router_weights(D, r, L, seed=int(z["weight_seed"]))
    router = ContentRouter(ContentRouterConfig(head_dim=D, n_heads=6, seq_len=L, proj_dim=r))
    with torch.no_grad():
        router.q_proj[0].weight.copy_(wq)
        router.k_proj[0].weight.copy_(wk)
        router.pos_bias.weight.copy_(pb)
    router = router.to(DEV)
    full = router.topk(q.to(DEV), k.to(DEV), K)
    assert full.dtype == torch.int64
    # element for element: the reference's torch.topk(score, K).indices order
    np.testing.assert_array_equal(full.cpu().numpy(), z["ref_full_order"].astype(np.int64))
    full_sets = router.topk(q.to(DEV), k.to(DEV), K, order="index")
    _assert_same(full_sets.int(), z["ref_full_sets"].astype(np.int32))
    causal = router.topk(q.to(DEV), k.to(DEV), K, causal=True, order="index")
    _assert_same(causal.int(), z["ref_sets"].astype(np.int32))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B,H,Hkv,N,D,r,L,K,causal", [
    (1, 12, 2, 512, 128, 64, 512, 64, True),     # the small single-layer shape
    (2, 4, 2, 300, 128, 64, 256, 128, False),    # unmasked, wide K
    (1, 6, 3, 200, 64, 32, 128, 16, True),       # ragged, clamped pos_bias
])
def test_router_topk_score_order(dtype, B, H, Hkv, N, D, r, L, K, causal):
    """ContentRouter.topk's default order (torch.topk's): every row element for
    element equal to the oracle's sets ordered by (score desc, key asc)."""
    q, k, _ = cases.qkv(B, H, Hkv, N, D, seed=7 * N + K, scale=1.0 / math.sqrt(D))
    q, k = q.to(dtype), k.to(dtype)
    wq, wk, pb = _weights(D, r, L, seed=K)
    router = ContentRouter(ContentRouterConfig(head_dim=D, n_heads=H, seq_len=L, proj_dim=r))
    with torch.no_grad():
        router.q_proj[0].weight.copy_(wq)
        router.k_proj[0].weight.copy_(wk)
        router.pos_bias.weight.copy_(pb)
    router = router.to(DEV)
    got = router.topk(q.to(DEV), k.to(DEV), K, causal=causal, index_dtype=torch.int32)
    idx, sc = oracle.router_topk(q, k, wq, wk, pb, L, K, causal=causal, with_scores=True)
    _assert_same(got, oracle.order_by_score(idx, sc))


def test_all_ties_pick_lowest_indices():
    """Zero router weights and a constant bias: every score ties, so each row keeps
    its K lowest eligible keys."""
    B, H, Hkv, N, D, r, L, K = 1, 2, 1, 150, 64, 64, 150, 32
    q = torch.randn(B, H, N, D)
    k = torch.randn(B, Hkv, N, D)
    wq = torch.zeros(r, D)
    wk = torch.zeros(r, D)
    pb = torch.full((2 * L, 1), 0.5)
    got = router_topk(q.to(DEV), k.to(DEV), wq.to(DEV), wk.to(DEV), pb.to(DEV), L, K).cpu()
    for i in (0, 1, 31, 32, 149):
        m = min(K, i + 1)
        assert got[0, 0, i].tolist() == list(range(m)) + [-1] * (K - m)
    _assert_same(got, oracle.router_topk(q, k, wq, wk, pb, L, K))


def test_bias_only_ties_many_duplicates():
    """q = 0: scores are the pos_bias table, which repeats 4 values, so ties at
    the K-th boundary are everywhere; the tie-break must follow key order."""
    B, H, Hkv, N, D, r, L, K = 1, 3, 1, 400, 64, 32, 400, 64
    q = torch.zeros(B, H, N, D)
    k = torch.randn(B, Hkv, N, D)
    wq, wk, _ = _weights(D, r, L, seed=9)
    pb = (torch.arange(2 * L) % 4).float().view(-1, 1)
    got = router_topk(q.to(DEV), k.to(DEV), wq.to(DEV), wk.to(DEV), pb.to(DEV), L, K)
    _assert_same(got, oracle.router_topk(q, k, wq, wk, pb, L, K))


def test_nan_scores_rank_first():
    B, H, Hkv, N, D, K = 1, 1, 1, 64, 64, 4
    q = torch.randn(B, H, N, D)
    k = torch.randn(B, Hkv, N, D)
    k[0, 0, 10, 3] = float("nan")
    got = oracle_topk(q.to(DEV), k.to(DEV), K)
    ref = oracle.oracle_topk(q, k, K)
    _assert_same(got, ref)
    assert (got[0, 0, 10:] == 10).any(-1).all()


def test_full_size_config2_selection():
    """The single-layer bf16 workload (B=8, 12/2 heads, D=128, N=4096, K=64, random router):
    structural properties on every row and exact oracle agreement on a sample of
    rows from every (b, h)."""
    B, H, Hkv, N, D, r, K = 8, 12, 2, 4096, 128, 64, 64
    q, k, _ = cases.qkv(B, H, Hkv, N, D, seed=4096, scale=1.0 / math.sqrt(D))
    q, k = q.bfloat16(), k.bfloat16()
    wq, wk, pb = _weights(D, r, N, seed=3)
    got, fb, status = router_topk_with_status(q.to(DEV), k.to(DEV), wq.to(DEV), wk.to(DEV), pb.to(DEV), N, K)
    assert status == 0
    pos = torch.arange(N, device=DEV).view(1, 1, N, 1)
    valid = got >= 0
    assert torch.equal(valid.sum(-1), torch.clamp(torch.arange(N, device=DEV) + 1, max=K).expand(B, H, N))
    assert bool((got <= pos).all())
    big = torch.where(valid, got, torch.full_like(got, 1 << 30))
    asc = (big[..., 1:] > big[..., :-1]) | ~valid[..., 1:]
    assert bool(asc.all()), "valid indices must be strictly ascending, padding last"
    gen = np.random.default_rng(0)
    rows = []
    for bh in range(B * H):
        rows += list(bh * N + np.concatenate([[0, 62, 63, 64, N - 1], gen.integers(0, N, 3)]))
    rows = np.array(rows, dtype=np.int64)
    ref = oracle.router_topk_rows(q, k, wq, wk, pb, N, K, rows)
    _assert_same(got.reshape(-1, K)[torch.from_numpy(rows).to(DEV)], ref)


def _run_both(q, k, wq, wk, pb, L, K, causal=True):
    """Tensor-core selector (default for r = 64, K <= 128) and, forced through
    OSSA_ROUTER_SELECT=exact, the CUDA-core exact selector on the same inputs."""
    import os

    args = (q.to(DEV), k.to(DEV), wq.to(DEV), wk.to(DEV), pb.to(DEV), L, K)
    tc, fb, status = router_topk_with_status(*args, causal=causal)
    os.environ["OSSA_ROUTER_SELECT"] = "exact"
    try:
        ex = router_topk(*args, causal=causal)
    finally:
        del os.environ["OSSA_ROUTER_SELECT"]
    return tc, ex, fb, status


@pytest.mark.parametrize("N,K,causal", [
    (2048, 64, True), (777, 32, True), (640, 64, False), (300, 48, True), (4096, 16, True),
    # wide selection (64 < K <= 128): 256 column classes, global candidate lists
    (2048, 128, True), (777, 100, True), (640, 128, False), (4096, 96, True), (1500, 65, True),
])
def test_tensor_core_and_exact_selectors_agree(N, K, causal):
    B, H, Hkv, D, r = 2, 12, 2, 128, 64
    q, k, _ = cases.qkv(B, H, Hkv, N, D, seed=N + K, scale=1.0 / math.sqrt(D))
    q, k = q.bfloat16(), k.bfloat16()
    wq, wk, pb = _weights(D, r, N, seed=K)
    tc, ex, fb, status = _run_both(q, k, wq, wk, pb, N, K, causal)
    assert status == 0
    assert torch.equal(tc, ex), f"{(tc != ex).any(-1).sum().item()} rows differ"
    rows = np.arange(0, B * H * N, 97, dtype=np.int64)
    ref = oracle.router_topk_rows(q, k, wq, wk, pb, N, K, rows, causal=causal)
    _assert_same(tc.reshape(-1, K)[torch.from_numpy(rows).to(DEV)], ref)


@pytest.mark.parametrize("K", [64, 128])
def test_tensor_core_selector_content_dominated_scores(K):
    """Trained-router-like regime: content scores dominate the position bias, so
    the boundary band is decided by the q'.k' products the tensor cores compute."""
    B, H, Hkv, N, D, r = 1, 12, 2, 1024, 128, 64
    q, k, _ = cases.qkv(B, H, Hkv, N, D, seed=77)
    wq, wk, pb = _weights(D, r, N, seed=8, bias_scale=0.01)
    wq, wk = wq * 4, wk * 4
    tc, fb, status = router_topk_with_status(q.to(DEV), k.to(DEV), wq.to(DEV), wk.to(DEV), pb.to(DEV), N, K)
    assert status == 0
    _assert_same(tc, oracle.router_topk(q, k, wq, wk, pb, N, K))


@pytest.mark.parametrize("N,K", [(256, 64), (512, 128)])
def test_tensor_core_selector_ties_go_to_exact_fallback(N, K):
    """All scores tie: every row's candidate list overflows and is recomputed by
    the exact warp-per-row selector; the result is still the lowest indices."""
    B, H, Hkv, D, r, L = 1, 4, 2, 64, 64, 256
    q = torch.randn(B, H, N, D)
    k = torch.randn(B, Hkv, N, D)
    wq = torch.zeros(r, D)
    wk = torch.zeros(r, D)
    pb = torch.full((2 * L, 1), 0.25)
    got, fb, status = router_topk_with_status(q.to(DEV), k.to(DEV), wq.to(DEV), wk.to(DEV), pb.to(DEV), L, K)
    assert status == 0 and fb > 0
    _assert_same(got, oracle.router_topk(q, k, wq, wk, pb, L, K))


@pytest.mark.parametrize("K", [64, 128])
def test_long_rows_exact_fallback_split(K):
    """Rows of 8192 keys or more that go to the exact selector are split over the 8
    warps of a CTA and merged: with every score tied, each row still lists its
    lowest K key indices (all but the first few hundred rows of a head take that
    path: shorter rows fit their candidate lists)."""
    B, H, Hkv, N, D, r = 1, 2, 1, 8192, 64, 64
    q = torch.randn(B, H, N, D)
    k = torch.randn(B, Hkv, N, D)
    wq = torch.zeros(r, D)
    wk = torch.zeros(r, D)
    pb = torch.full((2 * N, 1), 0.25)
    got, fb, status = router_topk_with_status(q.to(DEV), k.to(DEV), wq.to(DEV), wk.to(DEV), pb.to(DEV), N, K)
    assert status == 0 and fb >= B * H * (N - 640)
    i = torch.arange(N).view(N, 1)
    j = torch.arange(K).view(1, K)
    expect = torch.where(j <= i, j, torch.full_like(j, -1)).to(torch.int32)
    assert torch.equal(got.cpu(), expect.expand(B, H, N, K))
    rows = np.array([0, K - 1, K, 5000, N - 1, 2 * N - 1], dtype=np.int64)
    _assert_same(got.reshape(-1, K)[torch.from_numpy(rows).to(DEV)],
                 oracle.router_topk_rows(q, k, wq, wk, pb, N, K, rows, causal=True))


@pytest.mark.parametrize("K", [16, 128])
def test_tensor_core_selector_non_finite_rows(K):
    """A key with an infinite component makes every score of that (b, kv head)
    non-finite: those rows go to the exact selector, which ranks NaN first as
    torch.topk does."""
    B, H, Hkv, N, D, r = 1, 4, 2, 200, 64, 64
    q, k, _ = cases.qkv(B, H, Hkv, N, D, seed=5)
    k[0, 1, 50, 7] = float("inf")
    wq, wk, pb = _weights(D, r, N, seed=6)
    got, fb, status = router_topk_with_status(q.to(DEV), k.to(DEV), wq.to(DEV), wk.to(DEV), pb.to(DEV), N, K)
    assert status == 0 and fb >= 2 * N
    _assert_same(got, oracle.router_topk(q, k, wq, wk, pb, N, K))


def test_long_context_tensor_core_selector():
    """Long sequence (N = 16384, the tensor-core selector with 128 key tiles per
    query block at the end): identical to the exact selector, sampled rows to the
    oracle."""
    B, H, Hkv, N, D, r, K = 1, 4, 2, 16384, 128, 64, 64
    q, k, _ = cases.qkv(B, H, Hkv, N, D, seed=16, scale=1.0 / math.sqrt(D))
    q, k = q.bfloat16(), k.bfloat16()
    wq, wk, pb = _weights(D, r, N, seed=16)
    tc, ex, fb, status = _run_both(q, k, wq, wk, pb, N, K, True)
    assert status == 0
    assert torch.equal(tc, ex), f"{(tc != ex).any(-1).sum().item()} rows differ"
    rows = np.concatenate([np.arange(0, B * H * N, 4099), np.array([N - 1, 2 * N - 1, B * H * N - 1])]).astype(np.int64)
    ref = oracle.router_topk_rows(q, k, wq, wk, pb, N, K, rows, causal=True)
    _assert_same(tc.reshape(-1, K)[torch.from_numpy(rows).to(DEV)], ref)


def test_long_context_k128_selectors():
    """Long-context shape at its smallest length (N = 32768, K = 128): the wide
    tensor-core selection equals the exact CUDA-core selector on every row, and
    sampled rows equal the oracle."""
    B, H, Hkv, N, D, r, K = 1, 2, 1, 32768, 128, 64, 128
    q, k, _ = cases.qkv(B, H, Hkv, N, D, seed=32, scale=1.0 / math.sqrt(D))
    q, k = q.bfloat16(), k.bfloat16()
    wq, wk, pb = _weights(D, r, N, seed=32)
    tc, ex, fb, status = _run_both(q, k, wq, wk, pb, N, K, True)
    assert status == 0
    assert torch.equal(tc, ex), f"{(tc != ex).any(-1).sum().item()} rows differ"
    rows = np.array([0, 1, 127, 128, 4096, 20000, N - 1, N, 2 * N - 1], dtype=np.int64)
    ref = oracle.router_topk_rows(q, k, wq, wk, pb, N, K, rows, causal=True)
    _assert_same(tc.reshape(-1, K)[torch.from_numpy(rows).to(DEV)], ref)


@pytest.mark.parametrize("K", [64, 128])
def test_tensor_core_selector_wide_error_band(K):
    """Model-like magnitudes (q, k entries of unit scale, Xavier router weights:
    |q'|, |k'| around 7 to 10): the rigorous fp16 error bound then spans a dozen
    or more candidates at the K-th boundary.  They are decided by canonical
    rescoring of the candidates, not by the full-row exact fallback, and the
    result equals the exact selector and the oracle."""
    B, H, Hkv, N, D, r = 1, 12, 2, 2048, 128, 64
    q, k, _ = cases.qkv(B, H, Hkv, N, D, seed=40 + K, scale=0.6)
    q, k = q.bfloat16(), k.bfloat16()
    wq, wk, pb = _weights(D, r, N, seed=41 + K)
    tc, ex, fb, status = _run_both(q, k, wq, wk, pb, N, K, True)
    assert status == 0
    assert torch.equal(tc, ex), f"{(tc != ex).any(-1).sum().item()} rows differ"
    assert fb < 0.01 * B * H * N, f"{fb} rows fell back to the full-row exact selector"
    rows = np.concatenate([np.arange(0, B * H * N, 1021), np.array([N - 1, B * H * N - 1])]).astype(np.int64)
    ref = oracle.router_topk_rows(q, k, wq, wk, pb, N, K, rows, causal=True)
    _assert_same(tc.reshape(-1, K)[torch.from_numpy(rows).to(DEV)], ref)


@pytest.mark.parametrize("K", [64, 128])
@pytest.mark.parametrize("qscale,bias_scale", [
    (1.0 / math.sqrt(128), 1.0),  # position bias dominates: many half tiles are skipped
    (0.6, 1.0),                   # model-like content magnitudes: the content bound is loose
    (1.0 / math.sqrt(128), 0.0),  # no bias at all: only the content bound
])
def test_tensor_core_selector_half_tile_skip(K, qscale, bias_scale):
    """Query blocks with 40 or more key tiles skip, in pass 2, the half tiles whose
    score bound (content bound of the row + largest bias term of the half tile) is
    below the row's candidate threshold for every row of a warp.  N = 6144 puts the
    last nine query blocks of each head on that path; every row must equal the exact
    CUDA-core selector, whatever dominates the scores."""
    B, H, Hkv, N, D, r = 1, 6, 2, 6144, 128, 64
    q, k, _ = cases.qkv(B, H, Hkv, N, D, seed=60 + K, scale=qscale)
    q, k = q.bfloat16(), k.bfloat16()
    wq, wk, pb = _weights(D, r, N, seed=61 + K, bias_scale=bias_scale)
    tc, ex, fb, status = _run_both(q, k, wq, wk, pb, N, K, True)
    assert status == 0
    assert torch.equal(tc, ex), f"{(tc != ex).any(-1).sum().item()} rows differ"
    rows = np.array([0, 5000, N - 1, 3 * N - 1, B * H * N - 1], dtype=np.int64)
    ref = oracle.router_topk_rows(q, k, wq, wk, pb, N, K, rows, causal=True)
    _assert_same(tc.reshape(-1, K)[torch.from_numpy(rows).to(DEV)], ref)


@pytest.mark.parametrize("K,causal", [(128, True), (128, False), (64, True)])
def test_tensor_core_selector_repeated_calls_identical(K, causal):
    """Hundreds of back-to-back calls on the same inputs return the same indices
    as the exact selector every time: the tensor-core kernel's accumulator and
    window buffers are reused every four key tiles, and an early release of a
    buffer shows up as an occasional wrong row under repetition."""
    B, H, Hkv, N, D, r = 2, 12, 2, 1000, 128, 64
    q, k, _ = cases.qkv(B, H, Hkv, N, D, seed=1334, scale=1.0 / math.sqrt(D))
    q, k = q.bfloat16(), k.bfloat16()
    wq, wk, pb = _weights(D, r, N, seed=1334)
    tc, ex, fb, status = _run_both(q, k, wq, wk, pb, N, K, causal)
    assert status == 0 and torch.equal(tc, ex)
    args = (q.to(DEV), k.to(DEV), wq.to(DEV), wk.to(DEV), pb.to(DEV), N, K)
    bad = 0
    for _ in range(400):
        bad += int(not torch.equal(router_topk(*args, causal=causal), ex))
    assert bad == 0, f"{bad} of 400 calls differ"


def _both_projections(q, k, wq, wk, pb, L, K, causal=True):
    """router_topk with the query operand made from q on the tensor cores (canonical
    q' rows computed only where the selection needs them), and with every q' row
    projected canonically first (OSSA_QPROJ=canonical)."""
    import os
    args = (q.to(DEV), k.to(DEV), wq.to(DEV), wk.to(DEV), pb.to(DEV), L, K)
    lazy, fb, status = router_topk_with_status(*args, causal=causal)
    os.environ["OSSA_QPROJ"] = "canonical"
    try:
        canon = router_topk(*args, causal=causal)
    finally:
        del os.environ["OSSA_QPROJ"]
    return lazy, canon, fb, status


@pytest.mark.parametrize("case", ["ties", "nonfinite_query", "large_rows", "rows_block"])
@pytest.mark.parametrize("K", [64, 128])
def test_tensor_core_query_operand_on_demand_rows(case, K):
    """bf16 q, head_dim 128, proj_dim 64: the selector's fp16 query operand comes
    from a tensor-core projection of q, and the canonical fp32 q' (fmaf chain) is
    computed only for the rows that rescore their boundary band or go to the exact
    selector.  Rows on both of those paths give the indices of the canonical
    projection and of the oracle: all-tied scores (every row to the exact
    selector), a query row with an infinite entry, rows of large magnitude (wide
    error bands), and a block of query rows at an offset."""
    B, H, Hkv, N, D, r = 1, 12, 2, 768, 128, 64
    q, k, _ = cases.qkv(B, H, Hkv, N, D, seed=90 + K, scale=1.0 / math.sqrt(D))
    wq, wk, pb = _weights(D, r, N, seed=91 + K)
    q0 = 0
    if case == "ties":
        wk = torch.zeros_like(wk)
        pb = torch.full_like(pb, 0.25)
    elif case == "nonfinite_query":
        q[0, 3, 400, 17] = float("inf")
        q[0, 7, 10, 0] = float("-inf")
    elif case == "large_rows":
        q[0, :4] *= 40.0
    q, k = q.bfloat16(), k.bfloat16()
    if case == "rows_block":
        q0 = 256
        qb = q[:, :, q0:q0 + 384].contiguous()
        args = (qb.to(DEV), k.to(DEV), wq.to(DEV), wk.to(DEV), pb.to(DEV), N, K)
        lazy = router_topk(*args, q_start=q0)
        import os
        os.environ["OSSA_QPROJ"] = "canonical"
        try:
            canon = router_topk(*args, q_start=q0)
        finally:
            del os.environ["OSSA_QPROJ"]
        assert torch.equal(lazy, canon), f"{(lazy != canon).any(-1).sum().item()} rows differ"
        rows = np.array([0, 1, 200, 383, 384, 3 * 384 - 1, 12 * 384 - 1], dtype=np.int64)
        full = oracle.router_topk_rows(q, k, wq, wk, pb, N, K,
                                       (rows // 384) * N + q0 + rows % 384, causal=True)
        _assert_same(lazy.reshape(-1, K)[torch.from_numpy(rows).to(DEV)], full)
        return
    lazy, canon, fb, status = _both_projections(q, k, wq, wk, pb, N, K)
    assert status == 0
    assert torch.equal(lazy, canon), f"{(lazy != canon).any(-1).sum().item()} rows differ"
    if case == "ties":
        assert fb > 0
        _assert_same(lazy, oracle.router_topk(q, k, wq, wk, pb, N, K))
    else:
        rows = np.concatenate([np.arange(0, B * H * N, 97),
                               np.array([3 * N + 400, 7 * N + 10, 7 * N + 11, N - 1])]).astype(np.int64)
        ref = oracle.router_topk_rows(q, k, wq, wk, pb, N, K, rows, causal=True)
        _assert_same(lazy.reshape(-1, K)[torch.from_numpy(rows).to(DEV)], ref)
