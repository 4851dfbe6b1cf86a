"""Pins the CPU oracle against the reference's own outputs (tests/golden).

The golden vectors were produced by running the reference implementation
(tests/golden/make_golden.py); here the oracle (oracle/ossa_oracle.c and
oracle/reference_port.py) must reproduce them.  These are CPU tests.
"""

import math

import numpy as np
import pytest
import torch

import cases
import oracle
from oracle import reference_port as rp


def _load(golden_dir, name):
    return np.load(golden_dir / name)


def test_checkpoint_router_c1_sets_and_logits(golden_dir):
    """The small single-layer workload (B=1, 12/2 heads, D=128, N=512, K=64, fp32) with the
    reference's trained layer-14 router: identical index sets on every row and
    bit-identical logits on the stored rows."""
    z = _load(golden_dir, "router_ckpt_c1.npz")
    q, k, v = cases.c1_inputs()
    assert np.array_equal(cases.checksum(q, k, v), z["checksum"]), "regenerated inputs differ"
    idx = oracle.router_topk(q, k, z["wq"], z["wk"], z["pos_bias"], int(z["seq_len"]), int(z["K"]))
    ref = z["ref_sets"].astype(np.int32)
    assert idx.shape == ref.shape
    assert np.array_equal(idx, ref), f"{(idx != ref).any(-1).sum()} rows differ"
    logits = oracle.router_scores(q, k, z["wq"], z["wk"], z["pos_bias"], int(z["seq_len"]))
    np.testing.assert_array_equal(logits[:, :, z["logit_rows"], :], z["ref_logits"])


def test_checkpoint_router_c1_score_order(golden_dir):
    """torch.topk's own order (descending score) on the same workload: the oracle's
    sets ordered by (score desc, key asc) equal the reference's top-64 indices
    element for element on every row's first min(64, i + 1) entries (the rest are
    masked future keys there and -1 here)."""
    z = _load(golden_dir, "router_ckpt_c1.npz")
    q, k, v = cases.c1_inputs()
    idx, sc = oracle.router_topk(q, k, z["wq"], z["wk"], z["pos_bias"], int(z["seq_len"]), int(z["K"]),
                                 with_scores=True)
    got = oracle.order_by_score(idx, sc)
    ref = z["ref_order"].astype(np.int32)
    N, K = got.shape[2], got.shape[3]
    prefix = np.arange(K)[None, :] < np.minimum(K, np.arange(N) + 1)[:, None]
    np.testing.assert_array_equal(np.where(prefix, got, -1), np.where(prefix, ref, -1))
    assert (got[..., ~prefix] == -1).all()


def test_checkpoint_router_c1_output(golden_dir):
    z = _load(golden_dir, "router_ckpt_c1.npz")
    q, k, v = cases.c1_inputs()
    idx = torch.from_numpy(z["ref_sets"].astype(np.int64))
    out = rp.masked_index_attention(q, k, v, idx)
    heads = list(z["out_heads"])
    np.testing.assert_allclose(out[:, heads].float().numpy(), z["ref_out"], atol=1e-5, rtol=1e-5)


def test_random_router_gqa_causal_and_full(golden_dir):
    """Random-init router, 6/3 heads, ragged N=200, r=32, seq_len 128 < N so the
    pos_bias clamp is exercised; causal selection and the unmasked
    ContentRouter.topk (router.py:202-203)."""
    z = _load(golden_dir, "router_random_gqa.npz")
    q, k, v = cases.gqa_small_inputs()
    D = q.shape[-1]
    r, L, K = int(z["r"]), int(z["seq_len"]), int(z["K"])
    wq, wk, pb = cases.router_weights(D, r, L, seed=int(z["weight_seed"]))
    assert np.array_equal(cases.checksum(q, k, v, wq, wk, pb), z["checksum"])
    idx = oracle.router_topk(q, k, wq, wk, pb, L, K, causal=True)
    assert np.array_equal(idx, z["ref_sets"].astype(np.int32))
    idx_full, sc_full = oracle.router_topk(q, k, wq, wk, pb, L, K, causal=False, with_scores=True)
    assert np.array_equal(idx_full, z["ref_full_sets"].astype(np.int32))
    # ContentRouter.topk's order: torch.topk(score, K).indices, element for element
    assert np.array_equal(oracle.order_by_score(idx_full, sc_full), z["ref_full_order"].astype(np.int32))
    logits = oracle.router_scores(q, k, wq, wk, pb, L)
    np.testing.assert_array_equal(logits[:, :, z["logit_rows"], :], z["ref_logits"])
    out = rp.masked_index_attention(q, k, v, torch.from_numpy(idx.astype(np.int64)))
    np.testing.assert_allclose(out.float().numpy(), z["ref_out"], atol=1e-5, rtol=1e-5)


def test_exact_dot_selector(golden_dir):
    """The oracle selector q.k/sqrt(D) (sparse_forward.py:194-196) in fp32."""
    z = _load(golden_dir, "oracle_select.npz")
    q, k, v = cases.oracle_inputs()
    assert np.array_equal(cases.checksum(q, k, v), z["checksum"])
    idx = oracle.oracle_topk(q, k, int(z["K"]))
    ref = z["ref_sets"].astype(np.int32)
    diff = (idx != ref).any(-1)
    # rows may only differ where the reference's own fp32 boundary gap is below
    # the BLAS-vs-fmaf rounding scale
    assert (z["ref_gap"][diff] < 1e-6).all(), z["ref_gap"][diff]
    assert diff.sum() <= 2
    out = rp.masked_index_attention(q, k, v, torch.from_numpy(ref.astype(np.int64)))
    heads = list(z["out_heads"])
    np.testing.assert_allclose(out[:, heads].float().numpy(), z["ref_out"], atol=1e-5, rtol=1e-5)


def test_reference_sparse_forward_known_answers(golden_dir):
    """The reference's own tests (tests/test_sparse_attention.py:12-71) restated
    on the port and compared with the reference's recorded outputs."""
    z = _load(golden_dir, "sparse_forward_ref.npz")
    q, k, v = cases.reference_test_inputs()
    assert np.array_equal(cases.checksum(q, k, v), z["checksum"])
    top = torch.from_numpy(z["topk"].astype(np.int64))
    full = rp.sparse_forward_full(q, k, v, top)
    chunk = rp.sparse_forward_chunked(q, k, v, top, chunk_size=16)
    np.testing.assert_allclose(full.numpy(), z["out_full"], atol=1e-5)
    np.testing.assert_allclose(chunk.numpy(), z["out_chunked"], atol=1e-5)
    B, H, N, D = q.shape
    all_idx = torch.arange(N).view(1, 1, 1, N).expand(B, H, N, N).contiguous()
    np.testing.assert_allclose(rp.sparse_forward_full(q, k, v, all_idx).numpy(), z["out_all_keys"], atol=1e-5)
    np.testing.assert_allclose(rp.dense_attention(q, k, v).numpy(), z["out_dense"], atol=1e-5)
    np.testing.assert_allclose(z["out_all_keys"], z["out_dense"], atol=1e-5)  # K = N equals dense


def test_masked_index_oracle_matches_chunked_port():
    torch.manual_seed(0)
    B, H, N, D, K = 1, 4, 64, 16, 16
    q, k, v = (torch.randn(B, H, N, D) for _ in range(3))
    s = (q @ k.transpose(-2, -1)).masked_fill(torch.triu(torch.ones(N, N, dtype=torch.bool), 1), float("-inf"))
    top = s.topk(K, dim=-1).indices
    a = rp.sparse_forward_chunked(q, k, v, top, chunk_size=16)
    # -1-padded ascending sets restricted to j <= i describe the same attention
    pos = torch.arange(N).view(1, 1, N, 1)
    sets = torch.sort(top.masked_fill(top > pos, 10 ** 9), dim=-1).values
    sets = sets.masked_fill(sets == 10 ** 9, -1)
    b = rp.masked_index_attention(q, k, v, sets)
    np.testing.assert_allclose(a.numpy(), b.float().numpy(), atol=1e-5)


def test_oracle_topk_ties_and_padding():
    """Total order: equal scores resolve to the lower key index; rows with fewer
    than K eligible keys are -1 padded; NaN ranks above every number."""
    B, H, N, D = 1, 1, 10, 4
    q = torch.zeros(B, H, N, D)
    k = torch.zeros(B, H, N, D)
    idx = oracle.oracle_topk(q, k, 3)  # all scores 0: lowest indices win
    for i in range(N):
        exp = list(range(min(3, i + 1))) + [-1] * (3 - min(3, i + 1))
        assert list(idx[0, 0, i]) == exp
    k2 = k.clone()
    k2[0, 0, 5, 0] = float("nan")
    q2 = torch.ones(B, H, N, D)
    idx2 = oracle.oracle_topk(q2, k2, 1)
    assert idx2[0, 0, 9, 0] == 5 and idx2[0, 0, 4, 0] == 0


def test_oracle_topk_matches_torch_topk_random():
    """Sets equal torch.topk's on continuous random scores (no ties)."""
    torch.manual_seed(3)
    B, H, Hkv, N, D, K = 2, 4, 2, 96, 32, 8
    q = torch.randn(B, H, N, D)
    k = torch.randn(B, Hkv, N, D)
    idx = oracle.oracle_topk(q, k, K, causal=False)
    kr = k.repeat_interleave(2, dim=1)
    s = torch.matmul(q, kr.transpose(-2, -1)) / math.sqrt(D)
    ref = torch.sort(s.topk(K, dim=-1).indices, dim=-1).values.numpy()
    assert np.array_equal(idx, ref.astype(np.int32))


@pytest.mark.parametrize("causal", [True, False])
def test_oracle_topk_rows_matches_full_selection(causal):
    """The row-subset oracle selector (used for full-size spot checks) returns
    exactly the full selection's rows."""
    q, k, _ = cases.qkv(1, 4, 2, 200, 128, seed=3, scale=1.0 / math.sqrt(128))
    full = oracle.oracle_topk(q, k, 16, causal=causal).reshape(-1, 16)
    rows = np.arange(0, 800, 7, dtype=np.int64)
    assert (oracle.oracle_topk_rows(q, k, 16, rows, causal=causal) == full[rows]).all()


def test_router_distillation_restatement(golden_dir):
    """The training loss (ossa/router.py:80-99 on router.py:171-190), restated in
    fp64 with the target given as index lists: equal to the reference's own loss
    and gradients (fp32) on its own target indices (torch.topk of the dense
    attention, masked ties included)."""
    z = _load(golden_dir, "router_distill.npz")
    q, k, _ = cases.distill_inputs()
    D = q.shape[-1]
    r, L = int(z["r"]), int(z["seq_len"])
    wq, wk, pb = cases.router_weights(D, r, L, seed=int(z["weight_seed"]))
    assert np.array_equal(cases.checksum(q, k, wq, wk, pb), z["checksum"])
    loss, dwq, dwk, dpb = rp.router_distillation(q, k, wq, wk, pb, L, torch.from_numpy(z["target_idx"].astype(np.int64)))
    np.testing.assert_allclose(float(loss), float(z["loss"]), rtol=1e-6)
    for got, ref in ((dwq, z["dwq"]), (dwk, z["dwk"]), (dpb, z["dpos_bias"])):
        np.testing.assert_allclose(got.numpy(), ref, rtol=1e-4, atol=1e-7 * np.abs(ref).max())

