"""Parity at the full sizes of the single-GPU workloads.

* Oracle top-K attention: exact q.k/sqrt(D) selection (ossa/bench/sparse_forward.py:194-202)
  at B=4, 12/2 heads, head_dim 128, N=8192, K in {32, 128}, bf16, unit-normal q/k plus a
  shared rank-8 component.  The tensor-core selection equals the CUDA-core exact selector
  on every row and the CPU oracle on 1,100+ sampled rows (every head's last row among
  them); the gather over those indices matches the fp64 attention oracle on sampled rows.
* Long context: router selection (ossa/router.py:171-190 + causal top-K) at B=1, 12/2
  heads, N in {65536, 131072}, K=128: sampled rows, including the last row of every head,
  equal the CPU oracle; the gather on sampled rows matches the fp64 attention oracle.
* The single-layer bf16 workload's gather (B=8, N=4096, K=64): 64 rows of every batch
  element against the fp64 attention oracle.
* The full model's patched attention (ossa/bench/sparse_forward.py:166-225) at the
  Qwen2.5-1.5B layer shape (hidden 1536, 12/2 heads, head_dim 128), bf16, N=4096, K=64,
  inside a Qwen2 decoder layer: the layer's own selected keys equal the CPU oracle on
  sampled rows and its attention output (the input of o_proj) matches the fp64
  attention oracle on them.

Indices must be equal; attention outputs within 2e-3 abs/rel (bf16) of the fp64
oracle, plus half a bf16 ulp of the oracle's value: the output is itself a bf16
number, so at unit-scale values (the oracle workload's V is unit-normal) its own
rounding is already about 2e-3.
"""

import math
import os

import numpy as np
import pytest
import torch

import oracle
from oracle import reference_port as rp
from ossa_b200 import oracle_topk, router_topk, topk_attention
from ossa_b200.bench.long_context import make_inputs as long_inputs
from ossa_b200.bench.oracle_select import make_inputs as oracle_inputs
from ossa_b200.select import oracle_topk_with_status, router_topk_with_status

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TOL = dict(atol=2e-3, rtol=2e-3)


def _sample_rows(B, H, N, n_random, seed):
    """Flat row ids (b*H + h)*N + i: n_random random rows plus rows 0, K-edge rows and
    the last row of every (b, h)."""
    rng = np.random.default_rng(seed)
    rnd = rng.integers(0, B * H * N, size=n_random)
    edges = [(bh * N + i) for bh in range(B * H) for i in (0, 31, 127, 128, N - 1)]
    return np.unique(np.concatenate([rnd, np.array(edges)])).astype(np.int64)


def _check_gather_rows(out, q, k, v, idx, rows, H, N):
    """Attention output rows (flat ids) against the fp64 oracle, one (b, h) at a time
    with that head's own kv head (no repeated K/V on the host)."""
    Hkv = k.shape[1]
    G = H // Hkv
    bh = rows // N
    for key in np.unique(bh):
        b, h = divmod(int(key), H)
        pos = torch.from_numpy(rows[bh == key] % N)
        g = h // G
        ref = rp.masked_index_attention(q[b:b + 1, h:h + 1, pos.to(q.device)].float().cpu(),
                                        k[b:b + 1, g:g + 1].float().cpu(), v[b:b + 1, g:g + 1].float().cpu(),
                                        idx[b:b + 1, h:h + 1, pos.to(idx.device)].cpu(), positions=pos)
        got = out[b:b + 1, h:h + 1, pos.to(out.device)].double().cpu()
        mag = ref.abs().clamp(min=2.0 ** -126)
        half_ulp = torch.exp2(torch.floor(torch.log2(mag)) - 8)  # bf16: 8 significant bits
        tol = TOL["atol"] + TOL["rtol"] * ref.abs() + half_ulp
        err = (got - ref).abs()
        assert bool((err <= tol).all()), (f"(b={b}, h={h}): {int((err > tol).sum())} elements beyond "
                                         f"2e-3 + half a bf16 ulp; worst excess {float((err - tol).max()):.3g}")


@pytest.mark.parametrize("K", [32, 128])
def test_oracle_selection_full_size(K):
    B, H, Hkv, N, D = 4, 12, 2, 8192, 128
    q, k, v = oracle_inputs(B, H, Hkv, N, D, DEV, seed=3)
    tc, fb, status = oracle_topk_with_status(q, k, K)
    assert status == 0
    assert fb < 0.001 * B * H * N, f"{fb} rows on the full-row exact fallback"
    os.environ["OSSA_ORACLE_SELECT"] = "exact"
    try:
        ex = oracle_topk(q, k, K)
    finally:
        del os.environ["OSSA_ORACLE_SELECT"]
    assert torch.equal(tc, ex), f"{(tc != ex).any(-1).sum().item()} rows differ from the exact selector"
    rows = _sample_rows(B, H, N, 1024, seed=K)
    assert len(rows) >= 1024
    ref = oracle.oracle_topk_rows(q.cpu(), k.cpu(), K, rows)
    got = tc.reshape(-1, K)[torch.from_numpy(rows).to(DEV)].cpu().numpy()
    bad = (got != ref).any(-1)
    assert not bad.any(), f"{bad.sum()} sampled rows differ from the oracle; first flat row {rows[bad][0]}"
    out = topk_attention(q, k, v, topk_indices=tc, causal=True)
    _check_gather_rows(out, q, k, v, tc, rows[::8], H, N)


@pytest.mark.parametrize("N", [65536, 131072])
def test_long_context_selection_full_size(N):
    B, H, Hkv, D, r, K = 1, 12, 2, 128, 64, 128
    q, k, v, wq, wk, pb = long_inputs(N, DEV, seed=N // 1024)
    idx, fb, status = router_topk_with_status(q, k, wq, wk, pb, N, K)
    assert status == 0
    rows = _sample_rows(B, H, N, 24, seed=N)
    ref = oracle.router_topk_rows(q.cpu(), k.cpu(), wq.cpu(), wk.cpu(), pb.cpu(), N, K, rows)
    got = idx.reshape(-1, K)[torch.from_numpy(rows).to(DEV)].cpu().numpy()
    bad = (got != ref).any(-1)
    assert not bad.any(), f"{bad.sum()} sampled rows differ from the oracle; first flat row {rows[bad][0]}"
    # a second call returns the same indices (no state carried between calls)
    assert torch.equal(router_topk(q, k, wq, wk, pb, N, K), idx)
    out = topk_attention(q, k, v, topk_indices=idx, causal=True)
    assert bool(torch.isfinite(out).all())
    _check_gather_rows(out, q, k, v, idx, rows, H, N)


def test_single_layer_gather_64_rows_per_batch_element():
    B, H, Hkv, N, D, K = 8, 12, 2, 4096, 128, 64
    g = torch.Generator(device=DEV)
    g.manual_seed(11)
    s = 1.0 / math.sqrt(D)
    q = (torch.randn(B, H, N, D, device=DEV, generator=g) * s).bfloat16()
    k = (torch.randn(B, Hkv, N, D, device=DEV, generator=g) * s).bfloat16()
    v = (torch.randn(B, Hkv, N, D, device=DEV, generator=g) * s).bfloat16()
    gc = torch.Generator().manual_seed(12)
    wq = (torch.rand(64, D, generator=gc) * 2 - 1) * math.sqrt(6.0 / (64 + D))
    wk = (torch.rand(64, D, generator=gc) * 2 - 1) * math.sqrt(6.0 / (64 + D))
    pb = torch.randn(2 * N, 1, generator=gc)
    idx = router_topk(q, k, wq.to(DEV), wk.to(DEV), pb.to(DEV), N, K)
    out = topk_attention(q, k, v, topk_indices=idx, causal=True)
    rng = np.random.default_rng(13)
    rows = []
    for b in range(B):
        pos = np.unique(np.concatenate([[0, 1, 62, 63, 64, N - 1], rng.integers(0, N, size=64)]))[:64]
        heads = rng.integers(0, H, size=len(pos))
        rows.append((b * H + heads) * N + pos)
    rows = np.concatenate(rows).astype(np.int64)
    assert len(rows) == 64 * B
    _check_gather_rows(out, q, k, v, idx, rows, H, N)


def test_full_model_layer_patched_attention_full_size():
    """One decoder layer of the full-model workload with random bf16 weights and a
    random-init router: the patched forward's q, k, v are recomputed from the layer's
    captured input with the same operations, its selection is checked row by row
    against the CPU oracle, and its attention output (captured where it enters o_proj)
    against the fp64 attention oracle over those indices."""
    from transformers import Qwen2Config, Qwen2ForCausalLM

    from ossa_b200 import ContentRouter, ContentRouterConfig
    from ossa_b200.bench.sparse_forward import patch_all_layers
    from ossa_b200.rope import rope_to_heads

    B, N, K, H, Hkv, D = 1, 4096, 64, 12, 2, 128
    cfg = Qwen2Config(hidden_size=1536, intermediate_size=8960, num_hidden_layers=1, num_attention_heads=H,
                      num_key_value_heads=Hkv, vocab_size=1024, max_position_embeddings=N, rope_theta=1e6)
    torch.manual_seed(21)
    model = Qwen2ForCausalLM(cfg).to(DEV).bfloat16().eval()
    router = ContentRouter(ContentRouterConfig(head_dim=D, n_heads=H, seq_len=N, proj_dim=64))
    torch.nn.init.xavier_uniform_(router.q_proj[0].weight)
    torch.nn.init.xavier_uniform_(router.k_proj[0].weight)
    router = router.to(DEV)
    restore = patch_all_layers(model, "router", K, routers={0: router})
    attn = model.model.layers[0].self_attn
    seen = {}
    h1 = attn.register_forward_pre_hook(lambda m, a, kw: seen.update(inp=kw), with_kwargs=True)
    h2 = attn.o_proj.register_forward_pre_hook(lambda m, a: seen.update(out=a[0].detach().clone()))
    ids = torch.randint(0, 1024, (B, N), generator=torch.Generator().manual_seed(22)).to(DEV)
    try:
        with torch.no_grad():
            model(input_ids=ids, use_cache=False)
    finally:
        h1.remove()
        h2.remove()
        restore()
    hs = seen["inp"]["hidden_states"]
    cos, sin = seen["inp"]["position_embeddings"]
    with torch.no_grad():
        q = rope_to_heads(attn.q_proj(hs), H, cos, sin)
        k = rope_to_heads(attn.k_proj(hs), Hkv, cos, sin)
        v = rope_to_heads(attn.v_proj(hs), Hkv)
        wq, wk, pb = router.q_proj[0].weight, router.k_proj[0].weight, router.pos_bias.weight
        idx = router_topk(q, k, wq, wk, pb, N, K)
    out = seen["out"].view(B, N, H, D).transpose(1, 2)
    rows = _sample_rows(B, H, N, 256, seed=23)
    ref = oracle.router_topk_rows(q.cpu(), k.cpu(), wq.detach().cpu(), wk.detach().cpu(), pb.detach().cpu(), N, K,
                                  rows)
    got = idx.reshape(-1, K)[torch.from_numpy(rows).to(DEV)].cpu().numpy()
    assert (got == ref).all(), f"{int((got != ref).any(-1).sum())} of {len(rows)} sampled rows differ"
    _check_gather_rows(out, q, k, v, idx, rows, H, N)
