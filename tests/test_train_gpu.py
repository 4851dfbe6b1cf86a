"""Router training step on the GPU (ossa_b200.train): the distillation loss of
ossa/router.py:80-99 and its gradients for q_proj, k_proj and pos_bias, computed
without the (B, H, N, N) logits.

Checked against the reference's own loss and gradients (tests/golden, made by
running the reference) and against the fp64 restatement in oracle/reference_port.py
on ragged GQA shapes, clamped position offsets and bf16 inputs.  Tolerances: the
loss within 1e-5 relative; each gradient within 1e-4 relative to its largest entry
(fp32 sums over up to ~10^7 (i, j) terms, in a different order than autograd's).
"""

import math

import numpy as np
import pytest
import torch

import cases
import oracle
from oracle import reference_port as rp
from ossa_b200 import ContentRouter, ContentRouterConfig
from ossa_b200.train import dense_topk_targets, distillation_loss

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _router(D, H, r, L, wq, wk, pb):
    router = ContentRouter(ContentRouterConfig(head_dim=D, n_heads=H, seq_len=L, proj_dim=r))
    with torch.no_grad():
        router.q_proj[0].weight.copy_(wq)
        router.k_proj[0].weight.copy_(wk)
        router.pos_bias.weight.copy_(pb)
    return router.to(DEV)


def _close_grad(got, ref):
    ref = torch.as_tensor(ref).double()
    err = (got.detach().double().cpu() - ref).abs().max().item()
    assert err <= 1e-4 * ref.abs().max().item() + 1e-12, f"max error {err:.3g} vs max |ref| {ref.abs().max():.3g}"


def test_matches_reference_golden(golden_dir):
    """The reference's own training step (its torch.topk targets of the dense attention)."""
    z = np.load(golden_dir / "router_distill.npz")
    q, k, _ = cases.distill_inputs()
    B, H, N, D = q.shape
    r, L, K = int(z["r"]), int(z["seq_len"]), int(z["K"])
    wq, wk, pb = cases.router_weights(D, r, L, seed=int(z["weight_seed"]))
    router = _router(D, H, r, L, wq, wk, pb)
    tgt = torch.from_numpy(z["target_idx"].astype(np.int32)).to(DEV)
    loss = distillation_loss(router, q.to(DEV), k.to(DEV), K, targets=tgt)
    loss.backward()
    assert abs(loss.item() - float(z["loss"])) <= 1e-5 * abs(float(z["loss"]))
    _close_grad(router.q_proj[0].weight.grad, z["dwq"])
    _close_grad(router.k_proj[0].weight.grad, z["dwk"])
    _close_grad(router.pos_bias.weight.grad, z["dpos_bias"])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B,H,Hkv,N,D,r,L,K", [
    (1, 12, 2, 512, 128, 64, 512, 64),   # the small single-layer shape, the reference's training length
    (2, 6, 3, 200, 64, 32, 64, 16),      # ragged tiles, offsets clamped (N > seq_len)
    (1, 4, 4, 130, 128, 128, 256, 40),   # repeated heads, r = 128
    (1, 2, 1, 70, 32, 16, 70, 8),        # r = 16
])
def test_matches_restatement(dtype, B, H, Hkv, N, D, r, L, K):
    q, k, _ = cases.qkv(B, H, Hkv, N, D, seed=N + r, scale=1.0 / math.sqrt(D))
    q, k = q.to(dtype), k.to(dtype)
    wq, wk, pb = cases.router_weights(D, r, L, seed=r + K)
    router = _router(D, H, r, L, wq, wk, pb)
    tgt = dense_topk_targets(q.to(DEV), k.to(DEV), K)
    loss = router.distillation_loss(q.to(DEV), k.to(DEV), K, targets=tgt)
    loss.backward()
    rl, rwq, rwk, rpb = rp.router_distillation(q.float(), k.float(), wq, wk, pb, L, tgt.cpu())
    assert abs(loss.item() - rl.item()) <= 1e-5 * abs(rl.item())
    _close_grad(router.q_proj[0].weight.grad, rwq)
    _close_grad(router.k_proj[0].weight.grad, rwk)
    _close_grad(router.pos_bias.weight.grad, rpb)


def test_dense_targets_are_the_dense_topk():
    """The default targets: the top-k of the causal dense attention softmax(q k^T / sqrt(D))
    (the sets the reference's torch.topk of the dense probabilities gives on rows with at
    least k eligible keys)."""
    B, H, Hkv, N, D, K = 1, 4, 2, 300, 128, 32
    q, k, _ = cases.qkv(B, H, Hkv, N, D, seed=9, scale=1.0 / math.sqrt(D))
    got = dense_topk_targets(q.to(DEV), k.to(DEV), K).cpu().numpy()
    np.testing.assert_array_equal(got, oracle.oracle_topk(q, k, K))
    kr = k.repeat_interleave(H // Hkv, dim=1)
    causal = torch.tril(torch.ones(N, N, dtype=torch.bool))
    dense = torch.softmax((q @ kr.transpose(-2, -1) / math.sqrt(D)).masked_fill(~causal, float("-inf")), dim=-1)
    ref = torch.sort(torch.topk(dense, K, dim=-1).indices, dim=-1).values.numpy()
    rows = np.arange(N) >= K - 1
    same = (got[:, :, rows] == ref[:, :, rows]).all(-1)
    assert same.mean() > 0.999, f"{(~same).sum()} rows differ"  # fp32 near-ties may order differently


def test_training_steps_reduce_the_loss():
    """A few AdamW steps of the reference loop (content_train.py:141-148) lower the loss."""
    B, H, Hkv, N, D, r, L, K = 1, 12, 2, 512, 128, 64, 512, 64
    q, k, _ = cases.qkv(B, H, Hkv, N, D, seed=77)
    q, k = q.to(DEV), k.to(DEV)
    wq, wk, pb = cases.router_weights(D, r, L, seed=78)
    router = _router(D, H, r, L, wq, wk, pb)
    opt = torch.optim.AdamW(router.parameters(), lr=1e-3)
    tgt = dense_topk_targets(q, k, K)
    losses = []
    for _ in range(20):
        loss = router.distillation_loss(q, k, K, targets=tgt)
        opt.zero_grad()
        loss.backward()
        opt.step()
        losses.append(loss.item())
    assert losses[-1] < losses[0]
