"""The patched Qwen2 attention forward (ossa_b200.bench.sparse_forward) on the
GPU against the reference's patched forward restated on the CPU
(oracle/reference_port.patch_reference_forward), random-init tiny Qwen2."""

import copy

import pytest
import torch

from oracle import reference_port as rp
from ossa_b200 import ContentRouter, ContentRouterConfig
from ossa_b200.bench.sparse_forward import PatchPlan, _patch_layer, patch_all_layers

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _model(seed=0):
    from transformers import Qwen2Config, Qwen2ForCausalLM

    cfg = Qwen2Config(hidden_size=256, intermediate_size=512, num_hidden_layers=3, num_attention_heads=4,
                      num_key_value_heads=2, vocab_size=211, max_position_embeddings=512, rope_theta=1e6)
    torch.manual_seed(seed)
    return Qwen2ForCausalLM(cfg).eval()


def _routers(model, seq_len, seed=0):
    torch.manual_seed(seed)
    out = {}
    for li, layer in enumerate(model.model.layers):
        a = layer.self_attn
        r = ContentRouter(ContentRouterConfig(head_dim=a.head_dim, n_heads=a.config.num_attention_heads,
                                              seq_len=seq_len, proj_dim=64))
        torch.nn.init.xavier_uniform_(r.q_proj[0].weight)
        torch.nn.init.xavier_uniform_(r.k_proj[0].weight)
        out[li] = r
    return out


@pytest.mark.parametrize("mode", ["router", "oracle"])
@pytest.mark.parametrize("impl", ["gather", "mask"])
def test_patched_model_matches_reference_forward(mode, impl):
    N, K = 160, 16
    model = _model()
    routers = _routers(model, N)
    ids = torch.randint(0, 211, (2, N), generator=torch.Generator().manual_seed(1))

    ref_model = copy.deepcopy(model).double()
    ref_routers = {i: copy.deepcopy(r).double() for i, r in routers.items()}
    restore = rp.patch_reference_forward(ref_model, mode, K, routers=ref_routers, impl=impl)
    with torch.no_grad():
        ref = ref_model(input_ids=ids, use_cache=False).logits
    restore()

    gpu_model = copy.deepcopy(model).to(DEV)
    gpu_routers = {i: copy.deepcopy(r).to(DEV) for i, r in routers.items()}
    restore = _patch_layer(gpu_model, PatchPlan(mode=mode, k=K, layers=(0, 1, 2), routers=gpu_routers, impl=impl))
    with torch.no_grad():
        got = gpu_model(input_ids=ids.to(DEV), use_cache=False).logits
    restore()
    torch.testing.assert_close(got.double().cpu(), ref, atol=2e-4, rtol=2e-4)


def test_patched_bf16_model_runs_and_tracks_fp32():
    N, K = 256, 32
    model = _model(seed=3)
    routers = _routers(model, N, seed=3)
    ids = torch.randint(0, 211, (2, N), generator=torch.Generator().manual_seed(2))
    m32 = copy.deepcopy(model).to(DEV)
    r32 = {i: copy.deepcopy(r).to(DEV) for i, r in routers.items()}
    patch_all_layers(m32, "router", K, routers=r32)
    m16 = copy.deepcopy(model).to(DEV).bfloat16()
    patch_all_layers(m16, "router", K, routers=r32)
    with torch.no_grad():
        a = m32(input_ids=ids.to(DEV), use_cache=False).logits
        b = m16(input_ids=ids.to(DEV), use_cache=False).logits.float()
    assert torch.isfinite(b).all()
    cos = torch.nn.functional.cosine_similarity(a.flatten(0, 1), b.flatten(0, 1), dim=-1)
    assert cos.mean() > 0.99


def test_full_model_runner_small(capsys):
    """The full-model prefill runner end to end on a 2-layer cut of the
    architecture: one JSON line with a positive rate and finite logits."""
    import json

    from ossa_b200.bench import full_model

    full_model.main(["--batch", "2", "--seq", "512", "--layers", "2", "--steps", "1", "--warmup", "1"])
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["value"] > 0 and line["logits_finite"] and line["config"]["layers"] == 2


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("B,cs_batch,D", [(2, 2, 128), (3, 1, 128), (1, 1, 64), (2, 2, 16)])
def test_rope_to_heads_equals_eager_rope(dtype, B, cs_batch, D):
    """The fused RoPE + head transpose returns exactly Qwen2's eager
    apply_rotary_pos_emb on the (B, heads, N, D) view, made contiguous, and the
    layout-only form exactly the contiguous view."""
    from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb

    from ossa_b200.rope import rope_to_heads

    g = torch.Generator().manual_seed(D + B)
    N, Hq, Hkv = 77, 6, 2
    xq = (torch.randn(B, N, Hq * D, generator=g) * 3).to(dtype).to(DEV)
    xk = (torch.randn(B, N, Hkv * D, generator=g) * 3).to(dtype).to(DEV)
    pos = torch.arange(N).float()
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2).float() / D))
    emb = torch.cat([pos[:, None] * inv[None], pos[:, None] * inv[None]], dim=-1)
    cos = emb.cos()[None].expand(cs_batch, N, D).to(dtype).to(DEV)
    sin = emb.sin()[None].expand(cs_batch, N, D).to(dtype).to(DEV)
    qv = xq.view(B, N, Hq, D).transpose(1, 2)
    kv = xk.view(B, N, Hkv, D).transpose(1, 2)
    rq, rk = apply_rotary_pos_emb(qv, kv, cos, sin)
    assert torch.equal(rope_to_heads(xq, Hq, cos, sin), rq.contiguous())
    assert torch.equal(rope_to_heads(xk, Hkv, cos, sin), rk.contiguous())
    assert torch.equal(rope_to_heads(xk, Hkv), kv.contiguous())
