"""Host-side behaviour of the Python API that needs no GPU: the drop-in
surface, checkpoint compatibility, argument checking, the loud refusal of CPU
tensors, and the model patch/restore mechanics."""

import inspect

import numpy as np
import pytest
import torch

import ossa_b200
from ossa_b200 import ContentRouter, ContentRouterConfig, topk_attention
from ossa_b200.bench.sparse_forward import PatchPlan, _patch_layer, select_indices


def test_public_surface_matches_reference_names():
    for name in ("dense_attention_reference", "sparse_attention_forward", "sparse_attention_forward_chunked",
                 "topk_attention", "HAS_TRITON"):
        assert hasattr(ossa_b200, name)
    from ossa_b200.triton_kernel import topk_attention as t2
    assert t2 is topk_attention
    sig = inspect.signature(topk_attention)
    # the reference's parameters, in order, then only additive keyword-only ones with defaults
    ref = ["q", "k", "v", "topk_indices", "causal", "block_m", "use_triton"]
    assert list(sig.parameters)[:len(ref)] == ref
    for extra in list(sig.parameters)[len(ref):]:
        prm = sig.parameters[extra]
        assert prm.kind is inspect.Parameter.KEYWORD_ONLY and prm.default is None
    assert sig.parameters["causal"].default is True and sig.parameters["block_m"].default == 32


def test_router_loads_reference_checkpoint_state_dict(golden_dir):
    z = np.load(golden_dir / "router_ckpt_c1.npz")
    r = ContentRouter(ContentRouterConfig(head_dim=128, n_heads=12, seq_len=512, proj_dim=64))
    sd = {"q_proj.0.weight": torch.from_numpy(z["wq"]), "k_proj.0.weight": torch.from_numpy(z["wk"]),
          "pos_bias.weight": torch.from_numpy(z["pos_bias"])}
    assert set(r.state_dict()) == set(sd)
    r.load_state_dict(sd)
    assert sum(p.numel() for p in r.parameters()) == 17408  # the reference's parameter count
    with pytest.raises(TypeError):
        r(torch.zeros(1, 1, 4, 128))


def test_cpu_tensors_are_rejected_loudly():
    q = torch.randn(1, 2, 8, 16)
    idx = torch.zeros(1, 2, 8, 4, dtype=torch.int64)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        topk_attention(q, q, q, topk_indices=idx)
    r = ContentRouter(ContentRouterConfig(head_dim=16, n_heads=2, seq_len=8, proj_dim=16))
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        r.topk(q, q, 4, causal=True)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        r.score(q, q)


@pytest.mark.parametrize("bad", [
    dict(k=torch.randn(1, 3, 8, 16), v=torch.randn(1, 3, 8, 16)),
    dict(idx=torch.zeros(1, 2, 7, 4, dtype=torch.int64)),
    dict(idx=torch.zeros(1, 2, 8, 4, dtype=torch.float32)),
    dict(v=torch.randn(1, 2, 8, 16).double()),
])
def test_topk_attention_argument_checks(bad):
    q = torch.randn(1, 2, 8, 16)
    a = dict(k=torch.randn(1, 2, 8, 16), v=torch.randn(1, 2, 8, 16), idx=torch.zeros(1, 2, 8, 4, dtype=torch.int64))
    a.update(bad)
    with pytest.raises((ValueError, TypeError)):
        topk_attention(q, a["k"], a["v"], topk_indices=a["idx"])


def test_router_topk_too_many_keys_unmasked():
    r = ContentRouter(ContentRouterConfig(head_dim=16, n_heads=2, seq_len=8, proj_dim=16))
    q = torch.randn(1, 2, 8, 16)
    with pytest.raises(RuntimeError, match="out of range"):
        r.topk(q, q, 9)


def _tiny_qwen():
    from transformers import Qwen2Config, Qwen2ForCausalLM

    cfg = Qwen2Config(hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, vocab_size=97, max_position_embeddings=64)
    torch.manual_seed(0)
    return Qwen2ForCausalLM(cfg).eval()


def test_patch_and_restore_mechanics():
    model = _tiny_qwen()
    attn = [layer.self_attn for layer in model.model.layers]
    before = [a.forward for a in attn]
    restore = _patch_layer(model, PatchPlan(mode="oracle", k=4, layers=(0, 1), impl="gather"))
    assert all(a.forward is not b for a, b in zip(attn, before))
    ids = torch.randint(0, 97, (1, 12))
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        model(input_ids=ids, use_cache=False)
    restore()
    # bound methods compare equal when they wrap the same function and instance
    assert all(a.forward == b for a, b in zip(attn, before))
    assert _patch_layer(model, PatchPlan(mode="dense", layers=(0,)))() is None


def test_select_indices_rejects_unknown_modes():
    q = torch.randn(1, 2, 8, 16)
    with pytest.raises(ValueError):
        select_indices(PatchPlan(mode="bogus", k=4, layers=(0,)), 0, q, q)
    with pytest.raises(KeyError):
        select_indices(PatchPlan(mode="router", k=4, layers=(0,), routers={}), 0, q, q)


def test_host_pipeline_argument_checks():
    from ossa_b200.host_pipeline import routed_attention_from_host

    q = torch.zeros(2, 4, 8, 16, dtype=torch.bfloat16)
    k = torch.zeros(2, 2, 8, 16, dtype=torch.bfloat16)
    w = torch.zeros(8, 16)
    pb = torch.zeros(16, 1)
    with pytest.raises(ValueError, match="out_host"):
        routed_attention_from_host(q, k, k, w, w, pb, 8, 4, torch.zeros(2, 4, 8, 16))
    with pytest.raises(ValueError, match="batch"):
        routed_attention_from_host(q, k[:1], k[:1], w, w, pb, 8, 4, torch.zeros_like(q))
    with pytest.raises(ValueError, match="chunk"):
        routed_attention_from_host(q, k, k, w, w, pb, 8, 4, torch.zeros_like(q), chunk=0)
    with pytest.raises(ValueError, match="groups must divide"):
        routed_attention_from_host(q, k, k, w, w, pb, 8, 4, torch.zeros_like(q), chunk=1, groups=3)
    with pytest.raises(ValueError, match="chunk=1"):
        routed_attention_from_host(q, k, k, w, w, pb, 8, 4, torch.zeros_like(q), chunk=2, groups=2)
    with pytest.raises(ValueError, match="edge_groups must divide"):
        routed_attention_from_host(q, k, k, w, w, pb, 8, 4, torch.zeros_like(q), chunk=1, edge_groups=3)
    with pytest.raises(ValueError, match="CUDA"):
        routed_attention_from_host(q, k, k, w, w, pb, 8, 4, torch.zeros_like(q))


def test_full_model_runner_config_and_routers():
    """The full-model prefill runner builds the Qwen2.5-1.5B architecture and one
    seeded Xavier-uniform router per layer (checked on the CPU at 2 layers)."""
    import math

    from ossa_b200.bench import full_model

    cfg = full_model.qwen25_15b_config(4096)
    assert (cfg.hidden_size, cfg.intermediate_size, cfg.num_hidden_layers) == (1536, 8960, 28)
    assert (cfg.num_attention_heads, cfg.num_key_value_heads, cfg.vocab_size) == (12, 2, 151936)
    rope = getattr(cfg, "rope_parameters", None) or {"rope_theta": getattr(cfg, "rope_theta", None)}
    assert rope["rope_theta"] == 1e6 and cfg.hidden_size // cfg.num_attention_heads == 128

    class _Attn:
        head_dim = 128

    class _Layer:
        self_attn = _Attn()

    class _Model:
        config = cfg

        class model:  # noqa: N801 - mirrors the Hugging Face attribute path
            layers = [_Layer(), _Layer()]

    a = full_model.build_routers(_Model, 4096, "cpu", seed=5)
    b = full_model.build_routers(_Model, 4096, "cpu", seed=5)
    assert sorted(a) == [0, 1]
    bound = math.sqrt(6.0 / (64 + 128))
    for li in a:
        wq = a[li].q_proj[0].weight.detach()
        assert wq.shape == (64, 128) and float(wq.abs().max()) <= bound
        assert a[li].pos_bias.weight.shape == (2 * 4096, 1)
        assert torch.equal(wq, b[li].q_proj[0].weight.detach())
    assert not torch.equal(a[0].q_proj[0].weight, a[1].q_proj[0].weight)


def test_router_with_seq_len_scores_like_the_clamped_table(golden_dir, tmp_path):
    """A router resized from its trained seq_len (512, the reference checkpoint)
    to 1024 scores every (i, j) of a 1024-token input exactly as the trained
    table does under the reference's clamped indexing; shrinking keeps every
    in-range offset.  _load_router(pos_bias="extend") loads that way."""
    import types

    import cases
    import oracle
    from ossa_b200.bench.sparse_forward import _load_router

    z = np.load(golden_dir / "router_ckpt_c1.npz")
    r = ContentRouter(ContentRouterConfig(head_dim=128, n_heads=12, seq_len=512, proj_dim=64))
    r.load_state_dict({"q_proj.0.weight": torch.from_numpy(z["wq"]), "k_proj.0.weight": torch.from_numpy(z["wk"]),
                       "pos_bias.weight": torch.from_numpy(z["pos_bias"])})
    q, k, _ = cases.qkv(1, 2, 1, 1024, 128, seed=11)
    wq, wk, pb = (t.detach() for t in r._params())
    ref = oracle.router_scores(q, k, wq, wk, pb, 512)
    big = r.with_seq_len(1024)
    assert big.pos_bias.weight.shape == (2048, 1)
    got = oracle.router_scores(q, k, *(t.detach() for t in big._params()), 1024)
    assert np.array_equal(got, ref)
    small = r.with_seq_len(200)
    qs, ks = q[:, :, :200], k[:, :, :200]
    assert np.array_equal(oracle.router_scores(qs, ks, *(t.detach() for t in small._params()), 200),
                          oracle.router_scores(qs, ks, wq, wk, pb, 512))

    class Attn(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.head_dim = 128
            self.config = types.SimpleNamespace(num_attention_heads=12)
            self.w = torch.nn.Parameter(torch.zeros(1))

    model = torch.nn.Module()
    model.model = torch.nn.Module()
    model.model.layers = torch.nn.ModuleList([torch.nn.Module()])
    model.model.layers[0].self_attn = Attn()
    ckpt = tmp_path / "router.pt"
    torch.save({"cfg": {"proj_dim": 64}, "state_dict": r.state_dict()}, ckpt)
    with pytest.raises(RuntimeError):
        _load_router(ckpt, model, 0, 1024)  # the reference's behaviour: the table does not fit
    loaded = _load_router(ckpt, model, 0, 1024, pos_bias="extend")
    assert torch.equal(loaded.pos_bias.weight, big.pos_bias.weight)
    assert not loaded.training


def test_router_key_cache_argument_checks():
    from ossa_b200.decode import RouterKeyCache

    r = ContentRouter(ContentRouterConfig(head_dim=16, n_heads=4, seq_len=32, proj_dim=16))
    cache = RouterKeyCache(r, batch=1, kv_heads=2, capacity=8, device="cpu")
    with pytest.raises(ValueError):
        cache.append(torch.zeros(1, 2, 9, 16))      # past the capacity
    with pytest.raises(ValueError):
        cache.append(torch.zeros(1, 3, 2, 16))      # wrong head count
    with pytest.raises(RuntimeError):
        cache.append(torch.zeros(1, 2, 2, 16))      # CPU tensors are refused, no CPU path
    with pytest.raises(ValueError):
        cache.topk(torch.zeros(1, 4, 1, 16), 4)     # nothing cached yet
