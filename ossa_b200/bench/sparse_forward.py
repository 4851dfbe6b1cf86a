"""Patched ``Qwen2Attention.forward`` running the sm_100a sparse path.

Mirrors ``PatchPlan`` / ``_patch_layer`` / ``_load_router`` of
ossa/bench/sparse_forward.py:122-239, 272-294, so code that patches a Hugging
Face Qwen2 model with the reference keeps working.  The patched forward
(reference :157-229) does q/k/v projections and RoPE with the layer's own
modules, then:

* selection in fp32 by one fused kernel (router: ContentRouter scores, :185-193;
  oracle: exact q.k/sqrt(D), :194-196), causal, no N x N selector in memory;
* the gathered sparse forward (reference :204-208) on GQA-native K/V
  (no ``repeat_interleave``, :175-178);
* ``impl="mask"`` keeps the reference's mask-path semantics (top-K set plus the
  forced diagonal, :209-222) but evaluates them on the same O(N*K) kernel by
  appending the diagonal to each index row instead of a dense N x N softmax;
* o_proj and the ``(out, None)`` return as the reference;
* (additive) RoPE and the head transpose of q/k/v run as one kernel pass per
  tensor (``rope_to_heads``), bit-identical to ``apply_rotary_pos_emb`` plus the
  layout copies.

Deliberate difference: the reference casts router logits to the model dtype
before ``torch.topk`` (:193), which ties ~15% of rows at the K-th boundary in
bf16; selection here is in fp32 (ties broken toward the lower key index).
Like the reference, the forward is prefill-only: ``attention_mask`` (padding)
and ``past_key_values`` are ignored.
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path
from typing import Optional

import torch

from .. import select
from ..rope import rope_to_heads
from ..router import ContentRouter, ContentRouterConfig
from ..topk_attention import topk_attention


@dataclass
class PatchPlan:
    mode: str                          # "dense" | "oracle" | "router"
    k: int = 64
    layers: tuple[int, ...] = ()       # which layers to patch; empty = none
    routers: dict[int, ContentRouter] | None = None  # layer_idx -> router
    impl: str = "mask"                 # "mask" (top-K + forced diagonal) | "gather"


def _router_params(router):
    """(wq, wk, pos_bias, seq_len) of a ContentRouter-shaped module (this package's
    or the reference's: both expose q_proj[0], k_proj[0], pos_bias, cfg.seq_len)."""
    try:
        return (router.q_proj[0].weight, router.k_proj[0].weight, router.pos_bias.weight,
                int(router.cfg.seq_len))
    except AttributeError as e:
        raise TypeError(
            "only ContentRouter-style routers (q_proj, k_proj, pos_bias) are supported; "
            f"got {type(router).__name__}") from e


def select_indices(plan: PatchPlan, layer_idx: int, q: torch.Tensor, k: torch.Tensor) -> torch.Tensor:
    """Causal top-K indices (B, H, N, K') for one patched layer, int32, -1 padded."""
    N = q.shape[2]
    k_eff = min(plan.k, N)
    if plan.mode == "router":
        if plan.routers is None or layer_idx not in plan.routers:
            raise KeyError(f"no router for layer {layer_idx}")
        wq, wk, pb, seq_len = _router_params(plan.routers[layer_idx])
        idx = select.router_topk(q, k, wq, wk, pb, seq_len, k_eff, causal=True)
    elif plan.mode == "oracle":
        idx = select.oracle_topk(q, k, k_eff, causal=True)
    else:
        raise ValueError(plan.mode)
    if plan.impl == "mask":
        idx = select.with_diagonal(idx)
    elif plan.impl != "gather":
        raise ValueError(f"unknown impl {plan.impl!r}")
    return idx


def _patch_layer(model, plan: PatchPlan):
    """Monkey-patches ``self_attn.forward`` of the chosen layers; returns a
    callable that undoes every patch."""
    if plan.mode == "dense" or not plan.layers:
        return lambda: None

    restores: list = []
    for layer_idx in plan.layers:
        layer_module = model.model.layers[layer_idx].self_attn
        original_forward = layer_module.forward

        def make_forward(layer_module=layer_module, captured_idx=layer_idx):
            def new_forward(hidden_states, attention_mask=None, position_ids=None,
                            past_key_values=None, output_attentions=False,
                            use_cache=False, cache_position=None,
                            position_embeddings=None, **kwargs):
                B, N, _ = hidden_states.shape
                head_dim = layer_module.head_dim
                n_heads = layer_module.config.num_attention_heads
                n_kv_heads = layer_module.config.num_key_value_heads

                # projections, then RoPE and the (B, heads, N, D) layout in one kernel
                # pass per tensor (bit-identical to apply_rotary_pos_emb + contiguous)
                cos, sin = position_embeddings if position_embeddings is not None else (None, None)
                q = rope_to_heads(layer_module.q_proj(hidden_states), n_heads, cos, sin)
                k = rope_to_heads(layer_module.k_proj(hidden_states), n_kv_heads, cos, sin)
                v = rope_to_heads(layer_module.v_proj(hidden_states), n_kv_heads)

                with torch.no_grad():
                    idx = select_indices(plan, captured_idx, q, k)
                out = topk_attention(q, k, v, topk_indices=idx, causal=True)

                out = out.transpose(1, 2).reshape(B, N, n_heads * head_dim)
                out = layer_module.o_proj(out)
                return out, None
            return new_forward

        layer_module.forward = make_forward()
        restores.append((layer_module, original_forward))

    def restore() -> None:
        for lm, orig in restores:
            lm.forward = orig

    return restore


def _load_router(checkpoint: Path, model, layer: int, seq_len: int, *, pos_bias: str = "exact"):
    """Loads a ContentRouter checkpoint ({"state_dict", "cfg"}, the reference's
    format, bench/content_train.py:172-175) sized for ``seq_len`` as the reference
    does (sparse_forward.py:272-294).  With ``pos_bias="exact"`` (the reference's
    behaviour) a checkpoint trained at another seq_len does not fit.  With
    ``pos_bias="extend"`` (additive) the router is built at its trained seq_len
    and resized with ``ContentRouter.with_seq_len``: its scores at any offset
    equal the trained router's clamped ones."""
    if pos_bias not in ("exact", "extend"):
        raise ValueError(f"pos_bias must be 'exact' or 'extend', got {pos_bias!r}")
    state = torch.load(checkpoint, map_location=next(model.parameters()).device, weights_only=False)
    cfg_dict = state["cfg"]
    state_dict = state["state_dict"]
    if not any(key.startswith("q_proj") or key.startswith("k_proj") for key in state_dict):
        raise TypeError("only ContentRouter checkpoints are supported (PerLayerRouter is out of scope)")
    layer_module = model.model.layers[layer].self_attn
    trained = state_dict["pos_bias.weight"].shape[0] // 2
    cfg = ContentRouterConfig(
        head_dim=layer_module.head_dim,
        n_heads=layer_module.config.num_attention_heads,
        seq_len=trained if pos_bias == "extend" else seq_len,
        proj_dim=cfg_dict.get("proj_dim", 64),
    )
    router = ContentRouter(cfg).to(next(model.parameters()).device)
    router.load_state_dict(state_dict)
    router.eval()
    if pos_bias == "extend" and trained != seq_len:
        router = router.with_seq_len(seq_len).eval()
    return router


def patch_all_layers(model, mode: str, k: int, routers: Optional[dict] = None, impl: str = "gather"):
    """Convenience: patch every decoder layer (the full-model configuration)."""
    n = len(model.model.layers)
    return _patch_layer(model, PatchPlan(mode=mode, k=k, layers=tuple(range(n)), routers=routers, impl=impl))
