"""The reference's PyTorch hot path, restated with torch CPU ops.

TEST INFRASTRUCTURE (see oracle/__init__.py).  Each function follows the cited
reference lines; the arithmetic is the same sequence of torch calls the
reference makes, so on CPU fp32 it reproduces the reference's outputs up to
BLAS threading.  It is both the attention-output oracle and the CPU baseline
that bench.py times (``cpu_baseline.kind == "port"``).
"""

from __future__ import annotations

import math

import torch


def router_score(q, k, wq, wk, pos_bias, seq_len: int) -> torch.Tensor:
    """ContentRouter.score, ossa/router.py:171-190.  q, k: (B, H, N, D) with the
    same head count (the reference repeats kv heads first)."""
    qh = torch.nn.functional.linear(q, wq)               # router.py:179
    kh = torch.nn.functional.linear(k, wk)               # router.py:180
    scale = 1.0 / math.sqrt(wq.shape[0])                  # router.py:181
    logits = torch.einsum("bhnd,bhmd->bhnm", qh, kh) * scale   # router.py:182
    n = q.shape[2]
    pq = torch.arange(n, device=q.device).unsqueeze(1)    # router.py:184-186
    pk = torch.arange(n, device=q.device).unsqueeze(0)
    offsets = (pq - pk + seq_len).clamp(min=0, max=2 * seq_len - 1)  # router.py:187-188
    bias = pos_bias.reshape(-1)[offsets]                   # router.py:188 (Embedding lookup)
    return logits + bias                                   # router.py:189


def router_distillation(q, k, wq, wk, pos_bias, seq_len: int, targets, dtype=torch.float64):
    """ContentRouter training loss and gradients: distillation_loss(router.score(q, k),
    dense, k) (ossa/router.py:80-99 on router.py:171-190) with the 0/1 target given
    explicitly as index lists (B, H, N, K), -1 padded, in place of the dense top-k.
    q (B, H, N, D), k (B, Hkv, N, D) are repeated to H heads as the reference's
    callers do.  Evaluated in ``dtype`` with autograd; returns (loss, dwq, dwk,
    dpos_bias)."""
    H, Hkv = q.shape[1], k.shape[1]
    wq = wq.detach().to(dtype).requires_grad_(True)
    wk = wk.detach().to(dtype).requires_grad_(True)
    pb = pos_bias.detach().to(dtype).requires_grad_(True)
    logits = router_score(q.to(dtype), repeat_kv(k.to(dtype), H // Hkv), wq, wk, pb, seq_len)
    idx = targets.long()
    t = torch.zeros_like(logits)
    # padding (-1) adds 0 at key 0, so it cannot clear a listed key 0; a key listed
    # twice is still one target
    t.scatter_add_(-1, idx.clamp(min=0), (idx >= 0).to(dtype))
    t = (t > 0).to(dtype)
    loss = torch.nn.functional.binary_cross_entropy_with_logits(logits, t)
    loss.backward()
    return loss.detach(), wq.grad, wk.grad, pb.grad


def repeat_kv(x: torch.Tensor, rep: int) -> torch.Tensor:
    """GQA expansion, ossa/bench/sparse_forward.py:175-178."""
    return x.repeat_interleave(rep, dim=1) if rep > 1 else x


def causal_topk(selector: torch.Tensor, k: int) -> torch.Tensor:
    """Causal mask + torch.topk, ossa/bench/sparse_forward.py:180, 200-202."""
    n = selector.shape[-1]
    causal = torch.tril(torch.ones(n, n, dtype=torch.bool, device=selector.device))
    masked = selector.masked_fill(~causal, float("-inf"))
    return torch.topk(masked, k=min(k, n), dim=-1).indices


def sparse_forward_chunked(q, k, v, idx, chunk_size: int = 64, causal: bool = True):
    """sparse_attention_forward_chunked, ossa/sparse_attention.py:87-137."""
    B, H, N, D = q.shape
    K = idx.shape[-1]
    scale = 1.0 / math.sqrt(D)
    out = torch.empty_like(q)
    BH = B * H
    kf = k.reshape(BH, N, D)
    vf = v.reshape(BH, N, D)
    bh = torch.arange(BH, device=q.device).view(BH, 1, 1)
    for s in range(0, N, chunk_size):
        e = min(s + chunk_size, N)
        C = e - s
        qc = q[:, :, s:e, :].reshape(BH, C, D)
        ic = idx[:, :, s:e, :].reshape(BH, C, K)
        bb = bh.expand(BH, C, K)
        kt = kf[bb, ic]
        vt = vf[bb, ic]
        sc = torch.einsum("bcd,bckd->bck", qc, kt) * scale
        if causal:
            pos = torch.arange(s, e, device=q.device).view(1, C, 1)
            sc = sc.masked_fill(ic > pos, float("-inf"))
        p = torch.nan_to_num(torch.softmax(sc, dim=-1), nan=0.0)
        out[:, :, s:e, :] = torch.einsum("bck,bckd->bcd", p, vt).reshape(B, H, C, D)
    return out


def sparse_forward_full(q, k, v, idx, causal: bool = True):
    """sparse_attention_forward, ossa/sparse_attention.py:29-79."""
    B, H, N, D = q.shape
    K = idx.shape[-1]
    scale = 1.0 / math.sqrt(D)
    ie = idx.unsqueeze(-1).expand(B, H, N, K, D)
    kt = torch.gather(k.unsqueeze(2).expand(B, H, N, N, D), 3, ie)
    vt = torch.gather(v.unsqueeze(2).expand(B, H, N, N, D), 3, ie)
    sc = (q.unsqueeze(-2) * kt).sum(-1) * scale
    if causal:
        pos = torch.arange(N, device=q.device).view(1, 1, N, 1)
        sc = sc.masked_fill(idx > pos, float("-inf"))
    p = torch.nan_to_num(torch.softmax(sc, dim=-1), nan=0.0)
    return (p.unsqueeze(-1) * vt).sum(-2)


def dense_attention(q, k, v, causal: bool = True):
    """dense_attention_reference, ossa/sparse_attention.py:140-151."""
    N = q.shape[2]
    sc = torch.matmul(q, k.transpose(-2, -1)) * (1.0 / math.sqrt(q.shape[-1]))
    if causal:
        m = torch.triu(torch.ones(N, N, dtype=torch.bool, device=q.device), diagonal=1)
        sc = sc.masked_fill(m, float("-inf"))
    return torch.matmul(torch.softmax(sc, dim=-1), v)


def masked_index_attention(q, k, v, idx, causal: bool = True, positions=None):
    """Attention over an explicit per-row key set given as indices with -1 padding
    (the ossa_b200 index convention): fp64 softmax over the listed keys j with
    0 <= j < N (and j <= position when causal), 0 for a row with none.
    q: (B, H, M, D) query rows at `positions` (default 0..M-1); k, v:
    (B, Hkv, N, D), Hkv dividing H.  The fp64 oracle of the gather kernel; on
    indices without padding it equals sparse_forward_chunked."""
    B, H, M, D = q.shape
    N = k.shape[2]
    rep = H // k.shape[1]
    kk = repeat_kv(k, rep).double()
    vv = repeat_kv(v, rep).double()
    qd = q.double()
    idx = idx.long()
    pos = (torch.arange(M) if positions is None else torch.as_tensor(positions)).view(1, 1, M, 1)
    valid = (idx >= 0) & (idx < N)
    if causal:
        valid &= idx <= pos
    safe = idx.clamp(min=0, max=N - 1)
    bh = torch.arange(B * H).view(B, H, 1, 1)
    kt = kk.reshape(B * H, N, D)[bh, safe]
    vt = vv.reshape(B * H, N, D)[bh, safe]
    sc = torch.einsum("bhnd,bhnkd->bhnk", qd, kt) / math.sqrt(D)
    sc = sc.masked_fill(~valid, float("-inf"))
    p = torch.nan_to_num(torch.softmax(sc, dim=-1), nan=0.0)
    return torch.einsum("bhnk,bhnkd->bhnd", p, vt)


def reference_layer_path(q, k, v, wq, wk, pos_bias, seq_len: int, top_k: int,
                         chunk_size: int = 64):
    """Router selection + gather forward exactly as the patched forward runs it
    (ossa/bench/sparse_forward.py:175-208) for fp32 inputs: repeat kv heads,
    router.score in fp32, causal topk, chunked sparse forward."""
    rep = q.shape[1] // k.shape[1]
    kr = repeat_kv(k, rep)
    vr = repeat_kv(v, rep)
    logits = router_score(q.float(), kr.float(), wq, wk, pos_bias, seq_len)
    idx = causal_topk(logits.to(q.dtype), top_k)
    return sparse_forward_chunked(q, kr, vr, idx, chunk_size=chunk_size, causal=True), idx


def patch_reference_forward(model, mode: str, k_top: int, routers=None, impl: str = "gather",
                            select_in_fp32: bool = True):
    """The reference's patched Qwen2Attention.forward
    (ossa/bench/sparse_forward.py:157-229) restated for every layer of `model`:
    projections, RoPE, repeat_interleave GQA, selector (router :185-193 /
    oracle :194-196), causal topk (:200-202), then the chunked gather forward
    (:204-208) or the dense masked path with forced diagonal (:209-222), o_proj.
    With select_in_fp32 the selector is not cast to the model dtype before topk
    (the one documented difference of the sm_100a path).  Returns restore()."""
    from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb

    saved = []
    for li, layer in enumerate(model.model.layers):
        attn = layer.self_attn

        def fwd(hidden_states, attention_mask=None, position_ids=None, past_key_values=None,
                output_attentions=False, use_cache=False, cache_position=None,
                position_embeddings=None, _attn=attn, _li=li, **kw):
            B, N, _ = hidden_states.shape
            D = _attn.head_dim
            H = _attn.config.num_attention_heads
            Hkv = _attn.config.num_key_value_heads
            q = _attn.q_proj(hidden_states).view(B, N, H, D).transpose(1, 2)
            k = _attn.k_proj(hidden_states).view(B, N, Hkv, D).transpose(1, 2)
            v = _attn.v_proj(hidden_states).view(B, N, Hkv, D).transpose(1, 2)
            cos, sin = position_embeddings
            q, k = apply_rotary_pos_emb(q, k, cos, sin)
            k = repeat_kv(k, H // Hkv)
            v = repeat_kv(v, H // Hkv)
            causal = torch.tril(torch.ones(N, N, dtype=torch.bool, device=q.device))
            if mode == "router":
                r = routers[_li]
                logits = router_score(q.float(), k.float(), r.q_proj[0].weight.float(),
                                      r.k_proj[0].weight.float(), r.pos_bias.weight.float(), r.cfg.seq_len)
                sel = logits if select_in_fp32 else logits.to(q.dtype)
            else:
                sel = torch.matmul(q.float() if select_in_fp32 else q,
                                   (k.float() if select_in_fp32 else k).transpose(-2, -1)) * (1.0 / math.sqrt(D))
            sel = sel.masked_fill(~causal, float("-inf"))
            top = torch.topk(sel, k=min(k_top, N), dim=-1).indices
            if impl == "gather":
                out = sparse_forward_chunked(q, k, v, top, chunk_size=64, causal=True)
            else:
                sc = torch.matmul(q, k.transpose(-2, -1)) * (1.0 / math.sqrt(D))
                keep = torch.zeros_like(sc, dtype=torch.bool)
                keep.scatter_(-1, top, True)
                d = torch.arange(N, device=q.device)
                keep[..., d, d] = True
                keep &= causal
                sc = sc.masked_fill(~keep, float("-inf"))
                out = torch.matmul(torch.nan_to_num(torch.softmax(sc, dim=-1), nan=0.0), v)
            out = out.transpose(1, 2).contiguous().view(B, N, H * D)
            return _attn.o_proj(out), None

        saved.append((attn, attn.forward))
        attn.forward = fwd

    def restore():
        for a, f in saved:
            a.forward = f
    return restore
