"""Routed sparse attention over host-resident tensors, with PCIe transfers
overlapped with the kernels.

A serving process that holds q/k/v in pinned host memory would otherwise run
copy-in, selection + gather, and copy-out back to back.  Here the batch is cut
into chunks of batch elements and each chunk moves through three CUDA streams:

    copy-in stream   : q, k, v of chunk c        (host -> device)
    compute stream   : router_topk + topk_attention of chunk c
    copy-out stream  : attention output of chunk c (device -> host)

so the transfers of chunk c overlap the kernels of chunks c-1 and c+1.  Every
chunk runs the same kernels as the device-tensor API (ossa_b200.router_topk,
ossa_b200.topk_attention); nothing is computed on the host.  The call is
asynchronous with respect to the host like any CUDA work: the caller's current
stream waits for the last copy-out, so synchronising that stream (or reading
``out_host`` after ``torch.cuda.current_stream().synchronize()``) sees the result.
"""

from __future__ import annotations

import torch

from .select import router_topk
from .topk_attention import topk_attention

__all__ = ["routed_attention_from_host"]

# The pipeline's three streams, created once per device and reused by every call.
_streams: dict = {}


def _pipeline_streams(dev: torch.device):
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    st = _streams.get(key)
    if st is None:
        st = _streams[key] = (torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev))
    return st


def routed_attention_from_host(q_host, k_host, v_host, wq, wk, pos_bias, seq_len: int, top_k: int,
                               out_host, *, causal: bool = True, chunk: int = 2, device=None):
    """ContentRouter selection + gathered sparse attention for host tensors.

    ``q_host`` (B, H, N, D), ``k_host``/``v_host`` (B, Hkv, N, D) and ``out_host``
    (B, H, N, D) are CPU tensors, pinned for the copies to be asynchronous;
    ``wq``, ``wk`` (r, D) and ``pos_bias`` (2*seq_len, 1) are device tensors.
    Semantics per batch element are those of ``router_topk`` followed by
    ``topk_attention(..., causal=causal)``.  ``chunk`` batch elements move
    through the pipeline at a time.
    """
    for name, t in (("q_host", q_host), ("k_host", k_host), ("v_host", v_host), ("out_host", out_host)):
        if t.is_cuda:
            raise ValueError(f"{name} must be a host tensor")
    if out_host.shape != q_host.shape or out_host.dtype != q_host.dtype:
        raise ValueError("out_host must match q_host in shape and dtype")
    B = q_host.shape[0]
    if k_host.shape[0] != B or v_host.shape[0] != B:
        raise ValueError("q_host, k_host and v_host must share the batch dimension")
    if chunk < 1:
        raise ValueError("chunk must be >= 1")
    dev = torch.device(device) if device is not None else wq.device
    if dev.type != "cuda":
        raise ValueError("the router weights must live on a CUDA device")
    caller = torch.cuda.current_stream(dev)
    s_in, s_comp, s_out = _pipeline_streams(dev)
    # work queued on the caller's stream before this call comes first
    s_in.wait_stream(caller)
    s_comp.wait_stream(caller)
    s_out.wait_stream(caller)
    for b0 in range(0, B, chunk):
        b1 = min(B, b0 + chunk)
        with torch.cuda.stream(s_in):
            qd = q_host[b0:b1].to(dev, non_blocking=True)
            kd = k_host[b0:b1].to(dev, non_blocking=True)
            vd = v_host[b0:b1].to(dev, non_blocking=True)
        s_comp.wait_stream(s_in)
        with torch.cuda.stream(s_comp):
            for t in (qd, kd, vd):
                t.record_stream(s_comp)
            idx = router_topk(qd, kd, wq, wk, pos_bias, seq_len, top_k, causal=causal)
            out = topk_attention(qd, kd, vd, topk_indices=idx, causal=causal)
        s_out.wait_stream(s_comp)
        with torch.cuda.stream(s_out):
            out.record_stream(s_out)
            out_host[b0:b1].copy_(out, non_blocking=True)
    caller.wait_stream(s_out)
    return out_host
