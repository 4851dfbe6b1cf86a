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

import math

import torch

from . import _lib

__all__ = ["routed_attention_from_host", "release_pipeline_buffers"]

# The pipeline's three streams, created once per device and reused by every call.
_streams: dict = {}
# Device buffers of the pipeline, one set per (device, shapes, dtype, chunk, K):
# allocated on the first call of a shape and reused, so a call allocates nothing.
_buffers: dict = {}


def _pipeline_streams(dev: torch.device):
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    st = _streams.get(key)
    if st is None:
        st = _streams[key] = (torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev))
    return st


class _ChunkBuffers:
    """Two sets (chunk parities) of device buffers for one chunk of batch elements:
    q, k, v, indices, output and selector workspace, plus the events that order
    their reuse: chunk c + 2 copies in only after chunk c's kernels are done with
    its inputs, and chunk c + 2's kernels write only after chunk c's output has
    been copied out."""

    def __init__(self, dev, q_shape, k_shape, dtype, top_k, ws_bytes):
        self.q = [torch.empty(q_shape, dtype=dtype, device=dev) for _ in range(2)]
        self.k = [torch.empty(k_shape, dtype=dtype, device=dev) for _ in range(2)]
        self.v = [torch.empty(k_shape, dtype=dtype, device=dev) for _ in range(2)]
        self.idx = [torch.empty(q_shape[:3] + (top_k,), dtype=torch.int32, device=dev) for _ in range(2)]
        self.out = [torch.empty(q_shape, dtype=dtype, device=dev) for _ in range(2)]
        self.ws = [torch.empty(ws_bytes, dtype=torch.uint8, device=dev) for _ in range(2)]
        self.ws_bytes = ws_bytes
        self.in_done = [torch.cuda.Event() for _ in range(2)]
        self.comp_done = [torch.cuda.Event() for _ in range(2)]
        self.out_done = [torch.cuda.Event() for _ in range(2)]


def release_pipeline_buffers() -> None:
    """Drops the device buffers kept for the shapes seen so far."""
    _buffers.clear()


def routed_attention_from_host(q_host, k_host, v_host, wq, wk, pos_bias, seq_len: int, top_k: int,
                               out_host, *, causal: bool = True, chunk: int = 2, device=None):
    """ContentRouter selection + gathered sparse attention for host tensors.

    ``q_host`` (B, H, N, D), ``k_host``/``v_host`` (B, Hkv, N, D) and ``out_host``
    (B, H, N, D) are CPU tensors, pinned for the copies to be asynchronous, float32
    or bfloat16; ``wq``, ``wk`` (r, D) and ``pos_bias`` (2*seq_len, 1) are device
    tensors.  Semantics per batch element are those of ``router_topk`` followed by
    ``topk_attention(..., causal=causal)``.  ``chunk`` batch elements move
    through the pipeline at a time.  The device buffers of a shape are allocated on
    its first call and kept for the next ones (``release_pipeline_buffers`` drops
    them).
    """
    for name, t in (("q_host", q_host), ("k_host", k_host), ("v_host", v_host), ("out_host", out_host)):
        if t.is_cuda:
            raise ValueError(f"{name} must be a host tensor")
    if out_host.shape != q_host.shape or out_host.dtype != q_host.dtype:
        raise ValueError("out_host must match q_host in shape and dtype")
    if q_host.dim() != 4 or k_host.dim() != 4 or v_host.shape != k_host.shape:
        raise ValueError("q_host must be (B, H, N, D) and k_host, v_host (B, Hkv, N, D)")
    B, H, N, D = q_host.shape
    if k_host.shape[0] != B or k_host.shape[2] != N or k_host.shape[3] != D:
        raise ValueError("q_host, k_host and v_host must share the batch dimension, N and D")
    Hkv = k_host.shape[1]
    if Hkv <= 0 or H % Hkv != 0:
        raise ValueError(f"query heads {H} must be a multiple of key heads {Hkv}")
    if q_host.dtype != k_host.dtype or q_host.dtype != v_host.dtype:
        raise ValueError("q_host, k_host and v_host must share a dtype")
    if chunk < 1:
        raise ValueError("chunk must be >= 1")
    dev = torch.device(device) if device is not None else wq.device
    if dev.type != "cuda":
        raise ValueError("the router weights must live on a CUDA device")
    code = _lib.dtype_code(q_host)
    r = wq.shape[0]
    if wq.shape != (r, D) or wk.shape != (r, D):
        raise ValueError(f"projection weights must be ({r}, {D}); got {tuple(wq.shape)}, {tuple(wk.shape)}")
    if pos_bias.numel() != 2 * seq_len:
        raise ValueError(f"pos_bias has {pos_bias.numel()} entries, expected 2*seq_len = {2 * seq_len}")
    if top_k < 1:
        raise ValueError(f"top_k must be >= 1, got {top_k}")
    if B == 0:
        return out_host
    wqc = wq.detach().to(dev, torch.float32).contiguous()
    wkc = wk.detach().to(dev, torch.float32).contiguous()
    pbc = pos_bias.detach().to(dev, torch.float32).contiguous()
    L = _lib.lib()
    c = min(chunk, B)
    key = (dev.index if dev.index is not None else torch.cuda.current_device(), tuple(q_host.shape),
           tuple(k_host.shape), q_host.dtype, c, int(top_k), r)
    buf = _buffers.get(key)
    if buf is None:
        with torch.cuda.device(dev):
            buf = _buffers[key] = _ChunkBuffers(dev, (c, H, N, D), (c, Hkv, N, D), q_host.dtype, int(top_k),
                                                L.ossa_router_workspace_size(c, H, Hkv, N, r, int(top_k)))
    caller = torch.cuda.current_stream(dev)
    s_in, s_comp, s_out = _pipeline_streams(dev)
    # work queued on the caller's stream before this call comes first
    s_in.wait_stream(caller)
    s_comp.wait_stream(caller)
    s_out.wait_stream(caller)
    scale = float(1.0 / math.sqrt(D))
    for i, b0 in enumerate(range(0, B, c)):
        b1 = min(B, b0 + c)
        n, par = b1 - b0, i & 1
        qd, kd, vd = buf.q[par][:n], buf.k[par][:n], buf.v[par][:n]
        idx, out = buf.idx[par][:n], buf.out[par][:n]
        s_in.wait_event(buf.comp_done[par])  # chunk i - 2 no longer reads these inputs
        with torch.cuda.stream(s_in):
            qd.copy_(q_host[b0:b1], non_blocking=True)
            kd.copy_(k_host[b0:b1], non_blocking=True)
            vd.copy_(v_host[b0:b1], non_blocking=True)
        buf.in_done[par].record(s_in)
        s_comp.wait_event(buf.in_done[par])
        s_comp.wait_event(buf.out_done[par])  # chunk i - 2's output has been copied out
        with torch.cuda.device(dev):
            _lib.check(L.ossa_router_topk(qd.data_ptr(), kd.data_ptr(), code, wqc.data_ptr(), wkc.data_ptr(),
                                          pbc.data_ptr(), n, H, Hkv, N, D, r, int(seq_len), int(top_k),
                                          1 if causal else 0, idx.data_ptr(), buf.ws[par].data_ptr(),
                                          buf.ws_bytes, s_comp.cuda_stream))
            _lib.check(L.ossa_topk_attention_fwd(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), idx.data_ptr(), 0,
                                                 code, n, H, Hkv, N, D, int(top_k), scale,
                                                 1 if causal else 0, out.data_ptr(), s_comp.cuda_stream))
        buf.comp_done[par].record(s_comp)
        s_out.wait_event(buf.comp_done[par])
        with torch.cuda.stream(s_out):
            out_host[b0:b1].copy_(out, non_blocking=True)
        buf.out_done[par].record(s_out)
    caller.wait_stream(s_out)
    return out_host
