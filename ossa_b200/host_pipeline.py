"""Routed sparse attention over host-resident tensors, with PCIe transfers
overlapped with the kernels.

A serving process that holds q/k/v in pinned host memory would otherwise run
copy-in, selection + gather, and copy-out back to back.  Here the batch is cut
into chunks of batch elements (or, with ``groups``, of kv-head groups of one
batch element) and each chunk moves through three CUDA streams:

    copy-in stream      : q, k, v of chunk c        (host -> device)
    compute streams     : router_topk + topk_attention of chunk c (one stream per
                          buffer set, so the kernels of consecutive chunks
                          overlap on the GPU: a chunk of one batch element is too
                          small to fill it)
    copy-out stream     : attention output of chunk c (device -> host)

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

# Device buffer sets the chunks rotate through (chunk c uses set c % _NBUF): the
# copy-in can run up to _NBUF chunks ahead of the copy-out.
_NBUF = 3
# The pipeline's streams (copy-in, one compute stream per buffer set, copy-out),
# created once per device and reused by every call.
_streams: dict = {}
# Device buffers of the pipeline, one set per (device, shapes, dtype, chunk, K):
# allocated on the first call of a shape and reused, so a call allocates nothing.
_buffers: dict = {}


def _pipeline_streams(dev: torch.device):
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    st = _streams.get(key)
    if st is None:
        st = _streams[key] = (torch.cuda.Stream(dev), tuple(torch.cuda.Stream(dev) for _ in range(_NBUF)),
                              torch.cuda.Stream(dev))
    return st


class _ChunkBuffers:
    """_NBUF sets of device buffers for one chunk of batch elements: q, k, v,
    indices, output and selector workspace, plus the events that order their
    reuse: chunk c + _NBUF copies in only after chunk c's kernels are done with
    its inputs, and chunk c + _NBUF's kernels write only after chunk c's output
    has been copied out."""

    def __init__(self, dev, q_shape, k_shape, dtype, top_k, ws_bytes):
        self.q = [torch.empty(q_shape, dtype=dtype, device=dev) for _ in range(_NBUF)]
        self.k = [torch.empty(k_shape, dtype=dtype, device=dev) for _ in range(_NBUF)]
        self.v = [torch.empty(k_shape, dtype=dtype, device=dev) for _ in range(_NBUF)]
        self.idx = [torch.empty(q_shape[:3] + (top_k,), dtype=torch.int32, device=dev) for _ in range(_NBUF)]
        self.out = [torch.empty(q_shape, dtype=dtype, device=dev) for _ in range(_NBUF)]
        self.ws = [torch.empty(ws_bytes, dtype=torch.uint8, device=dev) for _ in range(_NBUF)]
        self.ws_bytes = ws_bytes
        self.in_done = [torch.cuda.Event() for _ in range(_NBUF)]
        self.comp_done = [torch.cuda.Event() for _ in range(_NBUF)]
        self.out_done = [torch.cuda.Event() for _ in range(_NBUF)]


def release_pipeline_buffers() -> None:
    """Drops the device buffers kept for the shapes seen so far."""
    _buffers.clear()


def routed_attention_from_host(q_host, k_host, v_host, wq, wk, pos_bias, seq_len: int, top_k: int,
                               out_host, *, causal: bool = True, chunk: int = 2, groups: int = 1,
                               edge_groups: int = 1, device=None):
    """ContentRouter selection + gathered sparse attention for host tensors.

    ``q_host`` (B, H, N, D), ``k_host``/``v_host`` (B, Hkv, N, D) and ``out_host``
    (B, H, N, D) are CPU tensors, pinned for the copies to be asynchronous, float32
    or bfloat16; ``wq``, ``wk`` (r, D) and ``pos_bias`` (2*seq_len, 1) are device
    tensors.  Semantics per batch element are those of ``router_topk`` followed by
    ``topk_attention(..., causal=causal)``.  ``chunk`` batch elements move
    through the pipeline at a time; with ``chunk=1``, ``groups`` > 1 cuts each batch
    element into that many slices of whole GQA groups (``groups`` divides the kv
    head count; a slice is contiguous in the (B, heads, N, D) layouts), which halves
    or better the copy-in before the first kernels and the copy-out after the last
    ones; ``edge_groups`` > 1 slices only the first and the last batch element that
    way (the chunks between keep whole elements, whose kernels use the GPU better).
    The device buffers of a shape are allocated on its first call and kept for
    the next ones (``release_pipeline_buffers`` drops them).
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
    if groups < 1 or Hkv % groups != 0:
        raise ValueError(f"groups must divide the kv head count {Hkv}, got {groups}")
    if groups > 1 and chunk != 1:
        raise ValueError("groups > 1 needs chunk=1 (a slice of one batch element)")
    if edge_groups < 1 or Hkv % edge_groups != 0:
        raise ValueError(f"edge_groups must divide the kv head count {Hkv}, got {edge_groups}")
    if edge_groups > 1 and chunk != 1:
        raise ValueError("edge_groups > 1 needs chunk=1 (a slice of one batch element)")
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
    Hs, Hkvs = H // groups, Hkv // groups  # query and kv heads of the largest chunk (buffer shapes)
    key = (dev.index if dev.index is not None else torch.cuda.current_device(), tuple(q_host.shape),
           tuple(k_host.shape), q_host.dtype, c, groups, int(top_k), r)
    buf = _buffers.get(key)
    if buf is None:
        with torch.cuda.device(dev):
            buf = _buffers[key] = _ChunkBuffers(dev, (c, Hs, N, D), (c, Hkvs, N, D), q_host.dtype, int(top_k),
                                                L.ossa_router_workspace_size(c, Hs, Hkvs, N, r, int(top_k)))
    caller = torch.cuda.current_stream(dev)
    s_in, s_comps, s_out = _pipeline_streams(dev)
    # work queued on the caller's stream before this call comes first
    s_in.wait_stream(caller)
    for sc in s_comps:
        sc.wait_stream(caller)
        for t in (wqc, wkc, pbc):  # converted copies live until the compute streams are done
            t.record_stream(sc)
    s_out.wait_stream(caller)
    scale = float(1.0 / math.sqrt(D))
    # chunks: (first batch element, slices of it, slice index)
    units = []
    for b0 in range(0, B, c):
        ng = max(groups, edge_groups) if (b0 == 0 or b0 + c >= B) else groups
        units += [(b0, ng, gi) for gi in range(ng)]
    for i, (b0, ng, gi) in enumerate(units):
        b1 = min(B, b0 + c)
        n, par = b1 - b0, i % _NBUF
        hs, hks = H // ng, Hkv // ng
        hq = slice(gi * hs, (gi + 1) * hs)      # the chunk's query heads
        hk = slice(gi * hks, (gi + 1) * hks)    # and their kv heads
        # a slice uses the leading heads of the buffers (contiguous: n = 1 when ng > 1)
        qd, kd, vd = buf.q[par][:n, :hs], buf.k[par][:n, :hks], buf.v[par][:n, :hks]
        idx, out = buf.idx[par][:n, :hs], buf.out[par][:n, :hs]
        s_in.wait_event(buf.comp_done[par])  # chunk i - _NBUF no longer reads these inputs
        with torch.cuda.stream(s_in):
            qd.copy_(q_host[b0:b1, hq], non_blocking=True)
            kd.copy_(k_host[b0:b1, hk], non_blocking=True)
            vd.copy_(v_host[b0:b1, hk], non_blocking=True)
        buf.in_done[par].record(s_in)
        s_comp = s_comps[par]  # also orders chunk i after chunk i - _NBUF, which used the same buffers
        s_comp.wait_event(buf.in_done[par])
        s_comp.wait_event(buf.out_done[par])  # chunk i - _NBUF's output has been copied out
        with torch.cuda.device(dev):
            _lib.check(L.ossa_router_topk(qd.data_ptr(), kd.data_ptr(), code, wqc.data_ptr(), wkc.data_ptr(),
                                          pbc.data_ptr(), n, hs, hks, N, D, r, int(seq_len), int(top_k),
                                          1 if causal else 0, idx.data_ptr(), buf.ws[par].data_ptr(),
                                          buf.ws_bytes, s_comp.cuda_stream))
            _lib.check(L.ossa_topk_attention_fwd(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), idx.data_ptr(), 0,
                                                 code, n, hs, hks, N, D, int(top_k), scale,
                                                 1 if causal else 0, out.data_ptr(), s_comp.cuda_stream))
        buf.comp_done[par].record(s_comp)
        s_out.wait_event(buf.comp_done[par])
        with torch.cuda.stream(s_out):
            out_host[b0:b1, hq].copy_(out, non_blocking=True)
        buf.out_done[par].record(s_out)
    caller.wait_stream(s_out)
    return out_host
