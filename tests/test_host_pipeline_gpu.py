"""Host-buffer entry point (ossa_b200.host_pipeline): the chunked three-stream
pipeline returns exactly what the device-tensor API returns for the same
inputs, for ragged chunking and GQA."""

import pytest
import torch

from ossa_b200 import router_topk, topk_attention
from ossa_b200.host_pipeline import routed_attention_from_host

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.mark.parametrize("B,chunk,groups,edge", [(3, 2, 1, 1), (4, 1, 1, 1), (2, 5, 1, 1), (3, 1, 2, 1),
                                               (4, 1, 1, 2), (1, 1, 1, 2)])
def test_host_pipeline_matches_device_path(B, chunk, groups, edge):
    """groups = 2: each batch element moves as two slices of one GQA group each;
    edge = 2: only the first and the last batch element do."""
    H, Hkv, N, D, r, K, L = 4, 2, 384, 128, 64, 32, 512
    g = torch.Generator().manual_seed(B * 10 + chunk + groups + 5 * edge)
    s = D ** -0.5
    q = (torch.randn(B, H, N, D, generator=g) * s).bfloat16().pin_memory()
    k = (torch.randn(B, Hkv, N, D, generator=g) * s).bfloat16().pin_memory()
    v = (torch.randn(B, Hkv, N, D, generator=g) * s).bfloat16().pin_memory()
    wq = (torch.randn(r, D, generator=g) * 0.1).to(DEV)
    wk = (torch.randn(r, D, generator=g) * 0.1).to(DEV)
    pb = torch.randn(2 * L, 1, generator=g).to(DEV)
    out_h = torch.empty_like(q).pin_memory()
    routed_attention_from_host(q, k, v, wq, wk, pb, L, K, out_h, chunk=chunk, groups=groups, edge_groups=edge)
    torch.cuda.current_stream().synchronize()
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    idx = router_topk(qd, kd, wq, wk, pb, L, K)
    ref = topk_attention(qd, kd, vd, topk_indices=idx, causal=True).cpu()
    assert torch.equal(out_h, ref)


def test_host_pipeline_reuses_buffers_across_calls():
    """Back-to-back calls on one shape (buffers kept from the first call, no host
    synchronisation between calls) each return their own inputs' result, and the
    later calls allocate no device memory."""
    B, H, Hkv, N, D, r, K, L, chunk = 5, 4, 2, 256, 128, 64, 32, 256, 2
    g = torch.Generator().manual_seed(7)
    s = D ** -0.5
    wq = (torch.randn(r, D, generator=g) * 0.1).to(DEV)
    wk = (torch.randn(r, D, generator=g) * 0.1).to(DEV)
    pb = torch.randn(2 * L, 1, generator=g).to(DEV)
    inputs = [tuple((torch.randn(B, h, N, D, generator=g) * s).bfloat16().pin_memory() for h in (H, Hkv, Hkv))
              for _ in range(3)]
    outs = [torch.empty(B, H, N, D, dtype=torch.bfloat16).pin_memory() for _ in range(3)]
    routed_attention_from_host(*inputs[0], wq, wk, pb, L, K, outs[0], chunk=chunk)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for (q, k, v), o in zip(inputs, outs):
        routed_attention_from_host(q, k, v, wq, wk, pb, L, K, o, chunk=chunk)
    torch.cuda.current_stream().synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    for (q, k, v), o in zip(inputs, outs):
        qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
        idx = router_topk(qd, kd, wq, wk, pb, L, K)
        assert torch.equal(o, topk_attention(qd, kd, vd, topk_indices=idx, causal=True).cpu())
