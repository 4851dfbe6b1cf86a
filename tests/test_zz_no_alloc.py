"""The allocation-free router selection entry point (ossa_router_topk_noalloc).

Some callers cannot allocate device memory where they launch this work: a host
framework that owns every byte of device memory and forbids allocation while
enqueueing (an inference-server plugin, for instance), or an FFI caller with no
device allocator.  ossa_router_topk_noalloc serves them from a fixed scratch
array inside the library.  This test calls it through the C ABI twice in a row
(the second call reuses the array and its leftover contents) and checks each
result against ossa_router_topk with a caller-provided workspace.  Indices are
integers, so the tolerance is exact equality, as in the other selection tests.

The file sorts last so a run that stops at the first failure has already run
every other test; it also passes when run alone in a fresh process.
"""

import ctypes
import math

import pytest
import torch

import cases
from ossa_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _inputs(seed, B=1, H=12, Hkv=2, N=1024, D=128, r=64):
    q, k, _ = cases.qkv(B, H, Hkv, N, D, seed=seed, scale=1.0 / math.sqrt(D))
    wq, wk, pb = cases.router_weights(D, r, N, seed=seed + 3)
    return (q.bfloat16().to(DEV), k.bfloat16().to(DEV), wq.to(DEV), wk.to(DEV), pb.to(DEV))


def _with_workspace(q, k, wq, wk, pb, K):
    L = _lib.lib()
    B, H, N, D = q.shape
    Hkv, r = k.shape[1], wq.shape[0]
    out = torch.empty(B, H, N, K, dtype=torch.int32, device=DEV)
    ws_bytes = L.ossa_router_workspace_size(B, H, Hkv, N, r, K)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
    _lib.check(L.ossa_router_topk(q.data_ptr(), k.data_ptr(), _lib.OSSA_BF16, wq.data_ptr(), wk.data_ptr(),
                                  pb.data_ptr(), B, H, Hkv, N, D, r, N, K, 1, out.data_ptr(), ws.data_ptr(),
                                  ws_bytes, _lib.stream_ptr(q.device)))
    return out


def _no_alloc(q, k, wq, wk, pb, K):
    L = _lib.lib()
    B, H, N, D = q.shape
    Hkv, r = k.shape[1], wq.shape[0]
    out = torch.full((B, H, N, K), -7, dtype=torch.int32, device=DEV)
    _lib.check(L.ossa_router_topk_noalloc(q.data_ptr(), k.data_ptr(), _lib.OSSA_BF16, wq.data_ptr(),
                                          wk.data_ptr(), pb.data_ptr(), B, H, Hkv, N, D, r, N, K, 1,
                                          out.data_ptr(), _lib.stream_ptr(q.device)))
    return out


def _status():
    fb, st = ctypes.c_int(-1), ctypes.c_int(-1)
    _lib.check(_lib.lib().ossa_router_status_noalloc(ctypes.byref(fb), ctypes.byref(st)))
    return fb.value, st.value


def test_no_alloc_matches_workspace_entry_point_twice():
    K = 64
    first = _inputs(seed=101)
    second = _inputs(seed=202, N=1500)  # different shape: leftover scratch contents must not leak in
    a1 = _no_alloc(*first, K)
    a2 = _no_alloc(*second, K)
    torch.cuda.synchronize()
    b1 = _with_workspace(*first, K)
    b2 = _with_workspace(*second, K)
    torch.cuda.synchronize()
    assert torch.equal(a1, b1)
    assert torch.equal(a2, b2)
    # and once more on the first inputs after the second call used the scratch
    assert torch.equal(_no_alloc(*first, K), b1)
    torch.cuda.synchronize()
    assert _status()[1] == 0  # no bounded device wait expired


@pytest.mark.parametrize("K,N,exact", [
    (128, 512, False),   # 64 < K <= 128: candidate lists and final choice in the scratch
    (64, 40, False),     # fewer than 128 query rows per head group: CUDA-core selector
    (64, 700, True),     # the exact CUDA-core selector forced, after tensor-core calls left their data
])
def test_no_alloc_other_selector_paths(K, N, exact, monkeypatch):
    """The other selection paths through the shared scratch, each checked against the
    workspace entry point on two calls in a row, with the counters read back."""
    if exact:
        monkeypatch.setenv("OSSA_ROUTER_SELECT", "exact")
    x = _inputs(seed=300 + K + N, N=N)
    ref = _with_workspace(*x, K)
    for _ in range(2):
        assert torch.equal(_no_alloc(*x, K), ref)
        torch.cuda.synchronize()
        assert _status()[1] == 0


def test_no_alloc_allocates_nothing():
    """Free device memory is unchanged across calls once the output exists (after a
    warm-up call, which may load kernels)."""
    K = 64
    x = _inputs(seed=404, N=2048)
    out = torch.empty(1, 12, 2048, K, dtype=torch.int32, device=DEV)
    L = _lib.lib()

    def call():
        q, k, wq, wk, pb = x
        _lib.check(L.ossa_router_topk_noalloc(q.data_ptr(), k.data_ptr(), _lib.OSSA_BF16, wq.data_ptr(),
                                              wk.data_ptr(), pb.data_ptr(), 1, 12, 2, 2048, 128, 64, 2048, K, 1,
                                              out.data_ptr(), _lib.stream_ptr(q.device)))

    call()
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        call()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert torch.equal(out, _with_workspace(*x, K))


def test_no_alloc_rejects_shapes_beyond_its_scratch():
    L = _lib.lib()
    B, H, Hkv, N, D, r, K = 8, 12, 2, 4096, 128, 64, 64
    assert L.ossa_router_workspace_size(B, H, Hkv, N, r, K) > 32 << 20
    null = 16  # never dereferenced: the size check comes first
    st = L.ossa_router_topk_noalloc(null, null, _lib.OSSA_BF16, null, null, null, B, H, Hkv, N, D, r, N, K, 1,
                                    null, None)
    assert st == _lib.OSSA_ERR_WORKSPACE
    assert "built-in scratch" in L.ossa_last_error_string().decode()
