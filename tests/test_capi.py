"""C-ABI checks that need no GPU: the library loads, exports every function
declared in include/ossa_b200.h, and rejects bad requests before touching the
device (validation runs ahead of any CUDA call)."""

import ctypes
import re
import subprocess

import pytest

from ossa_b200 import _lib
from ossa_b200.build import INCLUDE, LIB_PATH


def _declared():
    text = (INCLUDE / "ossa_b200.h").read_text()
    return sorted(set(re.findall(r"OSSA_API\s+[\w\s\*]+?\b(ossa_\w+)\s*\(", text)))


def test_header_declares_every_binding():
    assert _declared() == sorted(_lib.EXPORTED)


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    for name in _declared():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (ossa_\w+)", out))
    assert set(_declared()) <= exported
    # nothing else leaks out of the shared object with default visibility
    assert exported == set(_declared())


def test_version_and_error_string():
    assert _lib.version() == "0.1.0"
    assert isinstance(_lib.lib().ossa_last_error_string(), bytes)


def _attn(**kw):
    a = dict(q=None, k=None, v=None, idx=None, idx_is_64=0, dtype=_lib.OSSA_BF16, B=1, H=12, Hkv=2, N=64,
             D=128, K=8, scale=0.1, causal=1, out=None, stream=None)
    a.update(kw)
    return _lib.lib().ossa_topk_attention_fwd(a["q"], a["k"], a["v"], a["idx"], a["idx_is_64"], a["dtype"],
                                              a["B"], a["H"], a["Hkv"], a["N"], a["D"], a["K"], a["scale"],
                                              a["causal"], a["out"], a["stream"])


def _err():
    return _lib.lib().ossa_last_error_string().decode()


@pytest.mark.parametrize("kw,code,msg", [
    (dict(H=12, Hkv=5), _lib.OSSA_ERR_INVALID, "multiple"),
    (dict(D=96), _lib.OSSA_ERR_UNSUPPORTED, "head_dim"),
    (dict(dtype=7), _lib.OSSA_ERR_INVALID, "dtype"),
    (dict(idx_is_64=2), _lib.OSSA_ERR_INVALID, "idx_is_64"),
    (dict(K=-1), _lib.OSSA_ERR_INVALID, "K"),
    (dict(scale=float("nan")), _lib.OSSA_ERR_INVALID, "scale"),
    (dict(), _lib.OSSA_ERR_INVALID, "null"),
    (dict(q=16, k=32, v=48, idx=64, out=72), _lib.OSSA_ERR_INVALID, "aligned"),
])
def test_attention_validation(kw, code, msg):
    assert _attn(**kw) == code
    assert msg in _err()


def test_attention_empty_is_ok():
    assert _attn(B=0) == _lib.OSSA_OK
    assert _attn(N=0) == _lib.OSSA_OK


def test_router_validation_and_workspace():
    L = _lib.lib()
    ws = L.ossa_router_workspace_size(8, 12, 2, 4096, 64, 64)
    # q' (B*H*N*r fp32) + k' (B*Hkv*N*r fp32), 256-byte aligned pieces
    assert ws >= 8 * 12 * 4096 * 64 * 4 + 8 * 2 * 4096 * 64 * 4
    args = [16, 16, _lib.OSSA_BF16, 16, 16, 16, 1, 12, 2, 64, 128, 64, 64, 64, 1, 16, None, 0, None]
    assert L.ossa_router_topk(*args) == _lib.OSSA_ERR_WORKSPACE
    assert "workspace" in _err()
    bad_r = list(args)
    bad_r[11] = 48
    assert L.ossa_router_topk(*bad_r) == _lib.OSSA_ERR_UNSUPPORTED
    big_k = list(args)
    big_k[13] = 4096
    big_k[16], big_k[17] = 256, ws
    assert L.ossa_router_topk(*big_k) == _lib.OSSA_ERR_UNSUPPORTED
    assert L.ossa_oracle_topk(16, 16, _lib.OSSA_BF16, 1, 12, 2, 64, 96, 0.1, 8, 1, 16, None) == \
        _lib.OSSA_ERR_UNSUPPORTED


def test_rope_key_cache_and_oracle_ws_validation():
    """The fused RoPE, the decode key-cache and the workspace oracle entry
    points reject bad requests before any CUDA call."""
    L = _lib.lib()
    bf, inv, ws_err, uns = _lib.OSSA_BF16, _lib.OSSA_ERR_INVALID, _lib.OSSA_ERR_WORKSPACE, _lib.OSSA_ERR_UNSUPPORTED
    # RoPE: D must be a multiple of 8; cos without sin; unaligned pointers
    assert L.ossa_rope_to_heads(16, 16, 16, 0, bf, 1, 4, 2, 12, 16, None) == inv
    assert L.ossa_rope_to_heads(16, 16, None, 0, bf, 1, 4, 2, 128, 16, None) == inv
    assert L.ossa_rope_to_heads(8, None, None, 0, bf, 1, 4, 2, 128, 16, None) == inv
    assert L.ossa_rope_to_heads(16, None, None, 0, 7, 1, 4, 2, 128, 16, None) == inv
    assert L.ossa_rope_to_heads(None, None, None, 0, bf, 0, 4, 2, 128, None, None) == _lib.OSSA_OK  # empty
    # key projection: unsupported r, null output
    assert L.ossa_router_project_keys(16, bf, 16, 10, 128, 48, 16, None) == uns
    assert L.ossa_router_project_keys(16, bf, 16, 10, 128, 64, None, None) == inv
    # selection against cached keys: its workspace has no k' region, and too small a one is refused
    full = L.ossa_router_workspace_size_rows(1, 12, 2, 1, 32768, 64, 64)
    kp_only = L.ossa_router_workspace_size_kp(1, 12, 2, 1, 32768, 64, 64)
    assert 0 < kp_only and full - kp_only >= 2 * 32768 * 64 * 4
    args = [16, bf, 16, 16, 16, 1, 12, 2, 1, 32768, 128, 64, 32768, 64, 1, 32767, 16, 16, 64, None]
    assert L.ossa_router_topk_rows_kp(*args) == ws_err
    # the workspace oracle: bad K and an undersized workspace
    n = L.ossa_oracle_workspace_size(1, 12, 2, 1024, 128, 64, bf)
    assert n > 256
    assert L.ossa_oracle_topk_ws(16, 16, bf, 1, 12, 2, 1024, 128, 0.088, 0, 1, 16, 16, n, None) == inv
    assert L.ossa_oracle_topk_ws(16, 16, bf, 1, 12, 2, 1024, 128, 0.088, 64, 1, 16, 16, n - 16, None) == ws_err
