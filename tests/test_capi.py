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
