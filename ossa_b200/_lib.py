"""ctypes binding of libossa_b200.so (the C ABI declared in include/ossa_b200.h).

The library is required: there is no CPU or eager-PyTorch fallback.  If it is
missing it is built from ``csrc/`` with nvcc; if that is impossible every entry
point raises.
"""

from __future__ import annotations

import ctypes
import threading

import torch

from . import build as _build

OSSA_OK = 0
OSSA_ERR_INVALID = 1
OSSA_ERR_CUDA = 2
OSSA_ERR_WORKSPACE = 3
OSSA_ERR_UNSUPPORTED = 4

OSSA_F32 = 0
OSSA_BF16 = 1

EXPORTED = (
    "ossa_version",
    "ossa_last_error_string",
    "ossa_launch_count",
    "ossa_topk_attention_fwd",
    "ossa_router_workspace_size",
    "ossa_router_topk",
    "ossa_router_topk_sorted",
    "ossa_router_status",
    "ossa_router_score",
    "ossa_oracle_topk",
    "ossa_router_topk_noalloc",
    "ossa_router_status_noalloc",
    "ossa_topk_attention_fwd_rows",
    "ossa_router_workspace_size_rows",
    "ossa_router_topk_rows",
    "ossa_oracle_workspace_size",
    "ossa_oracle_topk_ws",
    "ossa_rope_to_heads",
    "ossa_router_distill_workspace_size",
    "ossa_router_distill_grad",
    "ossa_router_workspace_size_kp",
    "ossa_router_project_keys",
    "ossa_router_topk_rows_kp",
)

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class OssaError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"ossa_b200 error {status}: {message}")
        self.status = status


def _declare(lib: ctypes.CDLL) -> None:
    vp, ci, cf, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
    lib.ossa_version.argtypes = []
    lib.ossa_version.restype = ctypes.c_char_p
    lib.ossa_last_error_string.argtypes = []
    lib.ossa_last_error_string.restype = ctypes.c_char_p
    lib.ossa_launch_count.argtypes = []
    lib.ossa_launch_count.restype = ctypes.c_uint64
    lib.ossa_topk_attention_fwd.argtypes = [vp, vp, vp, vp, ci, ci, ci, ci, ci, ci, ci, ci, cf, ci, vp, vp]
    lib.ossa_topk_attention_fwd.restype = ci
    lib.ossa_router_workspace_size.argtypes = [ci, ci, ci, ci, ci, ci]
    lib.ossa_router_workspace_size.restype = sz
    lib.ossa_router_topk.argtypes = [vp, vp, ci, vp, vp, vp, ci, ci, ci, ci, ci, ci, ci, ci, ci, vp, vp, sz, vp]
    lib.ossa_router_topk.restype = ci
    lib.ossa_router_topk_sorted.argtypes = [vp, vp, ci, vp, vp, vp, ci, ci, ci, ci, ci, ci, ci, ci, ci, vp, vp, sz, vp]
    lib.ossa_router_topk_sorted.restype = ci
    lib.ossa_router_status.argtypes = [vp, ctypes.POINTER(ci), ctypes.POINTER(ci)]
    lib.ossa_router_status.restype = ci
    lib.ossa_router_score.argtypes = [vp, vp, ci, vp, vp, vp, ci, ci, ci, ci, ci, ci, ci, vp, vp, sz, vp]
    lib.ossa_router_score.restype = ci
    lib.ossa_oracle_topk.argtypes = [vp, vp, ci, ci, ci, ci, ci, ci, cf, ci, ci, vp, vp]
    lib.ossa_oracle_topk.restype = ci
    lib.ossa_router_topk_noalloc.argtypes = [vp, vp, ci, vp, vp, vp, ci, ci, ci, ci, ci, ci, ci, ci, ci, vp, vp]
    lib.ossa_router_topk_noalloc.restype = ci
    lib.ossa_router_status_noalloc.argtypes = [ctypes.POINTER(ci), ctypes.POINTER(ci)]
    lib.ossa_router_status_noalloc.restype = ci
    lib.ossa_topk_attention_fwd_rows.argtypes = [vp, vp, vp, vp] + [ci] * 9 + [cf, ci, ci, vp, vp]
    lib.ossa_topk_attention_fwd_rows.restype = ci
    lib.ossa_router_workspace_size_rows.argtypes = [ci] * 7
    lib.ossa_router_workspace_size_rows.restype = sz
    lib.ossa_router_topk_rows.argtypes = [vp, vp, ci, vp, vp, vp] + [ci] * 11 + [vp, vp, sz, vp]
    lib.ossa_router_topk_rows.restype = ci
    lib.ossa_oracle_workspace_size.argtypes = [ci] * 7
    lib.ossa_oracle_workspace_size.restype = sz
    lib.ossa_oracle_topk_ws.argtypes = [vp, vp, ci, ci, ci, ci, ci, ci, cf, ci, ci, vp, vp, sz, vp]
    lib.ossa_oracle_topk_ws.restype = ci
    lib.ossa_rope_to_heads.argtypes = [vp, vp, vp, ci, ci, ci, ci, ci, ci, vp, vp]
    lib.ossa_rope_to_heads.restype = ci
    lib.ossa_router_distill_workspace_size.argtypes = [ci] * 5
    lib.ossa_router_distill_workspace_size.restype = sz
    lib.ossa_router_distill_grad.argtypes = [vp, vp, ci, vp, vp, vp] + [ci] * 7 + [vp, ci, vp, vp, vp, vp, vp, sz, vp]
    lib.ossa_router_distill_grad.restype = ci
    lib.ossa_router_workspace_size_kp.argtypes = [ci] * 7
    lib.ossa_router_workspace_size_kp.restype = sz
    lib.ossa_router_project_keys.argtypes = [vp, ci, vp, ctypes.c_longlong, ci, ci, vp, vp]
    lib.ossa_router_project_keys.restype = ci
    lib.ossa_router_topk_rows_kp.argtypes = [vp, ci, vp, vp, vp] + [ci] * 11 + [vp, vp, sz, vp]
    lib.ossa_router_topk_rows_kp.restype = ci


def lib() -> ctypes.CDLL:
    """The loaded library (built on first use when missing or out of date)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = _build.LIB_PATH
            if not path.exists() or _build.is_stale():
                try:
                    path = _build.build()
                except Exception as e:  # no silent fallback: surface why
                    if not path.exists():
                        raise RuntimeError(f"libossa_b200.so is missing and could not be built: {e}") from e
            l = ctypes.CDLL(str(path))
            _declare(l)
            _lib = l
    return _lib


def check(status: int) -> None:
    if status != OSSA_OK:
        msg = lib().ossa_last_error_string().decode(errors="replace")
        raise OssaError(status, msg)


def launch_count() -> int:
    """Kernels libossa_b200 has launched in this process."""
    return int(lib().ossa_launch_count())


def version() -> str:
    return lib().ossa_version().decode()


def dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return OSSA_F32
    if t.dtype == torch.bfloat16:
        return OSSA_BF16
    raise TypeError(f"ossa_b200 kernels take float32 or bfloat16 tensors, got {t.dtype}")


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def require_cuda(*ts: torch.Tensor) -> torch.device:
    dev = None
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError(
                "ossa_b200 runs on CUDA tensors only (sm_100a kernels; there is no CPU path); "
                f"got a tensor on {t.device}")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors are on different devices: {dev} and {t.device}")
    return dev
