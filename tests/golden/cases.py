"""Deterministic input builders shared by the golden-fixture generator and tests.

Inputs are drawn on the CPU from ``torch.Generator`` seeds (bit-stable for a
given torch build), so fixtures only store seeds, weights that are not
derivable from a seed, and the reference's outputs.  Each fixture also stores
input checksums; tests refuse to compare when the regenerated inputs differ.
"""

from __future__ import annotations

import math

import numpy as np
import torch


def gen(seed: int) -> torch.Generator:
    g = torch.Generator()
    g.manual_seed(seed)
    return g


def randn(shape, seed: int, scale: float = 1.0) -> torch.Tensor:
    return torch.randn(*shape, generator=gen(seed), dtype=torch.float32) * scale


def xavier(r: int, d: int, seed: int) -> torch.Tensor:
    w = torch.empty(r, d, dtype=torch.float32)
    torch.nn.init.xavier_uniform_(w, generator=gen(seed))
    return w


def router_weights(d: int, r: int, seq_len: int, seed: int):
    """A random-init ContentRouter of the reference's shape: Xavier-uniform q/k
    projections (r, d) and an N(0, 1) pos_bias table (2*seq_len, 1)."""
    wq = xavier(r, d, seed)
    wk = xavier(r, d, seed + 1)
    pb = randn((2 * seq_len, 1), seed + 2)
    return wq, wk, pb


def qkv(B: int, H: int, Hkv: int, N: int, D: int, seed: int, scale: float = 1.0):
    q = randn((B, H, N, D), seed, scale)
    k = randn((B, Hkv, N, D), seed + 1, scale)
    v = randn((B, Hkv, N, D), seed + 2, scale)
    return q, k, v


def checksum(*ts) -> np.ndarray:
    return np.array([float(t.double().sum()) for t in ts] + [float(t.double().abs().sum()) for t in ts])


def c1_inputs():
    """The small single-layer CPU workload: B=1, 12 query / 2 kv heads, D=128, N=512, N(0,1)."""
    return qkv(1, 12, 2, 512, 128, seed=0)


def gqa_small_inputs():
    """Ragged GQA case: B=2, 6 query / 3 kv heads, N=200, D=64."""
    return qkv(2, 6, 3, 200, 64, seed=11)


def oracle_inputs():
    """Exact-dot selection case: B=1, 4 query / 2 kv heads, N=256, D=128."""
    return qkv(1, 4, 2, 256, 128, seed=21, scale=1.0 / math.sqrt(128))


def reference_test_inputs():
    """The reference tests' own shape (tests/test_sparse_attention.py:29-46)."""
    return qkv(1, 4, 4, 64, 16, seed=31)


def distill_inputs():
    """Router training case: B=1, 4 query / 2 kv heads, N=96, D=64, N(0,1)."""
    return qkv(1, 4, 2, 96, 64, seed=51)
