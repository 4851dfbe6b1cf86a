"""The error bound behind the selector's tensor-core query operand (router_qtc.cu).

The operand kernel computes q'_tc = x W^T on the tensor cores from bf16 x and W
split into bf16 hi + lo parts, with fp32 accumulation, and widens the selector's
row bounds by eps = gamma |x| |W|_F, gamma = 2^-14 + 2^-16 + 2^-17, which must
cover |q'_tc - q'| where q' is the canonical fp32 fmaf chain over d = 0..127 (the
oracle's arithmetic, which the selection is exact against).  The tensor core's
accumulation order and rounding are not specified, so this CPU test emulates
pessimistic forms of it: every product exact (bf16 x bf16), the 256 products
added in a random order with round-toward-zero fp32 additions, or in blocks of 16
summed exactly and truncated once (a wide internal adder), and checks, per output,
|q'_tc,c - q'_c| <= gamma sum_d |x_d w_cd| and, per row, |q'_tc - q'| <= eps, on
random rows, rows built to cancel (q' tiny against sum |x w|) and rows whose
entries span many binades.  No GPU is involved.
"""

import numpy as np
import pytest

GAMMA = 2.0**-14 + 2.0**-16 + 2.0**-17


def bf16(a):
    """float32 -> bfloat16 (round to nearest even) -> float32."""
    u = np.asarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def canonical(x, w):
    """fmaf chain per output from 0.0f, d = 0..127: the exact product plus the
    running sum, rounded once to float32 (float64 holds the product exactly)."""
    acc = np.zeros(w.shape[0], dtype=np.float32)
    for d in range(x.shape[0]):
        acc = (acc.astype(np.float64) + np.float64(x[d]) * w[:, d].astype(np.float64)).astype(np.float32)
    return acc


def rz(s):
    """float64 values -> float32 rounded toward zero."""
    f = s.astype(np.float32)
    over = np.abs(f.astype(np.float64)) > np.abs(s)
    f[over] = np.nextafter(f[over], np.float32(0))
    return f


def tensor_core(x, whi, wlo, rng, block):
    """Products of bf16 x with W hi and lo (exact in float32), summed per output in
    one random order: one by one with truncating fp32 adds (block = 1), or in
    blocks summed exactly and truncated once before the truncating add."""
    terms = np.concatenate([x[None, :] * whi, x[None, :] * wlo], axis=1).astype(np.float64)  # (64, 256)
    terms = terms[:, rng.permutation(terms.shape[1])]
    acc = np.zeros(terms.shape[0], dtype=np.float32)
    for b0 in range(0, terms.shape[1], block):
        part = rz(terms[:, b0:b0 + block].sum(axis=1)) if block > 1 else terms[:, b0].astype(np.float32)
        acc = rz(acc.astype(np.float64) + part.astype(np.float64))
    return acc


def _weights(rng):
    a = np.sqrt(6.0 / (64 + 128))
    w = rng.uniform(-a, a, size=(64, 128)).astype(np.float32)
    whi = bf16(w)
    wlo = bf16(w - whi)
    return w, whi, wlo


def _rows(kind, w, rng, n):
    if kind == "random":
        return [bf16(rng.standard_normal(128) * 0.09) for _ in range(n)]
    if kind == "cancelling":
        # x nearly orthogonal to the first 48 rows of W: q' small against sum |x w|
        basis = np.linalg.qr(w[:48].T.astype(np.float64))[0]
        out = []
        for _ in range(n):
            v = rng.standard_normal(128)
            v -= basis @ (basis.T @ v)
            out.append(bf16(v * 3.0))
        return out
    # entries spanning many binades, mixed signs
    return [bf16(rng.choice([-1.0, 1.0], 128) * 2.0 ** rng.uniform(-20, 10, 128)) for _ in range(n)]


@pytest.mark.parametrize("kind", ["random", "cancelling", "wide_range"])
@pytest.mark.parametrize("block", [1, 16])
def test_tensor_core_query_operand_error_bound(kind, block):
    rng = np.random.default_rng({"random": 1, "cancelling": 2, "wide_range": 3}[kind] * 10 + block)
    w, whi, wlo = _weights(rng)
    wf = float(np.sqrt((w.astype(np.float64) ** 2).sum()))
    worst_c, worst_row = 0.0, 0.0
    for x in _rows(kind, w, rng, 24):
        ref = canonical(x, w).astype(np.float64)
        tc = tensor_core(x, whi, wlo, rng, block).astype(np.float64)
        diff = np.abs(tc - ref)
        s = np.abs(x.astype(np.float64))[None, :] @ np.abs(w.astype(np.float64)).T  # sum_d |x_d w_cd|
        bound_c = GAMMA * s[0]
        assert (diff <= bound_c).all(), f"{kind}: output error {diff.max():.3g} above gamma sum|x w|"
        eps = GAMMA * float(np.linalg.norm(x.astype(np.float64))) * wf
        assert np.linalg.norm(diff) <= eps, f"{kind}: row error {np.linalg.norm(diff):.3g} above eps {eps:.3g}"
        worst_c = max(worst_c, float((diff / np.maximum(bound_c, 1e-300)).max()))
        worst_row = max(worst_row, float(np.linalg.norm(diff) / eps))
    # the margin the bound keeps over these emulations (informative; the asserts above decide)
    assert worst_c < 1.0 and worst_row < 1.0
