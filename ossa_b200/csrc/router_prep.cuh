// Per-row preparation of the tensor-core selector's query operand, shared by the
// prep kernel that reads the canonical q' (router_tc.cu) and the tensor-core q
// projection that produces the operand straight from q (router_qtc.cu): the
// power-of-two scaling of the fp16 copy, the epilogue multiplier, the bound on
// |approximate score - canonical score| and the bound on (approximate score - bias
// term); and the canonical q' rows of single queries, for the rows that need them
// when only the tensor-core projection ran.
#pragma once

#include <cuda_bf16.h>

#include <cstdint>

#include "common.cuh"

namespace ossa {
namespace {

constexpr float kTwoPowM22 = 2.384185791015625e-07f;  // 2^-22

// Per (b, kv head) statistics, kStatWords words each: [0] max |k'| bits,
// [1] max_j |k'_j|_2 bits, [2] non-finite flag, [3] max_j |fp16(k'_j) - k'_j|_2 bits
// (the largest conversion error of a key row, written by kconvert_kernel).
constexpr int kStatWords = 4;

// Power-of-two exponent e with max_abs * 2^e in [2^12, 2^13).
__device__ __forceinline__ int scale_exponent(float max_abs) {
    int ex = 0;
    frexpf(max_abs, &ex);
    return max_abs > 0.f ? 13 - ex : 0;
}

// x * 2^e for the scalings above, with f = 2^e from pow2f: a multiply by the
// exact power of two when 2^e and 2^-e are normal floats (then the product equals
// ldexpf(x, e)), ldexpf otherwise.
__device__ __forceinline__ float pow2f(int e) {
    return (e > -126 && e < 127) ? __int_as_float((e + 127) << 23) : 0.f;
}
__device__ __forceinline__ float scale2(float x, int e, float f) { return f != 0.f ? x * f : ldexpf(x, e); }

// The row's multiplier m = scale * 2^-(eq + ek) and error bound delta into
// rowinfo[row], and rowub[row], from the row's exponent eq, a bound qn on |q'_row|
// (canonical), a bound dq on |q16_row / 2^eq - q'_row| and whether any value of the
// row is not finite.
template <int kD>
__device__ __forceinline__ void row_bounds_finish(long long row, int eq, float qn, float dq, bool bad, int bg,
                                                  float scale, const uint32_t* __restrict__ stats,
                                                  const uint32_t* __restrict__ gstats, float2* __restrict__ rowinfo,
                                                  float* __restrict__ rowub) {
    const int ek = scale_exponent(__uint_as_float(stats[kStatWords * bg + 0]));
    const float kmax = __uint_as_float(stats[kStatWords * bg + 1]);
    const float dkmax = __uint_as_float(stats[kStatWords * bg + 3]);
    const float bmax = __uint_as_float(gstats[0]);
    const bool nonfinite = bad || stats[kStatWords * bg + 2] != 0u || gstats[1] != 0u;
    const float m = ldexpf(scale, -(eq + ek));
    const float cross = scale * qn * kmax;
    // |approx - canonical| <= scale * |q'.dk + dq.k' + dq.dk| (fp16 conversion,
    // Cauchy-Schwarz with the measured errors) + scale * 2^-13 |q'| max|k'| (fp32
    // accumulation in the tensor core and in the canonical chain: 64 terms at a few
    // ulp each, twice that for 128) + 2^-22 (max|bias| + cross) (the final roundings)
    constexpr float kAcc = 1.220703125e-4f * (kD / 64);
    const float delta = scale * (qn * dkmax + dq * kmax + dq * dkmax) * 1.0001f + scale * kAcc * qn * kmax +
                        kTwoPowM22 * (bmax + cross) + 1e-30f;
    if (nonfinite || !isfinite(delta) || !(m >= 1.1754944e-38f) || !isfinite(m)) {
        rowinfo[row] = make_float2(__int_as_float(0x7fc00000), 0.f);  // NaN multiplier: exact fallback
        rowub[row] = INFINITY;
    } else {
        rowinfo[row] = make_float2(m, delta);
        // + max|bias| 2^-20: the final rounding of score + bias term, whatever the sign
        rowub[row] = (cross * 1.0001f + delta) * 1.0001f + bmax * 9.5367431640625e-07f;
    }
}

// The same from the canonical row itself: ss = sum of q'^2, dd = sum of the squared
// fp16 conversion errors in unscaled units.  Any summation order of ss and dd will
// do: both enter with a relative margin far above their rounding.
template <int kD>
__device__ __forceinline__ void row_finish(long long row, int eq, float ss, float dd, bool bad, int bg, float scale,
                                           const uint32_t* __restrict__ stats, const uint32_t* __restrict__ gstats,
                                           float2* __restrict__ rowinfo, float* __restrict__ rowub) {
    row_bounds_finish<kD>(row, eq, sqrtf(ss) * 1.0001f, sqrtf(dd) * 1.0001f, bad, bg, scale, stats, gstats, rowinfo,
                          rowub);
}

// Canonical q' of two query rows (bf16 x0, x1, 128 values each; x1 may repeat x0),
// the fmaf chain over d = 0..127 from 0.0f per output as in the projection kernels,
// computed by the 32 lanes of a warp (outputs 2 lane and 2 lane + 1) and stored to
// q0 and q1 (q1 null: one row).  The weights are Wq transposed in shared memory:
// wt_lo holds d = 0..63 and wt_hi d = 64..127, [d][64 c] each (256 bytes per d: one
// conflict-free 8-byte load per lane).  Lanes 0..15 load row x0 and lanes 16..31 row
// x1, 16 bytes each, and pass them around with shuffles.  The caller orders the
// stores before any read of the rows (__syncwarp, or the end of the kernel).
__device__ __forceinline__ void warp_canon_q2(const __nv_bfloat16* __restrict__ x0,
                                                   const __nv_bfloat16* __restrict__ x1, const float* wt_lo,
                                                   const float* wt_hi, float* q0, float* q1, int lane) {
    const uint4 xv = __ldg(reinterpret_cast<const uint4*>(lane < 16 ? x0 : x1) + (lane & 15));
    float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
#pragma unroll 4
    for (int c = 0; c < 16; ++c) {
        float xf[8], yf[8];
        unpack_bf16x2(__shfl_sync(kFull, xv.x, c), xf[0], xf[1]);
        unpack_bf16x2(__shfl_sync(kFull, xv.y, c), xf[2], xf[3]);
        unpack_bf16x2(__shfl_sync(kFull, xv.z, c), xf[4], xf[5]);
        unpack_bf16x2(__shfl_sync(kFull, xv.w, c), xf[6], xf[7]);
        unpack_bf16x2(__shfl_sync(kFull, xv.x, 16 + c), yf[0], yf[1]);
        unpack_bf16x2(__shfl_sync(kFull, xv.y, 16 + c), yf[2], yf[3]);
        unpack_bf16x2(__shfl_sync(kFull, xv.z, 16 + c), yf[4], yf[5]);
        unpack_bf16x2(__shfl_sync(kFull, xv.w, 16 + c), yf[6], yf[7]);
        const float* ws = (c < 8 ? wt_lo + c * 512 : wt_hi + (c - 8) * 512) + 2 * lane;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const float2 w = *reinterpret_cast<const float2*>(ws + u * 64);
            a0 = fmaf(xf[u], w.x, a0);
            a1 = fmaf(xf[u], w.y, a1);
            b0 = fmaf(yf[u], w.x, b0);
            b1 = fmaf(yf[u], w.y, b1);
        }
    }
    reinterpret_cast<float2*>(q0)[lane] = make_float2(a0, a1);
    if (q1 != nullptr) reinterpret_cast<float2*>(q1)[lane] = make_float2(b0, b1);
}

}  // namespace
}  // namespace ossa
