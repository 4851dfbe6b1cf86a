// The tensor-core selector's query operand straight from the bf16 query rows
// (head_dim 128, proj_dim 64), for the router path (ossa/router.py:171-190: q' =
// q_proj(q)).  The selector scores with fp16 copies of q' and needs the canonical
// fp32 q' (the fmaf chain over d = 0..127) only for the rows whose top-K boundary is
// rescored or that go to the exact selector, a few per cent of the rows; those rows
// compute it themselves (warp_canon_q).  So this kernel reads q once and writes
// only what the selector reads for every row:
//
//  * q' = x W^T on the tensor cores (mma.sync m16n8k16, bf16 operands, fp32
//    accumulation) with W split into bf16 hi + lo parts (the products are exact;
//    the split leaves 2^-16 |w| per weight);
//  * the fp16 copy q16 scaled by the row's power of two (as the prep kernel), the
//    epilogue multiplier, and delta / rowub from bounds that cover the canonical
//    row: |q'| <= |q'_tc| + eps and |q16 / 2^eq - q'| <= |q16 / 2^eq - q'_tc| + eps,
//    with eps >= |q'_tc - q'| from |x| |W|_F (Cauchy-Schwarz per output).
//
// Each warp takes 16 rows and all 64 outputs.  A lane loads 16-byte pieces of its
// two rows (g and g + 8) straight from global memory (pieces t, t + 4, t + 8, t + 12:
// each load instruction covers 64 contiguous bytes of 16 rows), and the MMA's
// reduction index is permuted to match: k-step (m, h) gives lane t the elements
// 8 (t + 4m) + 4h + {0, 1} (k = 2t, 2t + 1) and + {2, 3} (k = 2t + 8, 2t + 9), the same
// permutation on the W side, where one 16-byte shared-memory load brings a lane's
// B fragments of two k-steps (W rows at a 320-byte pitch: conflict-free).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdint>

#include "common.cuh"
#include "kernels.h"
#include "router_prep.cuh"

namespace ossa {
namespace {

constexpr int kQtThreads = 256;
constexpr int kQtWarps = kQtThreads / 32;
constexpr int kQtPitch = 160;  // bf16 per staged W row (320 bytes)

// eps per output, relative to sum_d |x_d w_cd|: 2^-16 from the hi/lo split, 2^-14 for
// the tensor core's fp32 accumulation of the 256 exact products (a few ulp per
// step: below 2^-16 of the sum, taken with a 4x margin), 2^-17 for the canonical
// chain's 128 roundings.
constexpr float kQtGamma = 6.103515625e-05f + 1.52587890625e-05f + 7.62939453125e-06f;

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float sum_sq_bf16x8(const uint4& v, float acc) {
    float f[8];
    unpack_bf16x2(v.x, f[0], f[1]);
    unpack_bf16x2(v.y, f[2], f[3]);
    unpack_bf16x2(v.z, f[4], f[5]);
    unpack_bf16x2(v.w, f[6], f[7]);
#pragma unroll
    for (int u = 0; u < 8; ++u) acc = fmaf(f[u], f[u], acc);
    return acc;
}

__global__ void __launch_bounds__(kQtThreads, 2) qproj_tc_kernel(const QPrepArgs p) {
    __shared__ __align__(16) __nv_bfloat16 whi[64 * kQtPitch];
    __shared__ __align__(16) __nv_bfloat16 wlo[64 * kQtPitch];
    __shared__ float wred[kQtWarps];
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    float wss = 0.f;
    for (int e = tid; e < 64 * 128; e += kQtThreads) {
        const int c = e >> 7, d = e & 127;
        const float v = __ldg(p.w + e);
        const __nv_bfloat16 h = __float2bfloat16_rn(v);
        whi[c * kQtPitch + d] = h;
        if (blockIdx.x == 0) p.wt[d * 64 + c] = v;
        wlo[c * kQtPitch + d] = __float2bfloat16_rn(v - __bfloat162float(h));  // v - h is exact
        wss = fmaf(v, v, wss);
    }
    wss = warp_sum(wss);
    if (lane == 0) wred[warp] = wss;
    __syncthreads();
    float wf = 0.f;
#pragma unroll
    for (int u = 0; u < kQtWarps; ++u) wf += wred[u];
    wf = sqrtf(wf) * 1.001f;  // >= |W|_F

    const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(p.x);
    __half* q16 = static_cast<__half*>(p.q16);
    const long long ntile = (p.rows + 15) >> 4;
    const long long stride = (long long)gridDim.x * kQtWarps;
    // x pieces of the warp's current tile; piece m of the next tile is loaded as
    // soon as the MMAs of piece m are issued
    uint4 xa[4], xb[4];
    auto load_piece = [&](long long tile, int m, uint4& a, uint4& b) {
        const long long r = tile * 16 + g;
        const uint4 z = make_uint4(0u, 0u, 0u, 0u);
        a = (tile < ntile && r < p.rows) ? __ldg(reinterpret_cast<const uint4*>(x + r * 128 + 8 * (t + 4 * m))) : z;
        b = (tile < ntile && r + 8 < p.rows)
                ? __ldg(reinterpret_cast<const uint4*>(x + (r + 8) * 128 + 8 * (t + 4 * m)))
                : z;
    };
    long long wt = (long long)blockIdx.x * kQtWarps + warp;
#pragma unroll
    for (int m = 0; m < 4; ++m) load_piece(wt, m, xa[m], xb[m]);
    for (; wt < ntile; wt += stride) {
        const long long ra = wt * 16 + g, rb = ra + 8;
        const bool va = ra < p.rows, vb = rb < p.rows;
        float xsa = 0.f, xsb = 0.f;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            xsa = sum_sq_bf16x8(xa[m], xsa);
            xsb = sum_sq_bf16x8(xb[m], xsb);
        }
        float acc[8][4];
#pragma unroll
        for (int n = 0; n < 8; ++n)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[n][c] = 0.f;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
#pragma unroll
            for (int part = 0; part < 2; ++part) {  // W hi, then W lo: 8 independent accumulators per pass
                const __nv_bfloat16* ws = part == 0 ? whi : wlo;
                uint4 bw[8];
#pragma unroll
                for (int n = 0; n < 8; ++n)
                    bw[n] = *reinterpret_cast<const uint4*>(ws + (8 * n + g) * kQtPitch + 8 * (t + 4 * m));
#pragma unroll
                for (int n = 0; n < 8; ++n)
                    mma_bf16_16816(acc[n], xa[m].x, xb[m].x, xa[m].y, xb[m].y, bw[n].x, bw[n].y);
#pragma unroll
                for (int n = 0; n < 8; ++n)
                    mma_bf16_16816(acc[n], xa[m].z, xb[m].z, xa[m].w, xb[m].w, bw[n].z, bw[n].w);
            }
            load_piece(wt + stride, m, xa[m], xb[m]);
        }
        // lane (g, t) holds outputs 8n + 2t, 8n + 2t + 1 of rows g (acc[n][0..1]) and
        // g + 8 (acc[n][2..3]); the four lanes of a quad hold a row's 64
        float mxa = 0.f, mxb = 0.f, ssa = 0.f, ssb = 0.f;
        bool bada = false, badb = false;
#pragma unroll
        for (int n = 0; n < 8; ++n) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                mxa = fmaxf(mxa, fabsf(acc[n][c]));
                mxb = fmaxf(mxb, fabsf(acc[n][2 + c]));
                ssa = fmaf(acc[n][c], acc[n][c], ssa);
                ssb = fmaf(acc[n][2 + c], acc[n][2 + c], ssb);
                bada = bada || !isfinite(acc[n][c]);
                badb = badb || !isfinite(acc[n][2 + c]);
            }
        }
#pragma unroll
        for (int o = 1; o <= 2; o <<= 1) {
            mxa = fmaxf(mxa, __shfl_xor_sync(kFull, mxa, o));
            mxb = fmaxf(mxb, __shfl_xor_sync(kFull, mxb, o));
            ssa += __shfl_xor_sync(kFull, ssa, o);
            ssb += __shfl_xor_sync(kFull, ssb, o);
            xsa += __shfl_xor_sync(kFull, xsa, o);
            xsb += __shfl_xor_sync(kFull, xsb, o);
            bada = __shfl_xor_sync(kFull, (int)bada, o) != 0 || bada;
            badb = __shfl_xor_sync(kFull, (int)badb, o) != 0 || badb;
        }
        const int eqa = scale_exponent(mxa), eqb = scale_exponent(mxb);
        const float upa = pow2f(eqa), dna = pow2f(-eqa), upb = pow2f(eqb), dnb = pow2f(-eqb);
        float dda = 0.f, ddb = 0.f;
#pragma unroll
        for (int n = 0; n < 8; ++n) {
            const __half2 ha = __floats2half2_rn(scale2(acc[n][0], eqa, upa), scale2(acc[n][1], eqa, upa));
            const __half2 hb = __floats2half2_rn(scale2(acc[n][2], eqb, upb), scale2(acc[n][3], eqb, upb));
            if (va) *reinterpret_cast<__half2*>(q16 + ra * 64 + 8 * n + 2 * t) = ha;
            if (vb) *reinterpret_cast<__half2*>(q16 + rb * 64 + 8 * n + 2 * t) = hb;
            // conversion errors in unscaled units (power-of-two scaling and the
            // difference of two values within a factor of 2 are exact)
            const float2 fa = __half22float2(ha), fb = __half22float2(hb);
            const float e0 = scale2(fa.x, -eqa, dna) - acc[n][0], e1 = scale2(fa.y, -eqa, dna) - acc[n][1];
            const float e2 = scale2(fb.x, -eqb, dnb) - acc[n][2], e3 = scale2(fb.y, -eqb, dnb) - acc[n][3];
            dda = fmaf(e0, e0, fmaf(e1, e1, dda));
            ddb = fmaf(e2, e2, fmaf(e3, e3, ddb));
        }
#pragma unroll
        for (int o = 1; o <= 2; o <<= 1) {
            dda += __shfl_xor_sync(kFull, dda, o);
            ddb += __shfl_xor_sync(kFull, ddb, o);
        }
        // lane t = 0 finishes row g, lane t = 1 row g + 8
        if (t < 2 && (t == 0 ? va : vb)) {
            const long long row = t == 0 ? ra : rb;
            const float xn = sqrtf(t == 0 ? xsa : xsb) * 1.0001f;
            const float eps = kQtGamma * xn * wf * 1.0001f + 1e-30f * (xn + wf + 1.f);
            const float qn = sqrtf(t == 0 ? ssa : ssb) * 1.0001f + eps;
            const float dq = sqrtf(t == 0 ? dda : ddb) * 1.0001f + eps;
            // the canonical chain's partial sums stay below |x| |W|_F: a row near the
            // float range goes to the exact selector
            const bool bad = (t == 0 ? bada : badb) || !(xn * wf < 1e37f);
            const long long bh = row / p.Nq;
            const int b = (int)(bh / p.H);
            const int h = (int)(bh - (long long)b * p.H);
            const int bg = b * p.Hkv + h / (p.H / p.Hkv);
            row_bounds_finish<64>(row, t == 0 ? eqa : eqb, qn, dq, bad, bg, p.scale, p.stats, p.gstats, p.rowinfo,
                                  p.rowub);
        }
    }
}

}  // namespace

bool qproj_tc_supported(const ProjectArgs& a) {
    return a.dtype == kBF16 && a.D == 128 && a.R == 64 && reinterpret_cast<uintptr_t>(a.x) % 16 == 0 &&
           reinterpret_cast<uintptr_t>(a.w) % 16 == 0;
}

cudaError_t launch_qproj_tc(const QPrepArgs& a, cudaStream_t stream) {
    if (a.rows <= 0) return cudaSuccess;
    const long long ntile = (a.rows + 15) / 16;
    const long long want = (ntile + kQtWarps - 1) / kQtWarps;
    const int grid = (int)std::min<long long>(want, 2LL * device_sm_count());
    qproj_tc_kernel<<<grid, kQtThreads, 0, stream>>>(a);
    const cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) note_launch();
    return e;
}

}  // namespace ossa
