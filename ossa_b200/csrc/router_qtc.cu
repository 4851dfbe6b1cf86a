// The tensor-core selector's query operand straight from the bf16 query rows
// (head_dim 128, proj_dim 64), for the router path (ossa/router.py:171-190: q' =
// q_proj(q)).  The selector scores with fp16 copies of q' and needs the canonical
// fp32 q' (the fmaf chain over d = 0..127) only for the rows whose top-K boundary is
// rescored or that go to the exact selector, about a tenth of the rows; those rows
// compute it themselves (warp_canon_q2).  So this kernel reads q once and
// writes only what the selector reads for every row:
//
//  * q' = x W^T on the 5th-generation tensor cores (tcgen05.mma kind::f16, bf16
//    operands, fp32 accumulator in TMEM) with W split into bf16 hi + lo parts: the
//    products are exact and the split leaves 2^-16 |w| per weight;
//  * the fp16 copy q16 scaled by the row's power of two (as the prep kernel), the
//    epilogue multiplier, and delta / rowub from bounds that cover the canonical
//    row: |q'| <= |q'_tc| + eps and |q16 / 2^eq - q'| <= |q16 / 2^eq - q'_tc| + eps,
//    with eps >= |q'_tc - q'| from |x| |W|_F (Cauchy-Schwarz per output).
//
// One persistent CTA per SM walks 128-row tiles: warp 0 streams x tiles (two
// 128 x 64 boxes, 128-byte swizzle) through a 6-stage ring with TMA, warp 1 issues
// 2 x 8 MMAs of 128 x 64 x 16 per tile (W hi, then W lo) into one of eight 64-column
// TMEM accumulators (tile t into t % 8), and six groups of four epilogue warps give
// every row to one thread: group g takes the tiles t with t % 6 == g, each warp the 32
// rows of its TMEM lane quadrant.  A thread reads |x|^2 from the staged tile and its row's 64
// outputs with tcgen05.ld in 16-column chunks, twice (the row maximum sets the fp16
// scaling before any value is converted; a compact loop keeps the code in the
// instruction cache), and writes q16, rowinfo and rowub.  W's two bf16 parts sit in shared memory for the whole kernel.  Every
// mbarrier wait is bounded; on expiry the kernel sets bit 32 of the selector's
// status word and winds down.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdint>

#include "common.cuh"
#include "kernels.h"
#include "router_prep.cuh"
#include "sm100.cuh"

namespace ossa {
namespace {

using namespace sm100;

constexpr int kQtRows = 128;                 // rows per tile (MMA M)
constexpr int kQtStages = 6;                 // x tile ring
constexpr int kQtTileB = kQtRows * 128 * 2;  // one x tile: two 128 x 64 boxes (32 KB)
constexpr int kQtWB = 64 * 128 * 2;          // one W part: two 64 x 64 sub-tiles (16 KB)
constexpr int kQtGroups = 6;                         // epilogue groups of 4 warps, one tile each in turn
constexpr int kQtEpiWarps = 4 * kQtGroups;
constexpr int kQtThreads = 32 * (2 + kQtEpiWarps);  // warp 0 TMA, warp 1 MMA, then the epilogue warps
constexpr int kQtAcc = 8;                    // 64-column TMEM accumulators (all 512 columns)
constexpr uint32_t kQtTmemCols = 64 * kQtAcc;
constexpr int kQtOffWhi = kQtStages * kQtTileB;
constexpr int kQtOffWlo = kQtOffWhi + kQtWB;
constexpr int kQtOffBar = kQtOffWlo + kQtWB;
constexpr int kQtNumBars = 2 * kQtStages + 2 * kQtAcc + 1;
constexpr int kQtOffRed = kQtOffBar + kQtNumBars * 8;
constexpr int kQtOffSlot = kQtOffRed + (kQtThreads / 32) * 4;
constexpr size_t kQtSmem = kQtOffSlot + 16 + 1024;  // + alignment slack
static_assert(kQtOffWhi % 1024 == 0 && kQtWB % 1024 == 0, "swizzled tiles need 1 KB alignment");
static_assert(kQtSmem <= 232448, "shared memory budget");

// eps per output, relative to sum_d |x_d w_cd|: 2^-16 from the hi/lo split, 2^-14 for
// the tensor core's fp32 accumulation of the 256 exact products (a few ulp per
// step: below 2^-16 of the sum, taken with a 4x margin), 2^-17 for the canonical
// chain's 128 roundings.
constexpr float kQtGamma = 6.103515625e-05f + 1.52587890625e-05f + 7.62939453125e-06f;

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

__global__ void __launch_bounds__(kQtThreads, 1)
qproj_umma_kernel(const __grid_constant__ CUtensorMap tmX, const QPrepArgs p) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
    uint8_t* sX = smem;
    uint8_t* sWhi = smem + kQtOffWhi;
    uint8_t* sWlo = smem + kQtOffWlo;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kQtOffBar);
    uint64_t* full = bars;
    uint64_t* empty = bars + kQtStages;
    uint64_t* afull = empty + kQtStages;
    uint64_t* aempty = afull + kQtAcc;
    uint64_t* mdone = aempty + kQtAcc;
    float* wred = reinterpret_cast<float*>(smem + kQtOffRed);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kQtOffSlot);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long ntiles = (p.rows + kQtRows - 1) / kQtRows;
    const int my_tiles = ntiles > blockIdx.x ? (int)((ntiles - 1 - blockIdx.x) / gridDim.x + 1) : 0;

    // W's bf16 parts in the K-major 128-byte-swizzled layout (row c = output, 16-byte
    // chunk j of a 64-column sub-tile at position j ^ (c & 7)); |W|_F; block 0 also
    // writes Wq transposed for the selector's on-demand q' rows
    float wss = 0.f;
    for (int e = threadIdx.x; e < 64 * 128; e += kQtThreads) {
        const int c = e >> 7, d = e & 127;
        const float v = __ldg(p.w + e);
        const __nv_bfloat16 h = __float2bfloat16_rn(v);
        const __nv_bfloat16 l = __float2bfloat16_rn(v - __bfloat162float(h));  // v - h is exact
        const int off = (d >> 6) * 8192 + c * 128 + ((((d & 63) >> 3) ^ (c & 7)) << 4) + (d & 7) * 2;
        *reinterpret_cast<__nv_bfloat16*>(sWhi + off) = h;
        *reinterpret_cast<__nv_bfloat16*>(sWlo + off) = l;
        wss = fmaf(v, v, wss);
        if (blockIdx.x == 0) p.wt[d * 64 + c] = v;
    }
    wss = warp_sum(wss);
    if (lane == 0) wred[warp] = wss;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kQtStages; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 1 + 4);  // MMA commit + the tile's 4 epilogue warps (|x| read)
        }
        for (int a = 0; a < kQtAcc; ++a) {
            mbar_init(afull + a, 1);
            mbar_init(aempty + a, 4);
        }
        mbar_init(mdone, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kQtTmemCols);
        tmem_relinquish();
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // W tiles visible to the tensor cores
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            bool ok = true;
            int issued = 0;
            for (int t = 0; t < my_tiles; ++t) {
                const int s = t % kQtStages;
                if (t >= kQtStages) ok = mbar_wait(empty + s, ((t / kQtStages) - 1) & 1);
                if (!ok) break;
                const int row0 = (int)(((long long)blockIdx.x + (long long)t * gridDim.x) * kQtRows);
                mbar_arrive_expect_tx(full + s, kQtTileB);
                tma_load_2d(sX + (size_t)s * kQtTileB, &tmX, full + s, 0, row0);
                tma_load_2d(sX + (size_t)s * kQtTileB + 16384, &tmX, full + s, 64, row0);
                issued = t + 1;
            }
            // the last loads land before the CTA can retire
            for (int t = max(0, issued - kQtStages); t < issued; ++t)
                mbar_wait(full + t % kQtStages, (t / kQtStages) & 1);
            if (!ok) atomicOr(p.status, 32);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_f16(1u, kQtRows, 64);
            bool ok = true;
            for (int t = 0; t < my_tiles && ok; ++t) {
                const int s = t % kQtStages, ab = t % kQtAcc;
                ok = mbar_wait(full + s, (t / kQtStages) & 1);
                if (ok && t >= kQtAcc) ok = mbar_wait(aempty + ab, ((t / kQtAcc) - 1) & 1);
                if (!ok) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(ab * 64);
                const uint8_t* xa = sX + (size_t)s * kQtTileB;
#pragma unroll
                for (int k = 0; k < 8; ++k) {  // 16 columns of d per MMA; a new 64-column box every 4
                    const uint64_t ad = umma_desc_sw128(xa + (k >> 2) * 16384) + 2u * (k & 3);
                    const uint64_t bd = umma_desc_sw128(sWhi + (k >> 2) * 8192) + 2u * (k & 3);
                    mma_f16(d, ad, bd, idesc, k > 0 ? 1u : 0u);
                }
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const uint64_t ad = umma_desc_sw128(xa + (k >> 2) * 16384) + 2u * (k & 3);
                    const uint64_t bd = umma_desc_sw128(sWlo + (k >> 2) * 8192) + 2u * (k & 3);
                    mma_f16(d, ad, bd, idesc, 1u);
                }
                mma_commit(empty + s);
                mma_commit(afull + ab);
            }
            mma_commit(mdone);  // completes once every MMA issued above has finished
            mbar_wait(mdone, 0);
            if (!ok) atomicOr(p.status, 32);
        }
    } else {
        // ------------------------------------------------ epilogue: one row per thread
        float wf = 0.f;
#pragma unroll
        for (int u = 0; u < kQtThreads / 32; ++u) wf += wred[u];
        wf = sqrtf(wf) * 1.001f;  // >= |W|_F
        const int qd = warp & 3;                // TMEM lane quadrant this warp may access
        const int par = (warp - 2) / 4;         // tiles t with t % kQtGroups == par
        const int r = qd * 32 + lane;
        __half* q16 = static_cast<__half*>(p.q16);
        bool ok = true;
        for (int t = par; t < my_tiles; t += kQtGroups) {
            const int s = t % kQtStages, ab = t % kQtAcc;
            const bool got = mbar_wait(afull + ab, (t / kQtAcc) & 1) && mbar_wait(full + s, (t / kQtStages) & 1);
            if (!__all_sync(kFull, got)) {
                ok = false;
                break;
            }
            tc_fence_after();
            // |x_row|^2 from the staged tile (chunk j of a box at position j ^ (r & 7))
            const uint8_t* xr = sX + (size_t)s * kQtTileB + r * 128;
            float xs4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
            for (int j = 0; j < 16; ++j)
                xs4[j & 3] = sum_sq_bf16x8(
                    *reinterpret_cast<const uint4*>(xr + (j >> 3) * 16384 + (((j & 7) ^ (r & 7)) << 4)), xs4[j & 3]);
            const float xs = (xs4[0] + xs4[1]) + (xs4[2] + xs4[3]);
            __syncwarp();
            if (lane == 0) mbar_arrive(empty + s);

            // pass 1: row maximum and sum of squares (four independent chains; a
            // non-finite value makes the sum non-finite)
            const uint32_t taddr = tmem + ((uint32_t)(qd * 32) << 16) + (uint32_t)(ab * 64);
            float mx4[4] = {0.f, 0.f, 0.f, 0.f}, ss4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
            for (int ch = 0; ch < 4; ++ch) {
                uint32_t v[16];
                tmem_ld16(taddr + 16u * ch, v);
                tmem_wait_ld();
                reg_fence(v);
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                    const float f = __uint_as_float(v[c]);
                    mx4[c & 3] = fmaxf(mx4[c & 3], fabsf(f));
                    ss4[c & 3] = fmaf(f, f, ss4[c & 3]);
                }
            }
            const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
            const float ss = (ss4[0] + ss4[1]) + (ss4[2] + ss4[3]);
            const int eq = scale_exponent(mx);
            const float up = pow2f(eq), dn = pow2f(-eq);
            const long long row = ((long long)blockIdx.x + (long long)t * gridDim.x) * kQtRows + r;
            const bool live = row < p.rows;
            // pass 2: fp16 copy and its conversion errors in unscaled units (power-of-two
            // scaling and the difference of two values within a factor of 2 are exact)
            float dd4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
            for (int ch = 0; ch < 4; ++ch) {
                uint32_t v[16];
                tmem_ld16(taddr + 16u * ch, v);
                tmem_wait_ld();
                reg_fence(v);
                uint32_t pk[8];
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const float f0 = __uint_as_float(v[2 * c]), f1 = __uint_as_float(v[2 * c + 1]);
                    const __half2 h2 = __floats2half2_rn(scale2(f0, eq, up), scale2(f1, eq, up));
                    pk[c] = *reinterpret_cast<const uint32_t*>(&h2);
                    const float2 b = __half22float2(h2);
                    const float e0 = scale2(b.x, -eq, dn) - f0, e1 = scale2(b.y, -eq, dn) - f1;
                    dd4[c & 3] = fmaf(e0, e0, fmaf(e1, e1, dd4[c & 3]));
                }
                if (live) {
                    uint4* o = reinterpret_cast<uint4*>(q16 + row * 64 + 16 * ch);
                    o[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                    o[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(aempty + ab);
            if (live) {
                const float dd = (dd4[0] + dd4[1]) + (dd4[2] + dd4[3]);
                const float xn = sqrtf(xs) * 1.0001f;
                const float eps = kQtGamma * xn * wf * 1.0001f + 1e-30f * (xn + wf + 1.f);
                // the canonical chain's partial sums stay below |x| |W|_F: a row near the
                // float range goes to the exact selector
                const bool nonfinite = !isfinite(ss) || !(xn * wf < 1e37f);
                const long long bh = row / p.Nq;
                const int b = (int)(bh / p.H);
                const int h = (int)(bh - (long long)b * p.H);
                const int bg = b * p.Hkv + h / (p.H / p.Hkv);
                row_bounds_finish<64>(row, eq, sqrtf(ss) * 1.0001f + eps, sqrtf(dd) * 1.0001f + eps, nonfinite, bg,
                                      p.scale, p.stats, p.gstats, p.rowinfo, p.rowub);
            }
        }
        if (!ok && lane == 0) atomicOr(p.status, 32);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kQtTmemCols);
    }
}

}  // namespace

bool qproj_tc_supported(const ProjectArgs& a) {
    return a.dtype == kBF16 && a.D == 128 && a.R == 64 && reinterpret_cast<uintptr_t>(a.x) % 16 == 0 &&
           reinterpret_cast<uintptr_t>(a.w) % 16 == 0 && a.rows < (1LL << 31);
}

cudaError_t launch_qproj_tc(const QPrepArgs& a, cudaStream_t stream) {
    if (a.rows <= 0) return cudaSuccess;
    CUtensorMap tm;
    if (!make_row_map_16(&tm, a.x, true, (unsigned long long)a.rows, 128, kQtRows)) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(qproj_umma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kQtSmem);
    if (e != cudaSuccess) return e;
    const long long ntiles = (a.rows + kQtRows - 1) / kQtRows;
    const int grid = (int)std::min<long long>(ntiles, device_sm_count());
    qproj_umma_kernel<<<grid, kQtThreads, kQtSmem, stream>>>(tm, a);
    e = cudaGetLastError();
    if (e == cudaSuccess) note_launch();
    return e;
}

}  // namespace ossa
