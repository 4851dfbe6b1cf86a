// Gathered top-K attention forward (the O(N*K*D) sparse forward).
//
// Computes, per (b, h, i), the same result as sparse_attention_forward_chunked
// (ossa/sparse_attention.py:87-137) and the never-launched Triton kernel
// (ossa/triton_kernel.py:80-167):
//   s_j = (q_i . k_{idx_j}) * scale, masked where idx_j is outside [0, N) or, when
//   causal, idx_j > i;  out_i = softmax(s) . V[idx]  (0 for an all-masked row).
//
// Design (HBM/L2-bound gather, ~1 flop per byte):
//  * One CTA owns (b, kv head g, a tile of QTILE queries) and walks every
//    (query, head) pair of the GQA group h in [g*G, (g+1)*G).  The G query heads
//    of one query read K/V rows of the same kv head, so rows that several heads
//    (or neighbouring queries) pick are served from L1 instead of L2/HBM.
//    K/V are never expanded to H heads.
//  * One warp per (query, head).  Keys go in chunks of 32.  For the q.k step each
//    lane owns D/32 consecutive dims: a warp reads a whole 2*D-byte K row per load
//    instruction (coalesced 8-16 B per lane), 32 rows back to back for memory-level
//    parallelism, then a 31-shuffle transpose-reduction leaves key m's score in
//    lane m.  Online softmax in fp32 (exp2 domain), then the same coalesced row
//    loads of V accumulate p_m * v_m into each lane's dims.
//  * Masked/padded slots read row 0 (always in bounds) and are zeroed, so the
//    unrolled load loops carry no branches.
#include "bf16_dot.cuh"
#include "common.cuh"
#include "kernels.h"

#include <math.h>

namespace ossa {

namespace {

constexpr int kGatherThreads = 256;
constexpr int kGatherWarps = kGatherThreads / 32;

// Sums part[0..31] across the warp so that lane m ends with the total of part[m].
__device__ __forceinline__ float transpose_reduce32(float (&part)[32], int lane) {
#pragma unroll
    for (int w = 16; w >= 1; w >>= 1) {
        const bool upper = (lane & w) != 0;
#pragma unroll
        for (int t = 0; t < w; ++t) {
            const float a = part[t], b = part[t + w];
            const float send = upper ? a : b;
            const float keep = upper ? b : a;
            part[t] = keep + __shfl_xor_sync(kFull, send, w);
        }
    }
    return part[0];
}

template <typename T, int D, typename IdxT>
__global__ void __launch_bounds__(kGatherThreads)
gather_attn_fwd_kernel(const T* __restrict__ q, const T* __restrict__ k,
                       const T* __restrict__ v, const IdxT* __restrict__ idx,
                       T* __restrict__ out, int H, int Hkv, int N, int Nq, int q0, int K,
                       float scale_log2, int causal, int qtile) {
    constexpr int DPL = D >= 32 ? D / 32 : 1;  // dims owned by one lane
    constexpr int ACTIVE = D / DPL;            // lanes that own dims
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int G = H / Hkv;
    const int bg = blockIdx.y;  // b * Hkv + g
    const int b = bg / Hkv;
    const int g = bg - b * Hkv;
    const int i0 = blockIdx.x * qtile;
    const int nq = min(qtile, Nq - i0);
    const int items = nq * G;
    const bool dim_lane = lane < ACTIVE;

    __shared__ int s_j[kGatherWarps][32];
    __shared__ float s_p[kGatherWarps][32];

    const T* kb = k + (size_t)bg * N * D + lane * DPL;
    const T* vb = v + (size_t)bg * N * D + lane * DPL;

    for (int w = warp; w < items; w += kGatherWarps) {
        const int il = i0 + w / G;  // query row (local); its key-sequence position is q0 + il
        const int i = q0 + il;
        const int h = g * G + (w - (w / G) * G);
        const size_t row = ((size_t)b * H + h) * Nq + il;

        float qv[DPL];
        if (dim_lane) {
            VecLoad<T, DPL>::load(q + row * D + lane * DPL, qv);
        } else {
#pragma unroll
            for (int t = 0; t < DPL; ++t) qv[t] = 0.f;
        }
#pragma unroll
        for (int t = 0; t < DPL; ++t) qv[t] *= scale_log2;

        const IdxT* irow = idx + row * K;
        float m_run = -INFINITY, l_run = 0.f;
        float acc[DPL];
#pragma unroll
        for (int t = 0; t < DPL; ++t) acc[t] = 0.f;

        for (int kc = 0; kc < K; kc += 32) {
            const int kk = kc + lane;
            const long long j = kk < K ? (long long)irow[kk] : -1ll;
            const bool valid = j >= 0 && j < N && (!causal || j <= i);
            s_j[warp][lane] = valid ? (int)j : -1;
            __syncwarp();

            float part[32];
#pragma unroll
            for (int m = 0; m < 32; ++m) {
                const int jm = s_j[warp][m];
                float kv[DPL];
                if (dim_lane) {
                    VecLoad<T, DPL>::load(kb + (size_t)max(jm, 0) * D, kv);
                } else {
#pragma unroll
                    for (int t = 0; t < DPL; ++t) kv[t] = 0.f;
                }
                float d = 0.f;
#pragma unroll
                for (int t = 0; t < DPL; ++t) d = fmaf(qv[t], kv[t], d);
                part[m] = d;
            }
            const float dot = transpose_reduce32(part, lane);
            const float s = valid ? dot : -INFINITY;
            const float m_new = fmaxf(m_run, warp_max(s));
            if (m_new == -INFINITY) {  // warp-uniform: nothing valid so far
                __syncwarp();
                continue;
            }
            const float p = valid ? exp2f(s - m_new) : 0.f;
            const float alpha = exp2f(m_run - m_new);
            l_run = l_run * alpha + warp_sum(p);
#pragma unroll
            for (int t = 0; t < DPL; ++t) acc[t] *= alpha;
            s_p[warp][lane] = p;
            __syncwarp();

#pragma unroll
            for (int m = 0; m < 32; ++m) {
                const int jm = s_j[warp][m];
                const float pm = s_p[warp][m];
                if (dim_lane) {
                    float vv[DPL];
                    VecLoad<T, DPL>::load(vb + (size_t)max(jm, 0) * D, vv);
                    const float pe = jm >= 0 ? pm : 0.f;
#pragma unroll
                    for (int t = 0; t < DPL; ++t) acc[t] = fmaf(pe, jm >= 0 ? vv[t] : 0.f, acc[t]);
                }
            }
            m_run = m_new;
            __syncwarp();
        }

        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        if (dim_lane) {
            T* orow = out + row * D + lane * DPL;
#pragma unroll
            for (int t = 0; t < DPL; ++t) store_from_f32(orow + t, acc[t] * inv);
        }
    }
}

// bf16, D = 128: half a warp per key row.  Each lane owns 8 consecutive dims
// (one 16-byte load per row), so one load instruction fetches two key rows;
// q.k and p.v use the mixed-precision fma with bf16 operands (no conversions).
// Key slot m of a 32-key chunk is handled by half (m & 1) at step m >> 1; its
// score, probability and index live in lane 16 * (m & 1) + (m >> 1).
// Numerics: fp32 dot products of the bf16 inputs, fp32 online softmax, and
// p rounded to bf16 for the p.v product (as the reference's bf16 einsum does).
//
// One (query, head) row, one warp: kb / vb point at this lane's 16-byte column of
// key / value row 0 of the kv head; irow is the row's K indices.
template <typename IdxT>
__device__ __forceinline__ void gather_row_bf16_d128(uint4 qv, const uint4* __restrict__ kb,
                                                     const uint4* __restrict__ vb, const IdxT* __restrict__ irow,
                                                     int K, int N, int i, int causal, float scale_log2,
                                                     __nv_bfloat16* __restrict__ orow, int lane) {
    constexpr int D = 128;
    const int half = lane >> 4;
    const int hl = lane & 15;
    const int myslot = 2 * hl + half;  // key slot held by this lane
    float m_run = -INFINITY, l_run = 0.f;
    float acc[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) acc[t] = 0.f;

    for (int kc = 0; kc < K; kc += 32) {
        const int kk = kc + myslot;
        const long long jl = kk < K ? (long long)irow[kk] : -1ll;
        const bool valid = jl >= 0 && jl < N && (!causal || jl <= i);
        const int jv = valid ? (int)jl : -1;
        int js[16];
        float part[16];
#pragma unroll
        for (int m = 0; m < 16; ++m) {
            js[m] = __shfl_sync(kFull, jv, 16 * half + m);
            const uint4 kr = __ldg(kb + (size_t)max(js[m], 0) * (D / 8));
            part[m] = dot8_bf16(qv, kr);
        }
        // lane l of half h now holds key slot 2 * (l & 15) + h
        const float dot = transpose_reduce16(part, lane);
        const float sc = valid ? dot * scale_log2 : -INFINITY;
        const float m_new = fmaxf(m_run, warp_max(sc));
        if (m_new == -INFINITY) continue;  // warp-uniform: nothing valid so far
        const float p = valid ? exp2f(sc - m_new) : 0.f;
        const float alpha = exp2f(m_run - m_new);
        l_run = l_run * alpha + warp_sum(p);
#pragma unroll
        for (int t = 0; t < 8; ++t) acc[t] *= alpha;
        const uint32_t pbits = bf16_pair_bits(p);
#pragma unroll
        for (int m = 0; m < 16; ++m) {
            const uint32_t pm = __shfl_sync(kFull, pbits, 16 * half + m);
            const uint4 vr = __ldg(vb + (size_t)max(js[m], 0) * (D / 8));
            axpy8_bf16(pm, vr, acc);
        }
        m_run = m_new;
    }
    store_row_bf16(acc, l_run, orow, lane);
}

template <typename IdxT>
__global__ void __launch_bounds__(kGatherThreads)
gather_attn_bf16_d128_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                             const __nv_bfloat16* __restrict__ v, const IdxT* __restrict__ idx,
                             __nv_bfloat16* __restrict__ out, int H, int Hkv, int N, int Nq, int q0,
                             int K, float scale_log2, int causal, int qtile) {
    constexpr int D = 128;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int hl = lane & 15;
    const int G = H / Hkv;
    const int bg = blockIdx.y;
    const int b = bg / Hkv;
    const int g = bg - b * Hkv;
    const int i0 = blockIdx.x * qtile;
    const int nq = min(qtile, Nq - i0);
    const int items = nq * G;
    const uint4* kb = reinterpret_cast<const uint4*>(k + (size_t)bg * N * D) + hl;
    const uint4* vb = reinterpret_cast<const uint4*>(v + (size_t)bg * N * D) + hl;
    for (int w = warp; w < items; w += kGatherWarps) {
        const int il = i0 + w / G;  // query row (local); its key-sequence position is q0 + il
        const int h = g * G + (w - (w / G) * G);
        const size_t row = ((size_t)b * H + h) * Nq + il;
        const uint4 qv = __ldg(reinterpret_cast<const uint4*>(q + row * D) + hl);
        gather_row_bf16_d128<IdxT>(qv, kb, vb, idx + row * K, K, N, q0 + il, causal, scale_log2, out + row * D,
                                   lane);
    }
}

template <typename T, typename IdxT>
cudaError_t launch_typed(const GatherArgs& a, cudaStream_t stream) {
    const int qtile = 8;
    const int Nq = a.Nq > 0 ? a.Nq : a.N;
    dim3 grid((Nq + qtile - 1) / qtile, a.B * a.Hkv);
    dim3 block(kGatherThreads);
    const float scale_log2 = a.scale * 1.4426950408889634f;
    const T* q = static_cast<const T*>(a.q);
    const T* k = static_cast<const T*>(a.k);
    const T* v = static_cast<const T*>(a.v);
    const IdxT* ix = static_cast<const IdxT*>(a.idx);
    T* o = static_cast<T*>(a.out);
    if constexpr (sizeof(T) == 2) {
        if (a.D == 128) {
            gather_attn_bf16_d128_kernel<IdxT><<<grid, block, 0, stream>>>(q, k, v, ix, o, a.H, a.Hkv, a.N, Nq,
                                                                          a.q0, a.K, scale_log2, a.causal, qtile);
            cudaError_t e = cudaGetLastError();
            if (e == cudaSuccess) note_launch();
            return e;
        }
    }
    switch (a.D) {
#define OSSA_GATHER_CASE(DD)                                                              \
    case DD:                                                                              \
        gather_attn_fwd_kernel<T, DD, IdxT><<<grid, block, 0, stream>>>(                  \
            q, k, v, ix, o, a.H, a.Hkv, a.N, Nq, a.q0, a.K, scale_log2, a.causal, qtile); \
        break;
        OSSA_GATHER_CASE(16)
        OSSA_GATHER_CASE(32)
        OSSA_GATHER_CASE(64)
        OSSA_GATHER_CASE(128)
        OSSA_GATHER_CASE(256)
#undef OSSA_GATHER_CASE
        default:
            return cudaErrorInvalidValue;
    }
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) note_launch();
    return e;
}

}  // namespace

cudaError_t launch_gather_attn(const GatherArgs& a, cudaStream_t stream) {
    if (a.dtype == kF32) {
        return a.idx_is_64 ? launch_typed<float, int64_t>(a, stream)
                           : launch_typed<float, int32_t>(a, stream);
    }
    return a.idx_is_64 ? launch_typed<__nv_bfloat16, int64_t>(a, stream)
                       : launch_typed<__nv_bfloat16, int32_t>(a, stream);
}

}  // namespace ossa
