// Gathered top-K attention forward (the O(N*K*D) sparse forward).
//
// Computes, per (b, h, i), the same result as sparse_attention_forward_chunked
// (ossa/sparse_attention.py:87-137) and the never-launched Triton kernel
// (ossa/triton_kernel.py:80-167):
//   s_j = (q_i . k_{idx_j}) * scale, masked where idx_j is outside [0, N) or, when
//   causal, idx_j > i;  out_i = softmax(s) . V[idx]  (0 for an all-masked row).
//
// Design (HBM/L2-bound gather, ~1 flop per byte).  bf16 rows of head_dim 128 with
// 2-8 query heads per kv head take the tensor-core form below
// (gather_attn_bf16_d128_mma_kernel: one warp per query and all heads of its group,
// each selected key or value row loaded once for every head that picked it);
// everything else takes the per-(query, head) forms:
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

// ------------------------------------------- GQA heads on the tensor cores (bf16, D = 128)
//
// One warp per query and kv head, all G (2, 3, 4, 6 or 8) query heads of the group at once:
//  1. q: the G heads' rows as mma A fragments, loaded first so that their latency
//     overlaps the union build.
//  2. union of the heads' keys with head bits.  Direct form (N <= 4096, K <= 64): a
//     per-warp byte array indexed by the key holds the head bits, set by one atomicOr
//     per selected key (no probing, no compare-and-swap); a head bit that is already set
//     marks a repeated key.  Hash form: the G index rows must be in the selectors' form
//     (valid entries first, strictly ascending); every valid key goes into an
//     open-addressing hash with its head bit.  The union list (at most kMaxU keys) holds
//     each key once with its head bits.  A repeated key, a row out of form (hash form)
//     or a larger union sends the query through gather_row_bf16_d128 per head.
//  3. the union in chunks of 16 keys.  Key and value rows are copied to shared memory
//     with cp.async (16-byte pieces XOR-swizzled by row): the key rows of chunk c + 1
//     are in flight while chunk c is scored, the value rows of chunk c while its scores
//     and softmax run.  S = Q K^T on mma.sync m16n8k16 (bf16 operands, fp32
//     accumulation): A = the heads' q rows (rows G..15 zero), B = 8 keys per n-tile by
//     ldmatrix from the staged key rows.
//  4. online softmax per head over its selected keys (head bit set; others masked): a
//     head's scores sit in the four lanes of one quad, reduced by two shuffles; p is
//     rounded to bf16 for p.v, as in the per-head form.
//  5. O += P V with mma.sync: P from the score fragments (no shuffles), V as the B
//     operand by ldmatrix.trans from the staged value rows; at the end each head's row
//     is divided by its sum and stored as bf16.
// Results agree with the per-head form to rounding (tensor-core accumulation order).
constexpr int kMmaChunk = 16;                    // union keys per chunk: 2 score n-tiles, 1 value k-step
constexpr int kMmaWarps = 8;
constexpr int kRowBytes = 256;                   // one bf16 key or value row (D = 128)
constexpr int kChunkBytes = kMmaChunk * kRowBytes;
constexpr int kStageBytes = 3 * kChunkBytes;     // key rows of two chunks, value rows of one
constexpr int kDirectMaxN = 4096;                // keys covered by the direct head-bit array
template <int kSlotBits, bool kDirect>
constexpr int mma_max_union() { return kDirect ? 128 : (1 << kSlotBits) / 2; }
// Per warp: the staging area (the hash slots or the direct head-bit array use it while
// the union is built), then the union list (keys, head bits).
template <int kSlotBits, bool kDirect>
constexpr size_t mma_warp_smem() { return (size_t)kStageBytes + (size_t)8 * mma_max_union<kSlotBits, kDirect>(); }
template <int kSlotBits, bool kDirect>
constexpr size_t mma_smem_bytes() { return kMmaWarps * mma_warp_smem<kSlotBits, kDirect>(); }
static_assert(kDirectMaxN <= kStageBytes && ((size_t)8 << 9) <= (size_t)kStageBytes, "the union build fits in the staging area");
static_assert(mma_warp_smem<8, true>() % 16 == 0 && mma_warp_smem<9, false>() % 16 == 0, "warp areas stay 16-byte aligned");
static_assert(2 * (mma_smem_bytes<9, false>() + 1024) <= 233472, "two CTAs per SM");

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

// mma.sync m16n8k16 with all four A registers (rows 0..15).
__device__ __forceinline__ void mma_bf16_16816_a4(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                  uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Transpose of an 8 x 8 bf16 matrix held one 32-bit pair per lane (lane 4 r + c holds
// row r, columns 2 c, 2 c + 1; afterwards the same for the transpose).
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}

template <int kPending>
__device__ __forceinline__ void cp_async_wait_pending() {
    asm volatile("cp.async.wait_group %0;" ::"n"(kPending) : "memory");
}

template <typename IdxT, int G, int kSlotBits, bool kDirect>
__global__ void __launch_bounds__(kMmaWarps * 32, 2)
gather_attn_bf16_d128_mma_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                                 const __nv_bfloat16* __restrict__ v, const IdxT* __restrict__ idx,
                                 __nv_bfloat16* __restrict__ out, int H, int Hkv, int N, int Nq, int q0, int K,
                                 float scale_log2, int causal) {
    constexpr int D = 128;
    constexpr int kMaxU = mma_max_union<kSlotBits, kDirect>();
    constexpr int kSlots = 1 << kSlotBits;
    extern __shared__ __align__(128) uint8_t msm[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int gq = lane >> 2;  // MMA row of this lane: head gq
    const int c4 = lane & 3;   // position in the quad
    const unsigned lt = lanemask_lt();
    const int bg = blockIdx.y;
    const int b = bg / Hkv;
    const int g = bg - b * Hkv;
    const int il = blockIdx.x * kMmaWarps + warp;
    if (il >= Nq) return;  // warp-uniform; no CTA-wide barrier follows
    const int i = q0 + il;
    uint8_t* stage = msm + (size_t)warp * mma_warp_smem<kSlotBits, kDirect>();
    int* ukey = reinterpret_cast<int*>(stage + kStageBytes);  // the union list
    unsigned* umask = reinterpret_cast<unsigned*>(ukey + kMaxU);
    const __nv_bfloat16* kb = k + (size_t)bg * N * D;
    const __nv_bfloat16* vb = v + (size_t)bg * N * D;
    const size_t row0 = ((size_t)b * H + (size_t)g * G) * Nq + il;  // head t: row0 + t * Nq

    // ---- 1. q rows as A fragments: k-step s takes dims 16 s + 2 c4, +1 (a0) and
    // 16 s + 8 + 2 c4, +1 (a2) of head gq (rows G..15 zero)
    uint32_t qa[16];
    {
        const uint32_t* qw = reinterpret_cast<const uint32_t*>(q + (row0 + (size_t)(gq < G ? gq : 0) * Nq) * D);
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            qa[2 * s] = gq < G ? __ldg(qw + 8 * s + c4) : 0u;
            qa[2 * s + 1] = gq < G ? __ldg(qw + 8 * s + 4 + c4) : 0u;
        }
    }

    // ---- 2. union of the heads' keys with head bits into ukey / umask
    int x[G][4];
#pragma unroll
    for (int t = 0; t < G; ++t) {
        const IdxT* irow = idx + (row0 + (size_t)t * Nq) * K;
#pragma unroll
        for (int e = 0; e < 4; ++e) {  // K <= 128
            const int qi = lane + 32 * e;
            const long long jl = (32 * e < K && qi < K) ? (long long)irow[qi] : -1ll;
            x[t][e] = (jl >= 0 && jl < N && (!causal || jl <= i)) ? (int)jl : -1;
        }
    }
    bool canon = true;
    int U = 0;
    if constexpr (kDirect) {
        uint32_t* dbits = reinterpret_cast<uint32_t*>(stage);  // byte j: head bits of key j
        for (int w = lane; w < (N + 15) >> 4; w += 32) reinterpret_cast<uint4*>(dbits)[w] = make_uint4(0u, 0u, 0u, 0u);
        __syncwarp();
        bool dup = false;
#pragma unroll
        for (int t = 0; t < G; ++t) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int xv = x[t][e];
                if (32 * e < K && xv >= 0) {
                    const uint32_t sh = 8u * (uint32_t)(xv & 3) + (uint32_t)t;
                    const uint32_t old = atomicOr(&dbits[xv >> 2], 1u << sh);
                    dup = dup || ((old >> sh) & 1u) != 0u;
                }
            }
        }
        canon = !__any_sync(kFull, dup);
        __syncwarp();
        // the entry of the lowest head that selected a key appends it
#pragma unroll
        for (int t = 0; t < G; ++t) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                if (32 * e < K) {  // warp-uniform
                    const int xv = x[t][e];
                    unsigned mk = 0u;
                    bool own = false;
                    if (xv >= 0) {
                        mk = (dbits[xv >> 2] >> (8u * (uint32_t)(xv & 3))) & 0xffu;
                        own = (mk & ((1u << t) - 1u)) == 0u;
                    }
                    const unsigned bal = __ballot_sync(kFull, own);
                    if (own) {
                        const int pos = U + __popc(bal & lt);
                        if (pos < kMaxU) {
                            ukey[pos] = xv;
                            umask[pos] = mk;
                        }
                    }
                    U += __popc(bal);
                }
            }
        }
    } else {
        int* skey = reinterpret_cast<int*>(stage);  // hash slots (linear probing)
        unsigned* smask = reinterpret_cast<unsigned*>(skey + kSlots);
#pragma unroll
        for (int u = 0; u < kSlots / 32; ++u) {
            skey[lane + 32 * u] = -1;
            smask[lane + 32 * u] = 0u;
        }
        __syncwarp();
#pragma unroll
        for (int t = 0; t < G; ++t) {
            int prev31 = -1;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                if (32 * e < K) {  // warp-uniform
                    const int qi = lane + 32 * e;
                    const int xv = x[t][e];
                    int pv = __shfl_up_sync(kFull, xv, 1);
                    if (lane == 0) pv = prev31;
                    // the selectors' form: valid entries first, strictly ascending (so no
                    // key repeats within a head)
                    canon = canon && !__any_sync(kFull, xv >= 0 && qi > 0 && !(pv >= 0 && pv < xv));
                    prev31 = __shfl_sync(kFull, xv, 31);
                    if (xv >= 0) {
                        int slot = (int)(((uint32_t)xv * 2654435761u) >> (32 - kSlotBits));
                        for (int probe = 0; probe < kSlots; ++probe) {
                            const int old = atomicCAS(&skey[slot], -1, xv);
                            if (old == -1 || old == xv) {
                                atomicOr(&smask[slot], 1u << t);
                                break;
                            }
                            slot = (slot + 1) & (kSlots - 1);
                        }
                    }
                }
            }
        }
        __syncwarp();
        // occupied slots in slot order: lane owns slots S lane .. S lane + S - 1, S = kSlots / 32
        int kk[kSlots / 32];
        unsigned mk[kSlots / 32];
#pragma unroll
        for (int u = 0; u < kSlots / 32; ++u) {
            kk[u] = skey[(kSlots / 32) * lane + u];
            mk[u] = smask[(kSlots / 32) * lane + u];
        }
        int nmine = 0;
#pragma unroll
        for (int u = 0; u < kSlots / 32; ++u) nmine += kk[u] >= 0 ? 1 : 0;
        int before = nmine;  // inclusive prefix over lanes
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(kFull, before, o);
            if (lane >= o) before += y;
        }
        U = __shfl_sync(kFull, before, 31);
        int pos = before - nmine;
#pragma unroll
        for (int u = 0; u < kSlots / 32; ++u) {
            if (kk[u] >= 0) {
                if (pos < kMaxU) {
                    ukey[pos] = kk[u];
                    umask[pos] = mk[u];
                }
                ++pos;
            }
        }
    }
    __syncwarp();  // the union list is complete; the staging area is free
    if (!canon || U > kMaxU) {
#pragma unroll 1
        for (int t = 0; t < G; ++t) {
            const size_t row = row0 + (size_t)t * Nq;
            const uint4 qv = __ldg(reinterpret_cast<const uint4*>(q + row * D) + (lane & 15));
            gather_row_bf16_d128<IdxT>(qv, reinterpret_cast<const uint4*>(kb) + (lane & 15),
                                       reinterpret_cast<const uint4*>(vb) + (lane & 15), idx + row * K, K, N, i,
                                       causal, scale_log2, out + row * D, lane);
        }
        return;
    }

    // ---- 3.-5. the union in chunks of kMmaChunk keys
    const uint32_t st_s = (uint32_t)__cvta_generic_to_shared(stage);  // key rows: two chunk buffers
    const uint32_t vst_s = st_s + 2u * kChunkBytes;                    // value rows of one chunk
    // Staging: lane copies the 16-byte piece pc = lane % 16 of rows lane / 16 + 2 r of a
    // chunk; rows past the chunk's keys are zero-filled (source size 0).
    auto stage_rows = [&](uint32_t dst_base, const __nv_bfloat16* base, int c0) {
        const int nk = min(kMmaChunk, U - c0);
        const int pc = lane & 15;
#pragma unroll
        for (int r = 0; r < kMmaChunk / 2; ++r) {
            const int row = 2 * r + (lane >> 4);
            const bool valid = row < nk;
            const int key = valid ? ukey[c0 + row] : 0;
            const uint32_t dst = dst_base + (uint32_t)(row * kRowBytes + ((pc ^ (row & 7)) << 4));
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst),
                         "l"(base + (size_t)key * D + pc * 8), "r"(valid ? 16 : 0)
                         : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    // ldmatrix row addresses (16 rows of a chunk, 16-byte pieces).  Key rows, the A
    // operand of S^T (no transpose): lanes 0-7 / 8-15 / 16-23 / 24-31 give key rows
    // 0..7 / 8..15 / 0..7 / 8..15 at piece 2 s / 2 s / 2 s + 1 / 2 s + 1 (k-step s).
    // Value rows, the A operand of O^T (transposed): key rows 0..7 / 0..7 / 8..15 /
    // 8..15 at piece 2 mt / 2 mt + 1 / 2 mt / 2 mt + 1 (dims 16 mt .. 16 mt + 15).
    const int krow = (lane & 7) + ((lane >> 3) & 1) * 8, kpc = lane >> 4;
    const int vrow = (lane & 7) + (lane >> 4) * 8, vpc = (lane >> 3) & 1;
    // O^T accumulators: dims 16 mt + gq (+8) of heads 2 c4, 2 c4 + 1
    float oacc[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) oacc[n][0] = oacc[n][1] = oacc[n][2] = oacc[n][3] = 0.f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};  // heads 2 c4, 2 c4 + 1
    const int nch = (U + kMmaChunk - 1) / kMmaChunk;
    if (nch > 0) stage_rows(st_s, kb, 0);
    for (int c = 0; c < nch; ++c) {
        const int c0 = c * kMmaChunk;
        const int nk = min(kMmaChunk, U - c0);
        const bool more = c + 1 < nch;  // warp-uniform
        __syncwarp();  // chunk c - 1 is done with the value rows and with key buffer (c + 1) & 1
        stage_rows(vst_s, vb, c0);
        if (more) stage_rows(st_s + (uint32_t)(((c + 1) & 1) * kChunkBytes), kb, c0 + kMmaChunk);
        // groups in flight: key rows of c, value rows of c, key rows of c + 1 (if any)
        if (more) cp_async_wait_pending<2>();
        else cp_async_wait_pending<1>();
        __syncwarp();
        // S^T = K Q^T of the chunk: keys gq, gq + 8 x heads 2 c4, 2 c4 + 1
        const uint32_t kst = st_s + (uint32_t)((c & 1) * kChunkBytes);
        float sacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            const int piece = 2 * s + kpc;
            uint32_t a0, a1, a2, a3;
            asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                         : "=r"(a0), "=r"(a1), "=r"(a2), "=r"(a3)
                         : "r"(kst + (uint32_t)(krow * kRowBytes + ((piece ^ (krow & 7)) << 4))));
            mma_bf16_16816_a4(sacc, a0, a1, a2, a3, qa[2 * s], qa[2 * s + 1]);
        }
        // online softmax per head over its selected keys c0 + gq, c0 + gq + 8; a head's
        // scores sit in the eight lanes of equal c4
        bool sel[2][2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int ul = gq + 8 * h;
            const unsigned hb = ul < nk ? umask[c0 + ul] : 0u;
#pragma unroll
            for (int e = 0; e < 2; ++e) sel[h][e] = 2 * c4 + e < G && ((hb >> (2 * c4 + e)) & 1u);
        }
        float mx[2], alpha[2], pr[2][2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const float s0 = sel[0][e] ? sacc[e] * scale_log2 : -INFINITY;
            const float s1 = sel[1][e] ? sacc[2 + e] * scale_log2 : -INFINITY;
            float m = fmaxf(s0, s1);
            m = fmaxf(m, __shfl_xor_sync(kFull, m, 4));
            m = fmaxf(m, __shfl_xor_sync(kFull, m, 8));
            m = fmaxf(m, __shfl_xor_sync(kFull, m, 16));
            mx[e] = fmaxf(m_run[e], m);
            alpha[e] = mx[e] == -INFINITY ? 1.f : exp2f(m_run[e] - mx[e]);
            pr[0][e] = mx[e] == -INFINITY ? 0.f : exp2f(s0 - mx[e]);
            pr[1][e] = mx[e] == -INFINITY ? 0.f : exp2f(s1 - mx[e]);
            float sum = pr[0][e] + pr[1][e];
            sum += __shfl_xor_sync(kFull, sum, 4);
            sum += __shfl_xor_sync(kFull, sum, 8);
            sum += __shfl_xor_sync(kFull, sum, 16);
            l_run[e] = l_run[e] * alpha[e] + sum;
            m_run[e] = mx[e];
        }
#pragma unroll
        for (int n = 0; n < 8; ++n) {
            oacc[n][0] *= alpha[0];
            oacc[n][1] *= alpha[1];
            oacc[n][2] *= alpha[0];
            oacc[n][3] *= alpha[1];
        }
        // P^T as the B operand: each 8 x 8 (keys x heads) half of the score tile,
        // rounded to bf16, transposed across the warp
        const uint32_t pb0 = movmatrix_trans(pack_bf16x2(pr[0][0], pr[0][1]));
        const uint32_t pb1 = movmatrix_trans(pack_bf16x2(pr[1][0], pr[1][1]));
        // O^T += V^T P^T of the chunk
        if (more) cp_async_wait_pending<1>();
        else cp_async_wait_pending<0>();
        __syncwarp();
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
            const int pc = 2 * mt + vpc;
            uint32_t a0, a1, a2, a3;
            asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                         : "=r"(a0), "=r"(a1), "=r"(a2), "=r"(a3)
                         : "r"(vst_s + (uint32_t)(vrow * kRowBytes + ((pc ^ (vrow & 7)) << 4))));
            mma_bf16_16816_a4(oacc[mt], a0, a1, a2, a3, pb0, pb1);
        }
    }
    // each head's row divided by its sum; the 8 x 8 (dims x heads) halves of every O^T
    // tile transposed back, so lane (gq, c4) stores dims 2 c4, 2 c4 + 1 of head gq
    const float inv0 = l_run[0] > 0.f ? 1.f / l_run[0] : 0.f;
    const float inv1 = l_run[1] > 0.f ? 1.f / l_run[1] : 0.f;
    __nv_bfloat16* orow = out + (row0 + (size_t)(gq < G ? gq : 0) * Nq) * D + 2 * c4;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
        const uint32_t lo = movmatrix_trans(pack_bf16x2(oacc[mt][0] * inv0, oacc[mt][1] * inv1));
        const uint32_t hi = movmatrix_trans(pack_bf16x2(oacc[mt][2] * inv0, oacc[mt][3] * inv1));
        if (gq < G) {
            *reinterpret_cast<uint32_t*>(orow + 16 * mt) = lo;
            *reinterpret_cast<uint32_t*>(orow + 16 * mt + 8) = hi;
        }
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
        const int G = a.H / a.Hkv;
        if (a.D == 128 && a.K <= 128 && (G == 2 || G == 3 || G == 4 || G == 6 || G == 8)) {
            const bool big = a.K > 64;
            const bool direct = a.N <= kDirectMaxN && a.K <= 64;
#define OSSA_MMA_PICK(GG)                                                                      \
    (direct ? gather_attn_bf16_d128_mma_kernel<IdxT, GG, 8, true>                              \
            : (big ? gather_attn_bf16_d128_mma_kernel<IdxT, GG, 9, false>                      \
                   : gather_attn_bf16_d128_mma_kernel<IdxT, GG, 8, false>))
            auto kern = G == 2 ? OSSA_MMA_PICK(2)
                      : G == 3 ? OSSA_MMA_PICK(3)
                      : G == 4 ? OSSA_MMA_PICK(4)
                      : G == 6 ? OSSA_MMA_PICK(6)
                               : OSSA_MMA_PICK(8);
#undef OSSA_MMA_PICK
            const size_t kMmaSmem =
                direct ? mma_smem_bytes<8, true>() : (big ? mma_smem_bytes<9, false>() : mma_smem_bytes<8, false>());
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMmaSmem);
            if (e != cudaSuccess) return e;
            dim3 mgrid((Nq + kMmaWarps - 1) / kMmaWarps, a.B * a.Hkv);
            kern<<<mgrid, kMmaWarps * 32, kMmaSmem, stream>>>(q, k, v, ix, o, a.H, a.Hkv, a.N, Nq, a.q0, a.K,
                                                              scale_log2, a.causal);
            e = cudaGetLastError();
            if (e == cudaSuccess) note_launch();
            return e;
        }
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
