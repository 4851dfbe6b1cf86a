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
//  1. union: the G index rows must be in the selectors' form (valid entries first,
//     strictly ascending; else the query goes through gather_row_bf16_d128 per head).
//     Every valid key goes into an open-addressing hash in shared memory with its
//     head bit; the occupied slots, compacted in slot order, are the union (at most
//     kMmaMaxU keys, else per head).  The q rows are loaded before the union is built,
//     so their latency overlaps it.
//  2. the union in chunks of 32 keys: its value rows are copied to shared memory
//     (cp.async, 16-byte pieces XOR-swizzled by row) while the scores of the chunk
//     S = Q K_U^T run on mma.sync m16n8k16 (bf16 operands, fp32 accumulation): A =
//     the G heads' q rows (rows G..15 zero), B = 8 union keys per n-tile.  The
//     contraction runs over the head dims in a permuted order, the same for A and B
//     (lane c = lane % 4 of a quad supplies dims 32c .. 32c + 31, four per k-step),
//     so each lane loads one contiguous 64-byte piece of a key row per n-tile;
//  3. online softmax per head over its selected keys (head bit set; others masked):
//     a head's scores sit in the four lanes of one quad, reduced by two shuffles;
//     p is rounded to bf16 for p.v, as in the per-head form;
//  4. O += P V_chunk with mma.sync: P from the score fragments (no shuffles), V as
//     the B operand by ldmatrix.trans from the staged rows; at the end each head's
//     row is divided by its sum and stored as bf16.
// Results agree with the per-head form to rounding (tensor-core accumulation order).
// The union hash has 2^kSlotBits slots and holds at most half as many keys: 256
// slots (128 keys) for K <= 64, 512 slots (256 keys) above.  With N <= 4096 keys and
// K <= 64 the union is built instead in a per-warp byte array indexed by the key
// (kDirect): byte j holds the head bits of key j, set by one atomicOr per selected
// key, so there is no probing and no compare-and-swap; a head bit that is already set
// marks a repeated key (the per-head form then takes the query).  The entry of the
// lowest head that selected a key appends it to the union list.
constexpr int kMmaChunk = 32;     // union keys per chunk: 4 score n-tiles, 2 value k-steps
constexpr int kMmaWarps = 8;
constexpr int kDirectMaxN = 4096;  // keys covered by the direct head-bit array
constexpr int kDirectMaxU = 128;   // union entries of the direct form
// Per warp: the value rows of a chunk (kMmaChunk x 256 B; the direct head-bit array,
// kDirectMaxN bytes, uses the same space before the first chunk), then the hash
// slots / union list.
template <int kSlotBits, bool kDirect>
constexpr size_t mma_warp_smem() {
    return (size_t)kMmaChunk * 256 + (kDirect ? (size_t)kDirectMaxU * 8 : ((size_t)8 << kSlotBits));
}
static_assert(kDirectMaxN <= kMmaChunk * 256, "the direct head-bit array fits in the value staging area");
template <int kSlotBits, bool kDirect>
constexpr size_t mma_smem_bytes() { return kMmaWarps * mma_warp_smem<kSlotBits, kDirect>(); }
static_assert(mma_warp_smem<8, true>() % 16 == 0 && mma_warp_smem<9, false>() % 16 == 0, "warp areas stay 16-byte aligned");

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}

template <typename IdxT, int G, int kSlotBits, bool kDirect>
__global__ void __launch_bounds__(kMmaWarps * 32, 2)
gather_attn_bf16_d128_mma_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                                 const __nv_bfloat16* __restrict__ v, const IdxT* __restrict__ idx,
                                 __nv_bfloat16* __restrict__ out, int H, int Hkv, int N, int Nq, int q0, int K,
                                 float scale_log2, int causal) {
    constexpr int D = 128;
    constexpr int kMmaSlots = kDirect ? kDirectMaxU : 1 << kSlotBits;
    constexpr int kMmaMaxU = kDirect ? kDirectMaxU : kMmaSlots / 2;
    constexpr size_t kMmaWarpSmem = mma_warp_smem<kSlotBits, kDirect>();
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
    uint8_t* vs = msm + (size_t)warp * kMmaWarpSmem;  // [kMmaChunk][256 B], pieces swizzled
    int* ukey = reinterpret_cast<int*>(vs + kMmaChunk * 256);       // hash slots, then the union
    unsigned* umask = reinterpret_cast<unsigned*>(ukey + kMmaSlots);
    uint32_t* dbits = reinterpret_cast<uint32_t*>(vs);  // direct: head bits, 4 keys per word (until chunk 0)
    const __nv_bfloat16* kb = k + (size_t)bg * N * D;
    const __nv_bfloat16* vb = v + (size_t)bg * N * D;
    const size_t row0 = ((size_t)b * H + (size_t)g * G) * Nq + il;  // head t: row0 + t * Nq

    // ---- 1. union of the heads' keys with head bits into ukey / umask: the direct
    // head-bit array (kDirect), or an open-addressing hash in shared memory
    // (kMmaSlots slots, linear probing) compacted by ballot into the same arrays in
    // slot order
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
    // q rows of the heads as A fragments (dims 32 c4 .. 32 c4 + 31 of head gq), loaded
    // now so that their latency overlaps the union build
    uint32_t qa[16];
    {
        const uint4* qp = reinterpret_cast<const uint4*>(q + (row0 + (size_t)gq * Nq) * D + 32 * c4);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const uint4 xq = gq < G ? __ldg(qp + u) : make_uint4(0u, 0u, 0u, 0u);
            qa[4 * u + 0] = xq.x;
            qa[4 * u + 1] = xq.y;
            qa[4 * u + 2] = xq.z;
            qa[4 * u + 3] = xq.w;
        }
    }
    bool canon = true;
    int U = 0;
    if constexpr (kDirect) {
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
                        if (pos < kMmaMaxU) {
                            ukey[pos] = xv;
                            umask[pos] = mk;
                        }
                    }
                    U += __popc(bal);
                }
            }
        }
        __syncwarp();
    } else {
#pragma unroll
        for (int u = 0; u < kMmaSlots / 32; ++u) {
            ukey[lane + 32 * u] = -1;
            umask[lane + 32 * u] = 0u;
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
                        for (int probe = 0; probe < kMmaSlots; ++probe) {
                            const int old = atomicCAS(&ukey[slot], -1, xv);
                            if (old == -1 || old == xv) {
                                atomicOr(&umask[slot], 1u << t);
                                break;
                            }
                            slot = (slot + 1) & (kMmaSlots - 1);
                        }
                    }
                }
            }
        }
        __syncwarp();
        {
            int kk[kMmaSlots / 32];
            unsigned mk[kMmaSlots / 32];
#pragma unroll
            for (int u = 0; u < kMmaSlots / 32; ++u) {
                // lane owns slots S lane .. S lane + S - 1, S = kMmaSlots / 32
                kk[u] = ukey[(kMmaSlots / 32) * lane + u];
                mk[u] = umask[(kMmaSlots / 32) * lane + u];
            }
            __syncwarp();
            int nmine = 0;
#pragma unroll
            for (int u = 0; u < kMmaSlots / 32; ++u) nmine += kk[u] >= 0 ? 1 : 0;
            int before = nmine;  // inclusive prefix over lanes
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(kFull, before, o);
                if (lane >= o) before += y;
            }
            U = __shfl_sync(kFull, before, 31);
            int pos = before - nmine;
#pragma unroll
            for (int u = 0; u < kMmaSlots / 32; ++u) {
                if (kk[u] >= 0) {
                    if (pos < kMmaMaxU) {
                        ukey[pos] = kk[u];
                        umask[pos] = mk[u];
                    }
                    ++pos;
                }
            }
            __syncwarp();
        }
    }
    if (!canon || U > kMmaMaxU) {
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

    const uint32_t vs_s = (uint32_t)__cvta_generic_to_shared(vs);
    // ldmatrix.x4.trans: lanes 0-7 / 8-15 / 16-23 / 24-31 address rows of keys
    // +0..7 / +8..15 / +0..7 / +8..15 at dims 16 np (first two) and 16 np + 8 (last two)
    const int lrow = (lane & 7) + ((lane >> 3) & 1) * 8;
    const int lcol = lane >> 4;
    float oacc[16][4];
#pragma unroll
    for (int n = 0; n < 16; ++n) oacc[n][0] = oacc[n][1] = oacc[n][2] = oacc[n][3] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;

    for (int c0 = 0; c0 < U; c0 += kMmaChunk) {
        const int nk = min(kMmaChunk, U - c0);
        const int nt = (nk + 7) >> 3;      // score n-tiles of this chunk
        const int nks = (nk + 15) >> 4;    // value k-steps of this chunk
        // value rows of the chunk to shared memory (zero rows up to a multiple of 16)
        __syncwarp();  // the previous chunk's ldmatrix reads are done
        for (int e = lane; e < nks * 16 * 16; e += 32) {
            const int row = e >> 4, pc = e & 15;
            const uint32_t dst = vs_s + (uint32_t)(row * 256 + ((pc ^ (row & 7)) << 4));
            if (row < nk) {
                const void* src = vb + (size_t)ukey[c0 + row] * D + pc * 8;
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
            } else {
                asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(dst), "r"(0u) : "memory");
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        // scores of the chunk
        float sacc[kMmaChunk / 8][4];
#pragma unroll
        for (int t = 0; t < kMmaChunk / 8; ++t) {
            sacc[t][0] = sacc[t][1] = sacc[t][2] = sacc[t][3] = 0.f;
            if (t < nt) {
                const int u = c0 + 8 * t + gq;
                const int j = 8 * t + gq < nk ? ukey[u] : 0;
                const uint4* kp = reinterpret_cast<const uint4*>(kb + (size_t)j * D + 32 * c4);
                uint32_t kw[16];
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    const uint4 xk = __ldg(kp + w);
                    kw[4 * w + 0] = xk.x;
                    kw[4 * w + 1] = xk.y;
                    kw[4 * w + 2] = xk.z;
                    kw[4 * w + 3] = xk.w;
                }
#pragma unroll
                for (int s = 0; s < 8; ++s) mma_bf16_16816(sacc[t], qa[2 * s], qa[2 * s + 1], kw[2 * s], kw[2 * s + 1]);
            }
        }
        // online softmax of head gq over its selected keys c0 + 8 t + 2 c4 + e
        float mx = -INFINITY;
#pragma unroll
        for (int t = 0; t < kMmaChunk / 8; ++t) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int ul = 8 * t + 2 * c4 + e;
                const bool sel = ul < nk && gq < G && ((umask[c0 + ul] >> gq) & 1u);
                sacc[t][e] = sel ? sacc[t][e] * scale_log2 : -INFINITY;
                mx = fmaxf(mx, sacc[t][e]);
            }
        }
        mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 2));
        const float m_new = fmaxf(m_run, mx);
        const float alpha = m_new == -INFINITY ? 1.f : exp2f(m_run - m_new);
        float sum = 0.f;
        uint32_t pa[kMmaChunk / 8];
#pragma unroll
        for (int t = 0; t < kMmaChunk / 8; ++t) {
            const float p0 = m_new == -INFINITY ? 0.f : exp2f(sacc[t][0] - m_new);
            const float p1 = m_new == -INFINITY ? 0.f : exp2f(sacc[t][1] - m_new);
            sum += p0 + p1;
            pa[t] = pack_bf16x2(p0, p1);
        }
        sum += __shfl_xor_sync(kFull, sum, 1);
        sum += __shfl_xor_sync(kFull, sum, 2);
        l_run = l_run * alpha + sum;
        m_run = m_new;
#pragma unroll
        for (int n = 0; n < 16; ++n) {
            oacc[n][0] *= alpha;
            oacc[n][1] *= alpha;
        }
        // O += P V of the chunk
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncwarp();
#pragma unroll
        for (int ks = 0; ks < kMmaChunk / 16; ++ks) {
            if (ks < nks) {
                const int row = 16 * ks + lrow;
#pragma unroll
                for (int np = 0; np < 8; ++np) {
                    const int pc = 2 * np + lcol;
                    uint32_t r0, r1, r2, r3;
                    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                                 : "r"(vs_s + (uint32_t)(row * 256 + ((pc ^ (row & 7)) << 4))));
                    mma_bf16_16816(oacc[2 * np], pa[2 * ks], pa[2 * ks + 1], r0, r1);
                    mma_bf16_16816(oacc[2 * np + 1], pa[2 * ks], pa[2 * ks + 1], r2, r3);
                }
            }
        }
    }
    if (gq < G) {
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        __nv_bfloat16* orow = out + (row0 + (size_t)gq * Nq) * D + 2 * c4;
#pragma unroll
        for (int n = 0; n < 16; ++n)
            *reinterpret_cast<uint32_t*>(orow + 8 * n) = pack_bf16x2(oacc[n][0] * inv, oacc[n][1] * inv);
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
