// Fused causal top-K key selection with exact fp32 scores (CUDA cores).
//
// Replaces, per (b, h), the reference's materialised selector and torch.topk
// (ossa/router.py:171-190 + ossa/bench/sparse_forward.py:180-202 for the router,
// :194-202 for the exact-dot oracle): the N x N score matrix never exists.
//
// Score definition (bit-exact against the CPU oracle):
//   dot(i,j)   = fmaf-chain over c = 0..R-1 of a_i[c] * b_j[c]   (from 0.0f)
//   score(i,j) = fl(fl(dot * scale) + bias[clamp(i - j + L, 0, 2L-1)])   (router)
//              = fl(dot * scale)                                         (oracle)
// Selection: among j <= i (causal) or all j, the K largest by (score desc, j asc)
// with torch.topk's value order (NaN above +inf); emitted in ascending j, padded
// with -1.
//
// Structure: a CTA owns 128 query rows of one (b, h); thread t owns row i0 + t
// and keeps a_i in registers.  Keys stream in tiles of 32 (staged row-major in
// shared memory, read back as float4 broadcasts), 8 independent fmaf chains per
// thread.  Each row has a candidate buffer in shared memory (CAP = 32*EPL
// entries of {order key, j}, rotated by row to spread banks) and a threshold
// theta = key of the current K-th best: a score enters only if its key > theta.
// Because keys arrive in ascending j, a later key that ties theta loses the
// tie-break and is correctly dropped.  When a buffer nears CAP the warp compacts
// that row cooperatively: a 32-step radix select over the order keys finds the
// exact K-th key, then a stable ballot compaction keeps the K winners in
// position (= ascending j) order and raises theta.
#include "common.cuh"
#include "kernels.h"

namespace ossa {

namespace {

constexpr int kRows = 128;     // query rows per CTA (one per thread)
constexpr int kKeyTile = 32;   // keys per shared-memory tile

template <int EPL>
__device__ __forceinline__ void warp_compact_row(uint2* rowbuf, int rot, int cnt, int K, int lane,
                                                 uint32_t& theta_out, int& cnt_out) {
    constexpr int CAP = 32 * EPL;
    uint32_t u[EPL], jv[EPL];
    bool val[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
        const int p = lane + 32 * e;
        val[e] = p < cnt;
        int slot = p + rot;
        if (slot >= CAP) slot -= CAP;
        const uint2 t = val[e] ? rowbuf[slot] : make_uint2(0u, 0u);
        u[e] = t.x;
        jv[e] = t.y;
    }
    // Radix select: prefix becomes the K-th largest key, kk its rank among ties.
    uint32_t prefix = 0u, mask = 0u;
    int kk = K;
#pragma unroll 1
    for (int bit = 31; bit >= 0; --bit) {
        const uint32_t m2 = mask | (1u << bit);
        const uint32_t cand = prefix | (1u << bit);
        unsigned c = 0;
#pragma unroll
        for (int e = 0; e < EPL; ++e) c += (val[e] && (u[e] & m2) == cand) ? 1u : 0u;
        c = __reduce_add_sync(kFull, c);
        if ((int)c >= kk) prefix = cand; else kk -= (int)c;
        mask = m2;
    }
    __syncwarp();
    const unsigned lt = lanemask_lt();
    int outpos = 0, ties = 0;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
        const bool tie = val[e] && u[e] == prefix;
        const unsigned tb = __ballot_sync(kFull, tie);
        const bool keep = val[e] && (u[e] > prefix || (tie && ties + __popc(tb & lt) < kk));
        const unsigned kb = __ballot_sync(kFull, keep);
        if (keep) {
            int slot = outpos + __popc(kb & lt) + rot;
            if (slot >= CAP) slot -= CAP;
            rowbuf[slot] = make_uint2(u[e], jv[e]);
        }
        outpos += __popc(kb);
        ties += __popc(tb);
    }
    __syncwarp();
    theta_out = prefix;
    cnt_out = outpos;
}

template <int R, typename KT, bool BIAS, int EPL>
__global__ void __launch_bounds__(kRows, 1)
score_topk_kernel(const KT* __restrict__ qrows, const KT* __restrict__ krows,
                  const float* __restrict__ bias, int L, int H, int Hkv, int N, int Nq, int q0, int K,
                  float scale, int causal, int32_t* __restrict__ out, int nqb) {
    constexpr int CAP = 32 * EPL;
    constexpr int KS = R + 4;  // padded key-row stride in shared memory (float4 aligned)
    extern __shared__ float4 smem4[];
    float* Ks = reinterpret_cast<float*>(smem4);                  // [kKeyTile][KS]
    uint2* buf = reinterpret_cast<uint2*>(Ks + kKeyTile * KS);    // [kRows][CAP]

    const int BH = gridDim.x / nqb;
    const int order = blockIdx.x / BH;            // heavy (late) query blocks first
    const int bh = blockIdx.x - order * BH;
    const int qb = causal ? (nqb - 1 - order) : order;
    const int b = bh / H;
    const int h = bh - b * H;
    const int g = h / (H / Hkv);
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int i0 = qb * kRows;          // first query row of the block (local)
    const int il = i0 + tid;
    const bool active = il < Nq;
    const int i = q0 + il;              // its position in the key sequence

    float a[R];
    {
        const KT* qp = qrows + ((size_t)bh * Nq + (active ? il : 0)) * R;
#pragma unroll
        for (int c = 0; c < R; ++c) a[c] = active ? to_f32(qp[c]) : 0.f;
    }
    const KT* kb = krows + (size_t)(b * Hkv + g) * N * R;
    uint2* rowbuf = buf + (size_t)tid * CAP;
    const int rot = tid % CAP;

    uint32_t theta = 0u;  // order key threshold; 0 admits every real score
    int cnt = 0;
    const int jend = causal ? min(N, q0 + i0 + kRows) : N;

    for (int j0 = 0; j0 < jend; j0 += kKeyTile) {
        __syncthreads();
        for (int e = tid; e < kKeyTile * R; e += kRows) {
            const int jj = e / R, c = e - jj * R;
            const int j = j0 + jj;
            Ks[jj * KS + c] = j < N ? to_f32(kb[(size_t)j * R + c]) : 0.f;
        }
        __syncthreads();

#pragma unroll 1
        for (int jg = 0; jg < kKeyTile; jg += 8) {
            float acc[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) acc[t] = 0.f;
#pragma unroll
            for (int c4 = 0; c4 < R; c4 += 4) {
#pragma unroll
                for (int t = 0; t < 8; ++t) {
                    const float4 kv = *reinterpret_cast<const float4*>(Ks + (jg + t) * KS + c4);
                    acc[t] = fmaf(a[c4 + 0], kv.x, acc[t]);
                    acc[t] = fmaf(a[c4 + 1], kv.y, acc[t]);
                    acc[t] = fmaf(a[c4 + 2], kv.z, acc[t]);
                    acc[t] = fmaf(a[c4 + 3], kv.w, acc[t]);
                }
            }
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                const int j = j0 + jg + t;
                const bool valid = active && j < N && (!causal || j <= i);
                float s = __fmul_rn(acc[t], scale);
                if constexpr (BIAS) {
                    int bi = i - j + L;
                    bi = bi < 0 ? 0 : (bi > 2 * L - 1 ? 2 * L - 1 : bi);
                    s = __fadd_rn(s, __ldg(bias + bi));
                }
                const uint32_t u = order_key(s);
                if (valid && u > theta) {
                    int slot = cnt + rot;
                    if (slot >= CAP) slot -= CAP;
                    rowbuf[slot] = make_uint2(u, (uint32_t)j);
                    ++cnt;
                }
            }
        }

        // Rows that could overflow during the next tile are compacted now.
        unsigned need = __ballot_sync(kFull, cnt > CAP - kKeyTile);
        while (need) {
            const int src = __ffs(need) - 1;
            need &= need - 1;
            const int scnt = __shfl_sync(kFull, cnt, src);
            const int srot = __shfl_sync(kFull, rot, src);
            uint32_t nt;
            int nc;
            warp_compact_row<EPL>(buf + (size_t)((tid & ~31) + src) * CAP, srot, scnt, K, lane, nt, nc);
            if (lane == src) {
                theta = nt;
                cnt = nc;
            }
        }
    }

    // Final selection and coalesced write-out, one row of the warp at a time.
    const int wbase = tid & ~31;
    for (int src = 0; src < 32; ++src) {
        const int row_i = i0 + wbase + src;
        if (row_i >= Nq) break;  // warp-uniform
        int scnt = __shfl_sync(kFull, cnt, src);
        const int srot = __shfl_sync(kFull, rot, src);
        uint2* sbuf = buf + (size_t)(wbase + src) * CAP;
        if (scnt > K) {
            uint32_t nt;
            int nc;
            warp_compact_row<EPL>(sbuf, srot, scnt, K, lane, nt, nc);
            scnt = nc;
        }
        int32_t* orow = out + ((size_t)bh * Nq + row_i) * K;
        for (int p = lane; p < K; p += 32) {
            int32_t jv = -1;
            if (p < scnt) {
                int slot = p + srot;
                if (slot >= CAP) slot -= CAP;
                jv = (int32_t)sbuf[slot].y;
            }
            orow[p] = jv;
        }
        __syncwarp();
    }
}

template <int R, typename KT, bool BIAS, int EPL>
cudaError_t launch_cfg(const ScoreTopkArgs& a, cudaStream_t stream) {
    constexpr int CAP = 32 * EPL;
    const size_t smem = (size_t)kKeyTile * (R + 4) * sizeof(float) + (size_t)kRows * CAP * sizeof(uint2);
    auto kern = score_topk_kernel<R, KT, BIAS, EPL>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const int Nq = a.Nq > 0 ? a.Nq : a.N;
    const int nqb = (Nq + kRows - 1) / kRows;
    const long long nblk = (long long)nqb * a.B * a.H;
    if (nblk == 0) return cudaSuccess;
    kern<<<(unsigned)nblk, kRows, smem, stream>>>(
        static_cast<const KT*>(a.qrows), static_cast<const KT*>(a.krows), a.bias, a.L,
        a.H, a.Hkv, a.N, Nq, a.q0, a.K, a.scale, a.causal, a.out, nqb);
    cudaError_t err = cudaGetLastError();
    if (err == cudaSuccess) note_launch();
    return err;
}

// CAP must leave one key tile of room after a compaction to K entries.
inline int pick_epl(int K) {
    if (K + kKeyTile <= 64) return 2;
    if (K + kKeyTile <= 128) return 4;
    if (K + kKeyTile <= 192) return 6;
    return 0;
}

template <int R, typename KT, bool BIAS>
cudaError_t launch_epl(const ScoreTopkArgs& a, cudaStream_t stream) {
    switch (pick_epl(a.K)) {
        case 2: return launch_cfg<R, KT, BIAS, 2>(a, stream);
        case 4: return launch_cfg<R, KT, BIAS, 4>(a, stream);
        case 6: return launch_cfg<R, KT, BIAS, 6>(a, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

bool score_topk_supported(int R, int K) {
    return (R == 16 || R == 32 || R == 64 || R == 128) && K >= 1 && pick_epl(K) != 0;
}

cudaError_t launch_score_topk(const ScoreTopkArgs& a, cudaStream_t stream) {
    const bool bias = a.bias != nullptr;
    if (a.dtype == kF32) {
        switch (a.R) {
            case 16: return bias ? launch_epl<16, float, true>(a, stream) : launch_epl<16, float, false>(a, stream);
            case 32: return bias ? launch_epl<32, float, true>(a, stream) : launch_epl<32, float, false>(a, stream);
            case 64: return bias ? launch_epl<64, float, true>(a, stream) : launch_epl<64, float, false>(a, stream);
            case 128: return bias ? launch_epl<128, float, true>(a, stream) : launch_epl<128, float, false>(a, stream);
            default: return cudaErrorInvalidValue;
        }
    }
    // bf16 rows only occur for the exact-dot oracle selector (no bias).
    switch (a.R) {
        case 16: return launch_epl<16, __nv_bfloat16, false>(a, stream);
        case 32: return launch_epl<32, __nv_bfloat16, false>(a, stream);
        case 64: return launch_epl<64, __nv_bfloat16, false>(a, stream);
        case 128: return launch_epl<128, __nv_bfloat16, false>(a, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace ossa
