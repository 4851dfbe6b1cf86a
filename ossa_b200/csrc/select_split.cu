// Exact causal top-K for a few query rows against many keys: the decode shape
// (one new query per (b, h) against a long key cache), served through the
// query-row entry points (ossa_router_topk_rows with Nq = 1, q_start = the
// position).  The reference has no decode path: its patched forward is
// prefill-only (ossa/bench/sparse_forward.py:157-160); the scores and the
// selection rule are those of the router selector (ossa/router.py:171-190,
// sparse_forward.py:180-202), identical to score_topk.cu's.
//
// The CTA-per-128-rows selector of score_topk.cu gives such a row one thread,
// which walks every key alone.  Here the keys of a row are split into ranges of
// kSplitKeys:
//  1. split_scan_kernel: one warp per (row, range) computes the canonical fp32
//     scores of its range (lane = key) and keeps the range's K best in a
//     streaming warp list (threshold = the current K-th key, compaction in
//     position order, as the exact fallback selector does); the winners go to
//     global memory in ascending key order.
//  2. split_merge_kernel: one CTA per row.  Each range also reports its K-th
//     best order key; the largest of them is a lower bound on the row's K-th
//     best (that range alone has K keys at or above it), so only entries at or
//     above it enter the lists.  Warp w streams the winners of a contiguous
//     group of ranges, in range order, through the same streaming list; warp 0
//     then streams the 8 group lists in group order (keys still ascending) and
//     writes the K best ascending, -1 padded.
// Every key of the exact top K is among its range's K best, and ties at the
// K-th score go to the lower key index in both stages, so the result is the
// exact top K by (score desc, key asc).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "select_warp.cuh"

namespace ossa {

namespace {

constexpr int kSplitKeys = 1024;  // keys per warp range

// Streaming top-K of one warp over entries pushed 32 at a time in ascending key
// order.  An entry enters the list only if its order key beats the current
// K-th key (a later entry that ties it has a higher key index and loses); a
// list close to full keeps its K best in position order.  `wb` holds 32 * EPL
// entries (K + 32 <= 32 * EPL).
template <int EPL>
struct WarpStreamTopK {
    uint2* wb;
    int K;
    int cnt = 0;
    uint32_t theta = 0u;  // order keys of real scores are never 0

    __device__ __forceinline__ void keep_best(int lane, unsigned lt, bool raise_theta) {
        uint32_t u[EPL], jv[EPL];
        bool val[EPL], keep[EPL];
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
            const int q = lane + 32 * e;
            val[e] = q < cnt;
            const uint2 t = val[e] ? wb[q] : make_uint2(0u, 0u);
            u[e] = t.x;
            jv[e] = t.y;
        }
        uint32_t Tk;
        warp_topk_mask<EPL>(u, val, K, keep, &Tk);
        __syncwarp();
        int outpos = 0;
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
            const unsigned kb = __ballot_sync(kFull, keep[e]);
            if (keep[e]) wb[outpos + __popc(kb & lt)] = make_uint2(u[e], jv[e]);
            outpos += __popc(kb);
        }
        __syncwarp();
        cnt = outpos;
        if (raise_theta) theta = Tk;
    }

    __device__ __forceinline__ void push(bool valid, uint32_t key, uint32_t j, int lane, unsigned lt) {
        const bool adm = valid && key > theta;
        const unsigned bal = __ballot_sync(kFull, adm);
        if (adm) wb[cnt + __popc(bal & lt)] = make_uint2(key, j);
        cnt += __popc(bal);
        __syncwarp();
        if (cnt > 32 * EPL - 32) keep_best(lane, lt, true);
    }

    // Leaves the (at most K) winners in wb[0 .. return) in position order.
    __device__ __forceinline__ int finish(int lane, unsigned lt) {
        if (cnt > K) keep_best(lane, lt, false);
        return cnt;
    }
};

// Four warps per CTA.  Each warp stages the k' rows of its next 32 keys in
// shared memory, 64 columns at a time, with coalesced 16-byte loads (a lane
// loading its own 256-byte row would touch 32 lines per instruction); the row
// stride of CH + 4 floats makes each lane's 16-byte reads of its own row
// conflict-free.  Lane l then continues key l's fmaf chain over the chunk, so
// each score is the canonical one score_topk.cu selects on: the fmaf chain over
// c = 0..R-1 in order from 0, times scale, plus the position-bias term.
constexpr int kScanWarps = 4;

template <int R, bool kBias, int EPL>
__global__ void __launch_bounds__(32 * kScanWarps)
split_scan_kernel(const float* __restrict__ qp, const float* __restrict__ kp, const float* __restrict__ bias, int L,
                  int H, int Hkv, int N, int Nq, int q0, int K, float scale, int causal, long long rows, int nsplit,
                  uint2* __restrict__ cand, int* __restrict__ ccount, uint32_t* __restrict__ ckth) {
    constexpr int CH = R < 64 ? R : 64;  // columns per staged chunk
    constexpr int ST = CH + 4;            // row stride in floats
    __shared__ uint2 sbuf[kScanWarps][32 * EPL];
    __shared__ __align__(16) float stile[kScanWarps][32 * ST];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const long long gw = (long long)blockIdx.x * kScanWarps + warp;
    if (gw >= rows * nsplit) return;  // whole warps
    const unsigned lt = lanemask_lt();
    const long long row = gw / nsplit;
    const int sp = (int)(gw - row * nsplit);
    const long long bh = row / Nq;
    const int i = q0 + (int)(row - bh * Nq);
    const int b = (int)(bh / H);
    const int g = (int)(bh - (long long)b * H) / (H / Hkv);
    const float* qrow = qp + row * R;
    const float* kbase = kp + (size_t)(b * Hkv + g) * N * R;
    const int n = causal ? min(i + 1, N) : N;
    const int j0 = sp * kSplitKeys, j1 = min(j0 + kSplitKeys, n);
    float* tile = stile[warp];
    WarpStreamTopK<EPL> st{sbuf[warp], K};
    for (int jb = j0; jb < j1; jb += 32) {
        const int nk = min(32, j1 - jb);  // keys in this group
        float acc = 0.f;
#pragma unroll 1
        for (int c0 = 0; c0 < R; c0 += CH) {
            // stage rows jb .. jb + nk - 1, columns c0 .. c0 + CH - 1
            constexpr int V = CH / 4;  // float4 per staged row
#pragma unroll
            for (int t = 0; t < V; ++t) {
                const int f = lane + 32 * t;  // float4 index in the 32 x V block
                const int rr = f / V, cv = f - rr * V;
                float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
                if (rr < nk) x = __ldg(reinterpret_cast<const float4*>(kbase + (size_t)(jb + rr) * R + c0) + cv);
                *reinterpret_cast<float4*>(tile + rr * ST + 4 * cv) = x;
            }
            __syncwarp();
#pragma unroll
            for (int u = 0; u < V; ++u) {
                const float4 kk = *reinterpret_cast<const float4*>(tile + lane * ST + 4 * u);
                const float4 a = __ldg(reinterpret_cast<const float4*>(qrow + c0) + u);
                acc = fmaf(a.x, kk.x, acc);
                acc = fmaf(a.y, kk.y, acc);
                acc = fmaf(a.z, kk.z, acc);
                acc = fmaf(a.w, kk.w, acc);
            }
            __syncwarp();  // the tile is restaged next
        }
        const int j = jb + lane;
        const bool valid = lane < nk;
        float sc;
        if constexpr (kBias) {
            int bi = i - j + L;
            bi = bi < 0 ? 0 : (bi > 2 * L - 1 ? 2 * L - 1 : bi);
            sc = __fadd_rn(__fmul_rn(acc, scale), valid ? __ldg(bias + bi) : 0.f);
        } else {
            sc = __fmul_rn(acc, scale);
        }
        st.push(valid, valid ? order_key(sc) : 0u, (uint32_t)j, lane, lt);
    }
    const int m = st.finish(lane, lt);
    uint2* dst = cand + (size_t)gw * K;
    uint32_t kmin = 0xffffffffu;
    for (int t = lane; t < m; t += 32) {
        const uint2 e = st.wb[t];
        dst[t] = e;
        kmin = min(kmin, e.x);
    }
    kmin = __reduce_min_sync(kFull, kmin);
    if (lane == 0) {
        ccount[gw] = m;
        ckth[gw] = m == K ? kmin : 0u;  // the range's K-th best key (0: fewer than K)
    }
}

template <int EPL>
__global__ void __launch_bounds__(256)
split_merge_kernel(const uint2* __restrict__ cand, const int* __restrict__ ccount, const uint32_t* __restrict__ ckth,
                   int nsplit, int K, int32_t* __restrict__ out) {
    __shared__ uint2 sbuf[8][32 * EPL];
    __shared__ uint2 sfin[32 * EPL];
    __shared__ uint32_t swk[8];
    __shared__ int scnt[8];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const unsigned lt = lanemask_lt();
    const long long row = blockIdx.x;
    const size_t base = (size_t)row * nsplit;
    // lower bound on the row's K-th best key: the largest per-range K-th key
    uint32_t t0 = 0u;
    for (int s2 = threadIdx.x; s2 < nsplit; s2 += blockDim.x) t0 = max(t0, ckth[base + s2]);
    t0 = __reduce_max_sync(kFull, t0);
    if (lane == 0) swk[warp] = t0;
    __syncthreads();
    t0 = swk[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) t0 = max(t0, swk[w]);
    // warp w: ranges [w * per, (w + 1) * per)
    const int per = (nsplit + 7) / 8;
    WarpStreamTopK<EPL> st{sbuf[warp], K};
    st.theta = t0 > 0u ? t0 - 1u : 0u;  // admits keys >= t0
    const int s_lo = warp * per, s_hi = min(nsplit, s_lo + per);
    for (int sp = s_lo; sp < s_hi; ++sp) {
        const int c = ccount[base + sp];
        const uint2* src = cand + (base + sp) * K;
        for (int q0 = 0; q0 < c; q0 += 32) {
            const int t = q0 + lane;
            const bool valid = t < c;
            const uint2 e = valid ? src[t] : make_uint2(0u, 0u);
            st.push(valid, e.x, e.y, lane, lt);
        }
    }
    const int m = st.finish(lane, lt);
    if (lane == 0) scnt[warp] = m;
    __syncthreads();
    if (warp == 0) {
        WarpStreamTopK<EPL> fin{sfin, K};
        fin.theta = t0 > 0u ? t0 - 1u : 0u;
        for (int w = 0; w < 8; ++w) {
            const int c = scnt[w];
            for (int q0 = 0; q0 < c; q0 += 32) {
                const int t = q0 + lane;
                const bool valid = t < c;
                const uint2 e = valid ? sbuf[w][t] : make_uint2(0u, 0u);
                fin.push(valid, e.x, e.y, lane, lt);
            }
        }
        const int mf = fin.finish(lane, lt);
        int32_t* orow = out + row * K;
        for (int t = lane; t < K; t += 32) orow[t] = t < mf ? (int32_t)sfin[t].y : -1;
    }
}

int split_count(int N) { return (N + kSplitKeys - 1) / kSplitKeys; }

template <int R, bool kBias, int EPL>
cudaError_t launch_split(const SplitSelectArgs& a, cudaStream_t stream) {
    const int Nq = a.Nq > 0 ? a.Nq : a.N;
    const long long rows = (long long)a.B * a.H * Nq;
    const int nsplit = split_count(a.N);
    uint2* cand = static_cast<uint2*>(a.ws);
    int* ccount = reinterpret_cast<int*>(cand + (size_t)rows * nsplit * a.K);
    uint32_t* ckth = reinterpret_cast<uint32_t*>(ccount + (size_t)rows * nsplit);
    const long long warps = rows * nsplit;
    split_scan_kernel<R, kBias, EPL><<<(unsigned)((warps + kScanWarps - 1) / kScanWarps), 32 * kScanWarps, 0,
                                       stream>>>(
        a.qrows, a.krows, a.bias, a.L, a.H, a.Hkv, a.N, Nq, a.q0, a.K, a.scale, a.causal, rows, nsplit, cand,
        ccount, ckth);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    note_launch();
    split_merge_kernel<EPL><<<(unsigned)rows, 256, 0, stream>>>(cand, ccount, ckth, nsplit, a.K, a.out);
    e = cudaGetLastError();
    if (e == cudaSuccess) note_launch();
    return e;
}

template <int R, bool kBias>
cudaError_t launch_split_r(const SplitSelectArgs& a, cudaStream_t stream) {
    // candidate list of K + 32 entries per warp
    if (a.K <= 96) return launch_split<R, kBias, 4>(a, stream);
    return launch_split<R, kBias, 6>(a, stream);
}

template <bool kBias>
cudaError_t launch_split_b(const SplitSelectArgs& a, cudaStream_t stream) {
    switch (a.R) {
        case 16: return launch_split_r<16, kBias>(a, stream);
        case 32: return launch_split_r<32, kBias>(a, stream);
        case 64: return launch_split_r<64, kBias>(a, stream);
        case 128: return launch_split_r<128, kBias>(a, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

bool split_select_supported(int R, int K) {
    return (R == 16 || R == 32 || R == 64 || R == 128) && K >= 1 && K <= 160;
}

size_t split_select_workspace_bytes(long long rows, int N, int K) {
    const size_t n = (size_t)rows * split_count(N);
    return n * (size_t)K * sizeof(uint2) + n * (sizeof(int) + sizeof(uint32_t));
}

cudaError_t launch_split_select(const SplitSelectArgs& a, cudaStream_t stream) {
    if (!split_select_supported(a.R, a.K) || a.H % a.Hkv != 0) return cudaErrorInvalidValue;
    return a.bias ? launch_split_b<true>(a, stream) : launch_split_b<false>(a, stream);
}

}  // namespace ossa
