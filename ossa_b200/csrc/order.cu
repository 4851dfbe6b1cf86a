// Score order of selected index rows: the order torch.topk returns.
//
// The selectors emit each row's K keys in ascending key order (the order the
// gather wants).  ContentRouter.topk in the reference returns
// torch.topk(score, k).indices (ossa/router.py:202-203): keys by descending score.
// This kernel reorders rows in place to (score desc, key asc), the selection's
// own total order, with -1 padding last.
//
// One warp per row.  Each lane rescores its EPL entries with the canonical fp32
// formula (the fmaf chain the selectors decide on, from the projected rows the
// selection left in its workspace), packs (order key of the score, ~key) into a
// 64-bit word and the warp sorts the 32*EPL words with a bitonic network
// (entry x = lane + 32 e; partners 32 or more apart are in the same lane).
#include "common.cuh"
#include "kernels.h"

namespace ossa {

namespace {

__device__ __forceinline__ uint64_t shfl_xor_u64(uint64_t v, int m) {
    const uint32_t lo = __shfl_xor_sync(kFull, (uint32_t)v, m);
    const uint32_t hi = __shfl_xor_sync(kFull, (uint32_t)(v >> 32), m);
    return ((uint64_t)hi << 32) | lo;
}

// Sorts the warp's 32*EPL words into descending order (entry x = lane + 32 e).
template <int EPL>
__device__ __forceinline__ void warp_sort_desc(uint64_t (&v)[EPL], int lane) {
    constexpr int n = 32 * EPL;
#pragma unroll
    for (int k = 2; k <= n; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            if (j >= 32) {
                const int je = j >> 5;
#pragma unroll
                for (int e = 0; e < EPL; ++e) {
                    const int pe = e ^ je;
                    if (pe > e) {
                        // x and its partner share bit k (j < k), so both see one direction
                        const bool desc = ((lane + 32 * e) & k) == 0;
                        const uint64_t a = v[e], b = v[pe];
                        const bool sw = desc ? (a < b) : (a > b);
                        v[e] = sw ? b : a;
                        v[pe] = sw ? a : b;
                    }
                }
            } else {
#pragma unroll
                for (int e = 0; e < EPL; ++e) {
                    const int x = lane + 32 * e;
                    const uint64_t o = shfl_xor_u64(v[e], j);
                    const bool keep_max = (((x & j) == 0) == ((x & k) == 0));
                    v[e] = keep_max ? (v[e] > o ? v[e] : o) : (v[e] < o ? v[e] : o);
                }
            }
        }
    }
}

template <int EPL>
__global__ void __launch_bounds__(256) sort_rows_kernel(const float* __restrict__ qp, const float* __restrict__ kp,
                                                       const float* __restrict__ bias, int L, int H, int Hkv,
                                                       int N, int R, int K, float scale, long long rows,
                                                       int32_t* __restrict__ idx) {
    const int lane = threadIdx.x & 31;
    const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;  // warp-uniform
    const long long bh = row / N;
    const int i = (int)(row - bh * N);
    const int b = (int)(bh / H);
    const int g = (int)(bh - (long long)b * H) / (H / Hkv);
    const float* qrow = qp + (size_t)row * R;
    const float* kbase = kp + (size_t)(b * Hkv + g) * N * R;
    int32_t* orow = idx + (size_t)row * K;
    uint64_t v[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
        const int x = lane + 32 * e;
        const int j = x < K ? orow[x] : -1;
        v[e] = 0ull;
        if (j >= 0 && j < N) {
            const float* krow = kbase + (size_t)j * R;
            float acc = 0.f;
            for (int c = 0; c < R; c += 4) {
                const float4 a = __ldg(reinterpret_cast<const float4*>(qrow + c));
                const float4 w = __ldg(reinterpret_cast<const float4*>(krow + c));
                acc = fmaf(a.x, w.x, acc);
                acc = fmaf(a.y, w.y, acc);
                acc = fmaf(a.z, w.z, acc);
                acc = fmaf(a.w, w.w, acc);
            }
            float s = __fmul_rn(acc, scale);
            if (bias) {
                int bi = i - j + L;
                bi = bi < 0 ? 0 : (bi > 2 * L - 1 ? 2 * L - 1 : bi);
                s = __fadd_rn(s, __ldg(bias + bi));
            }
            // order keys of real scores are >= 1, so padding (0) sorts last
            v[e] = ((uint64_t)order_key(s) << 32) | (uint64_t)(0xffffffffu - (uint32_t)j);
        }
    }
    warp_sort_desc<EPL>(v, lane);
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
        const int x = lane + 32 * e;
        if (x < K) orow[x] = v[e] == 0ull ? -1 : (int32_t)(0xffffffffu - (uint32_t)v[e]);
    }
}

}  // namespace

bool sort_rows_supported(int R, int K) { return (R % 4) == 0 && R > 0 && K >= 1 && K <= 256; }

cudaError_t launch_sort_rows(const SortRowsArgs& a, cudaStream_t stream) {
    if (a.rows <= 0) return cudaSuccess;
    const unsigned blocks = (unsigned)((a.rows + 7) / 8);
    if (a.K <= 32)
        sort_rows_kernel<1><<<blocks, 256, 0, stream>>>(a.qp, a.kp, a.bias, a.L, a.H, a.Hkv, a.N, a.R, a.K, a.scale,
                                                        a.rows, a.idx);
    else if (a.K <= 64)
        sort_rows_kernel<2><<<blocks, 256, 0, stream>>>(a.qp, a.kp, a.bias, a.L, a.H, a.Hkv, a.N, a.R, a.K, a.scale,
                                                        a.rows, a.idx);
    else if (a.K <= 128)
        sort_rows_kernel<4><<<blocks, 256, 0, stream>>>(a.qp, a.kp, a.bias, a.L, a.H, a.Hkv, a.N, a.R, a.K, a.scale,
                                                        a.rows, a.idx);
    else
        sort_rows_kernel<8><<<blocks, 256, 0, stream>>>(a.qp, a.kp, a.bias, a.L, a.H, a.Hkv, a.N, a.R, a.K, a.scale,
                                                        a.rows, a.idx);
    const cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) note_launch();
    return e;
}

}  // namespace ossa
