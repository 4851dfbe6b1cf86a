// Router distillation loss and its gradient without the (B, H, N, N) logits.
//
// The reference trains ContentRouter by binary cross-entropy between its logits
// and a 0/1 target marking each query row's top-k keys of the dense attention
// (ossa/router.py:80-99, driven by ossa/bench/content_train.py:141-148):
//   loss = mean over all B*H*N*N entries (i, j) of
//          max(s, 0) - s * t + log(1 + exp(-|s|)),   s = score(i, j), t in {0, 1}
// with score(i, j) = (q'_i . k'_j) / sqrt(r) + pos_bias[clamp(i - j + L, 0, 2L - 1)]
// (ossa/router.py:171-190) over every (i, j), the masked ones included.  Its
// gradient is dL/ds = (sigmoid(s) - t) / (B*H*N*N), so
//   dq'_i = sum_j g_ij k'_j / sqrt(r),  dk'_j = sum_i g_ij q'_i / sqrt(r),
//   dpos_bias[o] = sum over (i, j) with clamp(i - j + L) = o of g_ij,
//   dWq = sum_rows dq'_row (x) q_row,  dWk = sum_rows dk'_row (x) k_row.
// Scores are the canonical fp32 ones of the selectors (fmaf chain over r from
// 0.0f, times 1/sqrt(r), plus the bias term).  The target rows are index lists
// (-1 padded, any order); key j of row i is a target when the row lists it.
//
// Three kernels, nothing quadratic in memory:
//  * distill_rows_kernel: a CTA per 64 query rows of one (b, h) streams all key
//    tiles of its kv head (64 keys): scores, loss terms and g into shared memory,
//    then dq' (4 threads per row, r/4 dims each) and the tile's bias diagonals;
//  * distill_cols_kernel: a CTA per 64 keys of one (b, kv head) streams the query
//    tiles of the group's heads, recomputes g and accumulates dk';
//  * weight_grad_kernel: dW = dP^T X over row blocks, atomically added.
#include "common.cuh"
#include "kernels.h"

#include <math.h>

namespace ossa {

namespace {

constexpr int kDT = 64;         // rows (queries or keys) per tile
constexpr int kDThreads = 256;  // 4 threads per tile row

// BCE-with-logits term and its derivative numerator for score s and target t.
__device__ __forceinline__ void bce_term(float s, float t, float& loss, float& dsig) {
    const float e = expf(-fabsf(s));
    loss = fmaxf(s, 0.f) - s * t + log1pf(e);
    const float sig = s >= 0.f ? 1.f / (1.f + e) : e / (1.f + e);
    dsig = sig - t;
}

// Canonical score of query row a (smem, stride rs) and key row c (smem).
template <int R>
__device__ __forceinline__ float tile_dot(const float* __restrict__ a, const float* __restrict__ c) {
    float acc = 0.f;
#pragma unroll
    for (int u = 0; u < R; u += 4) {
        const float4 x = *reinterpret_cast<const float4*>(a + u);
        const float4 y = *reinterpret_cast<const float4*>(c + u);
        acc = fmaf(x.x, y.x, acc);
        acc = fmaf(x.y, y.y, acc);
        acc = fmaf(x.z, y.z, acc);
        acc = fmaf(x.w, y.w, acc);
    }
    return acc;
}

// Loads `rows` rows of R floats (row stride R in global) into smem rows of stride
// R + 4, zero rows past `valid`.
template <int R>
__device__ __forceinline__ void load_rows(float* __restrict__ dst, const float* __restrict__ src, int valid) {
    constexpr int V = R / 4;
    for (int e = threadIdx.x; e < kDT * V; e += blockDim.x) {
        const int row = e / V, c = e - row * V;
        const float4 x = row < valid ? __ldg(reinterpret_cast<const float4*>(src + (size_t)row * R) + c)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(dst + row * (R + 4) + 4 * c) = x;
    }
}

// Target bits of the tile's 64 rows for keys [j0, j0 + 64): bit c of tmask[row]
// is set when the row's index list holds key j0 + c.
__device__ __forceinline__ void target_masks(const int32_t* __restrict__ trows, int K, int nrows, int j0,
                                             unsigned long long* tmask) {
    for (int row = threadIdx.x; row < kDT; row += blockDim.x) {
        unsigned long long m = 0ull;
        if (row < nrows) {
            const int32_t* t = trows + (size_t)row * K;
            for (int q = 0; q < K; ++q) {
                const int d = __ldg(t + q) - j0;
                if (d >= 0 && d < kDT) m |= 1ull << d;
            }
        }
        tmask[row] = m;
    }
}

template <int R>
__global__ void __launch_bounds__(kDThreads)
distill_rows_kernel(const float* __restrict__ qp, const float* __restrict__ kp, const float* __restrict__ bias, int L,
                    int H, int Hkv, int N, const int32_t* __restrict__ tgt, int K, float scale, float inv_count,
                    float* __restrict__ dqp, float* __restrict__ dbias, float* __restrict__ loss_part) {
    extern __shared__ float4 dsm4[];
    float* Qs = reinterpret_cast<float*>(dsm4);           // [kDT][R + 4]
    float* Ks = Qs + kDT * (R + 4);                        // [kDT][R + 4]
    float* Gs = Ks + kDT * (R + 4);                        // [kDT][kDT + 1]
    float* bins = Gs + kDT * (kDT + 1);                    // [2 * kDT - 1] diagonals of a tile
    unsigned long long* tmask = reinterpret_cast<unsigned long long*>(bins + 2 * kDT);  // [kDT]
    __shared__ float red[kDThreads / 32];
    const int bh = blockIdx.y;
    const int b = bh / H, h = bh - b * H, g = h / (H / Hkv);
    const int i0 = blockIdx.x * kDT;
    const int nrows = min(kDT, N - i0);
    const int tid = threadIdx.x, row = tid >> 2, part = tid & 3;
    const int i = i0 + row;
    load_rows<R>(Qs, qp + ((size_t)bh * N + i0) * R, nrows);
    const float* kbase = kp + (size_t)(b * Hkv + g) * N * R;
    const int32_t* trows = tgt + ((size_t)bh * N + i0) * K;
    float dq[R / 4];
#pragma unroll
    for (int c = 0; c < R / 4; ++c) dq[c] = 0.f;
    float lsum = 0.f;
    for (int j0 = 0; j0 < N; j0 += kDT) {
        const int nkeys = min(kDT, N - j0);
        __syncthreads();  // the previous tile's Ks, Gs, bins and masks are consumed
        load_rows<R>(Ks, kbase + (size_t)j0 * R, nkeys);
        target_masks(trows, K, nrows, j0, tmask);
        for (int e = tid; e < 2 * kDT - 1; e += kDThreads) bins[e] = 0.f;
        __syncthreads();
        const unsigned long long tm = tmask[row];
#pragma unroll 4
        for (int m = 0; m < kDT / 4; ++m) {
            const int c = part + 4 * m;
            const int j = j0 + c;
            float gv = 0.f;
            if (row < nrows && c < nkeys) {
                int bi = i - j + L;
                bi = bi < 0 ? 0 : (bi > 2 * L - 1 ? 2 * L - 1 : bi);
                const float s = __fadd_rn(__fmul_rn(tile_dot<R>(Qs + row * (R + 4), Ks + c * (R + 4)), scale),
                                          __ldg(bias + bi));
                float l, dsig;
                bce_term(s, (tm >> c) & 1ull ? 1.f : 0.f, l, dsig);
                lsum += l;
                gv = dsig * inv_count;
                atomicAdd(&bins[row - c + kDT - 1], gv);
            }
            Gs[row * (kDT + 1) + c] = gv;
        }
        __syncthreads();
        // dq' of this row: r/4 dims per thread (part-th quarter), keys in order
#pragma unroll 4
        for (int c = 0; c < kDT; ++c) {
            const float gv = Gs[row * (kDT + 1) + c];
            const float* kr = Ks + c * (R + 4) + part * (R / 4);
#pragma unroll
            for (int u = 0; u < R / 4; ++u) dq[u] = fmaf(gv, kr[u], dq[u]);
        }
        // the tile's bias diagonals d = i - j = (i0 - j0) + e - (kDT - 1)
        for (int e = tid; e < 2 * kDT - 1; e += kDThreads) {
            const float v = bins[e];
            if (v != 0.f) {
                int o = i0 - j0 + e - (kDT - 1) + L;
                o = o < 0 ? 0 : (o > 2 * L - 1 ? 2 * L - 1 : o);
                atomicAdd(dbias + o, v);
            }
        }
    }
    if (row < nrows) {
        float* o = dqp + ((size_t)bh * N + i) * R + part * (R / 4);
#pragma unroll
        for (int u = 0; u < R / 4; ++u) o[u] = dq[u] * scale;
    }
    // per-CTA loss partial (summed by the host side in a fixed order)
    const float w = warp_sum(lsum);
    if ((tid & 31) == 0) red[tid >> 5] = w;
    __syncthreads();
    if (tid == 0) {
        float t = 0.f;
        for (int u = 0; u < kDThreads / 32; ++u) t += red[u];
        loss_part[(size_t)blockIdx.y * gridDim.x + blockIdx.x] = t;
    }
}

template <int R>
__global__ void __launch_bounds__(kDThreads)
distill_cols_kernel(const float* __restrict__ qp, const float* __restrict__ kp, const float* __restrict__ bias, int L,
                    int H, int Hkv, int N, const int32_t* __restrict__ tgt, int K, float scale, float inv_count,
                    float* __restrict__ dkp) {
    extern __shared__ float4 dsm4[];
    float* Ks = reinterpret_cast<float*>(dsm4);  // [kDT][R + 4] this CTA's keys
    float* Qs = Ks + kDT * (R + 4);               // [kDT][R + 4]
    float* Gs = Qs + kDT * (R + 4);               // [kDT][kDT + 1], Gs[query][key]
    unsigned long long* tmask = reinterpret_cast<unsigned long long*>(Gs + kDT * (kDT + 1));
    const int bg = blockIdx.y;
    const int b = bg / Hkv, g = bg - b * Hkv;
    const int G = H / Hkv;
    const int j0 = blockIdx.x * kDT;
    const int nkeys = min(kDT, N - j0);
    const int tid = threadIdx.x, key = tid >> 2, part = tid & 3;
    const int j = j0 + key;
    load_rows<R>(Ks, kp + ((size_t)bg * N + j0) * R, nkeys);
    float dk[R / 4];
#pragma unroll
    for (int c = 0; c < R / 4; ++c) dk[c] = 0.f;
    for (int hh = 0; hh < G; ++hh) {
        const int bh = b * H + g * G + hh;
        for (int i0 = 0; i0 < N; i0 += kDT) {
            const int nrows = min(kDT, N - i0);
            __syncthreads();
            load_rows<R>(Qs, qp + ((size_t)bh * N + i0) * R, nrows);
            target_masks(tgt + ((size_t)bh * N + i0) * K, K, nrows, j0, tmask);
            __syncthreads();
#pragma unroll 4
            for (int m = 0; m < kDT / 4; ++m) {
                const int r = part + 4 * m;  // query row of the tile
                const int i = i0 + r;
                float gv = 0.f;
                if (r < nrows && key < nkeys) {
                    int bi = i - j + L;
                    bi = bi < 0 ? 0 : (bi > 2 * L - 1 ? 2 * L - 1 : bi);
                    const float s = __fadd_rn(__fmul_rn(tile_dot<R>(Qs + r * (R + 4), Ks + key * (R + 4)), scale),
                                              __ldg(bias + bi));
                    float l, dsig;
                    bce_term(s, (tmask[r] >> key) & 1ull ? 1.f : 0.f, l, dsig);
                    gv = dsig * inv_count;
                }
                Gs[r * (kDT + 1) + key] = gv;
            }
            __syncthreads();
#pragma unroll 4
            for (int r = 0; r < kDT; ++r) {
                const float gv = Gs[r * (kDT + 1) + key];
                const float* qr = Qs + r * (R + 4) + part * (R / 4);
#pragma unroll
                for (int u = 0; u < R / 4; ++u) dk[u] = fmaf(gv, qr[u], dk[u]);
            }
        }
    }
    if (key < nkeys) {
        float* o = dkp + ((size_t)bg * N + j) * R + part * (R / 4);
#pragma unroll
        for (int u = 0; u < R / 4; ++u) o[u] = dk[u] * scale;
    }
}

// dW[c][d] += sum over this CTA's rows of dp[row][c] * x[row][d]; a CTA takes
// kWRows rows, thread t owns output column d = t % D for r / (256 / D) of the c's.
constexpr int kWRows = 256;
template <typename T>
__global__ void __launch_bounds__(256)
weight_grad_kernel(const float* __restrict__ dp, const T* __restrict__ x, long long rows, int D, int R,
                   float* __restrict__ dw) {
    const long long r0 = (long long)blockIdx.x * kWRows;
    const int nr = (int)min((long long)kWRows, rows - r0);
    for (int o = threadIdx.x; o < R * D; o += blockDim.x) {
        const int c = o / D, d = o - c * D;
        float acc = 0.f;
        for (int rr = 0; rr < nr; ++rr)
            acc = fmaf(__ldg(dp + (size_t)(r0 + rr) * R + c), to_f32(x[(size_t)(r0 + rr) * D + d]), acc);
        atomicAdd(dw + o, acc);
    }
}

template <int R>
size_t rows_smem() { return (size_t)(2 * kDT * (R + 4) + kDT * (kDT + 1) + 2 * kDT) * 4 + kDT * 8; }

template <int R>
cudaError_t launch_r(const DistillArgs& a, cudaStream_t s) {
    const float scale = (float)(1.0 / sqrt((double)R));
    const float inv_count = (float)(1.0 / ((double)a.B * a.H * (double)a.N * (double)a.N));
    const int nt = (a.N + kDT - 1) / kDT;
    const size_t smem = rows_smem<R>();
    cudaError_t e = cudaFuncSetAttribute(distill_rows_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(distill_cols_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    distill_rows_kernel<R><<<dim3(nt, a.B * a.H), kDThreads, smem, s>>>(a.qp, a.kp, a.bias, a.L, a.H, a.Hkv, a.N,
                                                                       a.tgt, a.K, scale, inv_count, a.dqp, a.dbias,
                                                                       a.loss_part);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    note_launch();
    distill_cols_kernel<R><<<dim3(nt, a.B * a.Hkv), kDThreads, smem, s>>>(a.qp, a.kp, a.bias, a.L, a.H, a.Hkv, a.N,
                                                                          a.tgt, a.K, scale, inv_count, a.dkp);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    note_launch();
    return cudaSuccess;
}

template <typename T>
cudaError_t launch_wgrad(const float* dp, const void* x, long long rows, int D, int R, float* dw, cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    weight_grad_kernel<T><<<(unsigned)((rows + kWRows - 1) / kWRows), 256, 0, s>>>(dp, static_cast<const T*>(x), rows,
                                                                                 D, R, dw);
    const cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) note_launch();
    return e;
}

// loss = (sum of the per-CTA partials, in index order) / count, one thread.
__global__ void loss_reduce_kernel(const float* __restrict__ parts, long long n, double inv_count,
                                   float* __restrict__ out) {
    double t = 0.0;
    for (long long u = 0; u < n; ++u) t += (double)parts[u];
    *out = (float)(t * inv_count);
}

}  // namespace

size_t distill_loss_parts(int B, int H, int N) { return (size_t)B * H * ((N + kDT - 1) / kDT); }

cudaError_t launch_distill(const DistillArgs& a, cudaStream_t s) {
    cudaError_t e;
    switch (a.R) {
        case 16: e = launch_r<16>(a, s); break;
        case 32: e = launch_r<32>(a, s); break;
        case 64: e = launch_r<64>(a, s); break;
        case 128: e = launch_r<128>(a, s); break;
        default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return e;
    loss_reduce_kernel<<<1, 1, 0, s>>>(a.loss_part, (long long)distill_loss_parts(a.B, a.H, a.N),
                                       1.0 / ((double)a.B * a.H * (double)a.N * (double)a.N), a.loss_out);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    note_launch();
    const long long rq = (long long)a.B * a.H * a.N, rk = (long long)a.B * a.Hkv * a.N;
    if (a.dtype == kF32) {
        if ((e = launch_wgrad<float>(a.dqp, a.q, rq, a.D, a.R, a.dwq, s)) != cudaSuccess) return e;
        return launch_wgrad<float>(a.dkp, a.k, rk, a.D, a.R, a.dwk, s);
    }
    if ((e = launch_wgrad<__nv_bfloat16>(a.dqp, a.q, rq, a.D, a.R, a.dwq, s)) != cudaSuccess) return e;
    return launch_wgrad<__nv_bfloat16>(a.dkp, a.k, rk, a.D, a.R, a.dwk, s);
}

}  // namespace ossa
