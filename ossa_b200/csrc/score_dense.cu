// Materialised ContentRouter logits (ossa/router.py:171-190), (B, H, N, N) fp32.
//
// Same score definition as the fused selection kernel (fmaf chain over the R
// projected channels, then fl(fl(dot * scale) + bias)), so a caller that takes
// torch.topk of these logits sees exactly the values the fused path selects on.
// Thread t of a CTA owns key j = jb*128 + t (k'_j in registers) and walks every
// query row; q' rows are staged 32 at a time in shared memory and read as
// float4 broadcasts; stores are coalesced along j.
#include "common.cuh"
#include "kernels.h"

namespace ossa {

namespace {

constexpr int kKeys = 128;
constexpr int kRowTile = 32;

template <int R>
__global__ void __launch_bounds__(kKeys)
score_dense_kernel(const float* __restrict__ qrows, const float* __restrict__ krows,
                   const float* __restrict__ bias, int L, int H, int Hkv, int N,
                   float scale, float* __restrict__ out, int njb) {
    constexpr int QS = R + 4;
    __shared__ __align__(16) float Qs[kRowTile * QS];
    const int bh = blockIdx.x / njb;
    const int jb = blockIdx.x - bh * njb;
    const int b = bh / H;
    const int h = bh - b * H;
    const int g = h / (H / Hkv);
    const int tid = threadIdx.x;
    const int j = jb * kKeys + tid;
    const bool active = j < N;

    float kr[R];
    {
        const float* kp = krows + ((size_t)(b * Hkv + g) * N + (active ? j : 0)) * R;
#pragma unroll
        for (int c = 0; c < R; ++c) kr[c] = active ? kp[c] : 0.f;
    }
    const float* qb = qrows + (size_t)bh * N * R;
    float* ob = out + (size_t)bh * N * N;

    for (int i0 = 0; i0 < N; i0 += kRowTile) {
        __syncthreads();
        for (int e = tid; e < kRowTile * R; e += kKeys) {
            const int ii = e / R, c = e - ii * R;
            Qs[ii * QS + c] = (i0 + ii) < N ? qb[(size_t)(i0 + ii) * R + c] : 0.f;
        }
        __syncthreads();
#pragma unroll 1
        for (int ig = 0; ig < kRowTile; ig += 8) {
            float acc[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) acc[t] = 0.f;
#pragma unroll
            for (int c4 = 0; c4 < R; c4 += 4) {
#pragma unroll
                for (int t = 0; t < 8; ++t) {
                    const float4 qv = *reinterpret_cast<const float4*>(Qs + (ig + t) * QS + c4);
                    acc[t] = fmaf(qv.x, kr[c4 + 0], acc[t]);
                    acc[t] = fmaf(qv.y, kr[c4 + 1], acc[t]);
                    acc[t] = fmaf(qv.z, kr[c4 + 2], acc[t]);
                    acc[t] = fmaf(qv.w, kr[c4 + 3], acc[t]);
                }
            }
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                const int i = i0 + ig + t;
                if (active && i < N) {
                    float s = __fmul_rn(acc[t], scale);
                    if (bias != nullptr) {
                        int bi = i - j + L;
                        bi = bi < 0 ? 0 : (bi > 2 * L - 1 ? 2 * L - 1 : bi);
                        s = __fadd_rn(s, __ldg(bias + bi));
                    }
                    ob[(size_t)i * N + j] = s;
                }
            }
        }
    }
}

template <int R>
cudaError_t launch_r(const ScoreDenseArgs& a, cudaStream_t stream) {
    const int njb = (a.N + kKeys - 1) / kKeys;
    const long long nblk = (long long)njb * a.B * a.H;
    if (nblk == 0) return cudaSuccess;
    score_dense_kernel<R><<<(unsigned)nblk, kKeys, 0, stream>>>(
        a.qrows, a.krows, a.bias, a.L, a.H, a.Hkv, a.N, a.scale, a.out, njb);
    cudaError_t err = cudaGetLastError();
    if (err == cudaSuccess) note_launch();
    return err;
}

}  // namespace

cudaError_t launch_score_dense(const ScoreDenseArgs& a, cudaStream_t stream) {
    switch (a.R) {
        case 16: return launch_r<16>(a, stream);
        case 32: return launch_r<32>(a, stream);
        case 64: return launch_r<64>(a, stream);
        case 128: return launch_r<128>(a, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace ossa
