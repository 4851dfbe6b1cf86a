// Rotary position embedding fused with the head transpose of the patched layer.
//
// The patched forward (ossa/bench/sparse_forward.py:166-178) views each of the
// q/k/v projections (B, N, Hx*D) as (B, Hx, N, D), applies Qwen2's
// apply_rotary_pos_emb to q and k (x*cos + rotate_half(x)*sin, rotate_half =
// cat(-x2, x1)) and the selection and gather then read contiguous (B, Hx, N, D)
// rows.  In eager PyTorch that is a mul, a neg, a cat, a mul, an add and a
// layout copy per tensor; here it is one pass: each thread reads 4 values of the
// low half and the 4 matching values of the high half of one (b, n, h) row,
// with their cos/sin, and writes both groups of the rotated row at (b, h, n).
//
// Rounding follows the eager ops exactly: t1 = rnd(x*cos), t2 = rnd(rot*sin),
// out = rnd(t1 + t2), each product and the sum rounded to the tensor dtype
// (bf16: computed in fp32 and rounded to nearest even; fp32: no contraction),
// so the result is bit-identical to the unfused PyTorch ops.
// Without cos/sin the kernel is the plain layout copy (for v).
#include <algorithm>
#include <cstdint>

#include "common.cuh"
#include "kernels.h"

namespace ossa {

namespace {

template <typename T>
struct RopeIO;

template <>
struct RopeIO<float> {
    static __device__ __forceinline__ void load4(const float* p, float (&v)[4]) {
        const float4 x = __ldg(reinterpret_cast<const float4*>(p));
        v[0] = x.x;
        v[1] = x.y;
        v[2] = x.z;
        v[3] = x.w;
    }
    static __device__ __forceinline__ void store4(float* p, const float (&v)[4]) {
        *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    }
    static __device__ __forceinline__ float rnd(float x) { return x; }
};

template <>
struct RopeIO<__nv_bfloat16> {
    static __device__ __forceinline__ void load4(const __nv_bfloat16* p, float (&v)[4]) {
        const uint2 x = __ldg(reinterpret_cast<const uint2*>(p));
        unpack_bf16x2(x.x, v[0], v[1]);
        unpack_bf16x2(x.y, v[2], v[3]);
    }
    static __device__ __forceinline__ void store4(__nv_bfloat16* p, const float (&v)[4]) {
        const __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]);
        const __nv_bfloat162 b = __floats2bfloat162_rn(v[2], v[3]);
        uint2 o;
        o.x = *reinterpret_cast<const uint32_t*>(&a);
        o.y = *reinterpret_cast<const uint32_t*>(&b);
        *reinterpret_cast<uint2*>(p) = o;
    }
    static __device__ __forceinline__ float rnd(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
};

// One CTA per (b, n) position; thread t of it takes head h = t / (D/8) and
// columns c .. c+3 and c + D/2 .. c + D/2 + 3 of the low and high halves
// (c = 4 * (t mod D/8)).  32-bit index arithmetic only.
template <typename T, bool kRope>
__global__ void __launch_bounds__(256)
rope_heads_kernel(const T* __restrict__ x, const T* __restrict__ cosv, const T* __restrict__ sinv, int cs_batched,
                  int B, int N, int Hx, int D, T* __restrict__ out) {
    using IO = RopeIO<T>;
    const int hq = D / 8;  // threads per head row
    const int bn = blockIdx.x;
    const int b = bn / N;
    const int n = bn - b * N;
    const int half = D / 2;
    for (int t = threadIdx.x; t < Hx * hq; t += blockDim.x) {
        const int h = t / hq;
        const int c = 4 * (t - h * hq);
        const T* xr = x + ((size_t)bn * Hx + h) * D;
        float lo[4], hi[4];
        IO::load4(xr + c, lo);
        IO::load4(xr + half + c, hi);
        T* orow = out + (((size_t)b * Hx + h) * N + n) * D;
        if constexpr (kRope) {
            const size_t cr = ((size_t)(cs_batched ? b : 0) * N + n) * D;
            float cl[4], ch[4], sl[4], sh[4];
            IO::load4(cosv + cr + c, cl);
            IO::load4(cosv + cr + half + c, ch);
            IO::load4(sinv + cr + c, sl);
            IO::load4(sinv + cr + half + c, sh);
            float ol[4], oh[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                // low half: x1*cos - x2*sin; high half: x2*cos + x1*sin
                const float a1 = IO::rnd(__fmul_rn(lo[u], cl[u]));
                const float b1 = IO::rnd(__fmul_rn(-hi[u], sl[u]));
                ol[u] = IO::rnd(__fadd_rn(a1, b1));
                const float a2 = IO::rnd(__fmul_rn(hi[u], ch[u]));
                const float b2 = IO::rnd(__fmul_rn(lo[u], sh[u]));
                oh[u] = IO::rnd(__fadd_rn(a2, b2));
            }
            IO::store4(orow + c, ol);
            IO::store4(orow + half + c, oh);
        } else {
            IO::store4(orow + c, lo);
            IO::store4(orow + half + c, hi);
        }
    }
}

template <typename T>
cudaError_t launch_t(const RopeArgs& a, cudaStream_t stream) {
    const long long rows = (long long)a.B * a.N;
    if (rows == 0) return cudaSuccess;
    if (rows > 0x7fffffffLL) return cudaErrorInvalidValue;
    const unsigned grid = (unsigned)rows;
    const int per = a.Hx * (a.D / 8);  // threads' worth of work per position
    const unsigned block = (unsigned)std::min(256, (per + 31) / 32 * 32);
    const T* x = static_cast<const T*>(a.x);
    T* out = static_cast<T*>(a.out);
    if (a.cosv)
        rope_heads_kernel<T, true><<<grid, block, 0, stream>>>(x, static_cast<const T*>(a.cosv),
                                                            static_cast<const T*>(a.sinv), a.cs_batched, a.B, a.N,
                                                            a.Hx, a.D, out);
    else
        rope_heads_kernel<T, false><<<grid, block, 0, stream>>>(x, nullptr, nullptr, 0, a.B, a.N, a.Hx, a.D, out);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) note_launch();
    return e;
}

}  // namespace

cudaError_t launch_rope_heads(const RopeArgs& a, cudaStream_t stream) {
    if (a.D % 8 != 0 || a.D <= 0) return cudaErrorInvalidValue;
    return a.dtype == kF32 ? launch_t<float>(a, stream) : launch_t<__nv_bfloat16>(a, stream);
}

}  // namespace ossa
