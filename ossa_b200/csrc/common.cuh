// Shared device helpers for the ossa_b200 kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace ossa {

constexpr unsigned kFull = 0xffffffffu;

// ---------------------------------------------------------------------------
// Element loads: every kernel computes in fp32; inputs are fp32 or bf16.
// bf16 -> fp32 is exact (the bf16 bits are the high half of the fp32 word).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }

__device__ __forceinline__ void store_from_f32(float* p, float x) { *p = x; }
__device__ __forceinline__ void store_from_f32(__nv_bfloat16* p, float x) { *p = __float2bfloat16_rn(x); }

// Loads N consecutive elements (N*sizeof(T) bytes, naturally aligned) as fp32.
template <typename T, int N>
struct VecLoad;

template <int N>
struct VecLoad<float, N> {
    __device__ __forceinline__ static void load(const float* __restrict__ p, float* out) {
        if constexpr (N == 4) {
            float4 t = __ldg(reinterpret_cast<const float4*>(p));
            out[0] = t.x; out[1] = t.y; out[2] = t.z; out[3] = t.w;
        } else if constexpr (N == 8) {
            float4 a = __ldg(reinterpret_cast<const float4*>(p));
            float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
            out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
            out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
        } else if constexpr (N == 2) {
            float2 t = __ldg(reinterpret_cast<const float2*>(p));
            out[0] = t.x; out[1] = t.y;
        } else {
#pragma unroll
            for (int i = 0; i < N; ++i) out[i] = __ldg(p + i);
        }
    }
};

__device__ __forceinline__ void unpack_bf16x2(uint32_t w, float& lo, float& hi) {
    lo = __uint_as_float(w << 16);
    hi = __uint_as_float(w & 0xffff0000u);
}

template <int N>
struct VecLoad<__nv_bfloat16, N> {
    __device__ __forceinline__ static void load(const __nv_bfloat16* __restrict__ p, float* out) {
        if constexpr (N == 8) {
            uint4 t = __ldg(reinterpret_cast<const uint4*>(p));
            unpack_bf16x2(t.x, out[0], out[1]); unpack_bf16x2(t.y, out[2], out[3]);
            unpack_bf16x2(t.z, out[4], out[5]); unpack_bf16x2(t.w, out[6], out[7]);
        } else if constexpr (N == 4) {
            uint2 t = __ldg(reinterpret_cast<const uint2*>(p));
            unpack_bf16x2(t.x, out[0], out[1]); unpack_bf16x2(t.y, out[2], out[3]);
        } else if constexpr (N == 2) {
            uint32_t t = __ldg(reinterpret_cast<const unsigned int*>(p));
            unpack_bf16x2(t, out[0], out[1]);
        } else {
#pragma unroll
            for (int i = 0; i < N; ++i) out[i] = __bfloat162float(p[i]);
        }
    }
};

// ---------------------------------------------------------------------------
// Order-preserving map fp32 -> uint32: a > b (as torch.topk orders values,
// NaN above +inf) iff key(a) > key(b).  Every NaN maps to one key.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t order_key(float f) {
    uint32_t b = __float_as_uint(f);
    if (f != f) b = 0x7fc00000u;
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float key_to_float(uint32_t k) {
    uint32_t b = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    return __uint_as_float(b);
}

__device__ __forceinline__ unsigned lanemask_lt() {
    unsigned m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) x = fmaxf(x, __shfl_xor_sync(kFull, x, o));
    return x;
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) x += __shfl_xor_sync(kFull, x, o);
    return x;
}

}  // namespace ossa
