// bf16 dot-product helpers of the gather kernels (gather_attn.cu).
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include "common.cuh"

namespace ossa {

// d = a * b + c with a, b the low (HI = false) or high (HI = true) bf16 halves of
// 32-bit registers and c, d fp32: the bf16 x bf16 product is exact in fp32, so
// this equals fmaf(float(a), float(b), c) without the two conversions.
template <bool HI>
__device__ __forceinline__ float fma_bf16(uint32_t a, uint32_t b, float c) {
    float d;
    if constexpr (HI) {
        asm("{ .reg .b16 al, ah, bl, bh;\n mov.b32 {al, ah}, %1;\n mov.b32 {bl, bh}, %2;\n"
            " fma.rn.f32.bf16 %0, ah, bh, %3; }"
            : "=f"(d) : "r"(a), "r"(b), "f"(c));
    } else {
        asm("{ .reg .b16 al, ah, bl, bh;\n mov.b32 {al, ah}, %1;\n mov.b32 {bl, bh}, %2;\n"
            " fma.rn.f32.bf16 %0, al, bl, %3; }"
            : "=f"(d) : "r"(a), "r"(b), "f"(c));
    }
    return d;
}

// Dot product of two rows of 8 bf16 values (16 bytes each) in fp32: two fma chains
// (even and odd elements) of the mixed-precision fma, summed at the end.
__device__ __forceinline__ float dot8_bf16(uint4 a, uint4 b) {
    float d0 = fma_bf16<false>(a.x, b.x, 0.f);
    float d1 = fma_bf16<true>(a.x, b.x, 0.f);
    d0 = fma_bf16<false>(a.y, b.y, d0);
    d1 = fma_bf16<true>(a.y, b.y, d1);
    d0 = fma_bf16<false>(a.z, b.z, d0);
    d1 = fma_bf16<true>(a.z, b.z, d1);
    d0 = fma_bf16<false>(a.w, b.w, d0);
    d1 = fma_bf16<true>(a.w, b.w, d1);
    return d0 + d1;
}

// acc[0..7] += p * v[0..7], p a bf16 value in both halves of pm, v 8 bf16 values.
__device__ __forceinline__ void axpy8_bf16(uint32_t pm, uint4 v, float (&acc)[8]) {
    acc[0] = fma_bf16<false>(pm, v.x, acc[0]);
    acc[1] = fma_bf16<true>(pm, v.x, acc[1]);
    acc[2] = fma_bf16<false>(pm, v.y, acc[2]);
    acc[3] = fma_bf16<true>(pm, v.y, acc[3]);
    acc[4] = fma_bf16<false>(pm, v.z, acc[4]);
    acc[5] = fma_bf16<true>(pm, v.z, acc[5]);
    acc[6] = fma_bf16<false>(pm, v.w, acc[6]);
    acc[7] = fma_bf16<true>(pm, v.w, acc[7]);
}

// p rounded to bf16, in both halves of a 32-bit register (the fma operand).
__device__ __forceinline__ uint32_t bf16_pair_bits(float p) {
    return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(p)) * 0x10001u;
}

// Sums part[0..15] across each half-warp so that lane l of a half ends with the
// total of part[l & 15] over its half.
__device__ __forceinline__ float transpose_reduce16(float (&part)[16], int lane) {
#pragma unroll
    for (int w = 8; w >= 1; w >>= 1) {
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

// Output of one row from the two half-warps' partial accumulators (disjoint keys,
// same dims): summed, divided by the softmax denominator (0 for an empty row) and
// written as bf16 by the first half, 16 bytes per lane.
__device__ __forceinline__ void store_row_bf16(float (&acc)[8], float l_run, __nv_bfloat16* __restrict__ orow,
                                               int lane) {
#pragma unroll
    for (int t = 0; t < 8; ++t) acc[t] += __shfl_xor_sync(kFull, acc[t], 16);
    const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
    if (lane < 16) {
        uint4 o;
        uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const __nv_bfloat162 pr = __floats2bfloat162_rn(acc[2 * t] * inv, acc[2 * t + 1] * inv);
            ow[t] = *reinterpret_cast<const uint32_t*>(&pr);
        }
        *(reinterpret_cast<uint4*>(orow) + lane) = o;
    }
}

}  // namespace ossa
