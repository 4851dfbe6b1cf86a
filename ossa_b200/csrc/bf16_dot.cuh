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

}  // namespace ossa
