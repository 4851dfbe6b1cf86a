// ContentRouter projections q' = q Wq^T and k' = k Wk^T (ossa/router.py:179-180).
//
// Each output is one fp32 fused-multiply-add chain over d = 0..D-1 starting from
// 0.0f: acc = fmaf(x[d], w[c][d], acc).  That fixed order makes q'/k' bit-exact
// against the CPU oracle (which evaluates the same chain with C fmaf) and is the
// "fp32 projection" every selection decision downstream is defined on.
//
// Tiling: a CTA computes ROWS x R outputs with 256 threads; each thread owns a
// 4 x 4 register tile.  D is consumed in chunks of up to 128: the x chunk is
// fetched with 16-byte loads (all issued before the first use) and stored
// transposed in shared memory (float4 broadcast reads of 4 rows), W^T sits in
// shared memory (float4 reads of 4 output columns): two LDS.128 per 16 FFMA.
// The k projection is GQA-aware by construction: the caller runs it on the Hkv
// key heads only, never on repeated copies.
#include <algorithm>
#include <cstdint>

#include "common.cuh"
#include "kernels.h"

namespace ossa {

namespace {

constexpr int kProjThreads = 256;
constexpr int kDChunk = 128;

// Elements of x per 16-byte vector load.
template <typename T>
struct ChunkLoader {
    static constexpr int VEC = 16 / sizeof(T);  // elements per 16-byte load
};

template <typename T, int R>
__global__ void __launch_bounds__(kProjThreads)
project_kernel(const T* __restrict__ x, const float* __restrict__ w, float* __restrict__ out,
               long long rows, int D) {
    constexpr int CG = R / 4;                    // column groups
    constexpr int RG = kProjThreads / CG;        // row groups
    constexpr int ROWS = RG * 4;                 // rows per CTA
    constexpr int XS = ROWS + 4;                 // padded stride (keeps float4 alignment)
    constexpr int VEC = ChunkLoader<T>::VEC;
    extern __shared__ float4 smem4[];
    float* Xs = reinterpret_cast<float*>(smem4);  // [kDChunk][XS]
    float* Ws = Xs + kDChunk * XS;                // [kDChunk][R]

    const int tid = threadIdx.x;
    const int cg = tid % CG;
    const int rg = tid / CG;
    const long long row0 = (long long)blockIdx.x * ROWS;
    const bool vec_ok = (D % VEC) == 0;

    float acc[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[a][c] = 0.f;

    for (int dc = 0; dc < D; dc += kDChunk) {
        const int dn = min(kDChunk, D - dc);
        __syncthreads();
        if (vec_ok) {
            // ROWS rows x (dn / VEC) vectors; every load is issued before any store
            constexpr int kPer = (ROWS * kDChunk / VEC + kProjThreads - 1) / kProjThreads;
            const int nvec = dn / VEC;
            uint4 buf[kPer];
#pragma unroll
            for (int u = 0; u < kPer; ++u) {
                // consecutive threads take consecutive rows, so the transposed
                // shared-memory stores below hit consecutive banks
                const int e = tid + u * kProjThreads;
                const int vcol = e / ROWS, r = e - vcol * ROWS;
                const long long gr = row0 + r;
                buf[u] = make_uint4(0u, 0u, 0u, 0u);
                if (vcol < kDChunk / VEC && vcol < nvec && gr < rows)
                    buf[u] = __ldg(reinterpret_cast<const uint4*>(x + gr * D + dc) + vcol);
            }
#pragma unroll
            for (int u = 0; u < kPer; ++u) {
                const int e = tid + u * kProjThreads;
                const int vcol = e / ROWS, r = e - vcol * ROWS;
                if (vcol < kDChunk / VEC) {
                    float f[VEC];
                    if constexpr (sizeof(T) == 2) {
                        unpack_bf16x2(buf[u].x, f[0], f[1]);
                        unpack_bf16x2(buf[u].y, f[2], f[3]);
                        unpack_bf16x2(buf[u].z, f[4], f[5]);
                        unpack_bf16x2(buf[u].w, f[6], f[7]);
                    } else {
                        f[0] = __uint_as_float(buf[u].x);
                        f[1] = __uint_as_float(buf[u].y);
                        f[2] = __uint_as_float(buf[u].z);
                        f[3] = __uint_as_float(buf[u].w);
                    }
#pragma unroll
                    for (int t = 0; t < VEC; ++t) Xs[(vcol * VEC + t) * XS + r] = f[t];
                }
            }
        } else {
            for (int e = tid; e < ROWS * kDChunk; e += kProjThreads) {
                const int r = e / kDChunk, d = e - r * kDChunk;
                const long long gr = row0 + r;
                float val = 0.f;
                if (gr < rows && d < dn) val = to_f32(x[gr * D + dc + d]);
                Xs[d * XS + r] = val;
            }
        }
        for (int e = tid; e < R * kDChunk; e += kProjThreads) {
            const int d = e / R, c = e - d * R;
            Ws[d * R + c] = d < dn ? __ldg(w + (size_t)c * D + dc + d) : 0.f;
        }
        __syncthreads();
#pragma unroll 4
        for (int d = 0; d < dn; ++d) {
            const float4 xv = *reinterpret_cast<const float4*>(Xs + d * XS + rg * 4);
            const float4 wv = *reinterpret_cast<const float4*>(Ws + d * R + cg * 4);
            const float xa[4] = {xv.x, xv.y, xv.z, xv.w};
            const float wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[a][c] = fmaf(xa[a], wa[c], acc[a][c]);
        }
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const long long gr = row0 + rg * 4 + a;
        if (gr < rows) {
            *reinterpret_cast<float4*>(out + gr * R + cg * 4) =
                make_float4(acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
        }
    }
}

// 16-byte asynchronous global->shared copy; src_bytes = 0 zero-fills the slot.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc, int src_bytes) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(smem_dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(gsrc), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

// Persistent variant for D <= 128 with D a multiple of the 16-byte vector: W^T
// is staged in shared memory once per CTA, and the raw rows of the next tile
// stream in with cp.async while the current tile is converted and multiplied.
// Same per-output fmaf chain (d = 0..D-1 from 0.0f) as project_kernel.
template <typename T, int R>
__global__ void __launch_bounds__(kProjThreads)
project_persistent_kernel(const T* __restrict__ x, const float* __restrict__ w, float* __restrict__ out,
                          long long rows, int D, long long ntiles) {
    constexpr int CG = R / 4;
    constexpr int RG = kProjThreads / CG;
    constexpr int ROWS = RG * 4;
    constexpr int XS = ROWS + 4;
    constexpr int VEC = ChunkLoader<T>::VEC;
    constexpr int kStageVecs = ROWS * kDChunk / VEC;  // 16-byte vectors per stage (at D = 128)
    extern __shared__ float4 smem4[];
    float* Ws = reinterpret_cast<float*>(smem4);      // [kDChunk][R]
    float* Xs = Ws + kDChunk * R;                      // [kDChunk][XS]
    uint4* stage = reinterpret_cast<uint4*>(Xs + kDChunk * XS);  // 2 x [ROWS][D / VEC]

    const int tid = threadIdx.x;
    const int cg = tid % CG;
    const int rg = tid / CG;
    const int nvec = D / VEC;

    auto issue = [&](long long tile, int buf) {
        const long long row0 = tile * ROWS;
        uint4* st = stage + (size_t)buf * kStageVecs;
        for (int e = tid; e < ROWS * nvec; e += kProjThreads) {
            const int r = e / nvec, v = e - r * nvec;
            const long long gr = row0 + r;
            const bool in = gr < rows;
            const T* src = x + (in ? gr : 0) * (long long)D + v * VEC;
            cp_async16(st + e, src, in ? 16 : 0);
        }
        cp_async_commit();
    };

    for (int e = tid; e < R * D; e += kProjThreads) {
        const int d = e / R, c = e - d * R;
        Ws[d * R + c] = __ldg(w + (size_t)c * D + d);
    }
    long long tile = blockIdx.x;
    int buf = 0;
    if (tile < ntiles) issue(tile, 0);
    for (; tile < ntiles; tile += gridDim.x, buf ^= 1) {
        cp_async_wait_all();
        __syncthreads();  // stage[buf] landed for all threads; Xs is free again
        if (tile + gridDim.x < ntiles) issue(tile + gridDim.x, buf ^ 1);
        const uint4* st = stage + (size_t)buf * kStageVecs;
        // consecutive threads take consecutive rows: conflict-free transposed stores
        for (int e = tid; e < ROWS * nvec; e += kProjThreads) {
            const int v = e / ROWS, r = e - v * ROWS;
            const uint4 u = st[r * nvec + v];
            float f[VEC];
            if constexpr (sizeof(T) == 2) {
                unpack_bf16x2(u.x, f[0], f[1]);
                unpack_bf16x2(u.y, f[2], f[3]);
                unpack_bf16x2(u.z, f[4], f[5]);
                unpack_bf16x2(u.w, f[6], f[7]);
            } else {
                f[0] = __uint_as_float(u.x);
                f[1] = __uint_as_float(u.y);
                f[2] = __uint_as_float(u.z);
                f[3] = __uint_as_float(u.w);
            }
#pragma unroll
            for (int t = 0; t < VEC; ++t) Xs[(v * VEC + t) * XS + r] = f[t];
        }
        __syncthreads();
        float acc[4][4];
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[a][c] = 0.f;
#pragma unroll 4
        for (int d = 0; d < D; ++d) {
            const float4 xv = *reinterpret_cast<const float4*>(Xs + d * XS + rg * 4);
            const float4 wv = *reinterpret_cast<const float4*>(Ws + d * R + cg * 4);
            const float xa[4] = {xv.x, xv.y, xv.z, xv.w};
            const float wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[a][c] = fmaf(xa[a], wa[c], acc[a][c]);
        }
        const long long row0 = tile * ROWS;
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            const long long gr = row0 + rg * 4 + a;
            if (gr < rows) {
                *reinterpret_cast<float4*>(out + gr * R + cg * 4) =
                    make_float4(acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
            }
        }
    }
    cp_async_wait_all();
}

// (acc0, acc1) = (fma(x, w0, acc0), fma(x, w1, acc1)) as one fma.rn.f32x2: two
// IEEE fused multiply-adds, each rounded once, the same as two fmaf calls.
__device__ __forceinline__ void fma2(float& acc0, float& acc1, float x, float w0, float w1) {
    asm("{\n .reg .b64 ra, rb, rc;\n mov.b64 ra, {%2, %2};\n mov.b64 rb, {%3, %4};\n"
        " mov.b64 rc, {%0, %1};\n fma.rn.f32x2 rc, ra, rb, rc;\n mov.b64 {%0, %1}, rc;\n}"
        : "+f"(acc0), "+f"(acc1)
        : "f"(x), "f"(w0), "f"(w1));
}

// bf16 rows, D = 128, R = 64 (the ContentRouter shape of the product path).  A CTA
// takes 128-row tiles; warp w owns output columns 8w .. 8w+7 and lane l owns rows
// l, l+32, l+64, l+96, so a thread holds 4 x 8 accumulators.  For each d the warp
// reads W[d][8w .. 8w+7] at one address (a broadcast) and each lane unpacks its
// four x values from 16-byte row pieces it loaded for 8 consecutive d: per 32 FMA
// of a thread, two broadcast reads of W and half a 16-byte read of x.  The x rows
// stay bf16 in shared memory (272-byte pitch: the 8 lanes of a quarter warp read
// 8 consecutive rows from 8 distinct bank groups) and the next tile streams in
// with cp.async while the current one is multiplied.  Column pairs go through
// fma.rn.f32x2; every output keeps its fmaf chain d = 0..127 from 0.0f.
constexpr int kP2Rows = 128;                          // rows per tile
constexpr int kP2Pitch = 128 * 2 + 16;                // bytes per staged x row
constexpr int kP2StageBytes = kP2Rows * kP2Pitch;     // 34,816
constexpr int kP2Pieces = kP2Rows * 16 / kProjThreads;  // 16-byte pieces per thread per tile (8)
constexpr size_t kP2Smem = 128 * 64 * sizeof(float) + 2 * (size_t)kP2StageBytes;

// Element e (0..7) of 8 packed bf16, widened exactly.  The low half moves up with
// a byte permute and the high half is masked: both run on the integer pipe, which
// leaves the FMA pipe to the fma.rn.f32x2 stream.
__device__ __forceinline__ float bf16_elem(const uint4& u, int e) {
    const uint32_t wd = e < 2 ? u.x : (e < 4 ? u.y : (e < 6 ? u.z : u.w));
    return __uint_as_float((e & 1) ? (wd & 0xffff0000u) : __byte_perm(wd, 0u, 0x1054));
}

__global__ void __launch_bounds__(kProjThreads, 2)
project_bf16_d128_r64_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ w,
                             float* __restrict__ out, long long rows, long long ntiles) {
    extern __shared__ float4 smem4[];
    float* Ws = reinterpret_cast<float*>(smem4);                 // [128 d][64 c]
    uint8_t* stage = reinterpret_cast<uint8_t*>(Ws + 128 * 64);  // 2 x [128 rows][kP2Pitch]
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    for (int e = tid; e < 64 * 128; e += kProjThreads) {
        const int d = e / 64, c = e - d * 64;
        Ws[d * 64 + c] = __ldg(w + (size_t)c * 128 + d);
    }
    auto issue = [&](long long tile, int buf) {
        uint8_t* st = stage + (size_t)buf * kP2StageBytes;
#pragma unroll
        for (int u = 0; u < kP2Pieces; ++u) {
            const int e = tid + u * kProjThreads;
            const int r = e >> 4, v = e & 15;
            const long long gr = tile * kP2Rows + r;
            const bool in = gr < rows;
            cp_async16(st + r * kP2Pitch + v * 16, x + (in ? gr : 0) * 128 + v * 8, in ? 16 : 0);
        }
        cp_async_commit();
    };
    long long tile = blockIdx.x;
    int buf = 0;
    if (tile < ntiles) issue(tile, 0);
    const float* wrow = Ws + 8 * warp;
    for (; tile < ntiles; tile += gridDim.x, buf ^= 1) {
        cp_async_wait_all();
        __syncthreads();  // stage[buf] landed for every thread; stage[buf ^ 1] is free (and Ws is ready)
        if (tile + gridDim.x < ntiles) issue(tile + gridDim.x, buf ^ 1);
        const uint8_t* st = stage + (size_t)buf * kP2StageBytes + lane * kP2Pitch;
        float acc[4][8];
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int c = 0; c < 8; ++c) acc[a][c] = 0.f;
#pragma unroll 1
        for (int dc = 0; dc < 16; ++dc) {
            uint4 xr[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) xr[a] = *reinterpret_cast<const uint4*>(st + a * 32 * kP2Pitch + dc * 16);
#pragma unroll
            for (int dd = 0; dd < 8; ++dd) {
                const int d = dc * 8 + dd;
                const float4 w0 = *reinterpret_cast<const float4*>(wrow + d * 64);
                const float4 w1 = *reinterpret_cast<const float4*>(wrow + d * 64 + 4);
                const float wa[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                for (int a = 0; a < 4; ++a) {
                    const float xa = bf16_elem(xr[a], dd);
#pragma unroll
                    for (int c = 0; c < 8; c += 2) fma2(acc[a][c], acc[a][c + 1], xa, wa[c], wa[c + 1]);
                }
            }
        }
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            const long long gr = tile * kP2Rows + lane + 32 * a;
            if (gr < rows) {
                float4* o = reinterpret_cast<float4*>(out + gr * 64 + 8 * warp);
                o[0] = make_float4(acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
                o[1] = make_float4(acc[a][4], acc[a][5], acc[a][6], acc[a][7]);
            }
        }
    }
    cp_async_wait_all();
}

cudaError_t launch_bf16_d128_r64(const ProjectArgs& a, cudaStream_t stream) {
    auto kern = project_bf16_d128_r64_kernel;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kP2Smem);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 0, per_sm = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kProjThreads, kP2Smem)) != cudaSuccess)
        return e;
    const long long ntiles = (a.rows + kP2Rows - 1) / kP2Rows;
    if (ntiles == 0) return cudaSuccess;
    const long long grid = std::min<long long>(ntiles, (long long)sms * std::max(1, per_sm));
    kern<<<(unsigned)grid, kProjThreads, kP2Smem, stream>>>(static_cast<const __nv_bfloat16*>(a.x), a.w, a.out,
                                                           a.rows, ntiles);
    cudaError_t err = cudaGetLastError();
    if (err == cudaSuccess) note_launch();
    return err;
}

template <typename T, int R>
constexpr size_t persistent_smem_bytes();

template <typename T, int R>
cudaError_t launch_persistent(const ProjectArgs& a, cudaStream_t stream) {
    constexpr int ROWS = (kProjThreads / (R / 4)) * 4;
    const size_t smem = persistent_smem_bytes<T, R>();
    auto kern = project_persistent_kernel<T, R>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 0, per_sm = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kProjThreads, smem)) != cudaSuccess)
        return e;
    const long long ntiles = (a.rows + ROWS - 1) / ROWS;
    if (ntiles == 0) return cudaSuccess;
    const long long grid = std::min<long long>(ntiles, (long long)sms * std::max(1, per_sm));
    kern<<<(unsigned)grid, kProjThreads, smem, stream>>>(static_cast<const T*>(a.x), a.w, a.out, a.rows, a.D,
                                                          ntiles);
    cudaError_t err = cudaGetLastError();
    if (err == cudaSuccess) note_launch();
    return err;
}

template <typename T, int R>
constexpr size_t persistent_smem_bytes() {
    constexpr int ROWS = (kProjThreads / (R / 4)) * 4;
    return (size_t)kDChunk * R * sizeof(float) + (size_t)kDChunk * (ROWS + 4) * sizeof(float) +
           2 * (size_t)ROWS * kDChunk / ChunkLoader<T>::VEC * 16;
}

template <typename T, int R>
cudaError_t launch_r(const ProjectArgs& a, cudaStream_t stream) {
    if constexpr (sizeof(T) == 2 && R == 64) {
        if (a.D == 128 && reinterpret_cast<uintptr_t>(a.x) % 16 == 0) return launch_bf16_d128_r64(a, stream);
    }
    if constexpr (persistent_smem_bytes<T, R>() <= 200 * 1024) {
        if (a.D <= kDChunk && a.D % ChunkLoader<T>::VEC == 0 && reinterpret_cast<uintptr_t>(a.x) % 16 == 0)
            return launch_persistent<T, R>(a, stream);
    }
    constexpr int ROWS = (kProjThreads / (R / 4)) * 4;
    const size_t smem = (size_t)kDChunk * (ROWS + 4) * sizeof(float) + (size_t)kDChunk * R * sizeof(float);
    auto kern = project_kernel<T, R>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const long long nblk = (a.rows + ROWS - 1) / ROWS;
    if (nblk == 0) return cudaSuccess;
    kern<<<(unsigned)nblk, kProjThreads, smem, stream>>>(static_cast<const T*>(a.x), a.w, a.out, a.rows, a.D);
    cudaError_t err = cudaGetLastError();
    if (err == cudaSuccess) note_launch();
    return err;
}

template <typename T>
cudaError_t launch_t(const ProjectArgs& a, cudaStream_t stream) {
    switch (a.R) {
        case 16: return launch_r<T, 16>(a, stream);
        case 32: return launch_r<T, 32>(a, stream);
        case 64: return launch_r<T, 64>(a, stream);
        case 128: return launch_r<T, 128>(a, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

cudaError_t launch_project(const ProjectArgs& a, cudaStream_t stream) {
    return a.dtype == kF32 ? launch_t<float>(a, stream) : launch_t<__nv_bfloat16>(a, stream);
}

}  // namespace ossa
