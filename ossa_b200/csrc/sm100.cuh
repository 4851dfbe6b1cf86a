// Thin wrappers over the sm_100a PTX used by the tensor-core kernels:
// mbarriers, TMA tiled loads, tcgen05 (TMEM alloc, MMA, commit, loads, fences)
// and UMMA shared-memory / instruction descriptors.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace ossa {
namespace sm100 {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Shared-memory accesses by 32-bit shared address (no generic-address work).
__device__ __forceinline__ float4 lds_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ void sts_f32(uint32_t addr, float v) {
    asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v));
}
__device__ __forceinline__ void sts_f32_if(uint32_t addr, float v, bool pred) {
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %2, 0;\n @p st.shared.f32 [%0], %1;\n}"
                 ::"r"(addr), "f"(v), "r"(pred ? 1 : 0));
}
__device__ __forceinline__ uint2 lds_u2(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint4 lds_u4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}
// *addr = v when pred (an explicitly predicated store: no branch).
__device__ __forceinline__ void sts_u32_if(uint32_t addr, uint32_t v, bool pred) {
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %2, 0;\n @p st.shared.u32 [%0], %1;\n}"
                 ::"r"(addr), "r"(v), "r"(pred ? 1 : 0));
}
__device__ __forceinline__ uint32_t lds_u32_or(uint32_t addr, bool pred, uint32_t otherwise) {
    uint32_t v;
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %2, 0;\n mov.b32 %0, %3;\n @p ld.shared.u32 %0, [%1];\n}"
                 : "=r"(v) : "r"(addr), "r"(pred ? 1 : 0), "r"(otherwise));
    return v;
}
// value at addr when pred, else `otherwise` (an explicitly predicated load).
__device__ __forceinline__ float lds_f32_or(uint32_t addr, bool pred, float otherwise) {
    float v;
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %2, 0;\n mov.f32 %0, %3;\n @p ld.shared.f32 %0, [%1];\n}"
                 : "=f"(v) : "r"(addr), "r"(pred ? 1 : 0), "f"(otherwise));
    return v;
}

// ----------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: gives up after ~2^31 SM cycles (about a second) and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    const long long start = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - start > (1ll << 31)) return false;
    }
    return true;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Arrive once `dep` is available: the barrier address is computed from it (its
// value does not change the address), so the arrive cannot issue before the
// loads that produced `dep` have returned.
__device__ __forceinline__ void mbar_arrive_after(uint64_t* bar, uint32_t dep) {
    asm volatile(
        "{\n .reg .b32 z;\n and.b32 z, %1, 0;\n add.u32 z, z, %0;\n"
        " mbarrier.arrive.shared::cta.b64 _, [z];\n}" ::"r"(smem_u32(bar)), "r"(dep)
        : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// --------------------------------------------------------------------- TMA
// 2-D tiled load of one box into shared memory, completion counted on `bar`.
// x (the innermost coordinate) must keep x * element size a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(smem_u32(dst)), "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// 1-D bulk copy from global to this CTA's shared memory, completion counted on
// `bar`.  dst and src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// ------------------------------------------------------------------ tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t addr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(addr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D(tmem) (+)= A(smem desc) * B(smem desc)^T, kind::f16 (f16 or bf16 inputs, f32 accumulate).
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives once on `bar` when every tcgen05 op issued so far by this thread is done.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// 16 (tmem_ld16) or 32 (tmem_ld32) consecutive fp32 columns of this warp's 32 TMEM lanes
// (thread t <- lane base + t).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
          "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),
          "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),
          "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Pins the registers of a tcgen05.ld to this point: placed after tmem_wait_ld,
// it keeps the compiler from moving their uses above the wait.
template <int N>
__device__ __forceinline__ void reg_fence(uint32_t (&v)[N]) {
#pragma unroll
    for (int k = 0; k < N; ++k) asm volatile("" : "+r"(v[k]));
}

// UMMA shared-memory descriptor for a K-major operand tile stored with the
// 128-byte swizzle (rows of 128 bytes, 8-row / 1024-byte swizzle atoms, atoms
// 1024 bytes apart).  The tile must start on a 1024-byte boundary; advancing
// along K by 16 two-byte elements adds 32 bytes (2 encoded units) to the start.
__device__ __forceinline__ uint64_t umma_desc_sw128(const void* smem_tile) {
    const uint64_t addr = smem_u32(smem_tile);
    uint64_t d = (addr & 0x3FFFFull) >> 4;  // start address
    d |= 1ull << 16;                          // leading byte offset (unused for swizzled K-major)
    d |= (1024ull >> 4) << 32;                // stride byte offset: next 8-row atom
    d |= 1ull << 46;                          // descriptor version (sm_100)
    d |= 2ull << 61;                          // layout: 128-byte swizzle
    return d;
}

// Instruction descriptor, kind::f16: fp32 accumulator, A/B format (0 = f16,
// 1 = bf16), both K-major, M x N tile.
__host__ __device__ constexpr uint32_t umma_idesc_f16(uint32_t ab_format, uint32_t M, uint32_t N) {
    return (1u << 4) | (ab_format << 7) | (ab_format << 10) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

// 32x32b TMEM load of N (16 or 32) consecutive columns into v.
__device__ __forceinline__ void tmem_ld_chunk(uint32_t taddr, uint32_t (&v)[16]) { tmem_ld16(taddr, v); }
__device__ __forceinline__ void tmem_ld_chunk(uint32_t taddr, uint32_t (&v)[32]) { tmem_ld32(taddr, v); }

}  // namespace sm100
}  // namespace ossa
