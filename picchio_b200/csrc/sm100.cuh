// sm100.cuh - thin wrappers over the sm_100a instructions of the tensor-core
// path: bounded mbarrier waits, TMA tile loads, tcgen05 (TMEM allocation, MMA,
// commit, loads) and the shared-memory matrix descriptors they take.
//
// Descriptor and instruction-descriptor bit layouts follow the PTX ISA
// (tcgen05 "matrix descriptors" and "instruction descriptor" tables); every
// wait on an mbarrier is bounded (see mbar_wait).
#pragma once
#include <cuda.h>
#include <cstdint>

#include "ptx.cuh"

namespace pc {

__device__ __forceinline__ unsigned long long sm100_globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------- mbarrier ----
// (init / arrive / try_wait live in ptx.cuh)
__device__ __forceinline__ void mbar_init_fence() { fence_mbar_init(); }
// Waits for phase `parity` of bar to complete, for at most limit_ns; false on
// timeout (the caller records the error and winds down).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, unsigned long long limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = sm100_globaltimer();
    while (!mbar_try_wait(bar, parity))
        if (sm100_globaltimer() - t0 > limit_ns) return false;
    return true;
}

// ------------------------------------------------------------------- TMA ----
// 2-D tile load of a tensor map's box at (x = inner coordinate, y) into
// shared memory, completing on bar (transaction bytes).  No multicast.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
// 1-D bulk copy global -> shared completing on bar (transaction bytes); no
// multicast, no cache hint.  Both addresses 16-byte aligned, bytes a
// multiple of 16.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// Makes this thread's generic-proxy writes to shared memory visible to the
// async proxy (tcgen05.mma operands written with st.shared).
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ------------------------------------------------------- packed fp32 ----
// Two fp32 lanes per 64-bit register (low word = first), one instruction
// each: sub.rn.f32x2 / mul.rn.f32x2 round every lane as sub.rn / mul.rn do.
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// ---------------------------------------------------------------- tcgen05 ----
// TMEM allocation: one full warp; the base address is written to *slot.
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] x B[smem]^T, s8 x s8 -> s32, one CTA.
__device__ __forceinline__ void tc_mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}
// Arrives on bar once every tcgen05.mma issued so far by this thread is done.
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}
// 16 consecutive 32-bit TMEM columns of this thread's lane (32x32b shape):
// warp w of a warpgroup reads lanes 32 (w % 4) .. + 31.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major operand tile stored in the
// 128-byte swizzle layout: rows of 128 bytes, 8-row groups 1024 bytes apart
// (the stride byte offset), tile base 1024-byte aligned.  Advancing K by 32
// bytes inside the 128-byte row adds 2 to the encoded start address.
__device__ __forceinline__ uint64_t sw128_desc(const void *tile) {
    const uint64_t addr = (smem_u32(tile) & 0x3FFFFu) >> 4;
    return addr                     // start address, bits 0-13
           | (1ull << 16)           // leading byte offset (unused with swizzling)
           | ((1024ull >> 4) << 32) // stride byte offset: 8-row groups
           | (1ull << 46)           // descriptor version (sm_100)
           | (2ull << 61);          // layout: 128-byte swizzle
}

// D[tmem] (+)= A[smem] x B[smem]^T, f16 x f16 -> f32, one CTA.
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}
// Instruction descriptor: f16 x f16 -> f32, both operands K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
    return (1u << 4)                         // D format: f32
           | ((uint32_t)(N >> 3) << 17)      // N / 8 (A, B format 0: f16)
           | ((uint32_t)(M >> 4) << 24);     // M / 16
}
// Instruction descriptor: s8 x s8 -> s32, both operands K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
    return (2u << 4)                         // D format: s32
           | (1u << 7) | (1u << 10)          // A, B: signed 8-bit
           | ((uint32_t)(N >> 3) << 17)      // N / 8
           | ((uint32_t)(M >> 4) << 24);     // M / 16
}

}  // namespace pc
