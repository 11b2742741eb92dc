// tc05.cuh — 5th-generation tensor core (tcgen05) and TMA helpers shared by the tcgen05
// kernels (k_gemm.cu: grouped expert GEMM; k_dac.cu: DAC convolutions).
//
// Operand convention: both operands K-major in shared memory. The 128-byte-swizzle layout
// is the one a tiled TMA box with CU_TENSOR_MAP_SWIZZLE_128B writes: row n of a stage at
// n * 128 bytes, its 16-byte chunk c at chunk c ^ (n % 8), 8-row atoms 1024 bytes apart.
#pragma once

#include "common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

namespace z2b {

// Instruction descriptor, kind::f16: f32 accumulator, f16 A and B, both K-major, M x N.
__device__ __forceinline__ uint32_t idesc_f16(int m, int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// Shared-memory descriptor, K-major with the 128-byte swizzle: leading offset unused (1),
// 1024 B between 8-row atoms; the K16 slices of a 64-wide stage start 32 B apart inside
// the 128-byte rows.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}

// One tiled TMA load (this CTA only) of a 2-D box completing on `bar`. x times the element
// size is a multiple of 16 bytes (the callers pass multiples of 64 f16 elements).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        :: "r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)) : "memory");
}

// The same for a 3-D box (x innermost). y may be negative or past the extent: those rows
// read as zeros.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
        :: "r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}"
        :: "r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate) : "memory");
}

// Arrive on `bar` once every tcgen05.mma this thread issued before has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(bar)) : "memory");
}

// 16 consecutive f32 accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Bounded wait that also gives up as soon as another role of the block has given up.
__device__ __forceinline__ bool wait_ab(uint64_t* bar, uint32_t parity, uint32_t* err, volatile int* ab) {
    for (uint32_t i = 0; i < kMaxWaitPolls; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*ab) return false;
    }
    if (err) atomicOr(err, (uint32_t)DERR_WAIT_TIMEOUT);
    *ab = 1;
    return false;
}

// cuTensorMapEncodeTiled from the driver, looked up once (null if unavailable).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

}  // namespace z2b
