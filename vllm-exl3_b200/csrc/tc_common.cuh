// tc_common.cuh -- sm_100a tensor-core (tcgen05 / TMEM) and TMA primitives.
//
// Encodings follow the PTX ISA for sm_100a (the same bit layouts as CUTLASS's
// cute/arch/mma_sm100_desc.hpp):
//  * shared-memory matrix descriptor (64-bit): start address >> 4 in [0,14),
//    leading-dimension byte offset >> 4 in [16,30), stride-dimension byte
//    offset >> 4 in [32,46), version 1 in [46,48), base offset [49,52),
//    layout type in [61,64) (2 = 128-byte swizzle);
//  * instruction descriptor for kind::f16 (32-bit): D format [4,6) (1 = f32),
//    A format [7,10) and B format [10,13) (0 = f16), A/B major [15], [16]
//    (0 = K-major), N >> 3 in [17,23), M >> 4 in [24,29).
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "exl3_common.cuh"

namespace exl3 {

// K-major operand with a SWB-byte swizzle (SWB = 128: layout type 2; SWB =
// 64: layout type 4): 8-row atoms of SWB-byte rows, atoms 8*SWB bytes apart
// (SBO), LBO unused (1).  `addr` must be aligned to the atom (8*SWB bytes) at
// the atom origin; a K offset inside the row is added to `addr`.
template <int SWB>
__device__ __forceinline__ uint64_t umma_desc_k_sw(uint32_t smem_addr) {
    static_assert(SWB == 64 || SWB == 128, "64- or 128-byte swizzle");
    uint64_t d = 0;
    d |= uint64_t((smem_addr >> 4) & 0x3FFF);
    d |= uint64_t(1) << 16;                          // LBO (ignored for swizzled K-major)
    d |= uint64_t((8 * SWB) >> 4) << 32;             // SBO: 8 rows x SWB bytes
    d |= uint64_t(1) << 46;                          // version 1 (sm_100)
    d |= uint64_t(SWB == 128 ? 2 : 4) << 61;         // SWIZZLE_128B / SWIZZLE_64B
    return d;
}
__device__ __forceinline__ uint64_t umma_desc_k_sw128(uint32_t smem_addr) { return umma_desc_k_sw<128>(smem_addr); }

__host__ __device__ constexpr uint32_t umma_idesc_f16_f32(int M, int N) {
    return (1u << 4)                          // D = f32
         | (0u << 7) | (0u << 10)             // A, B = f16
         | (0u << 15) | (0u << 16)            // K-major A and B
         | (uint32_t(N >> 3) << 17)
         | (uint32_t(M >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

// arrive on `bar` once every tcgen05 op issued so far by this thread completes
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }

// generic-proxy shared-memory writes -> visible to the async proxy (UMMA, TMA)
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols));
}

// 32 consecutive fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
    #pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 2-D TMA tile load (no multicast) into shared memory, completing on `bar`
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
            smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Byte offset of fp16 element (row, k) in a K-major 128-byte-swizzled tile
// of 64-element rows (the layout TMA writes with CU_TENSOR_MAP_SWIZZLE_128B
// and UMMA reads with layout type 2): 16-byte chunk ^= row % 8.
__device__ __forceinline__ uint32_t sw128_offset(int row, int k) {
    return uint32_t((row >> 3) * 1024 + (row & 7) * 128 + ((((k >> 3) ^ (row & 7)) & 7) << 4) + (k & 7) * 2);
}

// The same for 64-byte swizzled 32-element rows (CU_TENSOR_MAP_SWIZZLE_64B,
// UMMA layout type 4): address bits 4-5 ^= bits 7-8, i.e. 16-byte chunk ^=
// (row / 2) % 4 inside 512-byte atoms of 8 rows.
__device__ __forceinline__ uint32_t sw64_offset(int row, int k) {
    return uint32_t((row >> 3) * 512 + (row & 7) * 64 + ((((k >> 3) ^ (row >> 1)) & 3) << 4) + (k & 7) * 2);
}

// In-thread 128-point FWHT (strides 1..64), v in registers.
__device__ __forceinline__ void fwht128_thread(float (&v)[128]) {
    #pragma unroll
    for (int s = 1; s < 128; s <<= 1) {
        #pragma unroll
        for (int base = 0; base < 128; base += s << 1) {
            #pragma unroll
            for (int i = 0; i < s; ++i) {
                const float a = v[base + i], b = v[base + s + i];
                v[base + i] = a + b;
                v[base + s + i] = a - b;
            }
        }
    }
}

}  // namespace exl3
