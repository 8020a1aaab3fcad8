// exl3_common.cuh -- device primitives shared by the EXL3 sm_100a kernels.
//
// Packed EXL3 tensor (one projection W in R^{in x out}):
//   trellis int16 [in/16][out/16][16*K]   tile (kt, nt) = 16 in x 16 out
//   suh fp16 [in], svh fp16 [out]
// and W = diag(suh) * H * W~ * H * diag(svh) / 128 with H the block-diagonal
// 128-point Sylvester Hadamard matrix and W~ the decoded trellis.
// (vcruz305/vllm-exl3 src/vllm_exl3/exl3.py:4405-4481; csrc/bindings.cpp:15-100)
//
// Trellis decode of one tile (csrc/exl3_dequant.cuh:105-166,
// csrc/bindings.cpp:37-77): value t in [0,256) is the 16-bit window starting
// at stream bit (t + 257) * K - 16 (mod 256K) of the tile read as uint32
// words p[2i] | p[2i+1] << 16 with bits numbered MSB first, mapped through a
// procedural codebook.  Value t = 8*l + j lands on W~ row (k) 2*(l%4) + (j&1)
// + 8*((j>>1)&1) and column (n) l/4 + 8*(j>>2).  That is exactly the register
// layout of an mma.m16n8k16 A fragment of W~^T, so lane l of a warp decodes
// its own eight values straight into tensor-core operand registers.
#pragma once

#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "exl3_internal.h"

namespace exl3 {

enum Codebook : int { CB_3INST = 0, CB_MCG = 1, CB_MUL1 = 2 };

// Device-side status word (first word of every workspace).  Kernels never
// trap: a bad pointer, K or an expired wait records a code here and skips the
// work.  The host reads it on demand (exl3_device_status).
enum DevStatus : int {
    DEV_OK = 0,
    DEV_BAD_K = 1,          // per-expert K outside 2..8
    DEV_BAD_ALIGN = 2,      // trellis / suh / svh pointer not 16-byte aligned
    DEV_NULL_PTR = 3,       // null pointer in a pointer table
    DEV_WAIT_TIMEOUT = 4,   // an mbarrier wait exceeded its bound
    DEV_BAD_ROUTE = 5,      // routing table inconsistent (internal)
    DEV_BAD_LAUNCH = 6,     // launch shape inconsistent with the kernel's needs (internal)
    DEV_BAD_INDEX = 7,      // a row id outside its table (n-gram lookup); the row is written as zeros
};

__device__ __forceinline__ void set_status(int* status, int code) {
    if (status) atomicCAS(status, 0, code);
}

constexpr float kHadNorm = 0.08838834764831845f;  // 1/sqrt(128)

// ---------------------------------------------------------------------------
// Codebook: two 16-bit windows (in the low halves of wa, wb) -> one fp16x2
// register {lo = value(wa), hi = value(wb)}.
//
// MCG / 3INST: x = w * C (+ A); each half of (x & 0x8fff8fff) ^ 0x3b603b60 is
// a normal fp16 with exponent 12..15, so lo + hi is exact in fp32 and the
// reference's float add + round (exl3_dequant.cuh:88-90, 113-117) equals one
// f16x2 add.
// mul1: s = 0x6400 + bytesum(w * C) is the fp16 value 1024 + bytesum; the
// reference's float s*h(0x1eee) + h(0xc931) with two roundings
// (exl3_dequant.cuh:96-100, 119-123) is exact in fp32 (22- and 20-bit
// results), so it equals one f16x2 fma rounded once.
// ---------------------------------------------------------------------------
template <int CB>
__device__ __forceinline__ uint32_t decode_pair(uint32_t wa, uint32_t wb) {
    if constexpr (CB == CB_MUL1) {
        const uint32_t xa = wa * 0x83DCD12Du;
        const uint32_t xb = wb * 0x83DCD12Du;
        // sa = {0x6400 + bytesum(xa), 0x6400}, sb = bytesum(xb) (<= 1020, no
        // carries): s = {lo: 0x6400 + sum_a, hi: 0x6400 + sum_b}, packed by a
        // multiply-add on the FMA pipe instead of a byte permute on the ALU
        const uint32_t sa = __dp4a(xa, 0x01010101u, 0x64006400u);
        const uint32_t sb = __dp4a(xb, 0x01010101u, 0u);
        uint32_t s;
        asm("mad.lo.u32 %0, %1, 65536, %2;" : "=r"(s) : "r"(sb), "r"(sa));
        uint32_t r;
        asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(s), "r"(0x1eee1eeeu), "r"(0xc931c931u));
        return r;
    } else {
        uint32_t xa, xb;
        if constexpr (CB == CB_MCG) {
            xa = wa * 0xCBAC1FEDu;
            xb = wb * 0xCBAC1FEDu;
        } else {
            xa = wa * 89226354u + 64248484u;
            xb = wb * 89226354u + 64248484u;
        }
        xa = (xa & 0x8fff8fffu) ^ 0x3b603b60u;
        xb = (xb & 0x8fff8fffu) ^ 0x3b603b60u;
        // lo + hi of each word as one f16 add, then pack the two sums.
        // Measured fastest of the forms tried on B200 (pairing the halves
        // with a bit-select and byte permute, or shifting them with
        // multiplies, both issued more integer instructions).
        uint32_t r;
        asm("{\n .reg .f16 a0, a1, b0, b1, sa, sb;\n"
            " mov.b32 {a0, a1}, %1;\n mov.b32 {b0, b1}, %2;\n"
            " add.rn.f16 sa, a0, a1;\n add.rn.f16 sb, b0, b1;\n"
            " mov.b32 %0, {sa, sb};\n}\n"
            : "=r"(r) : "r"(xa), "r"(xb));
        return r;
    }
}

// ---------------------------------------------------------------------------
// Window extraction.  Lane l's eight windows start at bits b0 + j*K with
// b0 = ((8l + 257) * K - 16) mod 256K.  With u0 = b0 / 16 (a 16-bit unit;
// unit u of the stream is int16 element u ^ 1 of the tile) and o0 = b0 % 16,
// the lane assembles the 96-bit stream r0:r1:r2 starting at unit u0 and reads
// window j as the top 16 bits of funnel_shift_left(r_{q+1}:r_q, o) where
// o = o0 + j*K (- 32 q).  For even K, o0 = K for every lane; the unit parity
// is constant for K = 4 and K = 8.
// `tile` points at the tile's 8K uint32 words (shared or global memory).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t win_at(uint32_t hi, uint32_t lo, int o) {
    return __funnelshift_lc(lo, hi, o) >> 16;
}

template <int K>
__device__ __forceinline__ void tile_windows(const uint32_t* __restrict__ tile, int lane,
                                             uint32_t (&w)[8]) {
    constexpr int N32 = 8 * K;  // uint32 words per tile
    if constexpr (K == 4) {
        // b0 = 32l - 12 (mod 1024): with S = word(l-1):word(l) (64 bits, MSB
        // first), window j sits at S offset 20 + 4j, i.e. (S >> (28 - 4j)) &
        // 0xffff.  Byte-aligned windows are one byte permute; the odd-nibble
        // ones share one funnel shift q = S >> 12.
        const uint32_t wa = tile[(lane + N32 - 1) & (N32 - 1)];
        const uint32_t wb = tile[lane];
        const uint32_t r0 = __byte_perm(wb, wa, 0x5432);  // S >> 16
        const uint32_t q = __funnelshift_r(wb, wa, 12);    // S >> 12
        w[0] = q >> 16;
        w[1] = __byte_perm(r0, 0u, 0x4421);
        w[2] = __byte_perm(q, 0u, 0x4421);
        w[3] = wb >> 16;
        w[4] = q & 0xffffu;
        w[5] = __byte_perm(wb, 0u, 0x4421);
        w[6] = (wb >> 4) & 0xffffu;
        w[7] = wb & 0xffffu;
    } else {
        constexpr int UNITS = 16 * K;  // 16-bit units per tile
        const int b0 = ((8 * lane + 257) * K - 16) % (256 * K);
        const int u0 = (b0 >> 4) % UNITS;
        // b0 mod 16 = (8*lane*K + K) mod 16: K for every lane when K is even
        // (a compile-time shift the compiler can fold), K or K + 8 when odd
        const int o0 = (K % 2 == 0) ? K : (b0 & 15);
        const int i0 = u0 >> 1;
        const bool odd = (u0 & 1) != 0;
        const uint32_t sel = odd ? 0x1076u : 0x3210u;
        const uint32_t wa = tile[i0];
        const uint32_t wb = tile[(i0 + 1) % N32];
        const uint32_t wc = tile[(i0 + 2) % N32];
        const uint32_t r0 = __byte_perm(wa, wb, sel);
        const uint32_t r1 = __byte_perm(wb, wc, sel);
        if constexpr (K <= 4) {
            // o0 + 7K <= 32 for K <= 4: every window lies in r0:r1.
            #pragma unroll
            for (int j = 0; j < 8; ++j) w[j] = win_at(r0, r1, o0 + j * K);
        } else {
            const uint32_t wd = tile[(i0 + 3) % N32];
            const uint32_t r2 = __byte_perm(wc, wd, sel);
            #pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int o = o0 + j * K;
                w[j] = (o <= 32) ? win_at(r0, r1, o) : win_at(r1, r2, o - 32);
            }
        }
    }
}

// Decode lane's share of one tile into the mma.m16n8k16 A fragment of W~^T
// (16 output features x 16 input features): a[0] = values j0,j1; a[1] = j4,j5;
// a[2] = j2,j3; a[3] = j6,j7.
template <int K, int CB>
__device__ __forceinline__ void decode_tile_afrag(const uint32_t* __restrict__ tile, int lane,
                                                  uint32_t (&a)[4]) {
    uint32_t w[8];
    tile_windows<K>(tile, lane, w);
    a[0] = decode_pair<CB>(w[0], w[1]);
    a[1] = decode_pair<CB>(w[4], w[5]);
    a[2] = decode_pair<CB>(w[2], w[3]);
    a[3] = decode_pair<CB>(w[6], w[7]);
}

// MCG / 3INST hash of one 16-bit window, stopped before the final add: the
// fp16x2 word {lo, hi} whose sum is the decoded weight.
template <int CB>
__device__ __forceinline__ uint32_t hash_word(uint32_t w) {
    uint32_t x;
    if constexpr (CB == CB_MCG) x = w * 0xCBAC1FEDu;
    else x = w * 89226354u + 64248484u;
    return (x & 0x8fff8fffu) ^ 0x3b603b60u;
}

// MCG / 3INST for the MMA: the lane's eight windows hashed but not summed
// (h[j] = {lo, hi} of value j).  Multiplied against an activation duplicated
// along K (both halves meet the same x), the tensor core forms
// lo*x + hi*x = (lo + hi)*x exactly in its fp32 accumulation, so the integer
// work per weight drops by the add and the fp16x2 repacking.  The weight is
// then used unrounded; the reference rounds lo + hi to fp16 first, a
// difference of at most half an fp16 ulp per weight.  Bit-exact fp16
// weights remain the job of the reconstruct path.
template <int K, int CB>
__device__ __forceinline__ void decode_tile_words(const uint32_t* __restrict__ tile, int lane,
                                                  uint32_t (&h)[8]) {
    uint32_t w[8];
    tile_windows<K>(tile, lane, w);
    #pragma unroll
    for (int j = 0; j < 8; ++j) h[j] = hash_word<CB>(w[j]);
}

// Position (fp16 element) of the first of the two copies of activation k
// (0..127) inside one 128-feature block of the duplicated layout used with
// decode_tile_words: per 16-feature k-tile 32 elements, two halves of 16,
// each holding k-pairs c = 0..7 for k = 2c (c < 4) or 2(c - 4) + 1 (c >= 4)
// -- the K order in which the lane's words meet the mma.m16n8k16 A fragment.
__device__ __forceinline__ int dup_pos(int k) {
    const int kl = k & 15;
    return (k >> 4) * 32 + (kl >> 3) * 16 + 2 * (((kl & 7) >> 1) + 4 * (kl & 1));
}

// Same decode, returning the eight fp16 values in j order as four fp16x2
// registers {j0,j1}, {j2,j3}, {j4,j5}, {j6,j7}.
template <int K, int CB>
__device__ __forceinline__ void decode_tile_pairs(const uint32_t* __restrict__ tile, int lane,
                                                  uint32_t (&v)[4]) {
    uint32_t w[8];
    tile_windows<K>(tile, lane, w);
    v[0] = decode_pair<CB>(w[0], w[1]);
    v[1] = decode_pair<CB>(w[2], w[3]);
    v[2] = decode_pair<CB>(w[4], w[5]);
    v[3] = decode_pair<CB>(w[6], w[7]);
}

// ---------------------------------------------------------------------------
// 128-point fast Walsh-Hadamard transform held by one warp, element
// lane + 32*i in v[i].  Stages run in the reference's order, strides
// 1, 2, 4, ..., 64 (exl3_dequant.cuh:168-179), each output being a + b or
// a - b of the same two fp32 inputs, so the result is bit-identical to the
// sequential transform.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void fwht128_warp(float (&v)[4], int lane) {
    #pragma unroll
    for (int s = 1; s < 32; s <<= 1) {
        const bool upper = (lane & s) != 0;
        #pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float p = __shfl_xor_sync(0xffffffffu, v[i], s);
            v[i] = upper ? __fsub_rn(p, v[i]) : __fadd_rn(v[i], p);
        }
    }
    {   // stride 32: (v0, v1), (v2, v3)
        const float a0 = v[0], b0 = v[1], a1 = v[2], b1 = v[3];
        v[0] = __fadd_rn(a0, b0); v[1] = __fsub_rn(a0, b0);
        v[2] = __fadd_rn(a1, b1); v[3] = __fsub_rn(a1, b1);
    }
    {   // stride 64: (v0, v2), (v1, v3)
        const float a0 = v[0], b0 = v[2], a1 = v[1], b1 = v[3];
        v[0] = __fadd_rn(a0, b0); v[2] = __fsub_rn(a0, b0);
        v[1] = __fadd_rn(a1, b1); v[3] = __fsub_rn(a1, b1);
    }
}

// Same transform with element 4*lane + i in v[i] (contiguous lanes, for
// vectorised row loads and stores).  Only the GEMV/GEMM activation paths use
// it; the bit-exact reconstruction keeps fwht128_warp.
__device__ __forceinline__ void fwht128_warp_contig(float (&v)[4], int lane) {
    {
        const float a0 = v[0], b0 = v[1], a1 = v[2], b1 = v[3];
        v[0] = a0 + b0; v[1] = a0 - b0; v[2] = a1 + b1; v[3] = a1 - b1;
    }
    {
        const float a0 = v[0], b0 = v[2], a1 = v[1], b1 = v[3];
        v[0] = a0 + b0; v[2] = a0 - b0; v[1] = a1 + b1; v[3] = a1 - b1;
    }
    #pragma unroll
    for (int s = 1; s < 32; s <<= 1) {
        const bool upper = (lane & s) != 0;
        #pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float p = __shfl_xor_sync(0xffffffffu, v[i], s);
            v[i] = upper ? p - v[i] : v[i] + p;
        }
    }
}

// ---------------------------------------------------------------------------
// Tensor-core fragments (register-fed mma.sync; the operands are decoded in
// registers, so no shared-memory round trip is needed for the weights).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t smem_addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_addr));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier + bulk async copy (TMA engine, 1-D form).  Every wait is bounded
// by a clock budget; on expiry it records DEV_WAIT_TIMEOUT and returns false.
// ---------------------------------------------------------------------------
constexpr long long kWaitBudgetCycles = 4000000000LL;  // ~2 s at 2 GHz

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}

// try_wait with a suspend-time hint: a thread whose phase is not complete
// sleeps (woken when the phase completes, or after at most the hint) instead
// of spinning, so waiting warps leave the issue slots to the working ones.
constexpr uint32_t kWaitSuspendNs = 1000000;  // 1 ms upper bound per try

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kWaitSuspendNs)
        : "memory");
    return ok != 0;
}

// Next slot of an S-deep ring; the phase parity flips on wrap-around
// (kept incrementally so no loop divides by the runtime depth).
__device__ __forceinline__ void ring_next(int& s, uint32_t& ph, int S) {
    if (++s == S) {
        s = 0;
        ph ^= 1u;
    }
}

// Returns false (and records the timeout) if the phase did not complete in
// the budget.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > kWaitBudgetCycles) {
            set_status(status, DEV_WAIT_TIMEOUT);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
            smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Programmatic dependent launch (griddepcontrol).  launch_dependents lets the
// next kernel of the stream, when it is launched with programmatic stream
// serialization, be scheduled before this one ends; wait blocks the calling
// thread until the kernel before it has completed and its writes are
// visible.  Both are no-ops for kernels launched the ordinary way.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ void named_bar_arrive(int id, int threads) {
    asm volatile("bar.arrive %0, %1;\n" ::"r"(id), "r"(threads) : "memory");
}

// dtype codes of the C ABI
enum DType : int { DT_F32 = 0, DT_F16 = 1, DT_BF16 = 2, DT_I32 = 3, DT_I64 = 4 };

__device__ __forceinline__ float load_as_float(const void* p, int64_t i, int dt) {
    if (dt == DT_F32) return static_cast<const float*>(p)[i];
    if (dt == DT_F16) return __half2float(static_cast<const __half*>(p)[i]);
    return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}

__device__ __forceinline__ void store_from_float(void* p, int64_t i, int dt, float v) {
    if (dt == DT_F32) static_cast<float*>(p)[i] = v;
    else if (dt == DT_F16) static_cast<__half*>(p)[i] = __float2half_rn(v);
    else static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

__device__ __forceinline__ int64_t load_id(const void* p, int64_t i, int dt) {
    return dt == DT_I64 ? static_cast<const int64_t*>(p)[i]
                        : static_cast<int64_t>(static_cast<const int32_t*>(p)[i]);
}

// Per-expert pointers of one projection family (tables) or a dense projection.
__device__ __forceinline__ const __half* proj_suh(const ProjRef& p, int e) {
    return p.suh_tbl ? reinterpret_cast<const __half*>(p.suh_tbl[e]) : static_cast<const __half*>(p.suh);
}
__device__ __forceinline__ const __half* proj_svh(const ProjRef& p, int e) {
    return p.svh_tbl ? reinterpret_cast<const __half*>(p.svh_tbl[e]) : static_cast<const __half*>(p.svh);
}
__device__ __forceinline__ const uint16_t* proj_trellis(const ProjRef& p, int e) {
    return p.trellis_tbl ? reinterpret_cast<const uint16_t*>(p.trellis_tbl[e])
                         : static_cast<const uint16_t*>(p.trellis);
}
__device__ __forceinline__ int proj_k(const ProjRef& p, int e) {
    return p.k_tbl ? int(p.k_tbl[e]) : p.k_uniform;
}

}  // namespace exl3
