// tc_gemm.cu -- routed grouped GEMM for prefill-sized batches on sm_100a:
// tcgen05 tensor cores with TMEM accumulators, TMA-fed activations and
// weights decoded from the trellis into shared memory.  The up projection's
// epilogue also applies the activation and the down projection's input
// rotation, so gate/up never make a second round trip through HBM.
//
// Replaces the reference's prefill tiers: ExLlamaV3 exl3_moe / exl3_moe_mixedk
// (expert-batched, src/vllm_exl3/exl3.py:3275-3579) and the fat-expert tier
// exl3_fat_gemm(_scatter) (csrc/exl3_fat_gemm.cu:65-305: 128x128 mma.sync
// tiles, K4 MCG only).
//
// Work item = one work tile (128 or 256 sorted rows of one expert: its
// routes, sorted and padded by the prep kernel) x one 128-column output block
// (= one 128-point Hadamard block); K runs in stages of 64.  One persistent
// CTA per SM walks the items with warp-specialised roles and three shared-
// memory rings, so no role waits on another's latency unless a ring is
// empty:
//   warp 0   activation producer: TMA 2-D loads of the 128x64 fp16 box per
//            128-row half (128-byte swizzle) into the A ring
//   warp 1   trellis producer: 1-D bulk copies of the stage's four k-tile
//            rows of compressed words into the (deep, small) raw ring
//   warp 2   TMEM allocator and the single MMA-issuing thread: tcgen05.mma
//            kind::f16 M128 N128 K16 (two accumulators for 256-row tiles),
//            fp32 in one of two TMEM accumulator buffers; tcgen05.commit
//            frees A and B slots and hands a finished buffer to the epilogue
//   warps 3-18 decoders: warp (d, half) decodes column tile d of two of the
//            stage's four k-tiles from the raw ring straight into the K-major
//            128-byte-swizzled B ring UMMA reads (conflict-free stores)
//   warps 19-22 epilogue: tcgen05.ld of each 128-row accumulator half into a
//            staging tile, release of the TMEM buffer, then per row a
//            warp-wide 128-point FWHT * svh / sqrt128 and the item's output
//            (fp32 rows, * route weight, the caller's dtype / scatter, or the
//            fused SwiGLU + down-input rotation), overlapping the next item's
//            main loop on the other TMEM buffer.
// Every mbarrier wait is bounded (a timeout records a status and aborts all
// roles, which then drain their in-flight copies and MMAs); no multicast.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "exl3_common.cuh"
#include "exl3_internal.h"
#include "tc_common.cuh"
#include "tc_gemm.h"

namespace exl3 {

// K per stage 64 (128-byte swizzled rows).  32-deep stages (64-byte swizzle)
// measured slower on B200: per-stage synchronisation outweighed the depth.
constexpr int kTcM = 128, kTcN = 128, kTcK = 64;
constexpr int kTcKt = kTcK / 16;            // k-tiles per stage
constexpr int kTcSwB = kTcK * 2;            // swizzle span = row bytes
constexpr int kTcABytes = kTcM * kTcK * 2;  // 16 KB per 128-row half
constexpr int kTcBBytes = kTcN * kTcK * 2;  // 16 KB
constexpr int kTcEpiPitch = 129;            // fp32 pitch of the staging tile (conflict-free row and column sweeps)
constexpr int kTcEpiBytes = kTcM * kTcEpiPitch * 4;

// warp roles
constexpr int kWarpProdA = 0, kWarpProdRaw = 1, kWarpMma = 2, kWarpDec0 = 3, kNumDec = 16;
constexpr int kWarpEpi0 = kWarpDec0 + kNumDec, kNumEpi = 4;
constexpr int kTcThreads = (kWarpEpi0 + kNumEpi) * 32;  // 736
constexpr int kEpiBarrier = 2;                           // named barrier of the epilogue warps

__host__ __device__ inline size_t tc_raw_bytes(int kmax) { return size_t(kTcKt) * 256 * kmax; }

// Shared-memory carve-up for ring depths (sa, sb, sr): A ring first (1024-
// aligned slots), then the B ring, the raw ring, the staging tile, barriers.
struct TcLayout {
    size_t a_off, b_off, raw_off, ep_off, bar_off, total;
    size_t a_slot, raw_slot;
};
__host__ __device__ inline TcLayout tc_layout(int kmax, int mt, int sa, int sb, int sr) {
    TcLayout L;
    L.a_slot = size_t(mt) * kTcABytes;
    L.raw_slot = (tc_raw_bytes(kmax) + 127) & ~size_t(127);
    L.a_off = 0;
    L.b_off = L.a_off + size_t(sa) * L.a_slot;
    L.raw_off = L.b_off + size_t(sb) * kTcBBytes;
    L.ep_off = L.raw_off + size_t(sr) * L.raw_slot;
    L.bar_off = (L.ep_off + kTcEpiBytes + 15) & ~size_t(15);
    L.total = L.bar_off + size_t(2 * (sa + sb + sr) + 5) * 8 + 16;
    return L;
}

__device__ __forceinline__ uint32_t tc_b_offset(int row, int k) {
    if constexpr (kTcSwB == 128) return sw128_offset(row, k);
    else return sw64_offset(row, k);
}

// Per-lane byte offsets of a decoder's stores into the swizzled weight tile.
// Lane (g, t) of column tile d writes, per k-tile kk, the fp16 pairs
// (n0, k0), (n0, k0 + 8), (n0 + 8, k0), (n0 + 8, k0 + 8) with n0 = 16d + g,
// k0 = 16kk + 2t.  k0 >> 3 is even, so k0 + 8 only flips bit 0 of the
// swizzled 16-byte chunk (offset ^ 16), and n0 + 8 is the next 8-row atom
// (+ 8 * kTcSwB): two offsets per k-tile cover all four stores.  A decoder
// warp owns two of the stage's four k-tiles: kk = 2 * half + {0, 1}.
struct TcStoreOffsets {
    uint32_t a[2], b[2];  // (n0, k0) and (n0, k0 + 8)
};

__device__ __forceinline__ TcStoreOffsets tc_store_offsets(int d, int half, int lane) {
    TcStoreOffsets o;
    const int n0 = 16 * d + (lane >> 2);
    #pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int k0 = 16 * (2 * half + i) + 2 * (lane & 3);
        o.a[i] = tc_b_offset(n0, k0);
        o.b[i] = tc_b_offset(n0, k0 + 8);
    }
    return o;
}

template <int K, int CB>
__device__ __forceinline__ void tc_decode_slice(const char* raw, char* bsm, int d, int half, int lane,
                                                const TcStoreOffsets& so) {
    // values j of lane l sit at n = 16d + l/4 (+8 for j >= 4),
    // k = 16kk + 2(l%4) (+1 for odd j, +8 for j&2)
    constexpr int kAtom = 8 * kTcSwB;  // bytes of 8 rows
    #pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int kk = 2 * half + i;
        const uint32_t* tile = reinterpret_cast<const uint32_t*>(raw) + (kk * 8 + d) * (8 * K);
        uint32_t v[4];
        decode_tile_pairs<K, CB>(tile, lane, v);
        char* pa = bsm + so.a[i];
        char* pb = bsm + so.b[i];
        *reinterpret_cast<uint32_t*>(pa) = v[0];
        *reinterpret_cast<uint32_t*>(pb) = v[1];
        *reinterpret_cast<uint32_t*>(pa + kAtom) = v[2];
        *reinterpret_cast<uint32_t*>(pb + kAtom) = v[3];
    }
}

__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, int* status, volatile int* abort_flag) {
    if (*abort_flag) return false;
    if (mbar_wait(bar, parity, status)) return true;
    *abort_flag = 1;
    return false;
}

// Per-item facts every role derives the same way.
struct TcItem {
    int e, p0, rows, cb, K, nh;
    bool ok;
    const uint16_t* trellis;
};

template <int MT>
__device__ __forceinline__ TcItem tc_item(const TcArgs& a, int64_t it) {
    TcItem I;
    const int4 T = a.tiles[it / a.ncb];
    I.cb = int(it % a.ncb);
    I.e = T.x, I.p0 = T.y, I.rows = T.z;
    I.K = proj_k(a.proj, I.e);
    I.trellis = proj_trellis(a.proj, I.e);
    I.ok = I.K >= 2 && I.K <= a.kmax && I.trellis != nullptr && (reinterpret_cast<uintptr_t>(I.trellis) & 15) == 0;
    I.nh = (MT == 2 && I.rows > 128) ? 2 : 1;
    return I;
}

// A decoder warp's stages of one item at a fixed bit width (K = 0: weights
// unusable, its slices are zeroed so the MMA adds nothing).
template <int K, int CB>
__device__ __forceinline__ bool tc_decode_item(char* smem, const TcLayout& L, int nst, int sb_n, int sr_n,
                                               uint64_t* raw_full, uint64_t* raw_empty, uint64_t* b_full,
                                               uint64_t* b_empty, int& rs, uint32_t& rph, int& bs, uint32_t& bph,
                                               int* status, volatile int* abort_flag, int d, int half, int lane,
                                               const TcStoreOffsets& so) {
    for (int ks = 0; ks < nst; ++ks) {
        if (!tc_wait(&raw_full[rs], rph, status, abort_flag)) return false;
        if (!tc_wait(&b_empty[bs], bph ^ 1u, status, abort_flag)) return false;
        char* bsm = smem + L.b_off + size_t(bs) * kTcBBytes;
        if constexpr (K != 0) {
            tc_decode_slice<K, CB>(smem + L.raw_off + size_t(rs) * L.raw_slot, bsm, d, half, lane, so);
        } else {
            for (int i = lane; i < 2 * 16 * 8; i += 32) {  // 2 k-tiles x 16 rows x 8 pairs
                const int kk = 2 * half + (i >> 7), n = 16 * d + ((i >> 3) & 15), k = 16 * kk + 2 * (i & 7);
                *reinterpret_cast<uint32_t*>(bsm + tc_b_offset(n, k)) = 0u;
            }
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&b_full[bs]);
            mbar_arrive(&raw_empty[rs]);
        }
        ring_next(rs, rph, sr_n);
        ring_next(bs, bph, sb_n);
    }
    return true;
}

template <int CB, int MT>
__global__ void __launch_bounds__(kTcThreads, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ TcArgs a) {
    extern __shared__ __align__(1024) char tc_smem_raw[];
    char* smem = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
    const int SA = a.sa, SB = a.sb, SR = a.sr;
    const TcLayout L = tc_layout(a.kmax, MT, SA, SB, SR);
    uint64_t* a_full = reinterpret_cast<uint64_t*>(smem + L.bar_off);
    uint64_t* a_empty = a_full + SA;
    uint64_t* b_full = a_empty + SA;
    uint64_t* b_empty = b_full + SB;
    uint64_t* raw_full = b_empty + SB;
    uint64_t* raw_empty = raw_full + SR;
    uint64_t* acc_full = raw_empty + SR;  // [2]
    uint64_t* acc_empty = acc_full + 2;   // [2]
    uint64_t* mma_done = acc_empty + 2;   // the MMA thread's final drain
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* epi_abort = abort_flag + 1;  // written only by epilogue warps, read after their barrier
    constexpr uint32_t kAccCols = uint32_t(kTcN) * MT;  // one accumulator buffer

    const int64_t n_items = int64_t(*a.ntiles) * a.ncb;
    const int nst = a.in_f / kTcK;
    const int ntiles_out = a.out_f / 16;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < SA; ++s) {
            mbar_init(&a_full[s], 1);
            mbar_init(&a_empty[s], 1);
        }
        for (int s = 0; s < SB; ++s) {
            mbar_init(&b_full[s], kNumDec);
            mbar_init(&b_empty[s], 1);
        }
        for (int s = 0; s < SR; ++s) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], kNumDec);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&acc_full[s], 1);
            mbar_init(&acc_empty[s], kNumEpi);
        }
        mbar_init(mma_done, 1);
        *abort_flag = 0;
        *epi_abort = 0;
        mbar_fence_init();
    }
    if (warp == kWarpMma) tmem_alloc(tmem_slot, 2 * kAccCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t taddr = *tmem_slot;

    if (warp == kWarpProdA) {
        // ------------------------- activation producer -------------------------
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0u, issued = 0u;
            for (int64_t it = blockIdx.x; it < n_items && !*abort_flag; it += gridDim.x) {
                const TcItem I = tc_item<MT>(a, it);
                for (int ks = 0; ks < nst; ++ks) {
                    if (!tc_wait(&a_empty[s], ph ^ 1u, a.status, abort_flag)) break;
                    char* st = smem + L.a_off + size_t(s) * L.a_slot;
                    mbar_arrive_expect_tx(&a_full[s], uint32_t(I.nh * kTcABytes));
                    for (int h = 0; h < I.nh; ++h)
                        tma_load_2d(st + h * kTcABytes, &amap, ks * kTcK, I.p0 + 128 * h, &a_full[s]);
                    ++issued;
                    ring_next(s, ph, SA);
                }
            }
            // drain: the last issued loads must land before the CTA exits
            for (uint32_t i = 0; i < uint32_t(SA) && i < issued; ++i) {
                s = (s + SA - 1) % SA;
                if (s == SA - 1) ph ^= 1u;
                mbar_wait(&a_full[s], ph, a.status);
            }
        }
    } else if (warp == kWarpProdRaw) {
        // --------------------------- trellis producer ---------------------------
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0u, issued = 0u;
            for (int64_t it = blockIdx.x; it < n_items && !*abort_flag; it += gridDim.x) {
                const TcItem I = tc_item<MT>(a, it);
                if (!I.ok)
                    set_status(a.status, I.K < 2 || I.K > a.kmax ? DEV_BAD_K : (I.trellis ? DEV_BAD_ALIGN : DEV_NULL_PTR));
                const int tw = 16 * I.K;
                for (int ks = 0; ks < nst; ++ks) {
                    if (!tc_wait(&raw_empty[s], ph ^ 1u, a.status, abort_flag)) break;
                    char* st = smem + L.raw_off + size_t(s) * L.raw_slot;
                    if (I.ok) {
                        mbar_arrive_expect_tx(&raw_full[s], uint32_t(kTcKt * 256 * I.K));
                        for (int kk = 0; kk < kTcKt; ++kk) {
                            const uint16_t* src =
                                I.trellis + (int64_t(ks * kTcKt + kk) * ntiles_out + int64_t(I.cb) * 8) * tw;
                            bulk_g2s(st + size_t(kk) * 256 * I.K, src, uint32_t(256 * I.K), &raw_full[s]);
                        }
                    } else {
                        mbar_arrive(&raw_full[s]);  // nothing to load: the decoders zero the slice
                    }
                    ++issued;
                    ring_next(s, ph, SR);
                }
            }
            for (uint32_t i = 0; i < uint32_t(SR) && i < issued; ++i) {
                s = (s + SR - 1) % SR;
                if (s == SR - 1) ph ^= 1u;
                mbar_wait(&raw_full[s], ph, a.status);
            }
        }
    } else if (warp == kWarpMma) {
        // ------------------------------ MMA issuer ------------------------------
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_f16_f32(kTcM, kTcN);
            int as = 0, bs = 0, ab = 0;
            uint32_t aph = 0u, bph = 0u, abph = 0u;
            for (int64_t it = blockIdx.x; it < n_items; it += gridDim.x) {
                const TcItem I = tc_item<MT>(a, it);
                if (!tc_wait(&acc_empty[ab], abph ^ 1u, a.status, abort_flag)) break;
                tc_fence_after();
                const uint32_t tacc = taddr + uint32_t(ab) * kAccCols;
                bool aborted = false;
                for (int ks = 0; ks < nst; ++ks) {
                    if (!tc_wait(&a_full[as], aph, a.status, abort_flag) ||
                        !tc_wait(&b_full[bs], bph, a.status, abort_flag)) {
                        aborted = true;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t abase = smem_u32(smem + L.a_off + size_t(as) * L.a_slot);
                    const uint32_t bbase = smem_u32(smem + L.b_off + size_t(bs) * kTcBBytes);
                    #pragma unroll
                    for (int k4 = 0; k4 < kTcK / 16; ++k4) {
                        const uint64_t bdesc = umma_desc_k_sw<kTcSwB>(bbase + 32 * k4);
                        for (int h = 0; h < I.nh; ++h)
                            umma_f16(tacc + uint32_t(kTcN * h), umma_desc_k_sw<kTcSwB>(abase + h * kTcABytes + 32 * k4),
                                     bdesc, idesc, (ks | k4) != 0);
                    }
                    umma_commit(&a_empty[as]);
                    umma_commit(&b_empty[bs]);
                    ring_next(as, aph, SA);
                    ring_next(bs, bph, SB);
                }
                umma_commit(&acc_full[ab]);  // also when aborted: the epilogue may be waiting on it
                ring_next(ab, abph, 2);
                if (aborted) break;
            }
            // every issued MMA has completed before TMEM is freed below
            umma_commit(mma_done);
            mbar_wait(mma_done, 0u, a.status);
        }
    } else if (warp < kWarpEpi0) {
        // ------------------------------- decoders -------------------------------
        const int dw = warp - kWarpDec0;
        const int d = dw & 7, half = dw >> 3;  // column tile, k-tile pair of each stage
        const TcStoreOffsets so = tc_store_offsets(d, half, lane);
        int rs = 0, bs = 0;
        uint32_t rph = 0u, bph = 0u;
        for (int64_t it = blockIdx.x; it < n_items; it += gridDim.x) {
            const TcItem I = tc_item<MT>(a, it);
            bool ok = true;
            #define EXL3_TC_DEC(KK)                                                                               \
                ok = tc_decode_item<KK, CB>(smem, L, nst, SB, SR, raw_full, raw_empty, b_full, b_empty, rs, rph, bs, \
                                            bph, a.status, abort_flag, d, half, lane, so)
            switch (I.ok ? I.K : 0) {
                case 2: EXL3_TC_DEC(2); break;
                case 3: EXL3_TC_DEC(3); break;
                case 4: EXL3_TC_DEC(4); break;
                case 5: EXL3_TC_DEC(5); break;
                case 6: EXL3_TC_DEC(6); break;
                case 7: EXL3_TC_DEC(7); break;
                case 8: EXL3_TC_DEC(8); break;
                default: EXL3_TC_DEC(0); break;
            }
            #undef EXL3_TC_DEC
            if (!ok) break;
        }
    } else {
        // ------------------------------- epilogue -------------------------------
        const int ew = warp - kWarpEpi0;  // 0..3: rows ew, ew + 4, ...
        const int q = warp & 3;           // TMEM lane quarter this warp may access
        float* ep = reinterpret_cast<float*>(smem + L.ep_off);  // [128][kTcEpiPitch]
        int ab = 0;
        uint32_t abph = 0u;
        for (int64_t it = blockIdx.x; it < n_items; it += gridDim.x) {
            const TcItem I = tc_item<MT>(a, it);
            if (!tc_wait(&acc_full[ab], abph, a.status, abort_flag)) {
                *epi_abort = 1;
                mbar_wait(&acc_full[ab], abph, a.status);  // issued MMAs must end before TMEM is reused
            }
            // one decision for all epilogue warps (their named barriers must match)
            named_bar_sync(kEpiBarrier, kNumEpi * 32);
            const bool got = *epi_abort == 0;
            tc_fence_after();
            const __half* svh = proj_svh(a.proj, I.e) + I.cb * 128;
            float sv[4];
            #pragma unroll
            for (int i = 0; i < 4; ++i) sv[i] = __half2float(svh[lane + 32 * i]) * kHadNorm;
            float su[4] = {0.f, 0.f, 0.f, 0.f};
            if (a.epi == TC_EPI_UPACT) {
                const __half* sup = proj_suh(a.down, I.e);  // every row of the tile is expert e
                #pragma unroll
                for (int i = 0; i < 4; ++i) su[i] = sup ? __half2float(sup[I.cb * 128 + lane + 32 * i]) : 0.f;
            }
            for (int h = 0; h < I.nh; ++h) {
                named_bar_sync(kEpiBarrier, kNumEpi * 32);  // the staging tile is free
                {
                    const int row = 32 * q + lane;
                    const uint32_t tbase = taddr + uint32_t(ab) * kAccCols + uint32_t(kTcN * h);
                    #pragma unroll 1
                    for (int c4 = 0; c4 < 4; ++c4) {
                        float part[32];
                        tmem_ld32(tbase + (uint32_t(32 * q) << 16) + uint32_t(32 * c4), part);
                        #pragma unroll
                        for (int i = 0; i < 32; ++i) ep[row * kTcEpiPitch + 32 * c4 + i] = part[i];
                    }
                }
                if (h == I.nh - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acc_empty[ab]);  // the TMEM buffer may take the next item
                }
                named_bar_sync(kEpiBarrier, kNumEpi * 32);  // staging complete
                if (!got) continue;
                const int rows_h = min(128, I.rows - 128 * h);
                // UPACT: the gate rows come from global memory; keep two rows in flight
                float gq[2][4];
                if (a.epi == TC_EPI_UPACT) {
                    #pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        const int rr = ew + kNumEpi * j;
                        const float* gr = a.g_rows + (I.p0 + 128 * h + rr) * int64_t(a.out_f) + I.cb * 128;
                        #pragma unroll
                        for (int i = 0; i < 4; ++i) gq[j][i] = rr < rows_h ? gr[lane + 32 * i] : 0.f;
                    }
                }
                for (int r = ew; r < rows_h; r += kNumEpi) {
                    float x[4];
                    #pragma unroll
                    for (int i = 0; i < 4; ++i) x[i] = ep[r * kTcEpiPitch + lane + 32 * i];
                    fwht128_warp(x, lane);
                    const int64_t p = I.p0 + 128 * h + r;
                    float wmul = 1.f;
                    if (a.epi == TC_EPI_DOWN) wmul = a.sorted_w[p];
                    #pragma unroll
                    for (int i = 0; i < 4; ++i) x[i] *= sv[i] * wmul;
                    if (a.epi == TC_EPI_LINEAR) {
                        const int tok = a.sorted_tok[p];
                        if (tok < 0) continue;
                        if (a.scatter_idx) {
                            // one route per destination row per call: plain read-modify-write
                            float* dst = static_cast<float*>(a.y) + a.scatter_idx[tok] * a.out_f + I.cb * 128;
                            const float w = __half2float(a.scatter_w[tok]);
                            #pragma unroll
                            for (int i = 0; i < 4; ++i) dst[lane + 32 * i] += w * x[i];
                        } else {
                            #pragma unroll
                            for (int i = 0; i < 4; ++i)
                                store_from_float(a.y, int64_t(tok) * a.out_f + I.cb * 128 + lane + 32 * i, a.y_dtype,
                                                 x[i]);
                        }
                    } else if (a.epi == TC_EPI_UPACT) {
                        // x = up; SwiGLU (+clamp) with the gate row, fp16 like the
                        // reference's act.half(), o suh_down, the down input's
                        // 128-point rotation (this column block is one Hadamard block)
                        float gv[4];
                        #pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            gv[i] = gq[0][i];
                            gq[0][i] = gq[1][i];
                        }
                        if (r + 2 * kNumEpi < rows_h) {
                            const float* gr = a.g_rows + (p + 2 * kNumEpi) * a.out_f + I.cb * 128;
                            #pragma unroll
                            for (int i = 0; i < 4; ++i) gq[1][i] = gr[lane + 32 * i];
                        }
                        #pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            float g = gv[i], u = x[i];
                            if (a.limit > 0.f) {
                                g = fminf(g, a.limit);
                                u = fminf(fmaxf(u, -a.limit), a.limit);
                            }
                            const float act = a.act == 3 ? (u + 1.0f) * g / (1.0f + expf(-1.702f * g))
                                                         : g / (1.0f + expf(-g)) * u;
                            x[i] = __half2float(__float2half_rn(act)) * su[i];
                        }
                        fwht128_warp(x, lane);
                        __half* dst = a.x2 + p * a.out_f + I.cb * 128;
                        #pragma unroll
                        for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = __float2half_rn(x[i] * kHadNorm);
                    } else {
                        float* dst = a.yrows + p * a.out_f + I.cb * 128;
                        #pragma unroll
                        for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = x[i];
                    }
                }
            }
            ring_next(ab, abph, 2);
            if (!got) break;
        }
    }
    __syncthreads();
    if (warp == kWarpMma) {
        tc_fence_after();
        tmem_dealloc(taddr, 2 * kAccCols);
    }
}

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// fp16 row-major [rows][cols] -> boxes of 128 rows x kTcK columns, kTcSwB-byte swizzle
static cudaError_t make_act_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
    const cuuint64_t strides[1] = {cuuint64_t(cols) * 2};
    const cuuint32_t box[2] = {kTcK, kTcM};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE,
                          kTcSwB == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

bool tc_pick_rings(int kmax, int mt, int& sa, int& sb, int& sr, size_t& smem) {
    // one CTA per SM: the raw ring is deep (small slots), B holds 3 (2 for
    // 256-row tiles), A takes what is left (>= 2)
    const size_t budget = 232448 - 1024 /* alignment slack */;
    sr = kmax <= 4 ? 8 : 6;
    sb = mt == 2 ? 2 : 3;
    for (sa = 6; sa >= 2; --sa) {
        const TcLayout L = tc_layout(kmax, mt, sa, sb, sr);
        if (L.total <= budget) {
            smem = L.total + 1024;
            return true;
        }
    }
    return false;
}

cudaError_t run_tc_gemm(int cb, int mt, const TcArgs& a, const void* act, int64_t act_rows, int64_t grid,
                        size_t smem, cudaStream_t s) {
    CUtensorMap map;
    cudaError_t e = make_act_map(&map, act, act_rows, a.in_f);
    if (e != cudaSuccess) return e;
    void (*kern)(CUtensorMap, TcArgs);
    if (mt == 2) {
        if (cb == CB_MCG) kern = tc_gemm_kernel<CB_MCG, 2>;
        else if (cb == CB_MUL1) kern = tc_gemm_kernel<CB_MUL1, 2>;
        else kern = tc_gemm_kernel<CB_3INST, 2>;
    } else {
        if (cb == CB_MCG) kern = tc_gemm_kernel<CB_MCG, 1>;
        else if (cb == CB_MUL1) kern = tc_gemm_kernel<CB_MUL1, 1>;
        else kern = tc_gemm_kernel<CB_3INST, 1>;
    }
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    // persistent: one CTA per SM (fewer if there cannot be that many items)
    grid = std::min<int64_t>(grid, num_sms_current());
    if (grid <= 0) return cudaSuccess;
    kern<<<unsigned(grid), kTcThreads, smem, s>>>(map, a);
    return cudaGetLastError();
}

}  // namespace exl3
