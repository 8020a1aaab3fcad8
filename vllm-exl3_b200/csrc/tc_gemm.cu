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
// One CTA computes one work tile (128 or 256 rows of one expert; rows =
// that expert's routes, sorted and padded by the prep kernel) x one
// 128-column output block (= one 128-point Hadamard block), looping over K
// in stages of 64:
//   warp 0   producer: TMA 2-D load of the 128x64 activation box per 128-row
//            half (128-byte swizzle) + 1-D bulk copies of the stage's four
//            k-tile rows of compressed trellis
//   warp 1   TMEM allocator and the single MMA-issuing thread:
//            tcgen05.mma kind::f16 M128 N128 K16, four per stage and half,
//            fp32 in TMEM; tcgen05.commit frees the stage
//   warps 2-9 decoders: each decodes its 16-column slice of the stage's
//            4 x 8 tiles in registers and stores fp16 pairs straight into the
//            K-major 128-byte-swizzled layout UMMA reads (conflict-free)
//   epilogue warps 2-5 move each 128-row accumulator half (tcgen05.ld, one
//            row per thread) into the now idle stage memory; warps 2-9 then
//            run a warp-wide 128-point FWHT per row, * 1/sqrt128 * svh, and
//            store rows coalesced (fp32 rows, * route weight, the caller's
//            dtype / scatter, or the fused SwiGLU + down-input rotation)
// Two CTAs per SM, so one CTA's prologue/epilogue overlaps the other's main
// loop and 16 decoder warps share the SM.  Every mbarrier wait is bounded; no
// multicast anywhere.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "exl3_common.cuh"
#include "exl3_internal.h"
#include "tc_common.cuh"
#include "tc_gemm.h"

namespace exl3 {

constexpr int kTcThreads = 320;
// K per stage 64 (128-byte swizzled rows).  32-deep stages (64-byte swizzle,
// twice as many stages in the same memory) measured slower on B200: the
// per-stage barrier and commit overhead outweighs the deeper pipeline.
constexpr int kTcM = 128, kTcN = 128, kTcK = 64;
constexpr int kTcKt = kTcK / 16;            // k-tiles per stage
constexpr int kTcSwB = kTcK * 2;            // swizzle span = row bytes
constexpr int kTcABytes = kTcM * kTcK * 2;  // 16 KB per 128-row half
constexpr int kTcBBytes = kTcN * kTcK * 2;  // 16 KB
constexpr int kTcMaxStages = 8;

__device__ __forceinline__ uint32_t tc_b_offset(int row, int k) {
    if constexpr (kTcSwB == 128) return sw128_offset(row, k);
    else return sw64_offset(row, k);
}

// Stage layout: mt activation halves of 128 rows (16 KB each, one TMA box
// apiece), the decoded 128 x 64 weight tile (16 KB), the raw trellis words.
__host__ __device__ inline size_t tc_raw_bytes(int kmax) { return size_t(kTcKt) * 256 * kmax; }
__host__ __device__ inline size_t tc_stage_bytes(int kmax, int mt) {
    return (size_t(mt) * kTcABytes + kTcBBytes + tc_raw_bytes(kmax) + 1023) & ~size_t(1023);
}

// Per-lane byte offsets of a decoder's stores into the swizzled weight tile.
// Lane (g, t) of column tile d writes, per k-tile kk, the fp16 pairs
// (n0, k0), (n0, k0 + 8), (n0 + 8, k0), (n0 + 8, k0 + 8) with n0 = 16d + g,
// k0 = 16kk + 2t.  k0 >> 3 is even, so k0 + 8 only flips bit 0 of the
// swizzled 16-byte chunk (offset ^ 16), and n0 + 8 is the next 8-row atom
// (+ 8 * kTcSwB): two offsets per kk cover all four stores.
struct TcStoreOffsets {
    uint32_t a[kTcKt], b[kTcKt];  // (n0, k0) and (n0, k0 + 8)
};

__device__ __forceinline__ TcStoreOffsets tc_store_offsets(int d, int lane) {
    TcStoreOffsets o;
    const int n0 = 16 * d + (lane >> 2);
    #pragma unroll
    for (int kk = 0; kk < kTcKt; ++kk) {
        const int k0 = 16 * kk + 2 * (lane & 3);
        o.a[kk] = tc_b_offset(n0, k0);
        o.b[kk] = tc_b_offset(n0, k0 + 8);
    }
    return o;
}

template <int K, int CB>
__device__ __forceinline__ void tc_decode_slice(const char* raw, char* bsm, int d, int lane,
                                                const TcStoreOffsets& so) {
    // k-tiles kk of this stage, 16-column tile d: values j of lane l sit at
    // n = 16d + l/4 (+8 for j >= 4), k = 16kk + 2(l%4) (+1 for odd j, +8 for j&2)
    constexpr int kAtom = 8 * kTcSwB;  // bytes of 8 rows
    #pragma unroll
    for (int kk = 0; kk < kTcKt; ++kk) {
        const uint32_t* tile = reinterpret_cast<const uint32_t*>(raw) + (kk * 8 + d) * (8 * K);
        uint32_t v[4];
        decode_tile_pairs<K, CB>(tile, lane, v);
        char* pa = bsm + so.a[kk];
        char* pb = bsm + so.b[kk];
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

// One decoder warp's whole K loop for a fixed bit width: the switch on the
// expert's K happens once per tile, not once per stage (an indirect branch
// per stage showed up as branch-resolve stalls).  K = 0: weights unusable,
// every stage's slice is zeroed so the MMA adds nothing.
template <int K, int CB>
__device__ __forceinline__ void tc_decoder_loop(char* smem, size_t stage_bytes, int S, int nst, int boff, int rawoff,
                                             uint64_t* full, uint64_t* dec, int* status, volatile int* abort_flag,
                                             int d, int lane) {
    const TcStoreOffsets so = tc_store_offsets(d, lane);
    int s = 0;         // stage slot and the parity of its current use
    uint32_t ph = 0u;
    for (int ks = 0; ks < nst; ++ks, ring_next(s, ph, S)) {
        const bool landed = tc_wait(&full[s], ph, status, abort_flag);
        char* st = smem + size_t(s) * stage_bytes;
        char* bsm = st + boff;
        if (K != 0 && landed) {
            tc_decode_slice<(K != 0 ? K : 2), CB>(st + rawoff, bsm, d, lane, so);
        } else {
            for (int i = lane; i < 16 * kTcK / 2; i += 32) {
                const int n = 16 * d + i / (kTcK / 2), k = 2 * (i % (kTcK / 2));
                *reinterpret_cast<uint32_t*>(bsm + tc_b_offset(n, k)) = 0u;
            }
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&dec[s]);
    }
}

constexpr int kTcEpiPitch = 129;  // fp32 pitch of the epilogue tile (conflict-free row and column sweeps)

// MT = 128-row halves per work tile: with MT = 2 one decoded weight tile
// feeds two M128 MMAs (two TMEM accumulators), halving the decode per FLOP.
template <int CB, int MT>
__global__ void __launch_bounds__(kTcThreads, 2)
tc_gemm_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ TcArgs a) {
    extern __shared__ __align__(1024) char tc_smem_raw[];
    char* smem = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));

    const int64_t n_base = int64_t(*a.ntiles) * a.ncb;
    const int nst_all = a.in_f / kTcK;
    // split-K count (CTA-uniform): the smallest s <= max_split minimising the
    // waves per unit of work, ceil(n_base * s / ctas) / s
    int nsplit = 1;
    if (a.max_split > 1 && n_base > 0) {
        int64_t best_w = (n_base + a.ctas - 1) / a.ctas;  // waves x s, compared as fractions
        for (int sp = 2; sp <= a.max_split && n_base * sp <= int64_t(gridDim.x); ++sp) {
            const int64_t w = (n_base * sp + a.ctas - 1) / a.ctas;
            if (w * nsplit < best_w * sp) {
                best_w = w;
                nsplit = sp;
            }
        }
    }
    const int64_t n_items = n_base * nsplit;
    // the grid is sized for the most tiles the routing could produce; CTAs
    // without work take the LOW block indices, which the hardware dispatches
    // first, so they exit while every SM slot is still free instead of
    // trickling through the few slots the working CTAs leave
    const int64_t item = int64_t(gridDim.x) - 1 - blockIdx.x;
    if (item >= n_items) return;  // whole CTA, before any barrier
    const int64_t base = item / nsplit;  // (tile, column block)
    const int split = int(item % nsplit);
    const int4 T = a.tiles[base / a.ncb];
    const int cb = int(base % a.ncb);
    const int e = T.x, p0 = T.y, rows = T.z;
    const int nh = (MT == 2 && rows > 128) ? 2 : 1;  // halves holding rows (CTA-uniform)

    // stage ring sized for this tile: a tile with one 128-row half needs no
    // room for a second activation box, which buys a deeper ring
    const size_t stage_bytes = tc_stage_bytes(a.kmax, nh);
    const int S = int(min(size_t(kTcMaxStages), size_t(a.stage_mem) / stage_bytes));
    if (S < 2 || size_t(S) * stage_bytes < size_t(128) * kTcEpiPitch * 4) {  // host sizing error: refuse
        if (threadIdx.x == 0) set_status(a.status, DEV_BAD_LAUNCH);
        return;
    }
    const int kBOff = nh * kTcABytes;             // decoded weight tile
    const int kRawOff = nh * kTcABytes + kTcBBytes;  // raw trellis words
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + size_t(S) * stage_bytes);
    uint64_t* dec = full + S;
    uint64_t* empty = dec + S;
    uint64_t* accf = empty + S;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accf + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);

    const int K = proj_k(a.proj, e);
    const uint16_t* trellis = proj_trellis(a.proj, e);
    const bool ok = K >= 2 && K <= a.kmax && trellis != nullptr && (reinterpret_cast<uintptr_t>(trellis) & 15) == 0;
    const int ks0 = int(int64_t(split) * nst_all / nsplit);  // this split's K stages [ks0, ks0 + nst)
    const int nst = int(int64_t(split + 1) * nst_all / nsplit) - ks0;
    const int ntiles_out = a.out_f / 16;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&dec[s], 8);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accf, 1);
        *abort_flag = 0;
        if (!ok) set_status(a.status, K < 2 || K > a.kmax ? DEV_BAD_K : (trellis ? DEV_BAD_ALIGN : DEV_NULL_PTR));
        mbar_fence_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, kTcN * MT);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t taddr = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            const int tw = 16 * K;
            int s = 0;
            uint32_t ph = 0u;
            for (int ks = 0; ks < nst; ++ks, ring_next(s, ph, S)) {
                if (!tc_wait(&empty[s], ph ^ 1u, a.status, abort_flag)) break;
                char* st = smem + size_t(s) * stage_bytes;
                const uint32_t rawb = ok ? uint32_t(kTcKt * 256 * K) : 0u;
                mbar_arrive_expect_tx(&full[s], uint32_t(nh * kTcABytes) + rawb);
                const int kg = ks0 + ks;  // K stage within the projection
                for (int h = 0; h < nh; ++h) tma_load_2d(st + h * kTcABytes, &amap, kg * kTcK, p0 + 128 * h, &full[s]);
                if (ok) {
                    for (int kk = 0; kk < kTcKt; ++kk) {
                        const uint16_t* src =
                            trellis + (int64_t(kg * kTcKt + kk) * ntiles_out + int64_t(cb) * 8) * tw;
                        bulk_g2s(st + kRawOff + size_t(kk) * 256 * K, src, uint32_t(256 * K), &full[s]);
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_f16_f32(kTcM, kTcN);
            int s = 0;
            uint32_t ph = 0u;
            for (int ks = 0; ks < nst; ++ks, ring_next(s, ph, S)) {
                if (!tc_wait(&full[s], ph, a.status, abort_flag)) break;
                if (!tc_wait(&dec[s], ph, a.status, abort_flag)) break;
                tc_fence_after();
                const uint32_t abase = smem_u32(smem + size_t(s) * stage_bytes);
                const uint32_t bbase = abase + kBOff;
                #pragma unroll
                for (int k4 = 0; k4 < kTcK / 16; ++k4) {
                    const uint64_t bdesc = umma_desc_k_sw<kTcSwB>(bbase + 32 * k4);
                    for (int h = 0; h < nh; ++h)
                        umma_f16(taddr + uint32_t(kTcN * h), umma_desc_k_sw<kTcSwB>(abase + h * kTcABytes + 32 * k4), bdesc,
                                 idesc, (ks | k4) != 0);
                }
                umma_commit(&empty[s]);
            }
            umma_commit(accf);  // also covers the no-MMA case: arrives at once
        }
        // free TMEM as soon as the epilogue warps have read the accumulators
        // (barrier 2: warp 1 + warps 2-5); the deallocation takes
        // microseconds and would otherwise sit on every CTA's exit path
        __syncwarp();
        named_bar_sync(2, 5 * 32);
        tc_fence_after();
        tmem_dealloc(taddr, kTcN * MT);
    } else {
        const int d = warp - 2;  // 16-column tile of the 128-column block
        const int kd = ok ? K : 0;
        #define EXL3_TC_DEC(KK) \
            tc_decoder_loop<KK, CB>(smem, stage_bytes, S, nst, kBOff, kRawOff, full, dec, a.status, abort_flag, d, lane)
        switch (kd) {
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

        // ---------------------------- epilogue ----------------------------
        // the stage memory is free once every MMA has completed (accf); one
        // 128-row half at a time goes TMEM -> smem tile -> FWHT -> rows
        float* ep = reinterpret_cast<float*>(smem);  // [128][kTcEpiPitch]
        const __half* svh = proj_svh(a.proj, e) + cb * 128;
        float sv[4];
        #pragma unroll
        for (int i = 0; i < 4; ++i) sv[i] = __half2float(svh[lane + 32 * i]) * kHadNorm;
        const int et = threadIdx.x - 64;  // epilogue thread 0..255
        // accumulator half h: TMEM -> epilogue tile (warps 2-5, one TMEM lane quarter each)
        auto tile_from_tmem = [&](int h) {
            if (warp < 6) {
                if (h == 0) {
                    // on an abort still wait (bounded) for issued MMAs before TMEM is read or freed
                    if (!tc_wait(accf, 0u, a.status, abort_flag)) mbar_wait(accf, 0u, a.status);
                    tc_fence_after();
                }
                const int q = warp & 3;  // TMEM lane quarter this warp may access
                const int row = 32 * q + lane;
                #pragma unroll 1
                for (int c4 = 0; c4 < 4; ++c4) {
                    float part[32];
                    tmem_ld32(taddr + (uint32_t(32 * q) << 16) + uint32_t(kTcN * h + 32 * c4), part);
                    #pragma unroll
                    for (int i = 0; i < 32; ++i) ep[row * kTcEpiPitch + 32 * c4 + i] = part[i];
                }
                tc_fence_before();
                if (h == nh - 1) named_bar_arrive(2, 5 * 32);  // last accumulator read: warp 1 may free TMEM
            }
            named_bar_sync(1, 8 * 32);
        };
        bool run_epi = true;
        float* parts = nullptr;
        if (nsplit > 1) {
            // every split stores its fp32 partial; the last split of the
            // (tile, column block) to arrive sums them in split order
            parts = a.part + size_t(base) * a.max_split * (128 * MT * 128);
            for (int h = 0; h < nh; ++h) {
                tile_from_tmem(h);
                const int rows_h = min(128, rows - 128 * h);
                float4* dst = reinterpret_cast<float4*>(parts + (size_t(split) * MT + h) * (128 * 128));
                for (int i = et; i < rows_h * 32; i += 256) {
                    const float* src = ep + (i >> 5) * kTcEpiPitch + 4 * (i & 31);
                    dst[i] = make_float4(src[0], src[1], src[2], src[3]);
                }
                named_bar_sync(1, 8 * 32);  // the tile is refilled next
            }
            // publish: the CTA barrier orders every thread's partial stores
            // before one thread's acquire-release add on the item's counter;
            // the last split reads the others after the barrier that follows
            // its acquire (no gpu-scope fence in every thread)
            named_bar_sync(1, 8 * 32);
            if (et == 0) {
                int prev;
                asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;"
                             : "=r"(prev)
                             : "l"(a.cnt + base)
                             : "memory");
                const bool last = prev == nsplit - 1;
                if (last) a.cnt[base] = 0;  // ready for the next launch
                *last_flag = last ? 1 : 0;
            }
            named_bar_sync(1, 8 * 32);
            run_epi = *last_flag != 0;
        }
        for (int h = 0; run_epi && h < nh; ++h) {
            const int rows_h = min(128, rows - 128 * h);
            if (nsplit > 1) {
                // sum in split order; four 16-byte loads per split in flight
                // per thread (one L2 round trip per 1024 vectors, not per element)
                const float4* src = reinterpret_cast<const float4*>(parts + size_t(h) * (128 * 128));
                const size_t sstride = size_t(MT) * (128 * 128) / 4;  // float4s between splits
                for (int i0 = et; i0 < rows_h * 32; i0 += 4 * 256) {
                    float4 v[4];
                    #pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int i = i0 + 256 * u;
                        v[u] = i < rows_h * 32 ? __ldcg(src + i) : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                    for (int sp = 1; sp < nsplit; ++sp) {
                        float4 w[4];
                        #pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int i = i0 + 256 * u;
                            w[u] = i < rows_h * 32 ? __ldcg(src + sp * sstride + i) : make_float4(0.f, 0.f, 0.f, 0.f);
                        }
                        #pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            v[u].x += w[u].x;
                            v[u].y += w[u].y;
                            v[u].z += w[u].z;
                            v[u].w += w[u].w;
                        }
                    }
                    #pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int i = i0 + 256 * u;
                        if (i < rows_h * 32) {
                            float* d = ep + (i >> 5) * kTcEpiPitch + 4 * (i & 31);
                            d[0] = v[u].x;
                            d[1] = v[u].y;
                            d[2] = v[u].z;
                            d[3] = v[u].w;
                        }
                    }
                }
                named_bar_sync(1, 8 * 32);
            } else {
                tile_from_tmem(h);
            }
            // UPACT: the gate rows are read from global memory; keep two rows
            // in flight ahead of the one being processed (latency hiding)
            float gq[2][4];
            float su[4] = {0.f, 0.f, 0.f, 0.f};
            const bool use_gate = a.epi == TC_EPI_UPACT && a.act != 2;  // act 2: non-gated relu^2
            if (a.epi == TC_EPI_UPACT) {
                const __half* sup = proj_suh(a.down, e);  // every row of the tile is expert e
                #pragma unroll
                for (int i = 0; i < 4; ++i) su[i] = sup ? __half2float(sup[cb * 128 + lane + 32 * i]) : 0.f;
                #pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const int rr = d + 8 * j;
                    const float* gr = a.g_rows + (p0 + 128 * h + rr) * int64_t(a.out_f) + cb * 128;
                    #pragma unroll
                    for (int i = 0; i < 4; ++i) gq[j][i] = (use_gate && rr < rows_h) ? gr[lane + 32 * i] : 0.f;
                }
            }
            for (int r = d; r < rows_h; r += 8) {
                float x[4];
                #pragma unroll
                for (int i = 0; i < 4; ++i) x[i] = ep[r * kTcEpiPitch + lane + 32 * i];
                fwht128_warp(x, lane);
                const int64_t p = p0 + 128 * h + r;
                float wmul = 1.f;
                if (a.epi == TC_EPI_DOWN) wmul = a.sorted_w[p];
                #pragma unroll
                for (int i = 0; i < 4; ++i) x[i] *= sv[i] * wmul;
                if (a.epi == TC_EPI_LINEAR) {
                    const int tok = a.sorted_tok[p];
                    if (tok < 0) continue;
                    if (a.scatter_idx) {
                        // one route per destination row per call: plain read-modify-write
                        float* dst = static_cast<float*>(a.y) + a.scatter_idx[tok] * a.out_f + cb * 128;
                        const float w = __half2float(a.scatter_w[tok]);
                        #pragma unroll
                        for (int i = 0; i < 4; ++i) dst[lane + 32 * i] += w * x[i];
                    } else {
                        #pragma unroll
                        for (int i = 0; i < 4; ++i)
                            store_from_float(a.y, int64_t(tok) * a.out_f + cb * 128 + lane + 32 * i, a.y_dtype, x[i]);
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
                    if (use_gate && r + 16 < rows_h) {
                        const float* gr = a.g_rows + (p + 16) * a.out_f + cb * 128;
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
                        float act;
                        if (a.act == 2) {
                            const float rl = fmaxf(u, 0.f);
                            act = rl * rl;
                        } else if (a.act == 3) {
                            act = (u + 1.0f) * g / (1.0f + expf(-1.702f * g));
                        } else {
                            act = g / (1.0f + expf(-g)) * u;
                        }
                        x[i] = __half2float(__float2half_rn(act)) * su[i];
                    }
                    fwht128_warp(x, lane);
                    __half* dst = a.x2 + p * a.out_f + cb * 128;
                    #pragma unroll
                    for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = __float2half_rn(x[i] * kHadNorm);
                } else {
                    float* dst = a.yrows + p * a.out_f + cb * 128;
                    #pragma unroll
                    for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = x[i];
                }
            }
            if (h + 1 < nh) named_bar_sync(1, 8 * 32);  // the tile is refilled with the next half
        }
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

bool tc_pick_stages(int kmax, int mt, int& stages, size_t& smem) {
    // two CTAs per SM; the epilogue tile [128][129] fp32 reuses the stages
    const size_t budget = (228 * 1024) / 2 - 1024 /* per-CTA reserve */ - 1024 /* alignment */ - 256;
    const size_t sb = tc_stage_bytes(kmax, mt);
    const size_t epi = size_t(128) * kTcEpiPitch * 4;
    int s = int(std::min<size_t>(kTcMaxStages, budget / sb));
    if (size_t(s) * sb < epi) s = int((epi + sb - 1) / sb);
    if (s < 2 || size_t(s) * sb > budget) return false;
    stages = s;
    // the whole budget: a tile with fewer rows than the launch's widest
    // sizes a deeper ring from the same memory
    smem = budget + 1024 + 256;
    return true;
}

int tc_split_ceiling(int64_t max_items, int in_f, int ctas) {
    if (max_items >= 2 * int64_t(ctas)) return 1;
    return std::max(1, std::min(kTcMaxSplit, in_f / kTcK / 8));
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
    if (grid <= 0) return cudaSuccess;
    kern<<<unsigned(grid), kTcThreads, smem, s>>>(map, a);
    return cudaGetLastError();
}


}  // namespace exl3
