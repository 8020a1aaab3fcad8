// moe.cu -- routed-expert EXL3 MoE forward (all tokens of a step in one
// pass) and the single-projection variants (dense linear, batched expert
// linear, fat GEMM), for sm_100a.
//
// Replaces the reference's per-token cooperative kernels p2b_fused_moe /
// p2b_fused_moe_mk / p2b_fused_moe_padded (csrc/p2b_moe.cu:643-2428), the
// m <= 8 GEMV exl3_gemv (csrc/exl3_gemv.cu:23-63) and its row-chunk loop
// exl3_gemm (csrc/exl3_gemm.cu:9-31).  The math is the reference's eager
// loop apply_exl3_python_loop (src/vllm_exl3/exl3.py:2357-2413):
//   per route (token t, local expert e, weight w):
//     g = x_t W_gate,e ; u = x_t W_up,e ; a = fp16(silu(min(g,L)) * clamp(u,L))
//     out_t += w * (a W_down,e)
// computed in the rotated domain x W = ((x o suh) H / sqrt128) W~ (H / sqrt128) o svh.
//
// Kernels, in stream order (no host synchronisation, graph-capturable):
//  1. prep     one CTA (chunked over CTAs for large batches): map ids to
//              local experts (expert_map, n_local sentinel;
//              exl3.py:2332-2354), counting sort of routes by expert (rows
//              claimed with warp-aggregated atomics, so their order within an
//              expert is free: no kernel mixes rows), each expert's rows
//              padded to 16, work slots of <= 16 rows, counters cleared.
//  2. rotate   fp16 H128(x o suh)/sqrt128 per (route, projection, 128-block),
//              stored [proj][kblock][row][136] (rows padded to 272 bytes so a
//              1-D bulk copy lands ldmatrix-conflict-free).
//  3. gemv<2>  gate+up: group = (slot, 128-column block), split stream-K:
//              every CTA takes the same number of 128-deep k stages of the
//              group sequence, so no wave is left half full.  A producer
//              thread streams the trellis rows and rotated inputs into a
//              shared-memory ring with cp.async.bulk; 8 consumer warps (one
//              16-column tile each, gate and up together) decode each 16x16
//              tile in registers straight into mma.m16n8k16 A fragments and
//              accumulate in fp32.  A group cut between CTAs is reduced in
//              stage order by the CTA that completes it (deterministic).
//              Epilogue: output FWHT o svh, SwiGLU (+clamp), fp16 round,
//              down-input rotation o suh_down -> rotated down inputs.
//  4. gemv<1>  down: same engine; epilogue FWHT o svh * route weight -> per-route rows.
//  5. combine  out_t = sum over t's routes in top-k order (no atomics).
#include <algorithm>
#include <utility>

#include "exl3_common.cuh"
#include "exl3_internal.h"
#include "tc_gemm.h"

namespace exl3 {

enum Epi : int { EPI_GATEUP = 0, EPI_DOWN = 1, EPI_LINEAR = 2, EPI_ROUTE = 3 };
enum Act : int { ACT_SILU = 0, ACT_RELU2 = 2, ACT_SWIGLU_OAI = 3 };

constexpr int kPrepThreads = 1024;
constexpr int kMaxLocal = 2048;
constexpr int kPrepChunk = 2048;       // routes per CTA when the prep is split over CTAs
constexpr int64_t kPrepSplitRoutes = 4 * kPrepChunk;  // split the prep from this many routes on
constexpr int kYsPitch = 132;          // fp32 pitch of the epilogue tile (conflict-free fragment stores)
constexpr int kXPitch = 136;           // fp16 pitch of a rotated-input row (272 B: ldmatrix conflict-free)
constexpr int kXSlice = 16 * kXPitch * 2;  // bytes of one 16-row x 128-column input slice
// MCG / 3INST: every activation stored twice in dup_pos order (256 + 8 pad,
// 528 B rows: still ldmatrix conflict-free), see decode_tile_words
constexpr int kXPitchD = 264;
constexpr int kXSliceD = 16 * kXPitchD * 2;
__host__ __device__ constexpr int x_pitch(bool dup) { return dup ? kXPitchD : kXPitch; }
__host__ __device__ constexpr int x_slice(bool dup) { return dup ? kXSliceD : kXSlice; }
constexpr int kCW = 8;                 // consumer warps: one per 16-column tile of a 128-column block
constexpr int kGemvThreads = (kCW + 1) * 32;

struct WsPtrs {
    int* status;
    int* nslots;
    int4* slots;  // {expert, first sorted row, rows, 0}
    int* route_pos;
    int* sorted_tok;
    int* sorted_route;
    int* sorted_exp;
    float* sorted_w;
    __half* xr;
    __half* a2;
    float* yd;
    float* part1;
    float* part2;
    int* cnt1;
    int* cnt2;
    int* ntiles128;
    float* tcpart;  // GEMM split-K partials
    int4* tiles128;  // {expert, first sorted row, rows <= tile_rows, 0}: the GEMM path's work tiles
    float* g;
    float* u;
    __half* x2;
    int* hist;  // split prep: [chunk][expert] counts, then first rows
};

static WsPtrs ws_ptrs(const MoePlan& p, void* ws) {
    char* b = static_cast<char*>(ws);
    WsPtrs w;
    w.status = reinterpret_cast<int*>(b + p.off_status);
    w.nslots = reinterpret_cast<int*>(b + p.off_nslots);
    w.slots = reinterpret_cast<int4*>(b + p.off_slots);
    w.route_pos = reinterpret_cast<int*>(b + p.off_route_pos);
    w.sorted_tok = reinterpret_cast<int*>(b + p.off_sorted_tok);
    w.sorted_route = reinterpret_cast<int*>(b + p.off_sorted_route);
    w.sorted_exp = reinterpret_cast<int*>(b + p.off_sorted_exp);
    w.sorted_w = reinterpret_cast<float*>(b + p.off_sorted_w);
    w.xr = reinterpret_cast<__half*>(b + p.off_xr);
    w.a2 = reinterpret_cast<__half*>(b + p.off_a2);
    w.yd = reinterpret_cast<float*>(b + p.off_yd);
    w.part1 = reinterpret_cast<float*>(b + p.off_part1);
    w.part2 = reinterpret_cast<float*>(b + p.off_part2);
    w.cnt1 = reinterpret_cast<int*>(b + p.off_cnt1);
    w.cnt2 = reinterpret_cast<int*>(b + p.off_cnt2);
    w.ntiles128 = reinterpret_cast<int*>(b + p.off_ntiles128);
    w.tcpart = reinterpret_cast<float*>(b + p.off_tcpart);
    w.tiles128 = reinterpret_cast<int4*>(b + p.off_tiles128);
    w.g = reinterpret_cast<float*>(b + p.off_g);
    w.u = reinterpret_cast<float*>(b + p.off_u);
    w.x2 = reinterpret_cast<__half*>(b + p.off_x2);
    w.hist = reinterpret_cast<int*>(b + p.off_hist);
    return w;
}

// ---------------------------------------------------------------------------
// 1. routing prep
// ---------------------------------------------------------------------------
struct PrepArgs {
    const void* ids;
    int ids_dtype;
    const void* weights;
    int w_dtype;
    const int32_t* expert_map;
    int64_t n_global;
    const int32_t* n_valid;
    int64_t t_max;
    int topk;
    int n_local;
    int linear;   // one expert, every row routed to it with weight 1
    int batched;  // ids is one expert list shared by every row: route r -> ids[r % topk]
    int cnt1_n;
    int cnt2_n;
    int tile_rows;  // GEMM path: rows per work tile (128 or 256)
    WsPtrs w;
};

__device__ __forceinline__ int local_expert(const PrepArgs& a, int64_t r) {
    if (a.linear) return 0;
    const int64_t g = load_id(a.ids, a.batched ? r % a.topk : r, a.ids_dtype);
    int64_t e = g;
    if (a.expert_map) e = (g >= 0 && g < a.n_global) ? int64_t(a.expert_map[g]) : -1;
    return (e >= 0 && e < a.n_local) ? int(e) : -1;
}

// Block-wide exclusive scan of one int per thread (kPrepThreads threads).
// Exclusive scan of three values at once (one pass: two barriers in the
// scan itself instead of two per value); sh96 holds 3 x 32 ints.
__device__ int3 block_excl_scan3(int3 v, int3* total, int* sh96) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int3 x = v;
    #pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y0 = __shfl_up_sync(0xffffffffu, x.x, o);
        const int y1 = __shfl_up_sync(0xffffffffu, x.y, o);
        const int y2 = __shfl_up_sync(0xffffffffu, x.z, o);
        if (lane >= o) {
            x.x += y0;
            x.y += y1;
            x.z += y2;
        }
    }
    if (lane == 31) {
        sh96[warp] = x.x;
        sh96[32 + warp] = x.y;
        sh96[64 + warp] = x.z;
    }
    __syncthreads();
    if (warp < 3) {
        int s = sh96[32 * warp + lane];
        #pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        sh96[32 * warp + lane] = s;
    }
    __syncthreads();
    int3 pre = make_int3(0, 0, 0);
    if (warp) pre = make_int3(sh96[warp - 1], sh96[32 + warp - 1], sh96[64 + warp - 1]);
    *total = make_int3(sh96[31], sh96[63], sh96[95]);
    __syncthreads();
    return make_int3(pre.x + x.x - v.x, pre.y + x.y - v.y, pre.z + x.z - v.z);
}

__device__ int block_excl_scan(int v, int* total, int* sh32) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
    #pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) sh32[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int s = sh32[lane];
        #pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        sh32[lane] = s;
    }
    __syncthreads();
    const int warp_prefix = warp ? sh32[warp - 1] : 0;
    *total = sh32[31];
    __syncthreads();
    return warp_prefix + x - v;
}

// Histogram of local experts over routes [r0, r1) into shared cnt[].
__device__ __forceinline__ void prep_histogram(const PrepArgs& a, int64_t r0, int64_t r1, int* cnt) {
    for (int64_t r = r0 + threadIdx.x; r < r1; r += kPrepThreads) {
        const int e = local_expert(a, r);
        if (e >= 0) atomicAdd(&cnt[e], 1);
    }
}

// From per-expert route counts: each expert's first sorted row (rows padded
// to 16) in poff[], the slot and work-tile tables, the padding rows and the
// totals.  Whole CTA; ends synchronised.
__device__ void prep_layout(const PrepArgs& a, const int* cnt, int* poff, int* sh32) {
    const int tid = threadIdx.x;
    const int E = a.n_local;
    const int per = (E + kPrepThreads - 1) / kPrepThreads;
    const int e0 = min(E, tid * per), e1 = min(E, e0 + per);
    const int TR = a.tile_rows;
    int sp = 0, ss = 0, st = 0;
    for (int e = e0; e < e1; ++e) {
        sp += (cnt[e] + 15) & ~15;
        ss += (cnt[e] + 15) >> 4;
        st += (cnt[e] + TR - 1) / TR;
    }
    int3 tot;
    const int3 x0 = block_excl_scan3(make_int3(sp, ss, st), &tot, sh32);
    int xp = x0.x, xs = x0.y, xt = x0.z;
    for (int e = e0; e < e1; ++e) {
        const int n = cnt[e];
        poff[e] = xp;
        for (int j = 0; j < ((n + 15) >> 4); ++j)
            a.w.slots[xs + j] = make_int4(e, xp + 16 * j, min(16, n - 16 * j), 0);
        if (a.w.tiles128)
            for (int j = 0; j < (n + TR - 1) / TR; ++j)
                a.w.tiles128[xt + j] = make_int4(e, xp + TR * j, min(TR, n - TR * j), 0);
        xt += (n + TR - 1) / TR;
        xp += (n + 15) & ~15;
        xs += (n + 15) >> 4;
    }
    if (tid == 0) {
        a.w.nslots[0] = tot.y;
        a.w.nslots[1] = tot.x;  // sorted rows in use (each expert padded to 16); rows past it are stale
        if (a.w.ntiles128) *a.w.ntiles128 = tot.z;
    }
    __syncthreads();
    // padding rows (fewer than 16 per expert): one warp per expert, one
    // coalesced store per array instead of one thread's serial row loop
    const int lane = tid & 31;
    for (int e = tid >> 5; e < E; e += kPrepThreads / 32) {
        const int n = cnt[e];
        if (lane < ((n + 15) & ~15) - n) {
            const int q = poff[e] + n + lane;
            a.w.sorted_tok[q] = -1;
            a.w.sorted_route[q] = -1;
            a.w.sorted_exp[q] = e;
            a.w.sorted_w[q] = 0.f;
        }
    }
    __syncthreads();
}

__device__ __forceinline__ float route_weight(const PrepArgs& a, int64_t r) {
    return (a.linear || a.batched) ? 1.f : load_as_float(a.weights, r, a.w_dtype);
}

// Placement of one route per thread: thread tid places route r (local expert
// e, -1 = not local or past r1; weight wgt) at the next free sorted row of
// its expert.  run[e] (shared memory) holds each expert's next row; the lanes
// of a warp that share an expert take one block of rows with a single atomic
// add by their leader.  The order of rows within an expert is not fixed, and
// need not be: every output row is computed from its own input row only (no
// kernel mixes rows), and the combine finds a route's row through route_pos.
// No barrier: rows are claimed atomically.
__device__ __forceinline__ void prep_place_step(const PrepArgs& a, int64_t r, int64_t r1, int64_t Rmax, int e,
                                                float wgt, int* run) {
    const int lane = threadIdx.x & 31;
    const unsigned mask = __match_any_sync(0xffffffffu, e);
    const int leader = __ffs(mask) - 1;
    int base = 0;
    if (e >= 0 && lane == leader) base = atomicAdd(&run[e], __popc(mask));
    base = __shfl_sync(0xffffffffu, base, leader);
    if (e >= 0) {
        const int p = base + __popc(mask & ((1u << lane) - 1u));
        a.w.route_pos[r] = p;
        a.w.sorted_tok[p] = int(r / a.topk);
        a.w.sorted_route[p] = int(r);
        a.w.sorted_exp[p] = e;
        a.w.sorted_w[p] = wgt;
    } else if (r < r1 && r < Rmax) {
        a.w.route_pos[r] = -1;
    }
}

// Placement of routes [r0, r1) within each expert's rows (run[] = first rows).
__device__ void prep_place(const PrepArgs& a, int64_t r0, int64_t r1, int64_t Rmax, int* run) {
    for (int64_t base = r0; base < r1; base += kPrepThreads) {
        const int64_t r = base + threadIdx.x;
        const int e = r < r1 ? local_expert(a, r) : -1;
        prep_place_step(a, r, r1, Rmax, e, e >= 0 ? route_weight(a, r) : 0.f, run);
    }
}

__device__ __forceinline__ int64_t prep_routes(const PrepArgs& a) {
    int64_t T = a.t_max;
    if (a.n_valid) T = min(T, int64_t(max(0, *a.n_valid)));
    return T * a.topk;
}

// Small batches: the whole prep in one CTA.
__global__ void __launch_bounds__(kPrepThreads) prep_kernel(const PrepArgs a) {
    __shared__ int cnt[kMaxLocal];
    __shared__ int poff[kMaxLocal];
    __shared__ int sh32[96];  // block scans of up to three values
    const int tid = threadIdx.x;
    const int E = a.n_local;
    const int64_t R = prep_routes(a), Rmax = a.t_max * a.topk;

    // every route's local expert and weight loaded once, up front (one
    // memory round trip instead of one per 1024-route step and pass)
    constexpr int kPer = int(kPrepSplitRoutes / kPrepThreads);
    int ev[kPer];
    float wv[kPer];
    #pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const int64_t r = int64_t(j) * kPrepThreads + tid;
        ev[j] = r < R ? local_expert(a, r) : -1;
    }
    #pragma unroll
    for (int j = 0; j < kPer; ++j) wv[j] = ev[j] >= 0 ? route_weight(a, int64_t(j) * kPrepThreads + tid) : 0.f;

    for (int i = tid; i < a.cnt1_n; i += kPrepThreads) a.w.cnt1[i] = 0;
    for (int i = tid; i < a.cnt2_n; i += kPrepThreads) a.w.cnt2[i] = 0;
    for (int e = tid; e < E; e += kPrepThreads) cnt[e] = 0;
    __syncthreads();
    #pragma unroll
    for (int j = 0; j < kPer; ++j) {  // warp-aggregated: one add per expert per warp
        const unsigned m = __match_any_sync(0xffffffffu, ev[j]);
        if (ev[j] >= 0 && (threadIdx.x & 31) == __ffs(m) - 1) atomicAdd(&cnt[ev[j]], __popc(m));
    }
    __syncthreads();
    prep_layout(a, cnt, poff, sh32);
    for (int e = tid; e < E; e += kPrepThreads) cnt[e] = poff[e];  // running positions
    __syncthreads();
    #pragma unroll
    for (int j = 0; j < kPer; ++j) {
        if (int64_t(j) * kPrepThreads >= R) break;  // CTA-uniform
        prep_place_step(a, int64_t(j) * kPrepThreads + tid, R, Rmax, ev[j], wv[j], cnt);
    }
    for (int64_t r = R + tid; r < Rmax; r += kPrepThreads) a.w.route_pos[r] = -1;
}

// Large batches: the same prep split over chunks of kPrepChunk routes.
// 1. per-chunk expert histograms hist[chunk][expert]
__global__ void __launch_bounds__(kPrepThreads) prep_count_kernel(const PrepArgs a) {
    __shared__ int cnt[kMaxLocal];
    const int E = a.n_local;
    const int64_t R = prep_routes(a);
    const int64_t r0 = int64_t(blockIdx.x) * kPrepChunk, r1 = min(R, r0 + kPrepChunk);
    for (int e = threadIdx.x; e < E; e += kPrepThreads) cnt[e] = 0;
    __syncthreads();
    prep_histogram(a, r0, r1, cnt);
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += kPrepThreads) a.w.hist[int64_t(blockIdx.x) * E + e] = cnt[e];
}

// 2. one CTA: totals, layout, and each chunk's first row per expert (in place of its histogram)
__global__ void __launch_bounds__(kPrepThreads) prep_plan_kernel(const PrepArgs a, int nchunks) {
    __shared__ int cnt[kMaxLocal];
    __shared__ int poff[kMaxLocal];
    __shared__ int sh32[96];  // block scans of up to three values
    const int tid = threadIdx.x;
    const int E = a.n_local;
    const int64_t R = prep_routes(a), Rmax = a.t_max * a.topk;
    for (int i = tid; i < a.cnt1_n; i += kPrepThreads) a.w.cnt1[i] = 0;
    for (int i = tid; i < a.cnt2_n; i += kPrepThreads) a.w.cnt2[i] = 0;
    for (int e = tid; e < E; e += kPrepThreads) {
        int n = 0;
        for (int c = 0; c < nchunks; ++c) n += a.w.hist[int64_t(c) * E + e];
        cnt[e] = n;
    }
    __syncthreads();
    prep_layout(a, cnt, poff, sh32);
    for (int e = tid; e < E; e += kPrepThreads) {
        int run = poff[e];
        for (int c = 0; c < nchunks; ++c) {
            const int v = a.w.hist[int64_t(c) * E + e];
            a.w.hist[int64_t(c) * E + e] = run;
            run += v;
        }
    }
    for (int64_t r = R + tid; r < Rmax; r += kPrepThreads) a.w.route_pos[r] = -1;
}

// 3. per chunk: placement from the chunk's first rows
__global__ void __launch_bounds__(kPrepThreads) prep_place_kernel(const PrepArgs a) {
    __shared__ int run[kMaxLocal];
    const int E = a.n_local;
    const int64_t R = prep_routes(a), Rmax = a.t_max * a.topk;
    const int64_t r0 = int64_t(blockIdx.x) * kPrepChunk, r1 = min(R, r0 + kPrepChunk);
    for (int e = threadIdx.x; e < E; e += kPrepThreads) run[e] = a.w.hist[int64_t(blockIdx.x) * E + e];
    __syncthreads();
    prep_place(a, r0, r1, Rmax, run);
}

// ---------------------------------------------------------------------------
// 2. input rotation
// ---------------------------------------------------------------------------
struct RotArgs {
    const void* x;
    int x_dtype;
    int in_f;
    int nproj;
    ProjRef proj[2];
    const int* nslots;
    const int4* slots;
    const int* sorted_tok;
    __half* xr;
    int64_t rpad;
    int* status;
    int prerotated;  // x already rotated (fp16): copy into the padded layout only
    int rowmajor;    // GEMM path: [proj][row][in] fp16, no padding
    int dup;         // GEMV path, MCG / 3INST: duplicated layout (dup_pos)
};


// Two consecutive activations (even index) as fp16x2, rounded like the
// reference's cast of the activations to fp16 (exl3.py:2384, 2856).
template <int XDT, bool VEC>
__device__ __forceinline__ uint32_t load_x2_h(const void* x, int64_t i) {
    if constexpr (VEC && XDT == DT_F16)
        return *reinterpret_cast<const uint32_t*>(static_cast<const __half*>(x) + i);
    __half2 h;
    if constexpr (VEC && XDT == DT_BF16) {
        const uint32_t u = *reinterpret_cast<const uint32_t*>(static_cast<const uint16_t*>(x) + i);
        h = __float22half2_rn(__bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u)));
    } else if constexpr (VEC && XDT == DT_F32) {
        h = __float22half2_rn(*reinterpret_cast<const float2*>(static_cast<const float*>(x) + i));
    } else {
        h = __floats2half2_rn(load_as_float(x, i, XDT), load_as_float(x, i + 1, XDT));
    }
    return *reinterpret_cast<const uint32_t*>(&h);
}

// Input rotation on tensor cores: H128 = H8 (x) H16, so one warp rotates 16 sorted
// rows x one 128-block as (a) eight mma.m16n8k16 of the fp16 rows' 16-feature
// blocks against diag(suh_block) H16 (exact +-suh operands, fp32
// accumulation: the strides 1..8 of the transform) and (b) an 8-point
// butterfly across the eight blocks held in each thread's accumulators (the
// strides 16, 32, 64) -- no shuffles.  Rows are grouped 16 at a time from a
// 16-aligned start, so a group never straddles two experts (each expert's
// rows are padded to 16); padding rows enter as zeros and are not stored.
// Output: GEMM path (rowmajor) fp16 [proj][row][in]; GEMV path fp16
// [proj][in/128][row][pitch], each feature stored twice in the dup_pos
// order for MCG / 3INST (dup).  Each warp assembles its 16 x 128 result in a
// shared-memory tile laid out like the destination rows (pitch 136, or 264
// for dup: conflict-free fragment stores) and writes it out with 16-byte
// stores: whole 256-byte rows (rowmajor) or the whole contiguous 16-row slice
// (GEMV layouts), instead of 4-byte stores scattered over 8 rows.  Padding
// rows of a group go out as zeros (their inputs are zero); no kernel reads
// them as data.
__device__ __forceinline__ void rot_store2(__half* row, int f, bool dup, float v0, float v1) {
    if (dup) {
        *reinterpret_cast<__half2*>(row + dup_pos(f)) = __half2half2(__float2half_rn(v0));
        *reinterpret_cast<__half2*>(row + dup_pos(f + 1)) = __half2half2(__float2half_rn(v1));
    } else {
        *reinterpret_cast<__half2*>(row + f) = __floats2half2_rn(v0, v1);
    }
}

enum RotLayout : int { ROT_ROWMAJOR = 0, ROT_PITCH = 1, ROT_DUP = 2 };

// fp16 pitch of a warp's shared-memory output tile
__host__ __device__ constexpr int rot_tile_pitch(int layout) { return layout == ROT_DUP ? kXPitchD : kXPitch; }

template <int XDT, bool VEC, int LAYOUT>
__global__ void __launch_bounds__(256) rotate_rows_mma_kernel(const RotArgs a, const int* __restrict__ sorted_exp) {
    constexpr int SP = rot_tile_pitch(LAYOUT);
    extern __shared__ __align__(16) __half rot_tiles[];
    __half* tile = rot_tiles + (threadIdx.x >> 5) * (16 * SP);
    pdl_launch_dependents();  // the GEMV that follows may start its prologue now
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int nkb = a.in_f / 128;
    const int64_t ngroups = min(int64_t(a.nslots[1]), int64_t(a.rpad)) / 16;
    // H16 signs of this thread's B-fragment entries: rows k in {2t, 2t+1,
    // 2t+8, 2t+9}, columns n = 8j + g
    __half2 hs[2][2];
    #pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int n = 8 * j + g;
        #pragma unroll
        for (int q = 0; q < 2; ++q) {
            const int k = 2 * t + 8 * q;
            hs[j][q] = __floats2half2_rn((__popc(k & n) & 1) ? -1.f : 1.f, (__popc((k + 1) & n) & 1) ? -1.f : 1.f);
        }
    }
    // warp w of CTA b takes items w * gridDim + b, ...: a small batch
    // spreads over every SM instead of filling the first CTAs' warps
    for (int64_t it = int64_t(threadIdx.x >> 5) * gridDim.x + blockIdx.x; it < ngroups * nkb;
         it += (int64_t(gridDim.x) * blockDim.x) >> 5) {
        const int64_t p0 = (it / nkb) * 16;
        const int kb = int(it % nkb);
        const int tok0 = a.sorted_tok[p0 + g], tok1 = a.sorted_tok[p0 + g + 8];
        const int e = sorted_exp[p0];
        uint32_t af[8][4];
        #pragma unroll
        for (int blk = 0; blk < 8; ++blk) {
            const int c = kb * 128 + 16 * blk + 2 * t;
            af[blk][0] = tok0 >= 0 ? load_x2_h<XDT, VEC>(a.x, int64_t(tok0) * a.in_f + c) : 0u;
            af[blk][1] = tok1 >= 0 ? load_x2_h<XDT, VEC>(a.x, int64_t(tok1) * a.in_f + c) : 0u;
            af[blk][2] = tok0 >= 0 ? load_x2_h<XDT, VEC>(a.x, int64_t(tok0) * a.in_f + c + 8) : 0u;
            af[blk][3] = tok1 >= 0 ? load_x2_h<XDT, VEC>(a.x, int64_t(tok1) * a.in_f + c + 8) : 0u;
        }
        constexpr bool dup = LAYOUT == ROT_DUP;
        // rows of the group that carry a route (row g: lane 4g's tok0; row g + 8: its tok1)
        const unsigned v0 = __ballot_sync(0xffffffffu, tok0 >= 0), v1 = __ballot_sync(0xffffffffu, tok1 >= 0);
        // the warp's tile -> output block kb of projection pj: 16-byte stores of
        // the rows in use (padding rows are never read as data)
        auto flush_tile = [&](int pj) {
            __syncwarp();
            if constexpr (LAYOUT == ROT_ROWMAJOR) {
                #pragma unroll 4
                for (int i = lane; i < 16 * 16; i += 32) {
                    const int r = i >> 4, c = (i & 15) * 8;
                    if ((((r < 8 ? v0 : v1) >> (4 * (r & 7))) & 1u) == 0) continue;
                    *reinterpret_cast<uint4*>(a.xr + (int64_t(pj) * a.rpad + p0 + r) * a.in_f + kb * 128 + c) =
                        *reinterpret_cast<const uint4*>(tile + r * SP + c);
                }
            } else {
                constexpr int RC = SP / 8;  // 16-byte chunks per row
                uint4* dst = reinterpret_cast<uint4*>(a.xr + ((int64_t(pj) * nkb + kb) * a.rpad + p0) * SP);
                const uint4* src = reinterpret_cast<const uint4*>(tile);
                #pragma unroll 4
                for (int i = lane; i < 16 * RC; i += 32) {
                    const int r = i / RC;
                    if ((((r < 8 ? v0 : v1) >> (4 * (r & 7))) & 1u) == 0) continue;
                    dst[i] = src[i];
                }
            }
            __syncwarp();
        };
        if (a.prerotated) {
            // input already rotated (the fat GEMM's contract): copy the fp16 rows
            #pragma unroll
            for (int blk = 0; blk < 8; ++blk)
                #pragma unroll
                for (int q = 0; q < 2; ++q) {
                    const int f = 16 * blk + 8 * q + 2 * t;
                    const float2 v0 = __half22float2(*reinterpret_cast<const __half2*>(&af[blk][2 * q]));
                    const float2 v1 = __half22float2(*reinterpret_cast<const __half2*>(&af[blk][2 * q + 1]));
                    rot_store2(tile + g * SP, f, dup, v0.x, v0.y);
                    rot_store2(tile + (g + 8) * SP, f, dup, v1.x, v1.y);
                }
            flush_tile(0);
            continue;
        }
        for (int pj = 0; pj < a.nproj; ++pj) {
            const __half* suh = proj_suh(a.proj[pj], e);
            if (suh == nullptr) {
                if (lane == 0) set_status(a.status, DEV_NULL_PTR);
                continue;
            }
            float d[8][2][4];
            #pragma unroll
            for (int blk = 0; blk < 8; ++blk) {
                const int k0 = kb * 128 + 16 * blk + 2 * t;
                // suh comes from the caller's tables: only 2-byte alignment is guaranteed
                const __half2 s01 = __halves2half2(suh[k0], suh[k0 + 1]);
                const __half2 s89 = __halves2half2(suh[k0 + 8], suh[k0 + 9]);
                #pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const __half2 b0 = __hmul2(s01, hs[j][0]), b1 = __hmul2(s89, hs[j][1]);
                    #pragma unroll
                    for (int i = 0; i < 4; ++i) d[blk][j][i] = 0.f;
                    mma_16816(d[blk][j], af[blk], *reinterpret_cast<const uint32_t*>(&b0),
                              *reinterpret_cast<const uint32_t*>(&b1));
                }
            }
            // strides 16, 32, 64: butterflies across the blocks, fp32
            #pragma unroll
            for (int st = 1; st < 8; st <<= 1)
                #pragma unroll
                for (int blk = 0; blk < 8; ++blk)
                    if ((blk & st) == 0)
                        #pragma unroll
                        for (int j = 0; j < 2; ++j)
                            #pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const float u = d[blk][j][i], v = d[blk + st][j][i];
                                d[blk][j][i] = __fadd_rn(u, v);
                                d[blk + st][j][i] = __fsub_rn(u, v);
                            }
            // D fragment (j, i): row g (i < 2) or g + 8, feature 16 blk + 8 j + 2 t + (i & 1)
            #pragma unroll
            for (int blk = 0; blk < 8; ++blk)
                #pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const int f = 16 * blk + 8 * j + 2 * t;
                    rot_store2(tile + g * SP, f, dup, d[blk][j][0] * kHadNorm, d[blk][j][1] * kHadNorm);
                    rot_store2(tile + (g + 8) * SP, f, dup, d[blk][j][2] * kHadNorm, d[blk][j][3] * kHadNorm);
                }
            flush_tile(pj);
        }
    }
}

template <int XDT, int LAYOUT>
static void launch_rotate_layout(const RotArgs& ra, const int* sorted_exp, int grid, cudaStream_t s) {
    const bool vec = (reinterpret_cast<uintptr_t>(ra.x) & 15) == 0;
    const int smem = 8 * 16 * rot_tile_pitch(LAYOUT) * 2;  // one 16-row tile per warp
    void (*k)(const RotArgs, const int*) = vec ? rotate_rows_mma_kernel<XDT, true, LAYOUT>
                                                : rotate_rows_mma_kernel<XDT, false, LAYOUT>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    k<<<grid, 256, smem, s>>>(ra, sorted_exp);
}

template <int XDT>
static void launch_rotate_rows(const RotArgs& ra, const int* sorted_exp, int grid, cudaStream_t s) {
    if (ra.rowmajor) launch_rotate_layout<XDT, ROT_ROWMAJOR>(ra, sorted_exp, grid, s);
    else if (ra.dup) launch_rotate_layout<XDT, ROT_DUP>(ra, sorted_exp, grid, s);
    else launch_rotate_layout<XDT, ROT_PITCH>(ra, sorted_exp, grid, s);
}

// ---------------------------------------------------------------------------
// 3/4. expert GEMV engine
// ---------------------------------------------------------------------------
struct GemvArgs {
    int* status;
    ProjRef proj[2];
    int in_f, out_f, ncb, stages, kmax;
    const int* nslots;
    const int4* slots;
    const __half* xin;
    int64_t rpad;
    // EPI_GATEUP
    ProjRef down;
    __half* a2;
    float limit;
    int act;
    // EPI_DOWN
    const float* sorted_w;
    float* yd;
    // EPI_LINEAR / EPI_ROUTE
    void* y;
    int y_dtype;
    const int* sorted_tok;
    const int* sorted_route;
    const int64_t* scatter_idx;  // EPI_LINEAR: y[scatter_idx[row]] += scatter_w[row] * v
    const __half* scatter_w;
    int64_t t_max;
    int topk;
    // split-K: partial tiles [2 * gridDim.x][kCW][NPROJ * 256], one counter per group
    float* part;
    int* cnt;
};

// Item ring: the producer stages each work item's description and the
// vectors its epilogue needs (svh slices, the down suh slice, per-row route
// data) in shared memory ahead of the consumers, so no consumer waits on a
// global load at an item's start or in its epilogue.  Slot j % kItemRing
// holds item j; the consumers release it after the item's epilogue.
constexpr int kItemRing = 4;
enum ItemField : int { IF_E = 0, IF_P0, IF_ROWS, IF_CB, IF_KT0, IF_KT1, IF_K0, IF_K1, IF_OK0, IF_OK1,
                       IF_SVH0, IF_SVH1, IF_DSUH };
// vector modes: 0 = absent (zeros), 1 = staged in the slot, 2 = read from global memory
struct ItemSlot {
    int info[16];
    __half svh[2][128];
    __half dsuh[128];
    float w[16];
    int tok[16];
    int route[16];
};
static_assert(sizeof(ItemSlot) == 1024, "item slot layout");

struct GemvSmem {
    uint64_t* full;
    uint64_t* empty;
    uint64_t* item_empty;  // [kItemRing]
    int* flags;  // [0] abort, [1] last-of-group
    ItemSlot* items;  // [kItemRing]
    float* ys;   // [NPROJ][16][kYsPitch]
    char* stages;
};

// stage = trellis region (NPROJ x 8 k-tile rows x 8 tiles, packed at each
// projection's own K, capacity kmax) + NPROJ rotated-input slices
__host__ __device__ inline size_t gemv_trellis_bytes(int nproj, int kmax) {
    return size_t(nproj) * kKtPerStage * 256 * kmax;
}
// nx: input slices per stage (one per projection; one for a paired launch,
// whose two column blocks share the input)
__host__ __device__ inline size_t gemv_stage_bytes(int nproj, int kmax, bool dup, int nx) {
    return (gemv_trellis_bytes(nproj, kmax) + size_t(nx) * x_slice(dup) + 127) & ~size_t(127);
}
__host__ __device__ inline size_t gemv_bar_bytes(int stages) {
    return (size_t(stages) * 2 * 8 + kItemRing * 8 + 8 * 4 + 127) & ~size_t(127);
}
__host__ __device__ inline size_t gemv_fixed_bytes(int nproj, int stages) {
    const size_t ys = (size_t(nproj) * 16 * kYsPitch * 4 + 127) & ~size_t(127);
    return gemv_bar_bytes(stages) + kItemRing * sizeof(ItemSlot) + ys;
}

__device__ __forceinline__ GemvSmem gemv_smem(char* base, int nproj, int stages) {
    GemvSmem s;
    s.full = reinterpret_cast<uint64_t*>(base);
    s.empty = s.full + stages;
    s.item_empty = s.empty + stages;
    s.flags = reinterpret_cast<int*>(s.item_empty + kItemRing);
    s.items = reinterpret_cast<ItemSlot*>(base + gemv_bar_bytes(stages));
    s.ys = reinterpret_cast<float*>(base + gemv_bar_bytes(stages) + kItemRing * sizeof(ItemSlot));
    s.stages = base + gemv_fixed_bytes(nproj, stages);
    return s;
}

// Stream-K work split.  The work is the sequence of (group, stage) pairs,
// group g = (slot g / ncb, 128-column block g % ncb) holding NS = in_f / 128
// stages; CTA i takes the stages [i W, (i + 1) W) with W = ceil(total / grid),
// so every CTA gets the same number of stages whatever the batch (no tail
// wave).  A group cut by CTA boundaries becomes pieces, one per CTA: each
// piece writes its fp32 partial tile, and the CTA that completes the group's
// count adds the pieces in stage order (deterministic) and runs the epilogue.
// A CTA cuts at most its first and last group, so the partials take two
// slots per CTA.  Every thread derives the same split from the slot count.
// (Stage counts stay far below 2^31: groups <= slots * out/128.)
struct StreamK {
    int groups, W, NS;
};

__device__ __forceinline__ StreamK gemv_streamk(const GemvArgs& a) {
    StreamK k;
    k.NS = a.in_f / 128;
    k.groups = *a.nslots * a.ncb;
    k.W = (k.groups * k.NS + int(gridDim.x) - 1) / int(gridDim.x);
    return k;
}

// first group of CTA c's range
__device__ __forceinline__ int sk_first_group(const StreamK& k, int c) { return c * k.W / k.NS; }

struct ItemInfo {
    int e, p0, rows, cb, kt0, kt1, group;
};

// the CTA's piece of group g (g inside the CTA's range)
__device__ __forceinline__ ItemInfo gemv_item(const GemvArgs& a, const StreamK& k, int g) {
    ItemInfo I;
    const int c = blockIdx.x;
    const int gs0 = g * k.NS;
    I.kt0 = (max(c * k.W, gs0) - gs0) * kKtPerStage;
    I.kt1 = (min((c + 1) * k.W, gs0 + k.NS) - gs0) * kKtPerStage;
    const int slot = g / a.ncb;
    I.cb = g - slot * a.ncb;
    const int4 sl = a.slots[slot];
    I.e = sl.x;
    I.p0 = sl.y;
    I.rows = sl.z;
    I.group = g;
    return I;
}

// CTAs holding the first and last pieces of group g
__device__ __forceinline__ int sk_cta0(const StreamK& k, int g) { return g * k.NS / k.W; }
__device__ __forceinline__ int sk_cta1(const StreamK& k, int g) { return (g * k.NS + k.NS - 1) / k.W; }
// partial slot of CTA c's piece of group g: its first group or its last
__device__ __forceinline__ int sk_pslot(const StreamK& k, int c, int g) {
    return 2 * c + (g == sk_first_group(k, c) ? 0 : 1);
}

// the CTA's group range [g0, g1)
__device__ __forceinline__ void sk_range(const StreamK& k, int& g0, int& g1) {
    const int c = blockIdx.x;
    const int s0 = c * k.W, s1 = min((c + 1) * k.W, k.groups * k.NS);
    if (s0 >= s1) {
        g0 = g1 = 0;
        return;
    }
    g0 = s0 / k.NS;
    g1 = (s1 - 1) / k.NS + 1;
}

// is projection usable for this expert (pointer present, aligned, K valid)?
__device__ __forceinline__ bool proj_ok(const ProjRef& p, int e, int kmax, int* status, bool report) {
    const int K = proj_k(p, e);
    const uint16_t* t = proj_trellis(p, e);
    if (K < 2 || K > kmax) {
        if (report) set_status(status, DEV_BAD_K);
        return false;
    }
    if (t == nullptr) {
        if (report) set_status(status, DEV_NULL_PTR);
        return false;
    }
    if (reinterpret_cast<uintptr_t>(t) & 15) {
        if (report) set_status(status, DEV_BAD_ALIGN);
        return false;
    }
    return true;
}

__device__ __forceinline__ bool guarded_wait(uint64_t* bar, uint32_t parity, int* status,
                                             volatile int* abort_flag) {
    if (*abort_flag) return false;
    if (mbar_wait(bar, parity, status)) return true;
    *abort_flag = 1;
    return false;
}

// One stage for NP projections that share one K: per k-tile, every
// projection's tile of this warp's 16 columns is decoded (independent chains
// for the scheduler) and multiplied by the 16-row input slice.
//   tiles: trellis region of the stage + this warp's tile offset (uint32 words)
//   xs:    per-lane ldmatrix address of projection 0's input slice
// SHX: every "projection" reads the same input slice (a paired launch: two
// column blocks of one projection)
template <int K, int CB, int NP, bool SHX = false>
__device__ __forceinline__ void stage_mma(const uint32_t* __restrict__ tiles, uint32_t xs, int lane,
                                          bool two, float (&acc)[NP][2][4]) {
    constexpr int ROW = 64 * K;                // words per k-tile row (8 tiles of 8K words)
    constexpr int REGION = kKtPerStage * ROW;  // words per projection region
    if constexpr (CB != CB_MUL1) {
        // unsummed {lo, hi} words against the duplicated activations: two
        // k16 MMAs per k-tile (k-pairs of j = 0,1,4,5 then j = 2,3,6,7)
        #pragma unroll
        for (int kk = 0; kk < kKtPerStage; ++kk) {
            uint32_t h[NP][8];
            #pragma unroll
            for (int p = 0; p < NP; ++p) decode_tile_words<K, CB>(tiles + p * REGION + kk * ROW, lane, h[p]);
            #pragma unroll
            for (int p = 0; p < NP; ++p) {
                uint32_t b[4], c[4];
                ldmatrix_x4(b, xs + (SHX ? 0 : p * kXSliceD) + kk * 64);
                ldmatrix_x4(c, xs + (SHX ? 0 : p * kXSliceD) + kk * 64 + 32);
                const uint32_t a0[4] = {h[p][0], h[p][4], h[p][1], h[p][5]};
                const uint32_t a1[4] = {h[p][2], h[p][6], h[p][3], h[p][7]};
                mma_16816(acc[p][0], a0, b[0], b[1]);
                mma_16816(acc[p][0], a1, c[0], c[1]);
                if (two) {
                    mma_16816(acc[p][1], a0, b[2], b[3]);
                    mma_16816(acc[p][1], a1, c[2], c[3]);
                }
            }
        }
    } else {
        #pragma unroll
        for (int kk = 0; kk < kKtPerStage; ++kk) {
            uint32_t af[NP][4];
            #pragma unroll
            for (int p = 0; p < NP; ++p) decode_tile_afrag<K, CB>(tiles + p * REGION + kk * ROW, lane, af[p]);
            #pragma unroll
            for (int p = 0; p < NP; ++p) {
                uint32_t b[4];
                ldmatrix_x4(b, xs + (SHX ? 0 : p * kXSlice) + kk * 32);
                mma_16816(acc[p][0], af[p], b[0], b[1]);
                if (two) mma_16816(acc[p][1], af[p], b[2], b[3]);
            }
        }
    }
}

template <int CB, int NP>
__device__ __forceinline__ void stage_mma_k(int K, const uint32_t* tiles, uint32_t xs, int lane, bool two,
                                            float (&acc)[NP][2][4]) {
    switch (K) {
        case 2: stage_mma<2, CB, NP>(tiles, xs, lane, two, acc); break;
        case 3: stage_mma<3, CB, NP>(tiles, xs, lane, two, acc); break;
        case 4: stage_mma<4, CB, NP>(tiles, xs, lane, two, acc); break;
        case 5: stage_mma<5, CB, NP>(tiles, xs, lane, two, acc); break;
        case 6: stage_mma<6, CB, NP>(tiles, xs, lane, two, acc); break;
        case 7: stage_mma<7, CB, NP>(tiles, xs, lane, two, acc); break;
        case 8: stage_mma<8, CB, NP>(tiles, xs, lane, two, acc); break;
        default: break;
    }
}

// A work item's stages when every projection has bit width K (the usual
// case); advances the ring position (s, ph).
template <int K, int CB, int NP, bool SHX>
__device__ __forceinline__ void gemv_same_k_loop(const GemvSmem& sm, int S, size_t stage_bytes, size_t xs_off,
                                                 uint32_t xs_lane, int cw, int kt0, int kt1, int& s, uint32_t& ph,
                                                 bool two, float (&acc)[NP][2][4], int* status,
                                                 volatile int* abort_flag, int lane) {
    for (int kt = kt0; kt < kt1; kt += kKtPerStage, ring_next(s, ph, S)) {
        if (guarded_wait(&sm.full[s], ph, status, abort_flag)) {
            const char* st = sm.stages + size_t(s) * stage_bytes;
            const uint32_t xs = smem_u32(st + xs_off) + xs_lane;
            stage_mma<K, CB, NP, SHX>(reinterpret_cast<const uint32_t*>(st) + cw * 8 * K, xs, lane, two, acc);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.empty[s]);
    }
}

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

template <int NPROJ, int EPI, int CB>
__global__ void __launch_bounds__(kGemvThreads, 2)
gemv_kernel(const __grid_constant__ GemvArgs a) {
    constexpr int NCT = kCW * 32;
    extern __shared__ __align__(128) char smem_raw[];
    pdl_launch_dependents();  // the next kernel may be scheduled as this one's CTAs retire
    constexpr bool DUP = CB != CB_MUL1;  // duplicated activation layout
    constexpr int XP = x_pitch(DUP), XS = x_slice(DUP);
    // paired launch (every single-projection epilogue): "projections" 0 and 1
    // are column blocks 2cb and 2cb + 1 of one projection; they share the
    // input slice, so a stage carries 16 tiles per warp on one slice, as
    // gate/up does
    constexpr bool PAIRED = EPI != EPI_GATEUP && NPROJ == 2;
    constexpr int NX = PAIRED ? 1 : NPROJ;
    const int S = a.stages;
    GemvSmem sm = gemv_smem(smem_raw, NPROJ, S);
    const size_t stage_bytes = gemv_stage_bytes(NPROJ, a.kmax, DUP, NX);
    const size_t xs_off = gemv_trellis_bytes(NPROJ, a.kmax);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    volatile int* abort_flag = sm.flags;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], kCW);
        }
        for (int j = 0; j < kItemRing; ++j) mbar_init(&sm.item_empty[j], 1);
        sm.flags[0] = 0;
        sm.flags[1] = 0;
        mbar_fence_init();
    }
    __syncthreads();

    const StreamK sk = gemv_streamk(a);
    int g0, g1;
    sk_range(sk, g0, g1);
    const int nkb = a.in_f / 128;
    const int ntiles_out = a.out_f / 16;

    if (warp == kCW) {
        // ------------------------------ producer ------------------------------
        if (lane != 0) return;
        bool pred_done = false;  // griddepcontrol.wait issued
        uint32_t q = 0;   // stages issued
        int ps = 0;       // ring slot and parity of stage q
        uint32_t pph = 0u;
        int ji = 0;  // item ring slot and parity
        uint32_t jph = 0u;
        for (int g = g0; g < g1 && !*abort_flag; ++g, ring_next(ji, jph, kItemRing)) {
            const ItemInfo I = gemv_item(a, sk, g);
            bool ok[NPROJ];
            int Kp[NPROJ];
            const uint16_t* tp[NPROJ];
            #pragma unroll
            for (int p = 0; p < NPROJ; ++p) {
                const ProjRef& pr = a.proj[PAIRED ? 0 : p];
                ok[p] = proj_ok(pr, I.e, a.kmax, a.status, p == 0 || !PAIRED);
                Kp[p] = proj_k(pr, I.e);
                tp[p] = proj_trellis(pr, I.e);
            }
            // output column block of "projection" p
            auto pcb = [&](int p) { return PAIRED ? 2 * I.cb + p : I.cb; };
            // the item's slot (free once the consumers finished item j - kItemRing)
            if (!guarded_wait(&sm.item_empty[ji], jph ^ 1u, a.status, abort_flag)) break;
            ItemSlot& is = sm.items[ji];
            is.info[IF_E] = I.e;
            is.info[IF_P0] = I.p0;
            is.info[IF_ROWS] = I.rows;
            is.info[IF_CB] = I.cb;
            is.info[IF_KT0] = I.kt0;
            is.info[IF_KT1] = I.kt1;
            #pragma unroll
            for (int p = 0; p < NPROJ; ++p) {
                is.info[IF_K0 + p] = Kp[p];
                is.info[IF_OK0 + p] = ok[p] ? 1 : 0;
            }
            // the item's vectors ride on its first stage's barrier
            const __half* vsrc[3] = {nullptr, nullptr, nullptr};
            void* vdst[3] = {is.svh[0], is.svh[1], is.dsuh};
            #pragma unroll
            for (int p = 0; p < NPROJ; ++p) vsrc[p] = proj_svh(a.proj[PAIRED ? 0 : p], I.e);
            if (EPI == EPI_GATEUP) vsrc[2] = proj_suh(a.down, I.e);
            uint32_t vbytes = 0;
            #pragma unroll
            for (int v = 0; v < 3; ++v) {
                if (v >= NPROJ && v < 2) continue;
                if (v == 2 && EPI != EPI_GATEUP) continue;
                int mode = 0;
                if (vsrc[v]) {
                    vsrc[v] += size_t(v < 2 ? pcb(v) : I.cb) * 128;
                    mode = (reinterpret_cast<uintptr_t>(vsrc[v]) & 15) ? 2 : 1;
                    if (mode == 1) vbytes += 256;
                }
                is.info[IF_SVH0 + v] = mode;
            }
            const void* rsrc = EPI == EPI_DOWN ? static_cast<const void*>(a.sorted_w + I.p0)
                             : EPI == EPI_LINEAR ? static_cast<const void*>(a.sorted_tok + I.p0)
                                                 : static_cast<const void*>(a.sorted_route + I.p0);
            void* rdst = EPI == EPI_DOWN ? static_cast<void*>(is.w)
                       : EPI == EPI_LINEAR ? static_cast<void*>(is.tok) : static_cast<void*>(is.route);
            const bool rows_v = EPI != EPI_GATEUP;
            if (rows_v) vbytes += 64;
            bool first_stage = true;
            for (int kt = I.kt0; kt < I.kt1; kt += kKtPerStage, ++q, ring_next(ps, pph, S)) {
                const int s = ps;
                if (!guarded_wait(&sm.empty[s], pph ^ 1u, a.status, abort_flag)) break;
                char* st = sm.stages + size_t(s) * stage_bytes;
                uint32_t bytes = NX * XS;
                if (first_stage) bytes += vbytes;
                #pragma unroll
                for (int p = 0; p < NPROJ; ++p)
                    if (ok[p]) bytes += kKtPerStage * 256 * Kp[p];
                mbar_arrive_expect_tx(&sm.full[s], bytes);
                size_t region = 0;
                #pragma unroll
                for (int p = 0; p < NPROJ; ++p) {
                    const int rowb = 256 * Kp[p];  // bytes of 8 tiles
                    if (ok[p]) {
                        const int tw = 16 * Kp[p];  // int16 per tile
                        for (int kk = 0; kk < kKtPerStage; ++kk) {
                            const uint16_t* src = tp[p] + (int64_t(kt + kk) * ntiles_out + int64_t(pcb(p)) * 8) * tw;
                            bulk_g2s(st + region + size_t(kk) * rowb, src, uint32_t(rowb), &sm.full[s]);
                        }
                    }
                    region += size_t(kKtPerStage) * (ok[p] ? rowb : 0);
                }
                const int kb = kt / kKtPerStage;
                // the inputs are the previous kernel's output (rotation, or
                // the gate/up epilogue): with a programmatic launch, the
                // routing tables, the item's metadata and this first stage's
                // trellis rows were fetched while that kernel was running
                if (!pred_done) {
                    pdl_wait();
                    pred_done = true;
                }
                #pragma unroll
                for (int p = 0; p < NX; ++p) {
                    const __half* src = a.xin + ((int64_t(p) * nkb + kb) * a.rpad + I.p0) * XP;
                    bulk_g2s(st + xs_off + size_t(p) * XS, src, uint32_t(XS), &sm.full[s]);
                }
                if (first_stage) {
                    #pragma unroll
                    for (int v = 0; v < 3; ++v)
                        if (is.info[IF_SVH0 + v] == 1 && (v < NPROJ || (v == 2 && EPI == EPI_GATEUP)))
                            bulk_g2s(vdst[v], vsrc[v], 256u, &sm.full[s]);
                    if (rows_v) bulk_g2s(rdst, rsrc, 64u, &sm.full[s]);
                    first_stage = false;
                }
            }
        }
        // drain: every issued stage must land before the CTA exits (the
        // consumers may have stopped early on an abort)
        const uint32_t first = q > uint32_t(S) ? q - uint32_t(S) : 0u;
        for (uint32_t r = first; r < q; ++r) {
            const int s = int(r % uint32_t(S));
            mbar_wait(&sm.full[s], (r / uint32_t(S)) & 1u, a.status);
        }
        return;
    }

    // ------------------------------ consumers ------------------------------
    // every consumer read and write comes after the previous kernel ends
    pdl_wait();
    const int cw = warp;  // 16-column tile of the 128-column block
    // per-lane ldmatrix row address inside an input slice (rows padded to 272 B)
    const int brow = (lane & 7) + ((lane >> 4) << 3);
    const uint32_t xs_lane = uint32_t(brow * XP * 2 + ((lane >> 3) & 1) * 16);
    int cs = 0;  // ring slot and parity of the next stage
    uint32_t cph = 0u;
    int ji = 0;  // item ring slot
    uint32_t jph = 0u;
    for (int g = g0; g < g1; ++g, ring_next(ji, jph, kItemRing)) {
        // the item's first stage has landed: its slot is filled
        if (!guarded_wait(&sm.full[cs], cph, a.status, abort_flag)) break;
        const ItemSlot& is = sm.items[ji];
        ItemInfo I;
        I.e = is.info[IF_E];
        I.p0 = is.info[IF_P0];
        I.rows = is.info[IF_ROWS];
        I.cb = is.info[IF_CB];
        I.kt0 = is.info[IF_KT0];
        I.kt1 = is.info[IF_KT1];
        I.group = g;
        bool ok[NPROJ];
        int Kp[NPROJ];
        #pragma unroll
        for (int p = 0; p < NPROJ; ++p) {
            ok[p] = is.info[IF_OK0 + p] != 0;
            Kp[p] = is.info[IF_K0 + p];
        }
        bool same = ok[0];
        #pragma unroll
        for (int p = 1; p < NPROJ; ++p) same = same && ok[p] && Kp[p] == Kp[0];
        const bool two = I.rows > 8;
        float acc[NPROJ][2][4];
        #pragma unroll
        for (int p = 0; p < NPROJ; ++p)
            #pragma unroll
            for (int i = 0; i < 8; ++i) acc[p][i >> 2][i & 3] = 0.f;
        // the common case (every projection at one K) runs a loop specialised
        // for that K: the switch on K happens once per item, not per stage
        #define EXL3_GEMV_SAME(KK)                                                                           \
            gemv_same_k_loop<KK, CB, NPROJ, PAIRED>(sm, S, stage_bytes, xs_off, xs_lane, cw, I.kt0, I.kt1, cs, cph, two, \
                                            acc, a.status, abort_flag, lane)
        if (same) {
            switch (Kp[0]) {
                case 2: EXL3_GEMV_SAME(2); break;
                case 3: EXL3_GEMV_SAME(3); break;
                case 4: EXL3_GEMV_SAME(4); break;
                case 5: EXL3_GEMV_SAME(5); break;
                case 6: EXL3_GEMV_SAME(6); break;
                case 7: EXL3_GEMV_SAME(7); break;
                default: EXL3_GEMV_SAME(8); break;
            }
        }
        #undef EXL3_GEMV_SAME
        for (int kt = I.kt0; !same && kt < I.kt1; kt += kKtPerStage, ring_next(cs, cph, S)) {
            const int s = cs;
            const bool landed = guarded_wait(&sm.full[s], cph, a.status, abort_flag);
            if (landed) {
                const char* st = sm.stages + size_t(s) * stage_bytes;
                const uint32_t xs = smem_u32(st + xs_off) + xs_lane;
                {
                    size_t region = 0;
                    #pragma unroll
                    for (int p = 0; p < NPROJ; ++p) {
                        if (ok[p]) {
                            const uint32_t* tiles =
                                reinterpret_cast<const uint32_t*>(st + region) + cw * 8 * Kp[p];
                            float (&accp)[1][2][4] = *reinterpret_cast<float (*)[1][2][4]>(&acc[p]);
                            stage_mma_k<CB, 1>(Kp[p], tiles, xs + (PAIRED ? 0 : p * XS), lane, two, accp);
                            region += size_t(kKtPerStage) * 256 * Kp[p];
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.empty[s]);
        }

        // ---- split group: the CTA completing it adds the pieces in stage order
        const int c0 = sk_cta0(sk, g), c1 = sk_cta1(sk, g);
        if (c0 != c1) {
            float* pp = a.part + (int64_t(sk_pslot(sk, blockIdx.x, g)) * kCW + cw) * (NPROJ * 256);
            #pragma unroll
            for (int p = 0; p < NPROJ; ++p)
                #pragma unroll
                for (int i = 0; i < 8; ++i) __stcg(pp + (p * 8 + i) * 32 + lane, acc[p][i >> 2][i & 3]);
            // publish the piece: the CTA barrier orders every thread's partial
            // stores before thread 0's acquire-release add on the group's
            // counter (one gpu-scope operation per piece instead of a fence in
            // every thread); the CTA that completes the count reads the other
            // pieces after the barrier that follows its acquire
            named_bar_sync(1, NCT);
            if (threadIdx.x == 0) {
                int old;
                asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;"
                             : "=r"(old)
                             : "l"(a.cnt + I.group)
                             : "memory");
                const int last = old == c1 - c0;
                if (last) a.cnt[I.group] = 0;
                sm.flags[1] = last;
            }
            named_bar_sync(1, NCT);
            if (!sm.flags[1]) {
                if (threadIdx.x == 0) mbar_arrive(&sm.item_empty[ji]);
                continue;
            }
            #pragma unroll
            for (int p = 0; p < NPROJ; ++p)
                #pragma unroll
                for (int i = 0; i < 8; ++i) acc[p][i >> 2][i & 3] = 0.f;
            for (int c = c0; c <= c1; ++c) {
                const float* rp = a.part + (int64_t(sk_pslot(sk, c, g)) * kCW + cw) * (NPROJ * 256);
                #pragma unroll
                for (int p = 0; p < NPROJ; ++p)
                    #pragma unroll
                    for (int i = 0; i < 8; ++i) acc[p][i >> 2][i & 3] += __ldcg(rp + (p * 8 + i) * 32 + lane);
            }
        }

        // ---- fragments -> [proj][token row][column] tile
        #pragma unroll
        for (int p = 0; p < NPROJ; ++p) {
            float* ys = sm.ys + p * 16 * kYsPitch;
            #pragma unroll
            for (int nb = 0; nb < 2; ++nb)
                #pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int m = cw * 16 + (lane >> 2) + 8 * (i >> 1);
                    const int n = nb * 8 + 2 * (lane & 3) + (i & 1);
                    ys[n * kYsPitch + m] = acc[p][nb][i];
                }
        }
        named_bar_sync(1, NCT);

        // ---- output rotation o svh
        for (int v = cw; v < NPROJ * I.rows; v += kCW) {
            const int p = v / I.rows, r = v % I.rows;
            float* row = sm.ys + (p * 16 + r) * kYsPitch;
            float x[4];
            #pragma unroll
            for (int i = 0; i < 4; ++i) x[i] = row[lane + 32 * i];
            fwht128_warp(x, lane);
            const int vm = is.info[IF_SVH0 + p];
            const __half* svh = vm == 1   ? is.svh[p]
                                : vm == 2 ? proj_svh(a.proj[PAIRED ? 0 : p], I.e) + (PAIRED ? 2 * I.cb + p : I.cb) * 128
                                          : nullptr;
            #pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float sv = svh ? __half2float(svh[lane + 32 * i]) : 0.f;
                row[lane + 32 * i] = x[i] * kHadNorm * sv;
            }
        }
        named_bar_sync(1, NCT);

        if constexpr (EPI == EPI_GATEUP) {
            // NPROJ == 2: gate (row block 0) and up (block 1); NPROJ == 1: the
            // up projection alone (non-gated relu^2)
            const int dm = is.info[IF_DSUH];
            const __half* dsuh = dm == 1 ? is.dsuh : dm == 2 ? proj_suh(a.down, I.e) + I.cb * 128 : nullptr;
            for (int r = cw; r < I.rows; r += kCW) {
                const float* gr = sm.ys + r * kYsPitch;
                const float* ur = sm.ys + ((NPROJ - 1) * 16 + r) * kYsPitch;
                float x[4];
                #pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int c = lane + 32 * i;
                    float g = gr[c], u = ur[c];
                    if (a.limit > 0.f) {
                        g = fminf(g, a.limit);
                        u = fminf(fmaxf(u, -a.limit), a.limit);
                    }
                    float act;
                    if (NPROJ == 1) {
                        const float rl = fmaxf(u, 0.f);
                        act = rl * rl;
                    } else if (a.act == ACT_SWIGLU_OAI) {
                        act = (u + 1.0f) * g / (1.0f + expf(-1.702f * g));
                    } else {
                        act = silu_f(g) * u;
                    }
                    const float h = __half2float(__float2half_rn(act));  // the reference's act.half()
                    x[i] = h * (dsuh ? __half2float(dsuh[c]) : 0.f);
                }
                fwht128_warp(x, lane);
                const int64_t p = I.p0 + r;
                __half* dst = a.a2 + (int64_t(I.cb) * a.rpad + p) * XP;
                if constexpr (DUP) {
                    #pragma unroll
                    for (int i = 0; i < 4; ++i)
                        *reinterpret_cast<__half2*>(dst + dup_pos(lane + 32 * i)) =
                            __half2half2(__float2half_rn(x[i] * kHadNorm));
                } else {
                    #pragma unroll
                    for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = __float2half_rn(x[i] * kHadNorm);
                }
            }
        } else if constexpr (EPI == EPI_DOWN) {
            for (int v = cw; v < NPROJ * I.rows; v += kCW) {
                const int pj = v / I.rows, r = v - pj * I.rows;
                const float* row = sm.ys + (pj * 16 + r) * kYsPitch;
                const int64_t p = I.p0 + r;
                const float w = is.w[r];
                float* dst = a.yd + p * a.out_f + (PAIRED ? 2 * I.cb + pj : I.cb) * 128;
                #pragma unroll
                for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = row[lane + 32 * i] * w;
            }
        } else if constexpr (EPI == EPI_LINEAR) {
            for (int v = cw; v < NPROJ * I.rows; v += kCW) {
                const int pj = v / I.rows, r = v - pj * I.rows;
                const float* row = sm.ys + (pj * 16 + r) * kYsPitch;
                const int col0 = (PAIRED ? 2 * I.cb + pj : I.cb) * 128;
                const int tok = is.tok[r];
                if (tok < 0) continue;
                if (a.scatter_idx) {
                    // one route per destination row per call: plain read-modify-write
                    float* dst = static_cast<float*>(a.y) + a.scatter_idx[tok] * a.out_f + col0;
                    const float w = __half2float(a.scatter_w[tok]);
                    #pragma unroll
                    for (int i = 0; i < 4; ++i) dst[lane + 32 * i] += w * row[lane + 32 * i];
                    continue;
                }
                #pragma unroll
                for (int i = 0; i < 4; ++i)
                    store_from_float(a.y, int64_t(tok) * a.out_f + col0 + lane + 32 * i, a.y_dtype,
                                     row[lane + 32 * i]);
            }
        } else {
            // EPI_ROUTE: route r = t * topk + j -> output row j * t_max + t
            for (int v = cw; v < NPROJ * I.rows; v += kCW) {
                const int pj = v / I.rows, r = v - pj * I.rows;
                const float* row = sm.ys + (pj * 16 + r) * kYsPitch;
                const int col0 = (PAIRED ? 2 * I.cb + pj : I.cb) * 128;
                const int rt = is.route[r];
                if (rt < 0) continue;
                const int64_t orow = int64_t(rt % a.topk) * a.t_max + rt / a.topk;
                #pragma unroll
                for (int i = 0; i < 4; ++i)
                    store_from_float(a.y, orow * a.out_f + col0 + lane + 32 * i, a.y_dtype, row[lane + 32 * i]);
            }
        }
        named_bar_sync(1, NCT);
        if (threadIdx.x == 0) mbar_arrive(&sm.item_empty[ji]);
    }
}

// ---------------------------------------------------------------------------
// 5. deterministic combine
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
combine_kernel(const int* __restrict__ route_pos, const float* __restrict__ yd, int64_t t_max, int topk,
               int hidden, const int32_t* n_valid, void* out, int out_dtype) {
    pdl_wait();  // the per-route rows come from the kernel before
    int64_t T = t_max;
    if (n_valid) T = min(T, int64_t(max(0, *n_valid)));
    const int h4 = hidden / 4;
    const int64_t total = t_max * h4;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t t = i / h4;
        const int c = int(i % h4) * 4;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        if (t < T) {
            // eight routes at a time: their row indices, then their rows, are
            // loaded together (two memory round trips per eight routes, not
            // two per route); the sum still runs in top-k order
            for (int k0 = 0; k0 < topk; k0 += 8) {
                int pos[8];
                #pragma unroll
                for (int u = 0; u < 8; ++u) pos[u] = k0 + u < topk ? route_pos[t * topk + k0 + u] : -1;
                float4 v[8];
                #pragma unroll
                for (int u = 0; u < 8; ++u)
                    v[u] = pos[u] >= 0 ? *reinterpret_cast<const float4*>(yd + int64_t(pos[u]) * hidden + c)
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
                #pragma unroll
                for (int u = 0; u < 8; ++u) {
                    if (pos[u] < 0) continue;
                    acc.x += v[u].x;
                    acc.y += v[u].y;
                    acc.z += v[u].z;
                    acc.w += v[u].w;
                }
            }
        }
        const int64_t o = t * hidden + c;
        store_from_float(out, o + 0, out_dtype, acc.x);
        store_from_float(out, o + 1, out_dtype, acc.y);
        store_from_float(out, o + 2, out_dtype, acc.z);
        store_from_float(out, o + 3, out_dtype, acc.w);
    }
}

// ---------------------------------------------------------------------------
// host: planning and launch
// ---------------------------------------------------------------------------
static constexpr size_t kSmemPerSm = 228 * 1024;
static constexpr int kCtasPerSm = 2;

static void pick_stages(int nproj, int kmax, bool dup, int nx, int& stages, size_t& smem) {
    const size_t per_cta = kSmemPerSm / kCtasPerSm - 1024;
    const size_t sb = gemv_stage_bytes(nproj, kmax, dup, nx);
    int s = 8;
    while (s > 2 && gemv_fixed_bytes(nproj, s) + size_t(s) * sb > per_cta) --s;
    stages = s;
    smem = gemv_fixed_bytes(nproj, s) + size_t(s) * sb;
}

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

bool plan_moe(MoePlan& p, int64_t t_max, int topk, int hidden, int inter, int n_local, int kmax,
              bool linear, int num_sms, bool allow_gemm, int cb) {
    if (t_max < 1 || topk < 1 || hidden < 128 || hidden % 128 || n_local < 1 || n_local > kMaxLocal)
        return false;
    if (inter < 128 || inter % 128) return false;
    if (kmax < 2 || kmax > 8) return false;
    p = MoePlan();
    p.t_max = t_max;
    p.topk = topk;
    p.hidden = hidden;  // single projection: in_features
    p.inter = inter;    // single projection: out_features
    p.n_local = n_local;
    p.kmax = kmax;
    p.linear = linear;
    p.routes = t_max * topk;
    const int64_t act_max = std::min<int64_t>(p.routes, n_local);
    p.smax = p.routes / 16 + act_max + 1;
    p.rpad = p.smax * 16;

    const int grid = num_sms * kCtasPerSm;
    p.ncb1 = inter / 128;
    p.dup = cb != CB_MUL1;  // unknown codebook (-1): size for the larger layout
    // single projection: pairs of 128-column blocks per work item when they pair up
    p.pair1 = linear && p.ncb1 % 2 == 0;
    pick_stages(linear && !p.pair1 ? 1 : 2, kmax, p.dup, linear ? 1 : 2, p.stages1, p.smem1);
    p.grid1 = grid;
    if (!linear) {
        p.ncb2 = hidden / 128;
        // down: pairs of 128-column blocks per work item when they pair up
        p.pair2 = p.ncb2 % 2 == 0;
        pick_stages(p.pair2 ? 2 : 1, kmax, p.dup, 1, p.stages2, p.smem2);
        p.grid2 = grid;
    }

    // prefill-sized batches (>= 32 rows per active expert on average) take the
    // tcgen05 GEMM path, which decodes each weight tile once per work tile of
    // 128 rows -- or of 256 rows (two accumulators sharing every decoded
    // tile) once experts average >= 192 rows and two such stages fit
    p.gemm = allow_gemm && p.routes >= 32 * act_max;
    p.tile_m = 128;
    if (p.routes >= 192 * act_max && tc_pick_stages(kmax, 2, p.tc_stages, p.tc_smem)) p.tile_m = 256;
    else tc_pick_stages(kmax, 1, p.tc_stages, p.tc_smem);
    p.t128max = p.routes / p.tile_m + act_max + 1;

    size_t o = 0;
    auto take = [&](size_t bytes) {
        const size_t at = o;
        o = align256(o + bytes);
        return at;
    };
    p.off_status = take(64);
    p.off_nslots = take(64);
    p.off_slots = take(size_t(p.smax) * 16);
    p.off_route_pos = take(size_t(p.routes) * 4);
    p.off_sorted_tok = take(size_t(p.rpad) * 4);
    p.off_sorted_route = take(size_t(p.rpad) * 4);
    p.off_sorted_exp = take(size_t(p.rpad) * 4);
    p.off_sorted_w = take(size_t(p.rpad) * 4);
    const int nproj1 = linear ? 1 : 2;
    p.prep_chunks = p.routes >= kPrepSplitRoutes ? int((p.routes + kPrepChunk - 1) / kPrepChunk) : 0;
    p.off_hist = take(size_t(p.prep_chunks) * n_local * 4);
    p.off_ntiles128 = take(p.gemm ? 64 : 0);
    p.off_tiles128 = take(p.gemm ? size_t(p.t128max) * 16 : 0);
    if (p.gemm) {
        p.off_xr = take(size_t(nproj1) * p.rpad * hidden * 2);
        p.off_g = take(linear ? 0 : size_t(p.rpad) * inter * 4);
        p.off_u = take(0);
        p.off_x2 = take(linear ? 0 : size_t(p.rpad) * inter * 2);
        p.off_yd = take(linear ? 0 : size_t(p.rpad) * hidden * 4);
        p.off_a2 = p.off_part1 = p.off_part2 = take(0);
        // split-K for the fused layer when few (tile, column block) items
        // can exist: fp32 partials per split and one counter per item
        if (!linear) {
            p.tc_split1 = tc_split_ceiling(p.t128max * p.ncb1, hidden, grid);
            p.tc_split2 = tc_split_ceiling(p.t128max * p.ncb2, inter, grid);
        }
        const int64_t items = p.t128max * std::max(p.ncb1, p.ncb2);
        const bool split = p.tc_split1 > 1 || p.tc_split2 > 1;
        const int64_t part_items = std::max(p.t128max * p.ncb1 * p.tc_split1, p.t128max * p.ncb2 * p.tc_split2);
        p.off_tcpart = take(split ? size_t(part_items) * p.tile_m * 128 * 4 : 0);
        p.off_tccnt = p.off_cnt1 = take(split ? size_t(items) * 4 : 0);
        p.off_cnt2 = take(0);
    } else {
        p.off_xr = take(size_t(nproj1) * (hidden / 128) * p.rpad * x_pitch(p.dup) * 2);
        p.off_a2 = take(linear ? 0 : size_t(inter / 128) * p.rpad * x_pitch(p.dup) * 2);
        p.off_yd = take(linear ? 0 : size_t(p.rpad) * hidden * 4);
        // stream-K partial tiles: two per CTA (exl3::gemv_item)
        p.off_part1 = take(size_t(2) * p.grid1 * kCW * (linear && !p.pair1 ? 1 : 2) * 256 * 4);
        p.off_part2 = take(linear ? 0 : size_t(2) * p.grid2 * kCW * (p.pair2 ? 2 : 1) * 256 * 4);
        p.off_cnt1 = take(size_t(p.smax) * p.ncb1 * 4);
        p.off_cnt2 = take(linear ? 0 : size_t(p.smax) * p.ncb2 * 4);
        p.off_g = p.off_u = p.off_x2 = take(0);
    }
    p.total = o;
    return true;
}

// Launch with programmatic stream serialization: the kernel may start while
// the one before it in the stream is still running and orders itself with
// griddepcontrol.wait (gemv_kernel, combine_kernel); captured into a CUDA
// graph as a programmatic edge.
template <typename... P, typename... A>
static cudaError_t launch_programmatic(void (*kern)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                       A&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<A>(args)...);
}

template <int NPROJ, int EPI>
static cudaError_t launch_gemv(int cb, const GemvArgs& g, int grid, size_t smem, cudaStream_t s) {
    void (*kern)(GemvArgs);
    if (cb == CB_MCG) kern = gemv_kernel<NPROJ, EPI, CB_MCG>;
    else if (cb == CB_MUL1) kern = gemv_kernel<NPROJ, EPI, CB_MUL1>;
    else kern = gemv_kernel<NPROJ, EPI, CB_3INST>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    return launch_programmatic(kern, dim3(grid), dim3(kGemvThreads), smem, s, g);
}

// ---------------------------------------------------------------------------
// phase timing for benchmarks (exl3_profile_*): events around each kernel
// phase, preceded by a bounded spin so the host has queued every launch
// before the GPU reaches the first event.  Not thread-safe; benchmark use only.
// ---------------------------------------------------------------------------
struct PhaseProfiler {
    bool on = false;
    long long delay_cycles = 0;
    int dev = -1;
    cudaEvent_t ev[8] = {};
    int n = 0;  // events recorded by the last call
};
static PhaseProfiler g_prof;

__global__ void spin_kernel(long long cycles) {
    const long long t0 = clock64();
    while (clock64() - t0 < cycles) {
    }
}

static void prof_begin(cudaStream_t s) {
    g_prof.n = 0;
    if (!g_prof.on) return;
    int dev = 0;
    cudaGetDevice(&dev);
    if (g_prof.dev != dev) {
        for (auto& e : g_prof.ev)
            if (e) cudaEventDestroy(e);
        for (auto& e : g_prof.ev) cudaEventCreate(&e);
        g_prof.dev = dev;
    }
    if (g_prof.delay_cycles > 0) spin_kernel<<<1, 1, 0, s>>>(g_prof.delay_cycles);
    cudaEventRecord(g_prof.ev[g_prof.n++], s);
}

static void prof_mark(cudaStream_t s) {
    if (g_prof.on && g_prof.n < 8) cudaEventRecord(g_prof.ev[g_prof.n++], s);
}

void profile_enable(bool on, long long delay_cycles) {
    g_prof.on = on;
    g_prof.delay_cycles = delay_cycles < 0 ? 0 : (delay_cycles > 4000000000LL ? 4000000000LL : delay_cycles);
}

int profile_read(float* ms, int max_phases) {
    const int n = g_prof.n - 1;
    if (n <= 0) return 0;
    if (cudaEventSynchronize(g_prof.ev[g_prof.n - 1]) != cudaSuccess) return -1;
    for (int i = 0; i < n && i < max_phases; ++i)
        if (cudaEventElapsedTime(&ms[i], g_prof.ev[i], g_prof.ev[i + 1]) != cudaSuccess) return -1;
    return n;
}

// prefill path: tcgen05 grouped GEMM (tc_gemm.cu) over 128-row expert tiles
static cudaError_t run_moe_gemm(const MoePlan& p, const MoeCall& c, const WsPtrs& w, int nsm, cudaStream_t s) {
    TcArgs t{};
    t.status = w.status;
    t.kmax = p.kmax;
    t.stage_mem = int(p.tc_smem - 1024 - 256);
    t.ntiles = w.ntiles128;
    t.tiles = w.tiles128;
    t.sorted_w = w.sorted_w;
    t.sorted_tok = w.sorted_tok;
    t.scatter_idx = c.scatter_idx;
    t.scatter_w = static_cast<const __half*>(c.scatter_w);
    t.ctas = nsm * kCtasPerSm;
    t.part = w.tcpart;
    t.cnt = w.cnt1;
    cudaError_t e;
    if (p.linear) {
        if (c.batched) return cudaErrorNotSupported;  // callers route batched linears to the GEMV path
        t.proj = c.up;
        t.in_f = p.hidden;
        t.out_f = p.inter;
        t.ncb = p.inter / 128;
        t.epi = TC_EPI_LINEAR;
        t.y = c.out;
        t.y_dtype = c.out_dtype;
        e = run_tc_gemm(c.cb, p.tile_m / 128, t, w.xr, p.rpad, p.t128max * t.ncb, p.tc_smem, s);
        prof_mark(s);
        return e;
    }
    // gate and up rows (fp32, after the output rotation o svh)
    t.in_f = p.hidden;
    t.out_f = p.inter;
    t.ncb = p.inter / 128;
    t.epi = TC_EPI_ROWS;
    t.proj = c.gate;
    t.yrows = w.g;
    t.max_split = p.tc_split1;
    const int mt = p.tile_m / 128;
    const bool gateless = c.act == ACT_RELU2;  // no gate projection: its launch is skipped
    if (!gateless &&
        (e = run_tc_gemm(c.cb, mt, t, w.xr, p.rpad, tc_grid(p.t128max * t.ncb, t.max_split, t.ctas), p.tc_smem,
                         s)) != cudaSuccess)
        return e;
    // up, fused with SwiGLU and the down input rotation (reads the gate rows)
    t.proj = c.up;
    t.epi = TC_EPI_UPACT;
    t.g_rows = w.g;
    t.x2 = w.x2;
    t.down = c.down;
    t.limit = c.limit;
    t.act = c.act;
    if ((e = run_tc_gemm(c.cb, mt, t, gateless ? w.xr : w.xr + size_t(p.rpad) * p.hidden, p.rpad,
                         tc_grid(p.t128max * t.ncb, t.max_split, t.ctas), p.tc_smem, s)) != cudaSuccess)
        return e;
    prof_mark(s);
    prof_mark(s);  // the activation phase is part of the up launch
    t.proj = c.down;
    t.in_f = p.inter;
    t.out_f = p.hidden;
    t.ncb = p.hidden / 128;
    t.epi = TC_EPI_DOWN;
    t.yrows = w.yd;
    t.max_split = p.tc_split2;
    if ((e = run_tc_gemm(c.cb, mt, t, w.x2, p.rpad, tc_grid(p.t128max * t.ncb, t.max_split, t.ctas), p.tc_smem, s)) !=
        cudaSuccess)
        return e;
    prof_mark(s);
    const int64_t total = p.t_max * (p.hidden / 4);
    const int64_t blocks = std::min<int64_t>((total + 255) / 256, int64_t(nsm) * 16);
    combine_kernel<<<unsigned(std::max<int64_t>(blocks, 1)), 256, 0, s>>>(
        w.route_pos, w.yd, p.t_max, p.topk, p.hidden, c.n_valid, c.out, c.out_dtype);
    e = cudaGetLastError();
    prof_mark(s);
    return e;
}

cudaError_t run_moe(const MoePlan& p, const MoeCall& c, void* ws, cudaStream_t s) {
    // the GEMV activation layout is fixed by the codebook the plan was made for
    if (!p.gemm && p.dup != (c.cb != CB_MUL1)) return cudaErrorInvalidValue;
    WsPtrs w = ws_ptrs(p, ws);
    if (!p.gemm) {
        w.ntiles128 = nullptr;
        w.tiles128 = nullptr;
    }
    const int nsm = std::max(1, p.grid1 / kCtasPerSm);

    PrepArgs pa;
    pa.ids = c.ids;
    pa.ids_dtype = c.ids_dtype;
    pa.weights = c.weights;
    pa.w_dtype = c.w_dtype;
    pa.expert_map = c.expert_map;
    pa.n_global = c.n_global;
    pa.n_valid = c.n_valid;
    pa.t_max = p.t_max;
    pa.topk = p.topk;
    pa.n_local = p.n_local;
    pa.linear = (p.linear && !c.batched) ? 1 : 0;
    pa.batched = c.batched ? 1 : 0;
    pa.cnt1_n = p.gemm ? ((p.tc_split1 > 1 || p.tc_split2 > 1) ? int(p.t128max * std::max(p.ncb1, p.ncb2)) : 0)
                       : int(p.smax * p.ncb1);
    pa.cnt2_n = (p.linear || p.gemm) ? 0 : int(p.smax * p.ncb2);
    pa.tile_rows = p.tile_m;
    pa.w = w;
    prof_begin(s);
    if (p.prep_chunks > 0) {
        prep_count_kernel<<<p.prep_chunks, kPrepThreads, 0, s>>>(pa);
        prep_plan_kernel<<<1, kPrepThreads, 0, s>>>(pa, p.prep_chunks);
        prep_place_kernel<<<p.prep_chunks, kPrepThreads, 0, s>>>(pa);
    } else {
        prep_kernel<<<1, kPrepThreads, 0, s>>>(pa);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    prof_mark(s);

    // non-gated relu^2: only the up projection exists (the gate tables are not read)
    const bool gateless = !p.linear && c.act == ACT_RELU2;
    RotArgs ra;
    ra.x = c.x;
    ra.x_dtype = c.x_dtype;
    ra.in_f = p.hidden;
    ra.nproj = (p.linear || gateless) ? 1 : 2;
    ra.proj[0] = (p.linear || gateless) ? c.up : c.gate;
    ra.proj[1] = c.up;
    ra.nslots = w.nslots;
    ra.slots = w.slots;
    ra.sorted_tok = w.sorted_tok;
    ra.xr = w.xr;
    ra.rpad = p.rpad;
    ra.status = w.status;
    ra.prerotated = c.prerotated ? 1 : 0;
    ra.rowmajor = p.gemm ? 1 : 0;
    ra.dup = p.dup ? 1 : 0;
    // one resident wave (two 256-thread CTAs per SM at <= 128 registers);
    // the warps loop over the (16-row group, 128-column block) items
    if (c.x_dtype == DT_F32) launch_rotate_rows<DT_F32>(ra, w.sorted_exp, nsm * 2, s);
    else if (c.x_dtype == DT_F16) launch_rotate_rows<DT_F16>(ra, w.sorted_exp, nsm * 2, s);
    else launch_rotate_rows<DT_BF16>(ra, w.sorted_exp, nsm * 2, s);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    prof_mark(s);
    if (p.gemm) return run_moe_gemm(p, c, w, nsm, s);

    GemvArgs g;
    g.status = w.status;
    g.nslots = w.nslots;
    g.slots = w.slots;
    g.rpad = p.rpad;
    g.kmax = p.kmax;
    g.sorted_tok = w.sorted_tok;
    g.sorted_route = w.sorted_route;
    g.sorted_w = w.sorted_w;
    g.scatter_idx = c.scatter_idx;
    g.scatter_w = static_cast<const __half*>(c.scatter_w);
    g.t_max = p.t_max;
    g.topk = p.topk;
    if (p.linear) {
        g.proj[0] = c.up;
        g.in_f = p.hidden;
        g.out_f = p.inter;
        g.ncb = p.pair1 ? p.ncb1 / 2 : p.ncb1;
        g.stages = p.stages1;
        g.xin = w.xr;
        g.y = c.out;
        g.y_dtype = c.out_dtype;
        g.part = w.part1;
        g.cnt = w.cnt1;
        if (p.pair1)
            e = c.batched ? launch_gemv<2, EPI_ROUTE>(c.cb, g, p.grid1, p.smem1, s)
                          : launch_gemv<2, EPI_LINEAR>(c.cb, g, p.grid1, p.smem1, s);
        else
            e = c.batched ? launch_gemv<1, EPI_ROUTE>(c.cb, g, p.grid1, p.smem1, s)
                          : launch_gemv<1, EPI_LINEAR>(c.cb, g, p.grid1, p.smem1, s);
        prof_mark(s);
        return e;
    }

    g.proj[0] = gateless ? c.up : c.gate;
    g.proj[1] = c.up;
    g.in_f = p.hidden;
    g.out_f = p.inter;
    g.ncb = p.ncb1;
    g.stages = p.stages1;
    g.xin = w.xr;
    g.down = c.down;
    g.a2 = w.a2;
    g.limit = c.limit;
    g.act = c.act;
    g.part = w.part1;
    g.cnt = w.cnt1;
    e = gateless ? launch_gemv<1, EPI_GATEUP>(c.cb, g, p.grid1, p.smem1, s)
                 : launch_gemv<2, EPI_GATEUP>(c.cb, g, p.grid1, p.smem1, s);
    if (e != cudaSuccess) return e;
    prof_mark(s);

    GemvArgs d = g;
    d.proj[0] = c.down;
    d.proj[1] = ProjRef();
    d.in_f = p.inter;
    d.out_f = p.hidden;
    d.ncb = p.pair2 ? p.ncb2 / 2 : p.ncb2;
    d.stages = p.stages2;
    d.xin = w.a2;
    d.yd = w.yd;
    d.part = w.part2;
    d.cnt = w.cnt2;
    e = p.pair2 ? launch_gemv<2, EPI_DOWN>(c.cb, d, p.grid2, p.smem2, s)
                : launch_gemv<1, EPI_DOWN>(c.cb, d, p.grid2, p.smem2, s);
    if (e != cudaSuccess) return e;
    prof_mark(s);

    const int64_t total = p.t_max * (p.hidden / 4);
    const int64_t blocks = std::min<int64_t>((total + 255) / 256, int64_t(nsm) * 16);
    e = launch_programmatic(combine_kernel, dim3(unsigned(std::max<int64_t>(blocks, 1))), dim3(256), 0, s,
                            static_cast<const int*>(w.route_pos), static_cast<const float*>(w.yd), p.t_max, p.topk,
                            p.hidden, static_cast<const int32_t*>(c.n_valid), c.out, c.out_dtype);
    prof_mark(s);
    return e;
}

int num_sms_current() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
    return n;
}

}  // namespace exl3
