// ep.cu -- expert-parallel dispatch/combine around the local routed-expert
// forward.
//
// Experts are split into `world` contiguous blocks of n_global/world (rank g
// owns experts [g*epr, (g+1)*epr)), the linear expert_map the reference's
// plugin consumes (src/vllm_exl3/exl3.py:2310-2354, map_topk_to_local at
// :2332).  A token is sent once to every rank that owns at least one of its
// routes (a "pair" (token, rank)); the pair carries the token row plus topk
// (local id, weight) slots, -1 / 0 for routes owned elsewhere, so the
// receiving rank runs the ordinary fused forward on it and returns one
// partial row: the weighted sum of that token's local routes.  The source
// adds its pairs' partial rows in rank order (no float atomics: the sum is
// deterministic).
//
// Send-buffer order is rank-major, token-ascending within a rank, so rank g's
// rows are one contiguous block: packed ([off_g, off_g + count_g), the split
// layout of an all-to-all with per-rank counts) or, given a capacity C >= the
// tokens of any rank, [g*C, g*C + count_g) of fixed C-row blocks whose empty
// slots carry no routes -- an equal-split all-to-all whose sizes never reach
// the host, so a whole step can be captured in a CUDA graph.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "exl3_common.cuh"
#include "exl3_internal.h"

namespace exl3 {
namespace {

constexpr int kEpPlanThreads = 1024;
constexpr int kEpWarps = kEpPlanThreads / 32;

struct EpPlanArgs {
    const void* ids;
    int ids_dtype;
    const void* weights;
    int w_dtype;
    int64_t tokens;
    int topk;
    int64_t n_global;
    int world;
    const int32_t* n_valid;
    int32_t* send_ids;
    float* send_w;
    int32_t* send_tok;
    int32_t* pair_idx;
    int32_t* send_counts;
    int64_t capacity;  // > 0: rank g's pairs start at row g * capacity
};

// A token's routes, loaded together (one memory round trip, not one per
// route): up to kEpRegTopk in registers; wider top-k reads the rest in place.
constexpr int kEpRegTopk = 16;

struct TokenRoutes {
    int32_t id[kEpRegTopk];  // global expert id, -1 if invalid or past topk
};

__device__ __forceinline__ int64_t route_id(const EpPlanArgs& a, const TokenRoutes& r, int64_t t, int k) {
    if (k < kEpRegTopk) return r.id[k];
    const int64_t id = load_id(a.ids, t * a.topk + k, a.ids_dtype);
    return (id >= 0 && id < a.n_global) ? id : -1;
}

__device__ __forceinline__ void load_routes(const EpPlanArgs& a, int64_t t, bool live, TokenRoutes& r) {
    #pragma unroll
    for (int k = 0; k < kEpRegTopk; ++k) {
        const int64_t id = (live && k < a.topk) ? load_id(a.ids, t * a.topk + k, a.ids_dtype) : -1;
        r.id[k] = (id >= 0 && id < a.n_global) ? int32_t(id) : -1;
    }
}

// bit g set <=> a route of token t is owned by rank g (invalid ids own nothing)
__device__ __forceinline__ uint64_t token_ranks(const EpPlanArgs& a, const TokenRoutes& r, int64_t t, int64_t epr) {
    uint64_t m = 0;
    #pragma unroll
    for (int k = 0; k < kEpRegTopk; ++k)
        if (r.id[k] >= 0) m |= uint64_t(1) << int(r.id[k] / epr);
    for (int k = kEpRegTopk; k < a.topk; ++k) {
        const int64_t id = route_id(a, r, t, k);
        if (id >= 0) m |= uint64_t(1) << int(id / epr);
    }
    return m;
}

// One CTA.  Pass 1 counts pairs per rank (warp ballots); pass 2 ranks every
// pair inside its rank's block, chunk by chunk, and writes the pair's meta.
__global__ void __launch_bounds__(kEpPlanThreads) ep_plan_kernel(const EpPlanArgs a) {
    __shared__ int wpos[kEpWarps][kEpMaxWorld];
    __shared__ int run[kEpMaxWorld];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = a.world;
    int64_t T = a.tokens;
    if (a.n_valid) T = min(T, int64_t(max(0, *a.n_valid)));
    const int64_t epr = a.n_global / G;
    const unsigned lt = (1u << lane) - 1u;

    if (tid < G) run[tid] = 0;
    __syncthreads();
    TokenRoutes rt;
    for (int64_t c = 0; c < T; c += kEpPlanThreads) {
        const int64_t t = c + tid;
        load_routes(a, t, t < T, rt);
        const uint64_t m = t < T ? token_ranks(a, rt, t, epr) : 0;
        for (int g = 0; g < G; ++g) {
            const unsigned b = __ballot_sync(0xffffffffu, (m >> g) & 1);
            if (lane == 0 && b) atomicAdd(&run[g], __popc(b));
        }
    }
    __syncthreads();
    if (tid == 0) {
        int s = 0;
        for (int g = 0; g < G; ++g) {
            const int n = run[g];
            a.send_counts[g] = n;
            run[g] = a.capacity > 0 ? int(g * a.capacity) : s;  // position of rank g's next pair
            s += n;
        }
    }
    __syncthreads();
    if (a.capacity > 0) {
        // empty slots of each rank's block: no token, no routes
        for (int g = 0; g < G; ++g) {
            const int64_t n = a.send_counts[g];
            for (int64_t i = n + tid; i < a.capacity; i += kEpPlanThreads) {
                const int64_t slot = g * a.capacity + i;
                a.send_tok[slot] = -1;
                for (int k = 0; k < a.topk; ++k) {
                    a.send_ids[slot * a.topk + k] = -1;
                    a.send_w[slot * a.topk + k] = 0.f;
                }
            }
        }
    }

    for (int64_t c = 0; c < T; c += kEpPlanThreads) {
        const int64_t t = c + tid;
        // a single chunk keeps pass 1's routes; later chunks reload theirs
        if (c > 0 || T > kEpPlanThreads) load_routes(a, t, t < T, rt);
        const uint64_t m = t < T ? token_ranks(a, rt, t, epr) : 0;
        float wr[kEpRegTopk];
        #pragma unroll
        for (int k = 0; k < kEpRegTopk; ++k)
            wr[k] = (m != 0 && k < a.topk) ? load_as_float(a.weights, t * a.topk + k, a.w_dtype) : 0.f;
        for (int g = 0; g < G; ++g) {
            const unsigned b = __ballot_sync(0xffffffffu, (m >> g) & 1);
            if (lane == 0) wpos[warp][g] = __popc(b);
        }
        __syncthreads();
        if (tid < G) {
            int s = run[tid];
            for (int w = 0; w < kEpWarps; ++w) {
                const int v = wpos[w][tid];
                wpos[w][tid] = s;
                s += v;
            }
            run[tid] = s;
        }
        __syncthreads();
        for (int g = 0; g < G; ++g) {
            const bool mine = (m >> g) & 1;
            const unsigned b = __ballot_sync(0xffffffffu, mine);
            if (mine) {
                const int pos = wpos[warp][g] + __popc(b & lt);
                a.pair_idx[t * G + g] = pos;
                a.send_tok[pos] = int32_t(t);
                #pragma unroll
                for (int k = 0; k < kEpRegTopk; ++k) {
                    if (k >= a.topk) break;
                    const int64_t id = rt.id[k];
                    const bool own = id >= 0 && id / epr == g;
                    a.send_ids[int64_t(pos) * a.topk + k] = own ? int32_t(id - g * epr) : -1;
                    a.send_w[int64_t(pos) * a.topk + k] = own ? wr[k] : 0.f;
                }
                for (int k = kEpRegTopk; k < a.topk; ++k) {
                    const int64_t id = route_id(a, rt, t, k);
                    const bool own = id >= 0 && id / epr == g;
                    a.send_ids[int64_t(pos) * a.topk + k] = own ? int32_t(id - g * epr) : -1;
                    a.send_w[int64_t(pos) * a.topk + k] = own ? load_as_float(a.weights, t * a.topk + k, a.w_dtype) : 0.f;
                }
            } else if (t < T) {
                a.pair_idx[t * G + g] = -1;
            }
        }
        __syncthreads();  // wpos is rewritten by the next chunk
    }
    // rows past n_valid own no pairs
    for (int64_t i = T * G + tid; i < a.tokens * G; i += kEpPlanThreads) a.pair_idx[i] = -1;
}

// One warp copies a row of nvec 16-byte vectors, eight vectors per lane
// loaded before any is stored (the source and destination may alias as far
// as the compiler knows, which would otherwise serialise load -> store).
__device__ __forceinline__ void copy_row_warp(uint4* dst, const uint4* src, int64_t nvec, int lane) {
    constexpr int B = 8;
    for (int64_t v0 = lane; v0 < nvec; v0 += 32 * B) {
        uint4 r[B];
        #pragma unroll
        for (int b = 0; b < B; ++b)
            if (v0 + 32 * b < nvec) r[b] = src[v0 + 32 * b];
        #pragma unroll
        for (int b = 0; b < B; ++b)
            if (v0 + 32 * b < nvec) dst[v0 + 32 * b] = r[b];
    }
}

// Copy each pair's token row into the send buffer: warp per pair, 16-byte
// vectors (rows are whole multiples of 256 bytes).
// With a capacity the rows are the world * capacity slots; empty slots
// (send_tok -1) are skipped and keep whatever the buffer held.
__global__ void __launch_bounds__(256) ep_gather_kernel(const uint4* __restrict__ x, int64_t row_vecs,
                                                        const int32_t* __restrict__ send_tok,
                                                        const int32_t* __restrict__ send_counts, int world,
                                                        int64_t capacity, uint4* __restrict__ send_x) {
    __shared__ int64_t total;
    if (threadIdx.x == 0) {
        int64_t s = 0;
        for (int g = 0; g < world; ++g) s += send_counts[g];
        total = capacity > 0 ? world * capacity : s;
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int64_t nw = (int64_t(gridDim.x) * blockDim.x) >> 5;
    for (int64_t p = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; p < total; p += nw) {
        const int tok = send_tok[p];
        if (tok < 0) continue;
        copy_row_warp(send_x + p * row_vecs, x + int64_t(tok) * row_vecs, row_vecs, lane);
    }
}

__device__ __forceinline__ void load4(const void* p, int64_t i, int dt, float (&v)[4]) {
    if (dt == DT_F32) {
        const float4 f = *reinterpret_cast<const float4*>(static_cast<const float*>(p) + i);
        v[0] = f.x, v[1] = f.y, v[2] = f.z, v[3] = f.w;
    } else {
        const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(p) + i);
        if (dt == DT_F16) {
            const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
            const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
            v[0] = a.x, v[1] = a.y, v[2] = b.x, v[3] = b.y;
        } else {
            const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
            const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
            v[0] = a.x, v[1] = a.y, v[2] = b.x, v[3] = b.y;
        }
    }
}

__device__ __forceinline__ void store4(void* p, int64_t i, int dt, const float (&v)[4]) {
    if (dt == DT_F32) {
        *reinterpret_cast<float4*>(static_cast<float*>(p) + i) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
        uint2 u;
        if (dt == DT_F16) {
            const __half2 a = __floats2half2_rn(v[0], v[1]), b = __floats2half2_rn(v[2], v[3]);
            u.x = *reinterpret_cast<const uint32_t*>(&a);
            u.y = *reinterpret_cast<const uint32_t*>(&b);
        } else {
            const __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]), b = __floats2bfloat162_rn(v[2], v[3]);
            u.x = *reinterpret_cast<const uint32_t*>(&a);
            u.y = *reinterpret_cast<const uint32_t*>(&b);
        }
        *reinterpret_cast<uint2*>(static_cast<uint16_t*>(p) + i) = u;
    }
}

// out[t] = sum over ranks g (ascending) of partial[pair_idx[t][g]].  Warp
// per (token, 128-feature chunk), lanes holding 4 consecutive features; the
// ranks' rows are loaded eight at a time before they are added in rank order
// (deterministic, and one memory round trip per eight ranks).  Rows past
// n_valid are zero.
__global__ void __launch_bounds__(256) ep_combine_kernel(const void* __restrict__ partial, int pdt,
                                                         const int32_t* __restrict__ pair_idx, int64_t tokens,
                                                         int world, int hidden, const int32_t* n_valid,
                                                         void* __restrict__ out, int odt, uint32_t* epoch) {
    constexpr int B = 8;
    const int lane = threadIdx.x & 31;
    // NVLink transport: this step is over once the combine runs (every wait
    // that reads the epoch came before it on the stream): advance the epoch
    if (epoch && blockIdx.x == 0 && threadIdx.x == 0) *epoch += 1u;
    int64_t T = tokens;
    if (n_valid) T = min(T, int64_t(max(0, *n_valid)));
    const int nch = hidden / 128;
    const int64_t tasks = tokens * nch;
    const int64_t nw = (int64_t(gridDim.x) * blockDim.x) >> 5;
    for (int64_t task = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; task < tasks; task += nw) {
        const int64_t t = task / nch;
        const int c0 = int(task % nch) * 128 + 4 * lane;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        if (t < T) {
            for (int g0 = 0; g0 < world; g0 += B) {
                int pj[B];
                #pragma unroll
                for (int j = 0; j < B; ++j) pj[j] = g0 + j < world ? pair_idx[t * world + g0 + j] : -1;
                float v[B][4];
                #pragma unroll
                for (int j = 0; j < B; ++j)
                    if (pj[j] >= 0) load4(partial, int64_t(pj[j]) * hidden + c0, pdt, v[j]);
                #pragma unroll
                for (int j = 0; j < B; ++j)
                    if (pj[j] >= 0)
                        #pragma unroll
                        for (int i = 0; i < 4; ++i) acc[i] += v[j][i];
            }
        }
        store4(out, t * hidden + c0, odt, acc);
    }
}

static int combine_grid(int64_t tokens, int hidden) {
    const int64_t tasks = tokens * (hidden / 128);
    return int(std::max<int64_t>(1, std::min<int64_t>((tasks + 7) / 8, int64_t(num_sms_current()) * 8)));
}

// ---------------------------------------------------------------------------
// NVLink transport: every rank owns a window (same geometry everywhere) that
// its peers map through CUDA IPC.  Sources store pair rows straight into the
// owners' windows and raise a per-step flag; owners run the local forward on
// their window and store the partial rows back into the sources' windows.
// A step completes the whole round trip before the next one starts (a
// source's next dispatch follows its combine, which waited for every owner's
// return, which followed that owner's forward), so one buffer per direction
// suffices and every pointer is fixed: a step can be captured in a graph.
// Flags hold the step number (monotonic), read from the window's own epoch.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

struct EpP2pArgs {
    const uint4* x;
    int64_t row_vecs;  // 16-byte vectors per x row
    int world, rank, topk;
    int64_t cap;
    EpWindow L;
    char* window;
    const int64_t* peers;
};

// True in the last CTA of the grid to get here.  The CTA barrier orders
// every thread's earlier stores (peer memory included) before thread 0's
// count, a system-scope acquire-release add: its release half is cumulative,
// so it publishes the whole CTA's stores, and in the last CTA its acquire
// half makes every other CTA's published stores visible to the threads that
// signal after the second barrier.  One fence per CTA, not one per thread.
// The counter (zero on entry) is reset by the last CTA.
__device__ __forceinline__ bool ep_last_cta(int* ctr) {
    __shared__ int s_last;
    __syncthreads();
    if (threadIdx.x == 0) {
        int prev;
        asm volatile("atom.acq_rel.sys.global.add.s32 %0, [%1], 1;" : "=r"(prev) : "l"(ctr) : "memory");
        s_last = prev == int(gridDim.x) - 1;
        if (s_last) *ctr = 0;
    }
    __syncthreads();
    return s_last != 0;
}

// raise this step's flag (arrival or return) in every peer's window; with
// counts, first tell each owner how many pairs it gets from this rank
__device__ __forceinline__ void ep_raise_flags(const EpP2pArgs& a, size_t flag_off, size_t counts_off,
                                               const int32_t* send_counts) {
    const int g = threadIdx.x;
    if (g >= a.world) return;
    const uint32_t epoch = *reinterpret_cast<const uint32_t*>(a.window + kEpCtlEpoch);
    char* dst = reinterpret_cast<char*>(a.peers[g]);
    if (send_counts) reinterpret_cast<volatile int32_t*>(dst + counts_off)[a.rank] = send_counts[g];
    // the release store orders the count above (and, cumulatively, what the
    // CTA acquired in ep_last_cta) before the flag
    st_release_sys(reinterpret_cast<uint32_t*>(dst + flag_off) + a.rank, epoch + 1u);
}

// source: pair slots (g, idx) of the capacity layout -> owner g's window at
// [rank * cap + idx]; empty slots carry ids -1 / weight 0 (rows untouched).
// The last CTA to finish raises the arrival flags.
__global__ void __launch_bounds__(256) ep_p2p_scatter_kernel(const EpP2pArgs a) {
    const int lane = threadIdx.x & 31;
    const int32_t* counts = reinterpret_cast<const int32_t*>(a.window + a.L.send_counts);
    const int32_t* tok = reinterpret_cast<const int32_t*>(a.window + a.L.send_tok);
    const int32_t* sid = reinterpret_cast<const int32_t*>(a.window + a.L.send_ids);
    const float* sw = reinterpret_cast<const float*>(a.window + a.L.send_w);
    const int64_t total = int64_t(a.world) * a.cap;
    const int64_t nw = (int64_t(gridDim.x) * blockDim.x) >> 5;
    for (int64_t it = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; it < total; it += nw) {
        const int g = int(it / a.cap);
        const int64_t idx = it % a.cap;
        char* dst = reinterpret_cast<char*>(a.peers[g]);
        const int64_t slot = int64_t(a.rank) * a.cap + idx;
        int32_t* did = reinterpret_cast<int32_t*>(dst + a.L.recv_ids) + slot * a.topk;
        float* dw = reinterpret_cast<float*>(dst + a.L.recv_w) + slot * a.topk;
        if (idx < counts[g]) {
            copy_row_warp(reinterpret_cast<uint4*>(dst + a.L.recv_x) + slot * a.row_vecs,
                          a.x + int64_t(tok[it]) * a.row_vecs, a.row_vecs, lane);
            for (int k = lane; k < a.topk; k += 32) {
                did[k] = sid[it * a.topk + k];
                dw[k] = sw[it * a.topk + k];
            }
        } else {
            for (int k = lane; k < a.topk; k += 32) {
                did[k] = -1;
                dw[k] = 0.f;
            }
        }
    }
    if (ep_last_cta(reinterpret_cast<int*>(a.window + kEpCtlScatterDone)))
        ep_raise_flags(a, a.L.arrive, a.L.counts, counts);
}

// owner: its partial rows of source g's pairs -> source g's window at
// [rank * cap + idx]; the last CTA to finish raises the return flags
__global__ void __launch_bounds__(256) ep_p2p_return_kernel(const uint4* __restrict__ partial, int64_t row_vecs,
                                                            const EpP2pArgs a) {
    const int lane = threadIdx.x & 31;
    const int32_t* counts = reinterpret_cast<const int32_t*>(a.window + a.L.counts);  // pairs from each source
    const int64_t total = int64_t(a.world) * a.cap;
    const int64_t nw = (int64_t(gridDim.x) * blockDim.x) >> 5;
    for (int64_t it = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; it < total; it += nw) {
        const int g = int(it / a.cap);
        const int64_t idx = it % a.cap;
        if (idx >= counts[g]) continue;
        char* dst = reinterpret_cast<char*>(a.peers[g]);
        copy_row_warp(reinterpret_cast<uint4*>(dst + a.L.back) + (int64_t(a.rank) * a.cap + idx) * row_vecs,
                      partial + it * row_vecs, row_vecs, lane);
    }
    if (ep_last_cta(reinterpret_cast<int*>(a.window + kEpCtlReturnDone))) ep_raise_flags(a, a.L.ret, 0, nullptr);
}

// wait (bounded) until every peer raised this step's flag in our window;
// on timeout record DEV_WAIT_TIMEOUT in the window's status word and return
__global__ void ep_p2p_wait_kernel(char* window, int world, size_t flag_off) {
    const int g = threadIdx.x;
    if (g >= world) return;
    const uint32_t target = *reinterpret_cast<const uint32_t*>(window + kEpCtlEpoch) + 1u;
    const uint32_t* flag = reinterpret_cast<const uint32_t*>(window + flag_off) + g;
    const long long t0 = clock64();
    while (int32_t(ld_acquire_sys(flag) - target) < 0) {
        if (clock64() - t0 > kWaitBudgetCycles) {
            atomicCAS(reinterpret_cast<int*>(window + kEpCtlStatus), 0, DEV_WAIT_TIMEOUT);
            return;
        }
        __nanosleep(200);
    }
}

__global__ void ep_p2p_epoch_kernel(char* window) {
    uint32_t* e = reinterpret_cast<uint32_t*>(window + kEpCtlEpoch);
    *e = *e + 1u;
}

}  // namespace

cudaError_t run_ep_p2p(const EpP2pCall& c, cudaStream_t s) {
    const EpWindow L = ep_window(c.world, c.capacity, c.hidden, c.topk, c.x_esize, c.p_esize);
    char* win = static_cast<char*>(c.window);
    EpP2pArgs a;
    a.world = c.world;
    a.rank = c.rank;
    a.topk = c.topk;
    a.cap = c.capacity;
    a.L = L;
    a.window = win;
    a.peers = c.peers;
    const int64_t slots = int64_t(c.world) * c.capacity;
    const int grid = int(std::max<int64_t>(1, std::min<int64_t>((slots + 7) / 8, int64_t(num_sms_current()) * 8)));
    cudaError_t e = cudaSuccess;
    if (c.phase == EP_P2P_DISPATCH) {
        EpPlanArgs p;
        p.ids = c.ids;
        p.ids_dtype = c.ids_dtype;
        p.weights = c.weights;
        p.w_dtype = c.w_dtype;
        p.tokens = c.tokens;
        p.topk = c.topk;
        p.n_global = c.n_global;
        p.world = c.world;
        p.n_valid = c.n_valid;
        p.send_ids = reinterpret_cast<int32_t*>(win + L.send_ids);
        p.send_w = reinterpret_cast<float*>(win + L.send_w);
        p.send_tok = reinterpret_cast<int32_t*>(win + L.send_tok);
        p.pair_idx = c.pair_idx;
        p.send_counts = reinterpret_cast<int32_t*>(win + L.send_counts);
        p.capacity = c.capacity;
        ep_plan_kernel<<<1, kEpPlanThreads, 0, s>>>(p);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        a.x = static_cast<const uint4*>(c.x);
        a.row_vecs = c.hidden * int64_t(c.x_esize) / 16;
        ep_p2p_scatter_kernel<<<grid, 256, 0, s>>>(a);
    } else if (c.phase == EP_P2P_WAIT_ARRIVE || c.phase == EP_P2P_WAIT_RETURN) {
        ep_p2p_wait_kernel<<<1, 64, 0, s>>>(win, c.world, c.phase == EP_P2P_WAIT_ARRIVE ? L.arrive : L.ret);
    } else if (c.phase == EP_P2P_RETURN) {
        ep_p2p_return_kernel<<<grid, 256, 0, s>>>(static_cast<const uint4*>(c.partial),
                                                  c.hidden * int64_t(c.p_esize) / 16, a);
    } else if (c.phase == EP_P2P_COMBINE) {
        if (c.tokens > 0)
            ep_combine_kernel<<<combine_grid(c.tokens, int(c.hidden)), 256, 0, s>>>(
                win + L.back, c.p_dtype, c.pair_idx, c.tokens, c.world, c.hidden, c.n_valid, c.out, c.out_dtype,
                reinterpret_cast<uint32_t*>(win + kEpCtlEpoch));
        else
            ep_p2p_epoch_kernel<<<1, 1, 0, s>>>(win);
    } else {
        return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t run_ep_dispatch(const EpDispatchCall& c, cudaStream_t s) {
    EpPlanArgs a;
    a.ids = c.ids;
    a.ids_dtype = c.ids_dtype;
    a.weights = c.weights;
    a.w_dtype = c.w_dtype;
    a.tokens = c.tokens;
    a.topk = c.topk;
    a.n_global = c.n_global;
    a.world = c.world;
    a.n_valid = c.n_valid;
    a.send_ids = c.send_ids;
    a.send_w = c.send_w;
    a.send_tok = c.send_tok;
    a.pair_idx = c.pair_idx;
    a.send_counts = c.send_counts;
    a.capacity = c.capacity;
    ep_plan_kernel<<<1, kEpPlanThreads, 0, s>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || c.tokens == 0) return e;
    const int64_t row_vecs = c.hidden * int64_t(c.x_esize) / 16;
    const int64_t max_pairs =
        c.capacity > 0 ? c.world * c.capacity : c.tokens * int64_t(std::min(c.world, c.topk));
    const int grid = int(std::max<int64_t>(1, std::min<int64_t>((max_pairs + 7) / 8, int64_t(num_sms_current()) * 8)));
    ep_gather_kernel<<<grid, 256, 0, s>>>(static_cast<const uint4*>(c.x), row_vecs, c.send_tok, c.send_counts,
                                          c.world, c.capacity, static_cast<uint4*>(c.send_x));
    return cudaGetLastError();
}

cudaError_t run_ep_combine(const void* partial, int pdt, const int32_t* pair_idx, int64_t tokens, int world,
                           int hidden, const int32_t* n_valid, void* out, int odt, cudaStream_t s) {
    if (tokens == 0) return cudaSuccess;
    ep_combine_kernel<<<combine_grid(tokens, hidden), 256, 0, s>>>(partial, pdt, pair_idx, tokens, world, hidden, n_valid, out, odt,
                                                                  nullptr);
    return cudaGetLastError();
}

}  // namespace exl3
