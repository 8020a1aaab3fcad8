// exl3_internal.h -- host-side launch plans shared by the kernels and the C ABI.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace exl3 {

constexpr int kRowsPerSlot = 16;  // token rows one expert work slot carries (two m16n8 mma columns)
constexpr int kKtPerStage = 8;    // k-tiles (16 input features each) per pipeline stage = one 128 block

// One projection family (gate, up or down) of a layer: either per-expert
// pointer tables (int64 device arrays of data_ptr values, the reference's
// build_exl3_fused_state layout, src/vllm_exl3/exl3.py:2475-2508) or, for a
// dense linear, direct pointers.
struct ProjRef {
    const int64_t* trellis_tbl = nullptr;
    const int64_t* suh_tbl = nullptr;
    const int64_t* svh_tbl = nullptr;
    const int8_t* k_tbl = nullptr;  // per-expert K; nullptr -> k_uniform
    const void* trellis = nullptr;  // direct (dense linear)
    const void* suh = nullptr;
    const void* svh = nullptr;
    int k_uniform = 0;
};

// Workspace carve-up for one forward call.  All offsets are bytes from the
// workspace base, 256-byte aligned.
struct MoePlan {
    // geometry
    int64_t t_max = 0;  // token rows of x / out
    int topk = 0;
    int hidden = 0;
    int inter = 0;
    int n_local = 0;
    int kmax = 8;
    bool linear = false;  // one projection (dense linear, batched expert linear): no activation
    bool dup = true;      // GEMV activations in the duplicated layout (MCG / 3INST)
    int64_t routes = 0;   // t_max * topk
    int64_t rpad = 0;     // sorted rows incl. per-expert padding to 16
    int64_t smax = 0;     // max work slots
    // per GEMV phase: column blocks, grid, ring stages
    int ncb1 = 0, grid1 = 0, stages1 = 0;
    int ncb2 = 0, grid2 = 0, stages2 = 0;
    bool pair1 = false;  // single-projection GEMV: two 128-column blocks per work item (ncb1 even)
    bool pair2 = false;  // down GEMV: two 128-column blocks per work item (ncb2 even)
    size_t smem1 = 0, smem2 = 0;
    // prefill path: tcgen05 grouped GEMM over 128-row expert tiles
    bool gemm = false;
    int tile_m = 128;      // rows per GEMM work tile: 128 or 256
    int prep_chunks = 0;   // > 0: routing prep split over this many CTAs (large batches)
    int64_t t128max = 0;   // max work tiles
    int tc_stages = 0;
    size_t tc_smem = 0;
    // split-K ceiling per GEMM projection (gate/up, down): the kernel picks
    // 1..ceiling on the device from the real tile count
    int tc_split1 = 1, tc_split2 = 1;
    size_t off_tcpart = 0, off_tccnt = 0;
    // offsets
    size_t off_status = 0, off_nslots = 0, off_slots = 0, off_route_pos = 0, off_sorted_tok = 0,
           off_sorted_route = 0, off_ntiles128 = 0, off_tiles128 = 0, off_g = 0, off_u = 0, off_x2 = 0,
           off_sorted_exp = 0, off_sorted_w = 0, off_xr = 0, off_a2 = 0, off_yd = 0,
           off_part1 = 0, off_part2 = 0, off_cnt1 = 0, off_cnt2 = 0, off_hist = 0;
    size_t total = 0;
};

// Fill a plan; returns false if the geometry is unsupported.  cb is the
// codebook of the call (its GEMV activation layout), or -1 for a size query
// that must cover every codebook.
bool plan_moe(MoePlan& p, int64_t t_max, int topk, int hidden, int inter, int n_local, int kmax,
              bool linear, int num_sms, bool allow_gemm = true, int cb = -1);

struct MoeCall {
    const void* x = nullptr;
    int x_dtype = 1;
    const void* ids = nullptr;
    int ids_dtype = 3;
    const void* weights = nullptr;
    int w_dtype = 0;
    const int32_t* expert_map = nullptr;
    int64_t n_global = 0;
    const int32_t* n_valid = nullptr;
    ProjRef gate, up, down;
    int cb = 1;
    int act = 0;
    float limit = 0.f;
    void* out = nullptr;
    int out_dtype = 0;
    bool gateless = false;
    // single-projection variants (plan.linear)
    bool batched = false;              // ids = expert list shared by all rows; out [n_active][m][out]
    bool prerotated = false;           // x already carries H(x o suh)/sqrt128 (fat GEMM input)
    const int64_t* scatter_idx = nullptr;  // out[scatter_idx[row]] += scatter_w[row] * y[row]
    const void* scatter_w = nullptr;       // fp16
};

cudaError_t run_moe(const MoePlan& p, const MoeCall& c, void* ws, cudaStream_t s);

cudaError_t run_reconstruct(int K, int cb, bool full, const void* trellis, const void* suh,
                            const void* svh, int64_t in_f, int64_t out_f, void* w, cudaStream_t s);
cudaError_t run_had128(const void* x, void* y, int64_t rows, int64_t n, const void* pre,
                       const void* post, float scale, cudaStream_t s);

// Expert-parallel dispatch (source side): rank g owns experts
// [g * n_global / world, (g + 1) * n_global / world).
constexpr int kEpMaxWorld = 64;

struct EpDispatchCall {
    const void* x = nullptr;  // [tokens][hidden], element size x_esize
    int x_esize = 2;
    int64_t tokens = 0;
    int hidden = 0;
    const void* ids = nullptr;
    int ids_dtype = 3;
    const void* weights = nullptr;
    int w_dtype = 0;
    int topk = 0;
    int64_t n_global = 0;
    int world = 1;
    const int32_t* n_valid = nullptr;
    void* send_x = nullptr;        // [pairs][hidden]
    int32_t* send_ids = nullptr;   // [pairs][topk] local expert id or -1
    float* send_w = nullptr;       // [pairs][topk]
    int32_t* send_tok = nullptr;   // [pairs] source token
    int32_t* pair_idx = nullptr;   // [tokens][world] pair row or -1
    int32_t* send_counts = nullptr;  // [world]
    int64_t capacity = 0;            // > 0: fixed blocks of capacity rows per rank
};

cudaError_t run_ep_dispatch(const EpDispatchCall& c, cudaStream_t s);

// NVLink transport window of one rank (byte offsets; same geometry on every
// rank).  Control word 0: step epoch; word 1: status.  Peers write arrive[],
// counts[], ret[], recv_*[] and back[]; the send_* scratch is local.
constexpr size_t kEpCtlEpoch = 0, kEpCtlStatus = 4;
// completion counters of the scatter / return grids (the last CTA raises the
// step's flags and resets its counter)
constexpr size_t kEpCtlScatterDone = 8, kEpCtlReturnDone = 12;
struct EpWindow {
    size_t arrive, counts, ret, send_counts, recv_x, recv_ids, recv_w, back, send_tok, send_ids, send_w, total;
};
__host__ __device__ inline EpWindow ep_window(int world, int64_t cap, int64_t hidden, int topk, int xsize,
                                             int psize) {
    auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
    const size_t slots = size_t(world) * size_t(cap);
    EpWindow L;
    L.arrive = 256;
    L.counts = L.arrive + 256;
    L.ret = L.counts + 256;
    L.send_counts = L.ret + 256;
    L.recv_x = L.send_counts + 256;
    L.recv_ids = up(L.recv_x + slots * size_t(hidden) * xsize);
    L.recv_w = up(L.recv_ids + slots * topk * 4);
    L.back = up(L.recv_w + slots * topk * 4);
    L.send_tok = up(L.back + slots * size_t(hidden) * psize);
    L.send_ids = up(L.send_tok + slots * 4);
    L.send_w = up(L.send_ids + slots * topk * 4);
    L.total = up(L.send_w + slots * topk * 4);
    return L;
}

enum EpP2pPhase : int { EP_P2P_DISPATCH = 0, EP_P2P_WAIT_ARRIVE = 1, EP_P2P_RETURN = 2, EP_P2P_WAIT_RETURN = 3,
                        EP_P2P_COMBINE = 4 };
struct EpP2pCall {
    int phase = 0;
    int world = 1, rank = 0, topk = 0;
    int64_t capacity = 0, hidden = 0, tokens = 0, n_global = 0;
    int x_esize = 2, p_esize = 4, p_dtype = 0;
    void* window = nullptr;
    const int64_t* peers = nullptr;
    // dispatch
    const void* x = nullptr;
    const void* ids = nullptr;
    int ids_dtype = 3;
    const void* weights = nullptr;
    int w_dtype = 0;
    const int32_t* n_valid = nullptr;
    int32_t* pair_idx = nullptr;
    // return
    const void* partial = nullptr;
    // combine
    void* out = nullptr;
    int out_dtype = 0;
};
cudaError_t run_ep_p2p(const EpP2pCall& c, cudaStream_t s);
cudaError_t run_ep_combine(const void* partial, int pdt, const int32_t* pair_idx, int64_t tokens, int world,
                           int hidden, const int32_t* n_valid, void* out, int odt, cudaStream_t s);

// n-gram embedding rows (ngram.cu): decode `n` packed rows given in order
// (ids == nullptr, heads per row) or gather rows `ids` of a table of n_rows
// (heads from head_offsets)
cudaError_t run_ngram(const uint16_t* rows, int64_t n, int64_t n_rows, int bits, const void* ids, int ids_dtype,
                      const int32_t* heads, const int64_t* head_offsets, int num_heads, const void* head_bias,
                      void* out, int out_dtype, int* status, cudaStream_t s);

int num_sms_current();
// stages and dynamic smem of the GEMM for mt 128-row halves per tile; false
// if two stages do not fit at two CTAs per SM
bool tc_pick_stages(int kmax, int mt, int& stages, size_t& smem);
void profile_enable(bool on, long long delay_cycles);
int profile_read(float* ms, int max_phases);

}  // namespace exl3
