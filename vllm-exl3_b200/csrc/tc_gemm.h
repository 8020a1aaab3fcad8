// tc_gemm.h -- launch interface of the tcgen05 grouped GEMM (tc_gemm.cu).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "exl3_internal.h"

namespace exl3 {

// epilogues: ROWS = fp32 rows; DOWN = fp32 rows x route weight; LINEAR =
// the caller's dtype per token (or weighted scatter); UPACT = the up
// projection fused with the activation: reads the gate rows, writes the
// fp16 down input H128(act o suh_down)/sqrt128
enum TcEpi : int { TC_EPI_ROWS = 0, TC_EPI_DOWN = 1, TC_EPI_LINEAR = 2, TC_EPI_UPACT = 3 };

struct TcArgs {
    int* status;
    ProjRef proj;
    int in_f, out_f, ncb, kmax;
    int stage_mem;  // dynamic shared memory for the stage ring (the kernel sizes
                    // its stages from the rows of its tile)
    const int* ntiles;
    const int4* tiles;  // {expert, first sorted row, rows <= 128 * mt, 0}
    int epi;
    float* yrows;           // TC_EPI_ROWS / TC_EPI_DOWN: [rows][out_f] fp32
    const float* sorted_w;  // TC_EPI_DOWN: route weight per sorted row
    void* y;                // TC_EPI_LINEAR: [tokens][out_f] in y_dtype (or scatter)
    int y_dtype;
    const int* sorted_tok;
    const int64_t* scatter_idx;
    const __half* scatter_w;
    // TC_EPI_UPACT
    const float* g_rows;  // [rows][out_f] gate rows (after o svh)
    __half* x2;           // [rows][out_f] fp16 down input
    ProjRef down;         // suh of the down projection
    float limit;          // SwiGLU clamp (0 = off)
    int act;              // 0 SiLU, 2 non-gated relu^2 (no gate rows), 3 SwiGLU-OAI
    // split-K: with max_split > 1 the kernel splits each (tile, column block)
    // over 1..max_split CTAs, chosen from the device-side tile count so the
    // CTAs fill `ctas` slots; each split writes fp32 partials to `part`
    // [(tile * ncb + cb) * max_split + split][128 * mt][128] and the last to
    // finish (counter `cnt[tile * ncb + cb]`, zero on entry, reset by it) sums
    // them in split order and runs the epilogue
    int max_split;
    int ctas;
    float* part;
    int* cnt;
};


// act: fp16 row-major [act_rows][in_f] activations (TMA source); mt: 128-row
// halves per work tile (1 or 2); grid: upper bound on tiles x column blocks x
// max(1, max_split) (extra CTAs exit at once)
// split-K ceiling for one projection: only when even the upper bound on
// work items leaves the CTA slots short, and only with >= 8 K stages a split
constexpr int kTcMaxSplit = 4;
int tc_split_ceiling(int64_t max_items, int in_f, int ctas);

// grid of a launch: every possible (tile, column block) item, times the
// split ceiling but at most two waves of CTAs (the kernel keeps its split
// count within the grid); CTAs without work still cost dispatch time
inline int64_t tc_grid(int64_t max_items, int max_split, int ctas) {
    if (max_split <= 1) return max_items;
    const int64_t g = max_items * max_split;
    return g < 2 * int64_t(ctas) ? g : (max_items > 2 * int64_t(ctas) ? max_items : 2 * int64_t(ctas));
}

cudaError_t run_tc_gemm(int cb, int mt, const TcArgs& a, const void* act, int64_t act_rows, int64_t grid,
                        size_t smem, cudaStream_t s);

}  // namespace exl3
