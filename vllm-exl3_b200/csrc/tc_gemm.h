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
    int in_f, out_f, ncb, kmax, stages;
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
    int act;              // 0 SiLU, 3 SwiGLU-OAI
};


// act: fp16 row-major [act_rows][in_f] activations (TMA source); mt: 128-row
// halves per work tile (1 or 2); grid: upper bound on tiles x column blocks
// (extra CTAs exit at once)
cudaError_t run_tc_gemm(int cb, int mt, const TcArgs& a, const void* act, int64_t act_rows, int64_t grid,
                        size_t smem, cudaStream_t s);

}  // namespace exl3
