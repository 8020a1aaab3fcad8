// tc_gemm.h -- launch interface of the tcgen05 grouped GEMM (tc_gemm.cu).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "exl3_internal.h"

namespace exl3 {

enum TcEpi : int { TC_EPI_ROWS = 0, TC_EPI_DOWN = 1, TC_EPI_LINEAR = 2 };

struct TcArgs {
    int* status;
    ProjRef proj;
    int in_f, out_f, ncb, kmax, stages;
    const int* ntiles;
    const int4* tiles;  // {expert, first sorted row, rows <= 128, 0}
    int epi;
    float* yrows;           // TC_EPI_ROWS / TC_EPI_DOWN: [rows][out_f] fp32
    const float* sorted_w;  // TC_EPI_DOWN: route weight per sorted row
    void* y;                // TC_EPI_LINEAR: [tokens][out_f] in y_dtype (or scatter)
    int y_dtype;
    const int* sorted_tok;
    const int64_t* scatter_idx;
    const __half* scatter_w;
};

struct ActArgs {
    const float* g;
    const float* u;
    __half* x2;
    ProjRef down;
    const int* ntiles;
    const int4* tiles;
    int inter;
    float limit;
    int act;
    int* status;
    int64_t rpad;
    const int* nrows;  // sorted rows in use (written by the prep kernel)
    const int* sorted_tok;
    const int* sorted_exp;
};

// act: fp16 row-major [act_rows][in_f] activations (TMA source); grid: upper
// bound on tiles x column blocks (extra CTAs exit at once)
cudaError_t run_tc_gemm(int cb, const TcArgs& a, const void* act, int64_t act_rows, int64_t grid, size_t smem,
                        cudaStream_t s);
cudaError_t run_tc_act(const ActArgs& a, int grid, cudaStream_t s);

}  // namespace exl3
