// reconstruct.cu -- trellis -> fp16 weights on the GPU, and the 128-point
// Hadamard rotation kernel.
//
//  * exl3_reconstruct: W = diag(suh) H W~ H diag(svh) / 128, bit-exact with
//    the reference's CPU dequant (csrc/bindings.cpp:15-100): the same fp32
//    butterflies in the same stage order, rows before columns, norm applied
//    after each pass and the final product taken left to right
//    (line * norm * suh[r] * svh[c]) before one round to fp16.
//  * exl3_decode_raw: W~ only (the analogue of ExLlamaV3's `reconstruct`).
//  * exl3_had128: y = fp16(H(x o pre) / sqrt(128) o post * scale) per
//    128-column block (the analogue of ExLlamaV3's `had_r_128`, called at
//    src/vllm_exl3/exl3.py:3039-3156).
//
// One CTA owns one 128 x 128 block: 8 warps decode its 64 tiles into shared
// memory (fp32, pitch 129 so row and column sweeps are conflict-free), then
// sweep rows and columns with the warp-wide FWHT.
#include "exl3_common.cuh"
#include "exl3_internal.h"

namespace exl3 {

constexpr int RC_PITCH = 129;
constexpr int RC_THREADS = 256;

template <int K, int CB, bool FULL>
__global__ void __launch_bounds__(RC_THREADS)
reconstruct_kernel(const uint32_t* __restrict__ trellis, const __half* __restrict__ suh,
                   const __half* __restrict__ svh, int ntiles_out, int64_t out_features,
                   __half* __restrict__ w) {
    extern __shared__ float sm[];  // [128][RC_PITCH]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bk = blockIdx.x, bn = blockIdx.y;  // 128-row / 128-col block
    const int64_t r0 = int64_t(bk) * 128, c0 = int64_t(bn) * 128;

    // 1. decode the block's 8 x 8 tiles
    for (int t = warp; t < 64; t += RC_THREADS / 32) {
        const int kt_l = t >> 3, nt_l = t & 7;
        const int64_t kt = int64_t(bk) * 8 + kt_l, nt = int64_t(bn) * 8 + nt_l;
        const uint32_t* tile = trellis + (kt * ntiles_out + nt) * (8 * K);
        uint32_t v[4];
        decode_tile_pairs<K, CB>(tile, lane, v);
        const int rbase = 2 * (lane & 3), cbase = lane >> 2;
        #pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t pr = v[j >> 1];
            const __half h = __ushort_as_half(static_cast<unsigned short>((j & 1) ? (pr >> 16) : (pr & 0xffffu)));
            const int row = kt_l * 16 + rbase + (j & 1) + 8 * ((j >> 1) & 1);
            const int col = nt_l * 16 + cbase + 8 * (j >> 2);
            if constexpr (FULL) {
                sm[row * RC_PITCH + col] = __half2float(h);
            } else {
                w[(r0 + row) * out_features + c0 + col] = h;
            }
        }
    }
    if constexpr (!FULL) return;
    __syncthreads();

    // 2. rows: FWHT then * norm
    for (int r = warp; r < 128; r += RC_THREADS / 32) {
        float v[4];
        #pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = sm[r * RC_PITCH + lane + 32 * i];
        fwht128_warp(v, lane);
        #pragma unroll
        for (int i = 0; i < 4; ++i) sm[r * RC_PITCH + lane + 32 * i] = __fmul_rn(v[i], kHadNorm);
    }
    __syncthreads();

    // 3. columns: FWHT then ((x * norm) * suh[r]) * svh[c]
    for (int c = warp; c < 128; c += RC_THREADS / 32) {
        float v[4];
        #pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = sm[(lane + 32 * i) * RC_PITCH + c];
        fwht128_warp(v, lane);
        const float sv = __half2float(svh[c0 + c]);
        #pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float su = __half2float(suh[r0 + lane + 32 * i]);
            sm[(lane + 32 * i) * RC_PITCH + c] = __fmul_rn(__fmul_rn(__fmul_rn(v[i], kHadNorm), su), sv);
        }
    }
    __syncthreads();

    // 4. coalesced fp16 store
    for (int r = warp; r < 128; r += RC_THREADS / 32) {
        #pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int c = lane + 32 * i;
            w[(r0 + r) * out_features + c0 + c] = __float2half_rn(sm[r * RC_PITCH + c]);
        }
    }
}

template <int K, int CB, bool FULL>
static cudaError_t launch_rc(const void* trellis, const void* suh, const void* svh, int64_t in_f,
                             int64_t out_f, void* w, cudaStream_t stream) {
    const size_t smem = FULL ? size_t(128) * RC_PITCH * sizeof(float) : 0;
    auto kern = reconstruct_kernel<K, CB, FULL>;
    if (FULL) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        if (e != cudaSuccess) return e;
    }
    dim3 grid(unsigned(in_f / 128), unsigned(out_f / 128));
    kern<<<grid, RC_THREADS, smem, stream>>>(static_cast<const uint32_t*>(trellis),
                                             static_cast<const __half*>(suh),
                                             static_cast<const __half*>(svh), int(out_f / 16), out_f,
                                             static_cast<__half*>(w));
    return cudaGetLastError();
}

template <bool FULL>
static cudaError_t dispatch_rc(int K, int cb, const void* trellis, const void* suh, const void* svh,
                               int64_t in_f, int64_t out_f, void* w, cudaStream_t s) {
#define EXL3_RC_CASE(KK)                                                                   \
    case KK:                                                                               \
        if (cb == CB_MCG) return launch_rc<KK, CB_MCG, FULL>(trellis, suh, svh, in_f, out_f, w, s); \
        if (cb == CB_MUL1) return launch_rc<KK, CB_MUL1, FULL>(trellis, suh, svh, in_f, out_f, w, s); \
        return launch_rc<KK, CB_3INST, FULL>(trellis, suh, svh, in_f, out_f, w, s);
    switch (K) {
        EXL3_RC_CASE(2)
        EXL3_RC_CASE(3)
        EXL3_RC_CASE(4)
        EXL3_RC_CASE(5)
        EXL3_RC_CASE(6)
        EXL3_RC_CASE(7)
        EXL3_RC_CASE(8)
        default: return cudaErrorInvalidValue;
    }
#undef EXL3_RC_CASE
}

cudaError_t run_reconstruct(int K, int cb, bool full, const void* trellis, const void* suh,
                            const void* svh, int64_t in_f, int64_t out_f, void* w, cudaStream_t s) {
    return full ? dispatch_rc<true>(K, cb, trellis, suh, svh, in_f, out_f, w, s)
                : dispatch_rc<false>(K, cb, trellis, suh, svh, in_f, out_f, w, s);
}

// ---------------------------------------------------------------------------
// Hadamard rotation of fp16 rows: one warp per (row, 128-block).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
had128_kernel(const __half* __restrict__ x, __half* __restrict__ y, int64_t rows, int64_t n,
              const __half* __restrict__ pre, const __half* __restrict__ post, float scale) {
    const int lane = threadIdx.x & 31;
    const int64_t nblk = n / 128;
    const int64_t total = rows * nblk;
    for (int64_t item = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; item < total;
         item += (int64_t(gridDim.x) * blockDim.x) >> 5) {
        const int64_t r = item / nblk, b = item % nblk;
        const __half* src = x + r * n + b * 128;
        float v[4];
        #pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int c = lane + 32 * i;
            float f = __half2float(src[c]);
            if (pre) f *= __half2float(pre[b * 128 + c]);
            v[i] = f;
        }
        fwht128_warp(v, lane);
        __half* dst = y + r * n + b * 128;
        #pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int c = lane + 32 * i;
            float f = v[i] * kHadNorm * scale;
            if (post) f *= __half2float(post[b * 128 + c]);
            dst[c] = __float2half_rn(f);
        }
    }
}

cudaError_t run_had128(const void* x, void* y, int64_t rows, int64_t n, const void* pre,
                       const void* post, float scale, cudaStream_t s) {
    const int64_t warps = rows * (n / 128);
    const int64_t blocks = (warps + 7) / 8;
    const unsigned grid = unsigned(blocks < 148 * 16 ? blocks : 148 * 16);
    had128_kernel<<<grid, 256, 0, s>>>(static_cast<const __half*>(x), static_cast<__half*>(y), rows,
                                       n, static_cast<const __half*>(pre),
                                       static_cast<const __half*>(post), scale);
    return cudaGetLastError();
}

}  // namespace exl3
