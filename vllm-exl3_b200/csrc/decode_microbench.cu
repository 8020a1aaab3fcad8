// decode_microbench.cu -- cost of the trellis decode that feeds the tcgen05
// GEMM, in isolation (no TMA, no MMA): per 16x16 tile, per bit width K and
// codebook, the instructions and SM sub-partition cycles of decode_tile_pairs
// plus the four swizzled shared-memory stores a decoder warp issues per tile
// (the same code tc_gemm.cu runs).  "windows" variants stop after the window
// extraction.  Raw words sit in shared memory; 296 CTAs x 8 warps, each warp
// re-decoding its four tiles `iters` times.
//
// Build: python -c "import sys; sys.path.insert(0,'vllm-exl3_b200'); \
//        from exl3_b200 import build; build.build_microbench()"
// Run:   vllm-exl3_b200/exl3_b200/decode_microbench   (one GPU; prints cycles/tile)
#include <cuda_runtime.h>

#include <cstdio>

#include "exl3_common.cuh"
#include "tc_common.cuh"

using namespace exl3;

namespace {

constexpr int kRawBytes = 4 * 256 * 8;  // four k-tile rows at K <= 8

template <int K, int CB, bool FULL, int MINB>
__global__ void __launch_bounds__(256, MINB) decode_slice_bench(const uint32_t* __restrict__ g, uint32_t* out,
                                                                 int iters) {
    __shared__ __align__(1024) char raw[kRawBytes];
    __shared__ __align__(1024) char bsm[16384];
    for (int i = threadIdx.x; i < kRawBytes / 4; i += blockDim.x) reinterpret_cast<uint32_t*>(raw)[i] = g[i];
    __syncthreads();
    const int d = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = 16 * d + (lane >> 2);
    uint32_t oa[4], ob[4];
    #pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
        oa[kk] = sw128_offset(n0, 16 * kk + 2 * (lane & 3));
        ob[kk] = sw128_offset(n0, 16 * kk + 2 * (lane & 3) + 8);
    }
    uint32_t acc = 0;
    for (int it = 0; it < iters; ++it) {
        #pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            const uint32_t* tile = reinterpret_cast<const uint32_t*>(raw) + (kk * 8 + d) * (8 * K);
            uint32_t v[4];
            if constexpr (FULL) {
                decode_tile_pairs<K, CB>(tile, lane, v);
            } else {
                uint32_t w[8];
                tile_windows<K>(tile, lane, w);
                v[0] = w[0] ^ w[1], v[1] = w[2] ^ w[3], v[2] = w[4] ^ w[5], v[3] = w[6] ^ w[7];
            }
            *reinterpret_cast<uint32_t*>(bsm + oa[kk]) = v[0];
            *reinterpret_cast<uint32_t*>(bsm + ob[kk]) = v[1];
            *reinterpret_cast<uint32_t*>(bsm + oa[kk] + 1024) = v[2];
            *reinterpret_cast<uint32_t*>(bsm + ob[kk] + 1024) = v[3];
        }
        __syncwarp();
        acc += *reinterpret_cast<const uint32_t*>(bsm + oa[it & 3]);
    }
    out[blockIdx.x * blockDim.x + threadIdx.x] = acc;  // keeps the work live
}

template <int K, int CB, bool FULL, int MINB = 2>
bool run(const uint32_t* g, uint32_t* o, const char* name) {
    constexpr int kCtas = 296, kIters = 2048;
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    decode_slice_bench<K, CB, FULL, MINB><<<kCtas, 256>>>(g, o, 16);  // warm-up
    cudaEventRecord(a);
    decode_slice_bench<K, CB, FULL, MINB><<<kCtas, 256>>>(g, o, kIters);
    cudaEventRecord(b);
    if (cudaEventSynchronize(b) != cudaSuccess) return false;
    float ms = 0.f;
    cudaEventElapsedTime(&ms, a, b);
    int sms = 148, clk_khz = 0, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&clk_khz, cudaDevAttrClockRate, dev);
    const double tiles_per_smsp = double(kCtas) * 8 * kIters * 4 / (sms * 4.0);
    std::printf("%-16s %8.3f ms  %6.1f cycles/tile/SMSP at %d MHz\n", name, ms,
                ms * 1e-3 * clk_khz * 1e3 / tiles_per_smsp, clk_khz / 1000);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    return true;
}

}  // namespace

int main() {
    uint32_t *g = nullptr, *o = nullptr;
    if (cudaMalloc(&g, kRawBytes) != cudaSuccess || cudaMalloc(&o, 296 * 256 * 4) != cudaSuccess) return 1;
    cudaMemset(g, 0x5a, kRawBytes);
    bool ok = run<2, CB_MUL1, true>(g, o, "K2 mul1") && run<3, CB_MUL1, true>(g, o, "K3 mul1") &&
              run<4, CB_MUL1, true>(g, o, "K4 mul1") && run<2, CB_MCG, true>(g, o, "K2 mcg") &&
              run<3, CB_MCG, true>(g, o, "K3 mcg") && run<4, CB_MCG, true>(g, o, "K4 mcg") &&
              run<2, CB_MCG, false>(g, o, "K2 windows") && run<3, CB_MCG, false>(g, o, "K3 windows") &&
              run<4, CB_MCG, false>(g, o, "K4 windows");
    const cudaError_t e = cudaDeviceSynchronize();
    std::printf("status: %s\n", cudaGetErrorString(e));
    cudaFree(g);
    cudaFree(o);
    return ok && e == cudaSuccess ? 0 : 1;
}
