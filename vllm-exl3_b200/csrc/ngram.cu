// ngram.cu -- row-wise EXL3 embedding tables (the n-gram format) on sm_100a.
//
// A table row holds one fp16 scale word and a tail-biting ring bitstream of
// 160 K-bit trellis states (1 + 160 K / 16 int16 words).  Element i's 16-bit
// state takes its bit m from stream bit ((i - m / K) mod 160) K + m % K (the
// stream read LSB-first inside each int16 word after the scale); its value is
// fp16(fp16(mul1(state)) * scale + head_bias[head][i]) with the mul1
// codebook of the trellis format (h = 1024 + bytesum(state * 0x83DCD12D),
// fp16(h * h(0x1eee) + h(0xc931)), fp32 arithmetic).
// (vcruz305/vllm-exl3 src/vllm_exl3/exl3.py:5170-5245 ngram_dequant_rows_torch,
// the restatement of ExLlamaV3's ngram_dequant; the lookup path of
// Exl3EmbeddingMethod._embedding_impl, exl3.py:5576-5587: gather the packed
// rows of the ids, head = searchsorted(head_offsets, id, right) - 1 clamped,
// decode.)
//
// One warp per row: the row's words are staged in shared memory, lane l
// decodes elements l, l + 32, ..., l + 128.  Gather, head search and decode
// are one launch.
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "exl3_common.cuh"
#include "exl3_internal.h"

namespace exl3 {

constexpr int kNgramDim = 160;
constexpr int kNgramWarps = 8;
constexpr int kNgramMaxWords = 1 + kNgramDim * 8 / 16;  // K = 8

struct NgramArgs {
    const uint16_t* rows;     // packed rows [n][words] (dequant) or the table [n_rows][words] (lookup)
    int64_t n;                // rows to produce
    int64_t n_rows;           // table rows (lookup)
    int bits;
    int words;
    const void* ids;          // lookup: row ids [n]; nullptr: rows are given in order (dequant)
    int ids_dtype;
    const int32_t* heads;     // dequant: head per row [n]
    const int64_t* head_offsets;  // lookup: first id of each head [num_heads], ascending
    int num_heads;
    const __half* head_bias;  // [num_heads][160]
    void* out;                // [n][160]
    int out_dtype;
    int* status;              // optional device status word (an id outside the table)
};

__device__ __forceinline__ float ngram_codebook(uint32_t state) {
    const uint32_t prod = state * 0x83DCD12Du;
    const float h = 1024.0f + float((prod & 0xffu) + ((prod >> 8) & 0xffu) + ((prod >> 16) & 0xffu) + (prod >> 24));
    const float kinv = __half2float(__ushort_as_half(0x1eee));
    const float kbias = __half2float(__ushort_as_half(0xc931));
    return __half2float(__float2half_rn(__fadd_rn(__fmul_rn(h, kinv), kbias)));
}

__global__ void __launch_bounds__(kNgramWarps * 32) ngram_kernel(const NgramArgs a) {
    __shared__ uint16_t srow[kNgramWarps][kNgramMaxWords + 3];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r = int64_t(blockIdx.x) * kNgramWarps + warp;
    if (r >= a.n) return;  // whole warp
    const int K = a.bits, W = a.words;
    int64_t src = r;
    int head = 0;
    bool valid = true;
    if (a.ids) {
        src = load_id(a.ids, r, a.ids_dtype);
        valid = src >= 0 && src < a.n_rows;
        // head = (number of offsets <= id) - 1, clamped to [0, num_heads)
        int count = 0;
        for (int h0 = 0; h0 < a.num_heads; h0 += 32) {
            const int h = h0 + lane;
            const bool le = h < a.num_heads && a.head_offsets[h] <= src;
            count += __popc(__ballot_sync(0xffffffffu, le));
        }
        head = min(max(count - 1, 0), a.num_heads - 1);
    } else {
        head = min(max(int(a.heads[r]), 0), a.num_heads - 1);
    }
    if (!valid) {
        if (lane == 0) set_status(a.status, DEV_BAD_INDEX);
        for (int i = lane; i < kNgramDim; i += 32) store_from_float(a.out, r * kNgramDim + i, a.out_dtype, 0.f);
        return;
    }
    const uint16_t* row = a.rows + src * int64_t(W);
    for (int w = lane; w < W; w += 32) srow[warp][w] = row[w];
    if (lane < 2) srow[warp][W + lane] = 0;
    __syncwarp();
    const float scale = __half2float(__ushort_as_half(srow[warp][0]));
    const uint16_t* stream = &srow[warp][1];
    const uint32_t kmask = (1u << K) - 1u;
    const __half* bias = a.head_bias + int64_t(head) * kNgramDim;
    for (int i = lane; i < kNgramDim; i += 32) {
        uint32_t state = 0;
        for (int g = 0; g * K < 16; ++g) {
            int j = i - g;
            if (j < 0) j += kNgramDim;
            const int b = j * K;  // < ring
            const int wi = b >> 4, sh = b & 15;
            const uint32_t win = uint32_t(stream[wi]) | (uint32_t(stream[wi + 1]) << 16);
            state |= ((win >> sh) & kmask) << (g * K);
        }
        state &= 0xffffu;
        const float v = __fadd_rn(__fmul_rn(ngram_codebook(state), scale), __half2float(bias[i]));
        const float h = __half2float(__float2half_rn(v));
        store_from_float(a.out, r * kNgramDim + i, a.out_dtype, h);
    }
}

cudaError_t run_ngram(const uint16_t* rows, int64_t n, int64_t n_rows, int bits, const void* ids, int ids_dtype,
                      const int32_t* heads, const int64_t* head_offsets, int num_heads, const void* head_bias,
                      void* out, int out_dtype, int* status, cudaStream_t s) {
    NgramArgs a;
    a.rows = rows;
    a.n = n;
    a.n_rows = n_rows;
    a.bits = bits;
    a.words = 1 + kNgramDim * bits / 16;
    a.ids = ids;
    a.ids_dtype = ids_dtype;
    a.heads = heads;
    a.head_offsets = head_offsets;
    a.num_heads = num_heads;
    a.head_bias = static_cast<const __half*>(head_bias);
    a.out = out;
    a.out_dtype = out_dtype;
    a.status = status;
    if (n <= 0) return cudaSuccess;
    const int64_t blocks = (n + kNgramWarps - 1) / kNgramWarps;
    ngram_kernel<<<unsigned(blocks), kNgramWarps * 32, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace exl3
