/*
 * exl3_oracle.c -- CPU restatement of the EXL3 trellis decode.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * kernels in vllm-exl3_b200/csrc.  Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / --impl reference legs may load it.  The product
 * path never calls it and has no CPU fallback.
 *
 * It restates, in plain C, the reference's own CPU dequant
 * (vcruz305/vllm-exl3 csrc/exl3_dequant.cuh and csrc/bindings.cpp:15-100).
 * Each function cites the reference lines whose arithmetic it follows.  The
 * restatement is pinned bit-for-bit against the reference compiled from its
 * own sources (oracle/Makefile target `ref`) and against the reference test
 * vectors (tests/test_oracle_*.py, tests/golden/).
 *
 * Build with -O2 -ffp-contract=off: the reference computes a*b + c in float
 * with two roundings (exl3_dequant.cuh:96-100) and the Hadamard butterflies as
 * separate adds; contraction into FMA would change bits.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define MCG_MUL 0xCBAC1FEDu  /* exl3_dequant.cuh:9 */
#define MUL1_MUL 0x83DCD12Du /* exl3_dequant.cuh:10 */

/* IEEE binary16 -> float (exl3_dequant.cuh:25-38). */
float oracle_half_to_float(uint16_t bits) {
    const uint32_t sign = (bits >> 15) & 1u;
    const uint32_t exp = (bits >> 10) & 0x1Fu;
    const uint32_t mant = bits & 0x3FFu;
    float v;
    if (exp == 0) {
        v = ldexpf((float)mant, -24);
    } else if (exp == 31) {
        if (mant) return NAN;
        v = INFINITY;
    } else {
        v = ldexpf(1.0f + (float)mant / 1024.0f, (int)exp - 15);
    }
    return sign ? -v : v;
}

/* float -> binary16, round to nearest even, NaN payload kept with the quiet
 * bit set (exl3_dequant.cuh:40-86). */
uint16_t oracle_float_to_half(float value) {
    uint32_t raw;
    memcpy(&raw, &value, sizeof raw);
    const uint32_t sign = (raw >> 16) & 0x8000u;
    const uint32_t e8 = (raw >> 23) & 0xFFu;
    const uint32_t mant = raw & 0x7FFFFFu;
    if (e8 == 0xFFu) {
        if (mant == 0) return (uint16_t)(sign | 0x7C00u);
        return (uint16_t)(sign | 0x7C00u | (((mant >> 13) | 0x200u) & 0x3FFu));
    }
    const int exp = (int)e8 - 127;
    if (exp < -14) {
        /* subnormal half: significand * 2^-24, RNE, may carry into 0x0400 */
        const uint32_t sig = mant | 0x800000u;
        const int shift = -exp - 1;
        if (shift >= 32) return (uint16_t)sign;
        uint32_t r = sig >> shift;
        const uint32_t rem = sig & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (r & 1u))) ++r;
        return (uint16_t)(sign | (r & 0x7FFu));
    }
    uint32_t rm = mant >> 13;
    const uint32_t rem = mant & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (rm & 1u))) ++rm;
    int he = exp + 15;
    if (rm == 0x400u) { rm = 0; ++he; }
    if (he >= 31) return (uint16_t)(sign | 0x7C00u);
    return (uint16_t)(sign | ((uint32_t)he << 10) | rm);
}

/* LOP3 with LUT 0x6A indexed a:b:c is c ^ (a & b) (exl3_dequant.cuh:12-23). */
static inline uint32_t lop3_6a(uint32_t a, uint32_t b, uint32_t c) { return c ^ (a & b); }

static inline uint16_t half_add(uint16_t a, uint16_t b) { /* :88-90 */
    return oracle_float_to_half(oracle_half_to_float(a) + oracle_half_to_float(b));
}

static inline uint16_t half_fma2(uint16_t a, uint16_t b, uint16_t c) { /* :96-100 */
    const float p = oracle_half_to_float(a) * oracle_half_to_float(b);
    return oracle_float_to_half(p + oracle_half_to_float(c));
}

/* One 16-bit trellis state -> fp16 bits, codebook cb: 0 = 3INST, 1 = MCG,
 * 2 = mul1 (exl3_dequant.cuh:105-124). */
uint16_t oracle_decode_codebook(uint16_t window, int cb) {
    uint32_t x = window;
    if (cb == 0 || cb == 1) {
        x = (cb == 0) ? x * 89226354u + 64248484u : x * MCG_MUL;
        x = lop3_6a(x, 0x8fff8fffu, 0x3b603b60u);
        return half_add((uint16_t)x, (uint16_t)(x >> 16));
    }
    x *= MUL1_MUL;
    const uint32_t s = 0x6400u + (x & 0xffu) + ((x >> 8) & 0xffu) + ((x >> 16) & 0xffu) + (x >> 24);
    return half_fma2((uint16_t)s, 0x1eeeu, 0xc931u);
}

/* Tail-biting 16-bit window of a tile holding `words` int16 values, read as
 * uint32 pairs with bits numbered MSB-first (exl3_dequant.cuh:141-159). */
uint16_t oracle_read_window(const uint16_t* p, size_t words, size_t bit) {
    bit %= words * 16;
    const size_t b1 = bit + 16;
    const size_t n32 = words / 2;
    const size_t i0 = (bit / 32) % n32;
    const size_t i1 = ((b1 - 1) / 32) % n32;
    const unsigned shift = (unsigned)((i1 + 1) * 32 - b1);
    const uint32_t a = (uint32_t)p[2 * i0] | ((uint32_t)p[2 * i0 + 1] << 16);
    const uint32_t b = (uint32_t)p[2 * i1] | ((uint32_t)p[2 * i1 + 1] << 16);
    const uint64_t merged = ((uint64_t)a << 32) | b;
    return (uint16_t)((merged >> shift) & 0xffffu);
}

/* Decode one 16x16 tile (16*K int16 words) into a row-major 16x16 block of
 * fp16 bits.  Value t = 8*l + j reads the window at (t + 257)*K - 16; lane
 * l's values land at the tensor-core fragment position below
 * (bindings.cpp:37-77): k-pair (l%4), column l/4, j selecting k+{0,1},
 * k+8+{0,1} and column +8 for j >= 4. */
void oracle_decode_tile(const uint16_t* tile, int K, int cb, uint16_t out[256]) {
    const size_t words = (size_t)16 * (size_t)K;
    for (int l = 0; l < 32; ++l) {
        const int r0 = (l % 4) * 2;
        const int c = l / 4;
        for (int j = 0; j < 8; ++j) {
            const size_t start = ((size_t)(8 * l + j) + 257u) * (size_t)K - 16u;
            const uint16_t v = oracle_decode_codebook(oracle_read_window(tile, words, start), cb);
            const int row = r0 + (j & 1) + ((j & 2) ? 8 : 0);
            const int col = c + ((j & 4) ? 8 : 0);
            out[row * 16 + col] = v;
        }
    }
}

/* Trellis [rows/16, cols/16, 16K] -> W~ [rows, cols] fp16 bits, no rotation. */
void oracle_decode_raw(const int16_t* trellis, int64_t rows, int64_t cols, int K, int cb,
                       uint16_t* out) {
    const int64_t kt_n = rows / 16, nt_n = cols / 16;
    const size_t words = (size_t)16 * (size_t)K;
    uint16_t blk[256];
    for (int64_t kt = 0; kt < kt_n; ++kt)
        for (int64_t nt = 0; nt < nt_n; ++nt) {
            const uint16_t* tile = (const uint16_t*)trellis + (size_t)(kt * nt_n + nt) * words;
            oracle_decode_tile(tile, K, cb, blk);
            for (int r = 0; r < 16; ++r)
                memcpy(out + (kt * 16 + r) * cols + nt * 16, blk + r * 16, 16 * sizeof(uint16_t));
        }
}

/* In-place unnormalised fast Walsh-Hadamard transform, strides 1..n/2,
 * (a+b, a-b) butterflies (exl3_dequant.cuh:168-179). */
void oracle_hadamard(float* v, int n) {
    for (int s = 1; s < n; s <<= 1)
        for (int base = 0; base < n; base += s << 1)
            for (int i = 0; i < s; ++i) {
                const float a = v[base + i], b = v[base + s + i];
                v[base + i] = a + b;
                v[base + s + i] = a - b;
            }
}

/* Full reconstruction W = diag(suh) H W~ H diag(svh) / 128 with the
 * reference's float rounding order (bindings.cpp:79-98): per 128x128 block,
 * rows transformed then scaled by norm, columns transformed then multiplied
 * left to right by norm, suh[r], svh[c], and rounded to fp16.
 * Returns 0, or -1 when rows/cols are not multiples of 128 (bindings.cpp:22). */
int oracle_dequant(const int16_t* trellis, const uint16_t* suh, const uint16_t* svh,
                   int64_t rows, int64_t cols, int K, int cb, uint16_t* out) {
    if (rows % 128 || cols % 128 || rows <= 0 || cols <= 0) return -1;
    float* m = (float*)malloc((size_t)rows * (size_t)cols * sizeof(float));
    uint16_t* raw = (uint16_t*)malloc((size_t)rows * (size_t)cols * sizeof(uint16_t));
    if (!m || !raw) { free(m); free(raw); return -2; }
    oracle_decode_raw(trellis, rows, cols, K, cb, raw);
    for (int64_t i = 0; i < rows * cols; ++i) m[i] = oracle_half_to_float(raw[i]);
    free(raw);
    const float norm = 0.08838834764831845f;
    float line[128];
    for (int64_t r0 = 0; r0 < rows; r0 += 128)
        for (int64_t c0 = 0; c0 < cols; c0 += 128) {
            for (int r = 0; r < 128; ++r) {
                float* row = m + (r0 + r) * cols + c0;
                for (int c = 0; c < 128; ++c) line[c] = row[c];
                oracle_hadamard(line, 128);
                for (int c = 0; c < 128; ++c) row[c] = line[c] * norm;
            }
            for (int c = 0; c < 128; ++c) {
                for (int r = 0; r < 128; ++r) line[r] = m[(r0 + r) * cols + c0 + c];
                oracle_hadamard(line, 128);
                const float sv = oracle_half_to_float(svh[c0 + c]);
                for (int r = 0; r < 128; ++r) {
                    const float v = line[r] * norm * oracle_half_to_float(suh[r0 + r]) * sv;
                    out[(r0 + r) * cols + c0 + c] = oracle_float_to_half(v);
                }
            }
        }
    free(m);
    return 0;
}

/* Batch helpers for the Python wrapper. */
void oracle_decode_codebook_many(const uint16_t* windows, int64_t n, int cb, uint16_t* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = oracle_decode_codebook(windows[i], cb);
}

void oracle_float_to_half_many(const float* v, int64_t n, uint16_t* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = oracle_float_to_half(v[i]);
}
