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
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

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

/* Lookup tables built once from the restated functions above: the codebook
 * of every 16-bit state for each codebook, and binary16 -> float.  They are
 * the same functions tabulated, so results stay bit-identical; they only
 * take the per-weight cost of the parity checker from ~160 ns to a few. */
static uint16_t g_cb_lut[3][65536];
static float g_h2f_lut[65536];
static pthread_once_t g_lut_once = PTHREAD_ONCE_INIT;

static void build_luts(void) {
    for (uint32_t w = 0; w < 65536u; ++w) {
        for (int cb = 0; cb < 3; ++cb) g_cb_lut[cb][w] = oracle_decode_codebook((uint16_t)w, cb);
        g_h2f_lut[w] = oracle_half_to_float((uint16_t)w);
    }
}

/* One 128x128 block (rows r0.., columns c0..) of the reconstruction, the
 * reference's float rounding order (bindings.cpp:79-98): rows transformed
 * then scaled by norm, columns transformed then multiplied left to right by
 * norm, suh[r], svh[c], then rounded to fp16.  `out` has row pitch `pitch`. */
static void dequant_block(const int16_t* trellis, const uint16_t* suh, const uint16_t* svh, int64_t cols,
                          int K, int cb, int64_t r0, int64_t c0, uint16_t* out, int64_t pitch) {
    const size_t words = (size_t)16 * (size_t)K;
    const int64_t nt_n = cols / 16;
    static const float norm = 0.08838834764831845f;
    float m[128][128];
    float line[128];
    for (int kt = 0; kt < 8; ++kt)
        for (int nt = 0; nt < 8; ++nt) {
            const uint16_t* tile =
                (const uint16_t*)trellis + (size_t)(((r0 / 16) + kt) * nt_n + (c0 / 16) + nt) * words;
            for (int l = 0; l < 32; ++l) {
                const int rr = (l % 4) * 2, cc = l / 4;
                for (int j = 0; j < 8; ++j) {
                    const size_t start = ((size_t)(8 * l + j) + 257u) * (size_t)K - 16u;
                    const uint16_t v = g_cb_lut[cb][oracle_read_window(tile, words, start)];
                    const int row = rr + (j & 1) + ((j & 2) ? 8 : 0);
                    const int col = cc + ((j & 4) ? 8 : 0);
                    m[kt * 16 + row][nt * 16 + col] = g_h2f_lut[v];
                }
            }
        }
    for (int r = 0; r < 128; ++r) {
        oracle_hadamard(m[r], 128);
        for (int c = 0; c < 128; ++c) m[r][c] = m[r][c] * norm;
    }
    for (int c = 0; c < 128; ++c) {
        for (int r = 0; r < 128; ++r) line[r] = m[r][c];
        oracle_hadamard(line, 128);
        const float sv = g_h2f_lut[svh[c0 + c]];
        for (int r = 0; r < 128; ++r) {
            const float v = line[r] * norm * g_h2f_lut[suh[r0 + r]] * sv;
            out[(size_t)r * (size_t)pitch + (size_t)c] = oracle_float_to_half(v);
        }
    }
}

struct dq_job {
    const int16_t* trellis;
    const uint16_t* suh;
    const uint16_t* svh;
    int64_t rows, cols, c0, c1;
    int K, cb;
    uint16_t* out;
    int64_t next;  /* next block index, claimed atomically */
};

static void* dq_worker(void* arg) {
    struct dq_job* j = (struct dq_job*)arg;
    const int64_t ncb = (j->c1 - j->c0) / 128, nblk = (j->rows / 128) * ncb;
    const int64_t pitch = j->c1 - j->c0;
    for (;;) {
        const int64_t b = __atomic_fetch_add(&j->next, 1, __ATOMIC_RELAXED);
        if (b >= nblk) break;
        const int64_t r0 = (b / ncb) * 128, cb0 = (b % ncb) * 128;
        dequant_block(j->trellis, j->suh, j->svh, j->cols, j->K, j->cb, r0, j->c0 + cb0,
                      j->out + (size_t)r0 * (size_t)pitch + (size_t)cb0, pitch);
    }
    return NULL;
}

static int oracle_threads(void) {
    const char* e = getenv("EXL3_ORACLE_THREADS");
    long n = e ? strtol(e, NULL, 10) : sysconf(_SC_NPROCESSORS_ONLN);
    if (n < 1) n = 1;
    if (n > 64) n = 64;
    return (int)n;
}

/* Columns [c0, c1) (multiples of 128) of W = diag(suh) H W~ H diag(svh) /
 * 128 as fp16 bits, out [rows][c1 - c0].  The 128x128 blocks are
 * independent, so any column range is exactly the corresponding columns of
 * the full reconstruction.  Blocks are spread over host threads.
 * Returns 0, -1 for dimensions that are not whole blocks (bindings.cpp:22). */
int oracle_dequant_cols(const int16_t* trellis, const uint16_t* suh, const uint16_t* svh, int64_t rows,
                        int64_t cols, int K, int cb, int64_t c0, int64_t c1, uint16_t* out) {
    if (rows % 128 || cols % 128 || rows <= 0 || cols <= 0) return -1;
    if (c0 < 0 || c1 > cols || c0 >= c1 || c0 % 128 || c1 % 128) return -1;
    if (K < 1 || K > 8 || cb < 0 || cb > 2) return -1;
    pthread_once(&g_lut_once, build_luts);
    struct dq_job job = {trellis, suh, svh, rows, cols, c0, c1, K, cb, out, 0};
    const int64_t nblk = (rows / 128) * ((c1 - c0) / 128);
    int nt = oracle_threads();
    if (nt > nblk) nt = (int)nblk;
    pthread_t th[64];
    int started = 0;
    for (int t = 1; t < nt; ++t)
        if (pthread_create(&th[started], NULL, dq_worker, &job) == 0) ++started;
    dq_worker(&job);
    for (int t = 0; t < started; ++t) pthread_join(th[t], NULL);
    return 0;
}

/* Full reconstruction (bindings.cpp:15-100): every column. */
int oracle_dequant(const int16_t* trellis, const uint16_t* suh, const uint16_t* svh,
                   int64_t rows, int64_t cols, int K, int cb, uint16_t* out) {
    return oracle_dequant_cols(trellis, suh, svh, rows, cols, K, cb, 0, cols, out);
}

/* Batch helpers for the Python wrapper. */
void oracle_decode_codebook_many(const uint16_t* windows, int64_t n, int cb, uint16_t* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = oracle_decode_codebook(windows[i], cb);
}

void oracle_float_to_half_many(const float* v, int64_t n, uint16_t* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = oracle_float_to_half(v[i]);
}
