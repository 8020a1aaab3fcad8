// capi.cu -- the extern "C" boundary (include/exl3_b200.h).  Host-side
// validation mirrors the reference's TORCH_CHECKs (csrc/bindings.cpp:117-147,
// csrc/p2b_moe.cu:2437-2466, 2346-2428): everything is rejected before launch
// with a message; nothing here reads device memory except exl3_device_status.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/exl3_b200.h"
#include "exl3_internal.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(EXL3_ERR_CUDA, "%s: CUDA error %d (%s)", what, int(e), cudaGetErrorString(e));
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

bool float_dtype(int d) { return d == EXL3_DT_F32 || d == EXL3_DT_F16 || d == EXL3_DT_BF16; }

int check_packed(const char* who, const void* trellis, const void* suh, const void* svh,
                 int64_t in_f, int64_t out_f, int K, int cb) {
    if (!trellis || !suh || !svh) return fail(EXL3_ERR_ARG, "%s: null trellis/suh/svh pointer", who);
    if (K < 2 || K > 8) return fail(EXL3_ERR_ARG, "%s: K must be in 2..8 (got %d)", who, K);
    if (cb < 0 || cb > 2) return fail(EXL3_ERR_ARG, "%s: codebook must be 0, 1 or 2 (got %d)", who, cb);
    if (in_f <= 0 || out_f <= 0 || in_f % 128 || out_f % 128)
        return fail(EXL3_ERR_ARG,
                    "%s: trellis dimensions must reconstruct whole 128-element Hadamard blocks "
                    "(in=%lld out=%lld)",
                    who, (long long)in_f, (long long)out_f);
    if (!aligned(trellis, 16)) return fail(EXL3_ERR_ARG, "%s: trellis must be 16-byte aligned", who);
    if (!aligned(suh, 2) || !aligned(svh, 2)) return fail(EXL3_ERR_ARG, "%s: suh/svh misaligned", who);
    return EXL3_OK;
}

}  // namespace

namespace exl3 {
// lets other translation units of the library report through exl3_last_error
void set_last_error(const char* msg) { g_last_error = msg; }
}  // namespace exl3

extern "C" {

int exl3_abi_version(void) { return EXL3_B200_ABI_VERSION; }

const char* exl3_last_error(void) { return g_last_error.c_str(); }

int exl3_device_status(const void* workspace, int clear, void* stream, int* status_out) {
    if (!workspace || !status_out) return fail(EXL3_ERR_ARG, "exl3_device_status: null argument");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int v = 0;
    cudaError_t e = cudaMemcpyAsync(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "exl3_device_status");
    if (clear && v) {
        e = cudaMemsetAsync(const_cast<void*>(workspace), 0, sizeof(int), s);
        if (e != cudaSuccess) return cuda_fail(e, "exl3_device_status");
    }
    *status_out = v;
    return EXL3_OK;
}

int exl3_reconstruct(const void* trellis, const void* suh, const void* svh, int64_t in_f, int64_t out_f,
                     int K, int cb, void* w_out, void* stream) {
    if (int rc = check_packed("exl3_reconstruct", trellis, suh, svh, in_f, out_f, K, cb)) return rc;
    if (!w_out) return fail(EXL3_ERR_ARG, "exl3_reconstruct: null output");
    cudaError_t e = exl3::run_reconstruct(K, cb, true, trellis, suh, svh, in_f, out_f, w_out,
                                          static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? EXL3_OK : cuda_fail(e, "exl3_reconstruct");
}

int exl3_decode_raw(const void* trellis, int64_t in_f, int64_t out_f, int K, int cb, void* w_out,
                    void* stream) {
    static const uint16_t one = 0x3c00;  // placeholder scales: unused by the raw decode
    if (int rc = check_packed("exl3_decode_raw", trellis, &one, &one, in_f, out_f, K, cb)) return rc;
    if (!w_out) return fail(EXL3_ERR_ARG, "exl3_decode_raw: null output");
    cudaError_t e = exl3::run_reconstruct(K, cb, false, trellis, nullptr, nullptr, in_f, out_f, w_out,
                                          static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? EXL3_OK : cuda_fail(e, "exl3_decode_raw");
}

int exl3_had128(const void* x, void* y, int64_t rows, int64_t n, const void* pre, const void* post,
                float scale, void* stream) {
    if (!x || !y) return fail(EXL3_ERR_ARG, "exl3_had128: null input/output");
    if (rows < 0 || n <= 0 || n % 128)
        return fail(EXL3_ERR_ARG, "exl3_had128: row width must be a positive multiple of 128");
    if (!std::isfinite(scale)) return fail(EXL3_ERR_ARG, "exl3_had128: scale must be finite");
    if (rows == 0) return EXL3_OK;
    cudaError_t e = exl3::run_had128(x, y, rows, n, pre, post, scale, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? EXL3_OK : cuda_fail(e, "exl3_had128");
}

size_t exl3_linear_workspace_size(int64_t m, int64_t in_f, int64_t out_f, int K) {
    exl3::MoePlan p;
    if (m < 1 || in_f > INT32_MAX || out_f > INT32_MAX) return 0;
    if (!exl3::plan_moe(p, m, 1, int(in_f), int(out_f), 1, K < 2 ? 8 : K, true, exl3::num_sms_current()))
        return 0;
    return p.total;
}

int exl3_linear(const void* x, int x_dtype, int64_t m, const void* trellis, const void* suh,
                const void* svh, int64_t in_f, int64_t out_f, int K, int cb, void* y, int y_dtype,
                void* ws, size_t ws_bytes, void* stream) {
    if (int rc = check_packed("exl3_linear", trellis, suh, svh, in_f, out_f, K, cb)) return rc;
    if (!x || !y) return fail(EXL3_ERR_ARG, "exl3_linear: null x/y");
    if (!float_dtype(x_dtype) || !float_dtype(y_dtype))
        return fail(EXL3_ERR_ARG, "exl3_linear: x/y dtype must be fp32, fp16 or bf16");
    if (m < 0) return fail(EXL3_ERR_ARG, "exl3_linear: m must be >= 0");
    if (m == 0) return EXL3_OK;
    if (in_f > INT32_MAX || out_f > INT32_MAX || m * in_f > (int64_t(1) << 40))
        return fail(EXL3_ERR_ARG, "exl3_linear: dimensions exceed kernel indexing");
    exl3::MoePlan p;
    if (!exl3::plan_moe(p, m, 1, int(in_f), int(out_f), 1, K, true, exl3::num_sms_current(), true, cb))
        return fail(EXL3_ERR_ARG, "exl3_linear: unsupported geometry");
    if (!ws || ws_bytes < p.total)
        return fail(EXL3_ERR_WORKSPACE, "exl3_linear: workspace of %zu bytes required (got %zu)", p.total,
                    ws_bytes);
    if (!aligned(ws, 256)) return fail(EXL3_ERR_WORKSPACE, "exl3_linear: workspace must be 256-byte aligned");
    exl3::MoeCall c;
    c.x = x;
    c.x_dtype = x_dtype;
    c.up.trellis = trellis;
    c.up.suh = suh;
    c.up.svh = svh;
    c.up.k_uniform = K;
    c.cb = cb;
    c.out = y;
    c.out_dtype = y_dtype;
    cudaError_t e = exl3::run_moe(p, c, ws, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? EXL3_OK : cuda_fail(e, "exl3_linear");
}

size_t exl3_moe_workspace_size(int64_t tokens, int topk, int64_t hidden, int64_t inter, int n_local,
                               int kmax) {
    exl3::MoePlan p;
    if (hidden > INT32_MAX || inter > INT32_MAX) return 0;
    if (!exl3::plan_moe(p, tokens, topk, int(hidden), int(inter), n_local, kmax, false,
                        exl3::num_sms_current()))
        return 0;
    return p.total;
}

int exl3_moe_forward(const void* x, int x_dtype, int64_t tokens, int64_t hidden, int64_t inter,
                     const int64_t* gt, const int64_t* gu, const int64_t* gv, const int64_t* ut,
                     const int64_t* uu, const int64_t* uv, const int64_t* dt, const int64_t* du,
                     const int64_t* dv, const void* ids, int ids_dtype, const void* weights,
                     int w_dtype, int topk, const int32_t* expert_map, int64_t n_global,
                     const int8_t* kg, const int8_t* ku, const int8_t* kd, int k_uniform, int kmax,
                     int n_local, int cb, int act, float limit, const int32_t* n_valid, void* out,
                     int out_dtype, void* ws, size_t ws_bytes, void* stream) {
    const char* who = "fused MoE";
    if (!x || !out) return fail(EXL3_ERR_ARG, "%s: null x/out", who);
    if (!gt || !gu || !gv || !ut || !uu || !uv || !dt || !du || !dv)
        return fail(EXL3_ERR_ARG, "%s: null pointer table", who);
    if (!ids || !weights) return fail(EXL3_ERR_ARG, "%s: null routing tensors", who);
    if (!float_dtype(x_dtype) || !float_dtype(out_dtype) || !float_dtype(w_dtype))
        return fail(EXL3_ERR_ARG, "%s: x/out/weights dtype must be fp32, fp16 or bf16", who);
    if (ids_dtype != EXL3_DT_I32 && ids_dtype != EXL3_DT_I64)
        return fail(EXL3_ERR_ARG, "%s: expert ids must be int32 or int64", who);
    if (tokens < 0) return fail(EXL3_ERR_ARG, "%s: tokens must be >= 0", who);
    if (hidden <= 0 || hidden % 128 || hidden > INT32_MAX)
        return fail(EXL3_ERR_ARG, "%s hidden width must be a positive multiple of 128", who);
    if (inter <= 0 || inter % 128 || inter > INT32_MAX)
        return fail(EXL3_ERR_ARG, "%s local intermediate width must be a positive multiple of 128", who);
    if (topk < 1) return fail(EXL3_ERR_ARG, "%s: topk must be >= 1", who);
    if (n_local < 1 || n_local > 2048) return fail(EXL3_ERR_ARG, "%s: n_local must be in 1..2048", who);
    if (!std::isfinite(limit) || limit < 0.f)
        return fail(EXL3_ERR_ARG,
                    "%s SwiGLU limit must be finite and nonnegative (0 disables clipping)", who);
    if (cb < 0 || cb > 2) return fail(EXL3_ERR_ARG, "%s: codebook must be 0, 1 or 2", who);
    if (act != EXL3_ACT_SILU && act != EXL3_ACT_SWIGLU_OAI && act != EXL3_ACT_RELU2)
        return fail(EXL3_ERR_ARG, "%s: unsupported activation %d", who, act);
    if (kmax < 2 || kmax > 8) return fail(EXL3_ERR_ARG, "%s: kmax must be in 2..8", who);
    const bool tables = kg || ku || kd;
    if (tables && !(kg && ku && kd))
        return fail(EXL3_ERR_ARG, "%s: K tables must be given together", who);
    if (!tables && (k_uniform < 2 || k_uniform > kmax))
        return fail(EXL3_ERR_ARG, "%s: uniform K must be in 2..kmax", who);
    if (expert_map && n_global < 1) return fail(EXL3_ERR_ARG, "%s: expert_map needs n_global >= 1", who);
    if (tokens == 0) return EXL3_OK;
    exl3::MoePlan p;
    if (!exl3::plan_moe(p, tokens, topk, int(hidden), int(inter), n_local, kmax, false,
                        exl3::num_sms_current(), true, cb))
        return fail(EXL3_ERR_ARG, "%s: unsupported geometry", who);
    if (!ws || ws_bytes < p.total)
        return fail(EXL3_ERR_WORKSPACE, "%s: workspace of %zu bytes required (got %zu)", who, p.total,
                    ws_bytes);
    if (!aligned(ws, 256)) return fail(EXL3_ERR_WORKSPACE, "%s: workspace must be 256-byte aligned", who);

    exl3::MoeCall c;
    c.x = x;
    c.x_dtype = x_dtype;
    c.ids = ids;
    c.ids_dtype = ids_dtype;
    c.weights = weights;
    c.w_dtype = w_dtype;
    c.expert_map = expert_map;
    c.n_global = n_global;
    c.n_valid = n_valid;
    c.gate = {gt, gu, gv, kg, nullptr, nullptr, nullptr, k_uniform};
    c.up = {ut, uu, uv, ku, nullptr, nullptr, nullptr, k_uniform};
    c.down = {dt, du, dv, kd, nullptr, nullptr, nullptr, k_uniform};
    c.cb = cb;
    c.act = act;
    c.limit = limit;
    c.out = out;
    c.out_dtype = out_dtype;
    cudaError_t e = exl3::run_moe(p, c, ws, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? EXL3_OK : cuda_fail(e, "fused MoE launch");
}

size_t exl3_batched_linear_workspace_size(int64_t m, int n_active, int64_t in_f, int64_t out_f,
                                          int n_table, int K) {
    exl3::MoePlan p;
    if (m < 1 || n_active < 1 || in_f > INT32_MAX || out_f > INT32_MAX) return 0;
    if (!exl3::plan_moe(p, m, n_active, int(in_f), int(out_f), n_table, K < 2 ? 8 : K, true,
                        exl3::num_sms_current(), false))
        return 0;
    return p.total;
}

int exl3_batched_linear(const void* x, int x_dtype, int64_t m, const int64_t* trellis_ptrs,
                        const int64_t* suh_ptrs, const int64_t* svh_ptrs, int n_table,
                        const int32_t* expert_indices, int n_active, int64_t in_f, int64_t out_f, int K,
                        int cb, void* y, int y_dtype, void* ws, size_t ws_bytes, void* stream) {
    const char* who = "batched GEMV";
    if (!x || !y || !trellis_ptrs || !suh_ptrs || !svh_ptrs || !expert_indices)
        return fail(EXL3_ERR_ARG, "%s: null argument", who);
    if (!float_dtype(x_dtype) || !float_dtype(y_dtype))
        return fail(EXL3_ERR_ARG, "%s: x/y dtype must be fp32, fp16 or bf16", who);
    if (K < 2 || K > 8) return fail(EXL3_ERR_ARG, "%s supports K in 2..8", who);
    if (cb < 0 || cb > 2) return fail(EXL3_ERR_ARG, "%s: codebook must be 0, 1 or 2", who);
    if (in_f <= 0 || out_f <= 0 || in_f % 128 || out_f % 128 || in_f > INT32_MAX || out_f > INT32_MAX)
        return fail(EXL3_ERR_ARG, "%s: in/out features must be positive multiples of 128", who);
    if (n_table < 1 || n_table > 2048) return fail(EXL3_ERR_ARG, "%s: table length must be in 1..2048", who);
    if (n_active < 1 || m < 1) return fail(EXL3_ERR_ARG, "%s: need m >= 1 and at least one expert", who);
    exl3::MoePlan p;
    if (!exl3::plan_moe(p, m, n_active, int(in_f), int(out_f), n_table, K, true, exl3::num_sms_current(), false,
                        cb))
        return fail(EXL3_ERR_ARG, "%s: unsupported geometry", who);
    if (!ws || ws_bytes < p.total)
        return fail(EXL3_ERR_WORKSPACE, "%s: workspace of %zu bytes required (got %zu)", who, p.total, ws_bytes);
    if (!aligned(ws, 256)) return fail(EXL3_ERR_WORKSPACE, "%s: workspace must be 256-byte aligned", who);
    exl3::MoeCall c;
    c.x = x;
    c.x_dtype = x_dtype;
    c.ids = expert_indices;
    c.ids_dtype = EXL3_DT_I32;
    c.up = {trellis_ptrs, suh_ptrs, svh_ptrs, nullptr, nullptr, nullptr, nullptr, K};
    c.cb = cb;
    c.out = y;
    c.out_dtype = y_dtype;
    c.batched = true;
    cudaError_t e = exl3::run_moe(p, c, ws, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? EXL3_OK : cuda_fail(e, who);
}

int exl3_fat_gemm(const void* a, int64_t m, const void* packed, const void* svh, int64_t in_f,
                  int64_t out_f, int K, int cb, float* out, const int64_t* token_idx,
                  const void* route_weight, void* ws, size_t ws_bytes, void* stream) {
    static const uint16_t one = 0x3c00;  // the input is pre-rotated: no suh is read
    if (int rc = check_packed("exl3_fat_gemm", packed, &one, svh, in_f, out_f, K, cb)) return rc;
    if (!a || !out) return fail(EXL3_ERR_ARG, "exl3_fat_gemm: null a/out");
    if ((token_idx == nullptr) != (route_weight == nullptr))
        return fail(EXL3_ERR_ARG, "exl3_fat_gemm: token_idx and route_weight go together");
    if (m < 0) return fail(EXL3_ERR_ARG, "exl3_fat_gemm: m must be >= 0");
    if (m == 0) return EXL3_OK;
    exl3::MoePlan p;
    if (in_f > INT32_MAX || out_f > INT32_MAX ||
        !exl3::plan_moe(p, m, 1, int(in_f), int(out_f), 1, K, true, exl3::num_sms_current(), true, cb))
        return fail(EXL3_ERR_ARG, "exl3_fat_gemm: unsupported geometry");
    if (!ws || ws_bytes < p.total)
        return fail(EXL3_ERR_WORKSPACE, "exl3_fat_gemm: workspace of %zu bytes required (got %zu)", p.total,
                    ws_bytes);
    if (!aligned(ws, 256)) return fail(EXL3_ERR_WORKSPACE, "exl3_fat_gemm: workspace must be 256-byte aligned");
    exl3::MoeCall c;
    c.x = a;
    c.x_dtype = EXL3_DT_F16;
    c.up.trellis = packed;
    c.up.svh = svh;
    c.up.k_uniform = K;
    c.cb = cb;
    c.out = out;
    c.out_dtype = EXL3_DT_F32;
    c.prerotated = true;
    c.scatter_idx = token_idx;
    c.scatter_w = route_weight;
    cudaError_t e = exl3::run_moe(p, c, ws, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? EXL3_OK : cuda_fail(e, "exl3_fat_gemm");
}

int exl3_ep_dispatch(const void* x, int x_dtype, int64_t tokens, int64_t hidden, const void* ids, int ids_dtype,
                     const void* weights, int w_dtype, int topk, int64_t n_global, int world,
                     const int32_t* n_valid, void* send_x, int32_t* send_ids, float* send_w, int32_t* send_tok,
                     int32_t* pair_idx, int32_t* send_counts, int64_t capacity, void* stream) {
    const char* who = "exl3_ep_dispatch";
    if (!x || !ids || !weights) return fail(EXL3_ERR_ARG, "%s: null x/ids/weights", who);
    if (!send_x || !send_ids || !send_w || !send_tok || !pair_idx || !send_counts)
        return fail(EXL3_ERR_ARG, "%s: null output buffer", who);
    if (!float_dtype(x_dtype) || !float_dtype(w_dtype))
        return fail(EXL3_ERR_ARG, "%s: x/weights dtype must be fp32, fp16 or bf16", who);
    if (ids_dtype != EXL3_DT_I32 && ids_dtype != EXL3_DT_I64)
        return fail(EXL3_ERR_ARG, "%s: expert ids must be int32 or int64", who);
    if (world < 1 || world > exl3::kEpMaxWorld)
        return fail(EXL3_ERR_ARG, "%s: world size must be in 1..%d", who, exl3::kEpMaxWorld);
    if (n_global < world || n_global % world)
        return fail(EXL3_ERR_ARG, "%s: %lld experts do not split evenly over %d ranks", who, (long long)n_global,
                    world);
    if (topk < 1 || topk > 64) return fail(EXL3_ERR_ARG, "%s: topk must be in 1..64", who);
    if (tokens < 0 || tokens * int64_t(world) > INT32_MAX)
        return fail(EXL3_ERR_ARG, "%s: tokens x world must fit int32", who);
    if (hidden <= 0 || hidden % 128 || hidden > INT32_MAX)
        return fail(EXL3_ERR_ARG, "%s: hidden width must be a positive multiple of 128", who);
    if (!aligned(x, 16) || !aligned(send_x, 16)) return fail(EXL3_ERR_ARG, "%s: x/send_x must be 16-byte aligned", who);
    if (capacity < 0 || (capacity > 0 && capacity < tokens) || capacity * int64_t(world) > INT32_MAX)
        return fail(EXL3_ERR_ARG, "%s: capacity must be 0 or in [tokens, INT32_MAX / world] (got %lld)", who,
                    (long long)capacity);
    exl3::EpDispatchCall c;
    c.x = x;
    c.x_esize = x_dtype == EXL3_DT_F32 ? 4 : 2;
    c.tokens = tokens;
    c.hidden = int(hidden);
    c.ids = ids;
    c.ids_dtype = ids_dtype;
    c.weights = weights;
    c.w_dtype = w_dtype;
    c.topk = topk;
    c.n_global = n_global;
    c.world = world;
    c.n_valid = n_valid;
    c.send_x = send_x;
    c.send_ids = send_ids;
    c.send_w = send_w;
    c.send_tok = send_tok;
    c.pair_idx = pair_idx;
    c.send_counts = send_counts;
    c.capacity = capacity;
    cudaError_t e = exl3::run_ep_dispatch(c, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? EXL3_OK : cuda_fail(e, who);
}

int exl3_ep_combine(const void* partial, int partial_dtype, const int32_t* pair_idx, int64_t tokens, int world,
                    int64_t hidden, const int32_t* n_valid, void* out, int out_dtype, void* stream) {
    const char* who = "exl3_ep_combine";
    if (!partial || !pair_idx || !out) return fail(EXL3_ERR_ARG, "%s: null argument", who);
    if (!float_dtype(partial_dtype) || !float_dtype(out_dtype))
        return fail(EXL3_ERR_ARG, "%s: partial/out dtype must be fp32, fp16 or bf16", who);
    if (world < 1 || world > exl3::kEpMaxWorld)
        return fail(EXL3_ERR_ARG, "%s: world size must be in 1..%d", who, exl3::kEpMaxWorld);
    if (tokens < 0 || tokens * int64_t(world) > INT32_MAX)
        return fail(EXL3_ERR_ARG, "%s: tokens x world must fit int32", who);
    if (hidden <= 0 || hidden % 128 || hidden > INT32_MAX)
        return fail(EXL3_ERR_ARG, "%s: hidden width must be a positive multiple of 128", who);
    if (!aligned(partial, 16) || !aligned(out, 16))
        return fail(EXL3_ERR_ARG, "%s: partial/out must be 16-byte aligned", who);
    cudaError_t e = exl3::run_ep_combine(partial, partial_dtype, pair_idx, tokens, world, int(hidden), n_valid, out,
                                         out_dtype, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? EXL3_OK : cuda_fail(e, who);
}

size_t exl3_ep_window_size(int world, int64_t capacity, int64_t hidden, int topk, int x_dtype, int partial_dtype) {
    if (world < 1 || world > exl3::kEpMaxWorld || capacity < 1 || hidden <= 0 || hidden % 128 || topk < 1 ||
        topk > 64 || !float_dtype(x_dtype) || !float_dtype(partial_dtype))
        return 0;
    return exl3::ep_window(world, capacity, hidden, topk, x_dtype == EXL3_DT_F32 ? 4 : 2,
                           partial_dtype == EXL3_DT_F32 ? 4 : 2)
        .total;
}

int exl3_ep_window_alloc(size_t bytes, void** window) {
    if (!window || bytes == 0) return fail(EXL3_ERR_ARG, "exl3_ep_window_alloc: bad arguments");
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
    if (e != cudaSuccess) {
        if (p) cudaFree(p);
        return cuda_fail(e, "exl3_ep_window_alloc");
    }
    *window = p;
    return EXL3_OK;
}

int exl3_ep_window_free(void* window) {
    if (!window) return EXL3_OK;
    cudaError_t e = cudaFree(window);
    return e == cudaSuccess ? EXL3_OK : cuda_fail(e, "exl3_ep_window_free");
}

int exl3_ep_ipc_handle(const void* window, void* handle) {
    if (!window || !handle) return fail(EXL3_ERR_ARG, "exl3_ep_ipc_handle: null argument");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(window));
    if (e != cudaSuccess) return cuda_fail(e, "exl3_ep_ipc_handle");
    memcpy(handle, &h, sizeof(h));
    return EXL3_OK;
}

int exl3_ep_ipc_open(const void* handle, void** mapped) {
    if (!handle || !mapped) return fail(EXL3_ERR_ARG, "exl3_ep_ipc_open: null argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(mapped, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? EXL3_OK : cuda_fail(e, "exl3_ep_ipc_open");
}

int exl3_ep_ipc_close(void* mapped) {
    if (!mapped) return EXL3_OK;
    cudaError_t e = cudaIpcCloseMemHandle(mapped);
    return e == cudaSuccess ? EXL3_OK : cuda_fail(e, "exl3_ep_ipc_close");
}

static int ep_p2p_common(const char* who, int world, int rank, int64_t capacity, int64_t hidden, int topk, int x_dtype,
                         int partial_dtype, const void* window, const int64_t* peers) {
    if (!window || !peers) return fail(EXL3_ERR_ARG, "%s: null window/peers", who);
    if (world < 1 || world > exl3::kEpMaxWorld || rank < 0 || rank >= world)
        return fail(EXL3_ERR_ARG, "%s: bad world/rank", who);
    if (capacity < 1 || capacity * int64_t(world) > INT32_MAX) return fail(EXL3_ERR_ARG, "%s: bad capacity", who);
    if (hidden <= 0 || hidden % 128 || hidden > INT32_MAX)
        return fail(EXL3_ERR_ARG, "%s: hidden width must be a positive multiple of 128", who);
    if (topk < 1 || topk > 64) return fail(EXL3_ERR_ARG, "%s: topk must be in 1..64", who);
    if (!float_dtype(x_dtype) || !float_dtype(partial_dtype)) return fail(EXL3_ERR_ARG, "%s: bad dtype", who);
    if (!aligned(window, 256)) return fail(EXL3_ERR_ARG, "%s: window must be 256-byte aligned", who);
    return EXL3_OK;
}

static exl3::EpP2pCall ep_p2p_call(int phase, int world, int rank, int64_t capacity, int64_t hidden, int topk,
                                   int x_dtype, int partial_dtype, void* window, const int64_t* peers) {
    exl3::EpP2pCall c;
    c.phase = phase;
    c.world = world;
    c.rank = rank;
    c.capacity = capacity;
    c.hidden = hidden;
    c.topk = topk;
    c.x_esize = x_dtype == EXL3_DT_F32 ? 4 : 2;
    c.p_esize = partial_dtype == EXL3_DT_F32 ? 4 : 2;
    c.p_dtype = partial_dtype;
    c.window = window;
    c.peers = peers;
    return c;
}

int exl3_ep_p2p_dispatch(const void* x, int x_dtype, int64_t tokens, int64_t hidden, const void* ids, int ids_dtype,
                         const void* weights, int w_dtype, int topk, int64_t n_global, int world, int rank,
                         int64_t capacity, const int32_t* n_valid, void* window, const int64_t* peers,
                         int partial_dtype, int32_t* pair_idx, void* stream) {
    const char* who = "exl3_ep_p2p_dispatch";
    if (int rc = ep_p2p_common(who, world, rank, capacity, hidden, topk, x_dtype, partial_dtype, window, peers))
        return rc;
    if (!x || !ids || !weights || !pair_idx) return fail(EXL3_ERR_ARG, "%s: null argument", who);
    if (ids_dtype != EXL3_DT_I32 && ids_dtype != EXL3_DT_I64)
        return fail(EXL3_ERR_ARG, "%s: expert ids must be int32 or int64", who);
    if (!float_dtype(w_dtype)) return fail(EXL3_ERR_ARG, "%s: bad weights dtype", who);
    if (n_global < world || n_global % world)
        return fail(EXL3_ERR_ARG, "%s: %lld experts do not split evenly over %d ranks", who, (long long)n_global,
                    world);
    if (tokens < 0 || tokens > capacity) return fail(EXL3_ERR_ARG, "%s: tokens must be in [0, capacity]", who);
    if (!aligned(x, 16)) return fail(EXL3_ERR_ARG, "%s: x must be 16-byte aligned", who);
    exl3::EpP2pCall c = ep_p2p_call(exl3::EP_P2P_DISPATCH, world, rank, capacity, hidden, topk, x_dtype,
                                    partial_dtype, window, peers);
    c.x = x;
    c.tokens = tokens;
    c.ids = ids;
    c.ids_dtype = ids_dtype;
    c.weights = weights;
    c.w_dtype = w_dtype;
    c.n_global = n_global;
    c.n_valid = n_valid;
    c.pair_idx = pair_idx;
    cudaError_t e = exl3::run_ep_p2p(c, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? EXL3_OK : cuda_fail(e, who);
}

int exl3_ep_p2p_wait(void* window, int world, int phase, void* stream) {
    const char* who = "exl3_ep_p2p_wait";
    if (!window || world < 1 || world > exl3::kEpMaxWorld || (phase != 0 && phase != 1))
        return fail(EXL3_ERR_ARG, "%s: bad arguments", who);
    exl3::EpP2pCall c;
    c.phase = phase == 0 ? exl3::EP_P2P_WAIT_ARRIVE : exl3::EP_P2P_WAIT_RETURN;
    c.world = world;
    c.window = window;
    cudaError_t e = exl3::run_ep_p2p(c, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? EXL3_OK : cuda_fail(e, who);
}

int exl3_ep_p2p_return(const void* partial, int partial_dtype, int world, int rank, int64_t capacity, int64_t hidden,
                       int topk, int x_dtype, void* window, const int64_t* peers, void* stream) {
    const char* who = "exl3_ep_p2p_return";
    if (int rc = ep_p2p_common(who, world, rank, capacity, hidden, topk, x_dtype, partial_dtype, window, peers))
        return rc;
    if (!partial || !aligned(partial, 16)) return fail(EXL3_ERR_ARG, "%s: partial must be 16-byte aligned", who);
    exl3::EpP2pCall c = ep_p2p_call(exl3::EP_P2P_RETURN, world, rank, capacity, hidden, topk, x_dtype,
                                    partial_dtype, window, peers);
    c.partial = partial;
    cudaError_t e = exl3::run_ep_p2p(c, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? EXL3_OK : cuda_fail(e, who);
}

int exl3_ep_p2p_combine(void* window, int world, int rank, int64_t capacity, int64_t hidden, int topk, int x_dtype,
                        int partial_dtype, const int32_t* pair_idx, int64_t tokens, const int32_t* n_valid, void* out,
                        int out_dtype, void* stream) {
    const char* who = "exl3_ep_p2p_combine";
    static const int64_t dummy = 0;
    if (int rc = ep_p2p_common(who, world, rank, capacity, hidden, topk, x_dtype, partial_dtype, window, &dummy))
        return rc;
    if (!pair_idx || !out || !aligned(out, 16)) return fail(EXL3_ERR_ARG, "%s: bad pair_idx/out", who);
    if (!float_dtype(out_dtype)) return fail(EXL3_ERR_ARG, "%s: bad out dtype", who);
    if (tokens < 0 || tokens > capacity) return fail(EXL3_ERR_ARG, "%s: tokens must be in [0, capacity]", who);
    exl3::EpP2pCall c = ep_p2p_call(exl3::EP_P2P_COMBINE, world, rank, capacity, hidden, topk, x_dtype,
                                    partial_dtype, window, nullptr);
    c.pair_idx = const_cast<int32_t*>(pair_idx);
    c.tokens = tokens;
    c.n_valid = n_valid;
    c.out = out;
    c.out_dtype = out_dtype;
    cudaError_t e = exl3::run_ep_p2p(c, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? EXL3_OK : cuda_fail(e, who);
}

int exl3_ep_window_recv(int world, int64_t capacity, int64_t hidden, int topk, int x_dtype, int partial_dtype,
                        size_t* x_off, size_t* ids_off, size_t* w_off) {
    if (!x_off || !ids_off || !w_off ||
        exl3_ep_window_size(world, capacity, hidden, topk, x_dtype, partial_dtype) == 0)
        return fail(EXL3_ERR_ARG, "exl3_ep_window_recv: bad geometry");
    const exl3::EpWindow L = exl3::ep_window(world, capacity, hidden, topk, x_dtype == EXL3_DT_F32 ? 4 : 2,
                                             partial_dtype == EXL3_DT_F32 ? 4 : 2);
    *x_off = L.recv_x;
    *ids_off = L.recv_ids;
    *w_off = L.recv_w;
    return EXL3_OK;
}

int exl3_profile_enable(int on, long long delay_cycles) {
    exl3::profile_enable(on != 0, delay_cycles);
    return EXL3_OK;
}

int exl3_profile_read(float* ms, int max_phases, int* n_phases) {
    if (!ms || !n_phases || max_phases < 1) return fail(EXL3_ERR_ARG, "exl3_profile_read: bad arguments");
    const int n = exl3::profile_read(ms, max_phases);
    if (n < 0) return fail(EXL3_ERR_CUDA, "exl3_profile_read: event query failed");
    *n_phases = n;
    return EXL3_OK;
}


int exl3_ngram_dequant(const void* packed, int64_t n, int bits, const int32_t* heads, const void* head_bias,
                       int num_heads, void* out, int out_dtype, void* stream) {
    const char* who = "exl3_ngram_dequant";
    if (n < 0) return fail(EXL3_ERR_ARG, "%s: n must be >= 0", who);
    if (bits < 1 || bits > 8) return fail(EXL3_ERR_ARG, "%s: bits must be in 1..8 (got %d)", who, bits);
    if (num_heads < 1) return fail(EXL3_ERR_ARG, "%s: num_heads must be >= 1", who);
    if (!float_dtype(out_dtype)) return fail(EXL3_ERR_ARG, "%s: out dtype must be fp32, fp16 or bf16", who);
    if (n == 0) return EXL3_OK;
    if (!packed || !heads || !head_bias || !out) return fail(EXL3_ERR_ARG, "%s: null pointer", who);
    if (!aligned(packed, 2) || !aligned(head_bias, 2)) return fail(EXL3_ERR_ARG, "%s: misaligned fp16/int16 data", who);
    cudaError_t e = exl3::run_ngram(static_cast<const uint16_t*>(packed), n, n, bits, nullptr, EXL3_DT_I32, heads,
                                    nullptr, num_heads, head_bias, out, out_dtype, nullptr,
                                    static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? EXL3_OK : cuda_fail(e, who);
}

int exl3_ngram_lookup(const void* table, int64_t n_rows, int bits, const void* ids, int ids_dtype, int64_t n,
                      const int64_t* head_offsets, int num_heads, const void* head_bias, void* out, int out_dtype,
                      int* status, void* stream) {
    const char* who = "exl3_ngram_lookup";
    if (n < 0 || n_rows < 0) return fail(EXL3_ERR_ARG, "%s: n and n_rows must be >= 0", who);
    if (bits < 1 || bits > 8) return fail(EXL3_ERR_ARG, "%s: bits must be in 1..8 (got %d)", who, bits);
    if (num_heads < 1) return fail(EXL3_ERR_ARG, "%s: num_heads must be >= 1", who);
    if (ids_dtype != EXL3_DT_I32 && ids_dtype != EXL3_DT_I64)
        return fail(EXL3_ERR_ARG, "%s: ids must be int32 or int64", who);
    if (!float_dtype(out_dtype)) return fail(EXL3_ERR_ARG, "%s: out dtype must be fp32, fp16 or bf16", who);
    if (n == 0) return EXL3_OK;
    if (!table || !ids || !head_offsets || !head_bias || !out) return fail(EXL3_ERR_ARG, "%s: null pointer", who);
    if (!aligned(table, 2) || !aligned(head_bias, 2)) return fail(EXL3_ERR_ARG, "%s: misaligned fp16/int16 data", who);
    cudaError_t e = exl3::run_ngram(static_cast<const uint16_t*>(table), n, n_rows, bits, ids, ids_dtype, nullptr,
                                    head_offsets, num_heads, head_bias, out, out_dtype, status,
                                    static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? EXL3_OK : cuda_fail(e, who);
}

}  // extern "C"
