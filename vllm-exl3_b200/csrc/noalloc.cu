// noalloc.cu -- the dense EXL3 linear (exl3_linear) for callers that cannot
// allocate device memory.
//
// Some callers of this library must not allocate GPU memory at the time they
// run a projection: a serving engine that has already given every free byte
// of HBM to its KV cache after its start-up profiling (a late cudaMalloc may
// fail or fragment that budget), and plain C or FFI hosts without a caching
// allocator, for which each cudaMalloc/cudaFree pair would also synchronise
// the device.  exl3_linear_noalloc serves them: it computes exactly what
// exl3_linear computes, but its work buffers live in one file-scope device
// array of EXL3_LINEAR_NOALLOC_SCRATCH_BYTES (16 MiB) that every GPU loading
// this library holds until the process exits.
//
// Rules that follow from the shared array:
//  * the array's device address is looked up once per device, with that
//    device current, by the first call made on it (cudaGetSymbolAddress);
//    make that first call before any stream capture, e.g. during warm-up;
//  * every call reuses the array and it keeps the previous call's contents;
//    the status word, the one word that must start at zero, is cleared on
//    the call's stream before the kernels run; the routing prep kernel then
//    rewrites the slot count and clears the split-K counters;
//  * calls whose GPU work overlaps (two streams, or two host threads on one
//    device without ordering) race on the array and corrupt each other;
//  * a call whose work buffers would exceed the array is rejected before
//    anything is launched.
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "../../include/exl3_b200.h"
#include "exl3_internal.h"

namespace exl3 {
void set_last_error(const char* msg);
}

namespace {

static __device__ __align__(256) unsigned char g_linear_scratch[EXL3_LINEAR_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

int noalloc_fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    exl3::set_last_error(buf);
    return code;
}

// Device address of g_linear_scratch on the current device (looked up once).
cudaError_t scratch_on_current_device(void** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (g_scratch_addr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_linear_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return cudaSuccess;
}

}  // namespace

extern "C" int exl3_linear_noalloc(const void* x, int x_dtype, int64_t m, const void* trellis,
                                   const void* suh, const void* svh, int64_t in_f, int64_t out_f,
                                   int K, int cb, void* y, int y_dtype, void* stream) {
    const char* who = "exl3_linear_noalloc";
    if (!x || !y || !trellis || !suh || !svh) return noalloc_fail(EXL3_ERR_ARG, "%s: null pointer", who);
    if (K < 2 || K > 8) return noalloc_fail(EXL3_ERR_ARG, "%s: K must be in 2..8 (got %d)", who, K);
    if (cb < 0 || cb > 2) return noalloc_fail(EXL3_ERR_ARG, "%s: codebook must be 0, 1 or 2", who);
    const bool fx = x_dtype == EXL3_DT_F32 || x_dtype == EXL3_DT_F16 || x_dtype == EXL3_DT_BF16;
    const bool fy = y_dtype == EXL3_DT_F32 || y_dtype == EXL3_DT_F16 || y_dtype == EXL3_DT_BF16;
    if (!fx || !fy) return noalloc_fail(EXL3_ERR_ARG, "%s: x/y dtype must be fp32, fp16 or bf16", who);
    if (in_f <= 0 || out_f <= 0 || in_f % 128 || out_f % 128 || in_f > INT32_MAX || out_f > INT32_MAX)
        return noalloc_fail(EXL3_ERR_ARG,
                            "%s: in/out features must be positive multiples of 128 (whole Hadamard blocks)",
                            who);
    if (reinterpret_cast<uintptr_t>(trellis) & 15)
        return noalloc_fail(EXL3_ERR_ARG, "%s: trellis must be 16-byte aligned", who);
    if ((reinterpret_cast<uintptr_t>(suh) & 1) || (reinterpret_cast<uintptr_t>(svh) & 1))
        return noalloc_fail(EXL3_ERR_ARG, "%s: suh/svh must be 2-byte aligned fp16 arrays", who);
    if (m < 0) return noalloc_fail(EXL3_ERR_ARG, "%s: m must be >= 0", who);
    if (m == 0) return EXL3_OK;
    exl3::MoePlan p;
    if (!exl3::plan_moe(p, m, 1, int(in_f), int(out_f), 1, K, true, exl3::num_sms_current(), true, cb))
        return noalloc_fail(EXL3_ERR_ARG, "%s: unsupported geometry", who);
    if (p.total > size_t(EXL3_LINEAR_NOALLOC_SCRATCH_BYTES))
        return noalloc_fail(EXL3_ERR_ARG,
                            "%s: this call needs %zu bytes of scratch but the built-in scratch holds %zu "
                            "bytes; use fewer rows, or exl3_linear with a caller-owned workspace",
                            who, p.total, size_t(EXL3_LINEAR_NOALLOC_SCRATCH_BYTES));
    void* ws = nullptr;
    cudaError_t e = scratch_on_current_device(&ws);
    if (e != cudaSuccess)
        return noalloc_fail(EXL3_ERR_CUDA, "%s: scratch lookup failed: CUDA error %d (%s)", who, int(e),
                            cudaGetErrorString(e));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // the previous call's status word (the prep kernel rewrites the slot
    // count and clears the counters itself)
    e = cudaMemsetAsync(ws, 0, 256, s);
    if (e != cudaSuccess)
        return noalloc_fail(EXL3_ERR_CUDA, "%s: CUDA error %d (%s)", who, int(e), cudaGetErrorString(e));
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
    e = exl3::run_moe(p, c, ws, s);
    if (e != cudaSuccess)
        return noalloc_fail(EXL3_ERR_CUDA, "%s: CUDA error %d (%s)", who, int(e), cudaGetErrorString(e));
    return EXL3_OK;
}
