// ref_stubs.cpp -- link stubs for building the reference's CPU dequant.
//
// TEST INFRASTRUCTURE ONLY (see oracle/Makefile, target `ref`).  The
// reference's pybind module (csrc/bindings.cpp) declares eight CUDA entry
// points that live in .cu files needing ExLlamaV3's un-vendored headers.  The
// CPU-only build of bindings.cpp therefore gets these definitions, which
// refuse to run.  Only dequant_trellis and the CPU branch of exl3_gemv
// (bindings.cpp:117-147) are used from the resulting module.
#include <torch/extension.h>

namespace {
[[noreturn]] void no_cuda(const char* name) {
    TORCH_CHECK(false, name, " requires the CUDA build of the reference");
}
}  // namespace

at::Tensor exl3_gemv_cuda(const at::Tensor&, const at::Tensor&, const at::Tensor&,
                          const at::Tensor&, int64_t, bool, int64_t) {
    no_cuda("exl3_gemv_cuda");
}

at::Tensor exl3_gemm_cuda(const at::Tensor&, const at::Tensor&, const at::Tensor&,
                          const at::Tensor&, int64_t, bool) {
    no_cuda("exl3_gemm_cuda");
}

at::Tensor p2b_gemv_batched_cuda(const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                 const at::Tensor&, const at::Tensor&, int64_t, bool,
                                 int64_t) {
    no_cuda("p2b_gemv_batched_cuda");
}

at::Tensor p2b_fused_moe_cuda(const at::Tensor&, at::Tensor&, const at::Tensor&,
                              const at::Tensor&, const at::Tensor&, const at::Tensor&,
                              const at::Tensor&, const at::Tensor&, const at::Tensor&,
                              const at::Tensor&, const at::Tensor&, const at::Tensor&,
                              const at::Tensor&, int64_t, int64_t, int64_t, bool, int64_t,
                              float) {
    no_cuda("p2b_fused_moe_cuda");
}

at::Tensor p2b_fused_moe_mk_cuda(const at::Tensor&, at::Tensor&, const at::Tensor&,
                                 const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                 const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                 const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                 const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                 const at::Tensor&, int64_t, bool, int64_t, float) {
    no_cuda("p2b_fused_moe_mk_cuda");
}

at::Tensor p2b_fused_moe_padded_cuda(const at::Tensor&, at::Tensor&, const at::Tensor&,
                                     const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                     const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                     const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                     const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                     const at::Tensor&, const at::Tensor&, int64_t, int64_t,
                                     bool, int64_t, float) {
    no_cuda("p2b_fused_moe_padded_cuda");
}

void exl3_fat_gemm(at::Tensor, at::Tensor, at::Tensor, at::Tensor, int64_t, bool, bool) {
    no_cuda("exl3_fat_gemm");
}

void exl3_fat_gemm_scatter(at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor,
                           at::Tensor, int64_t, bool, bool) {
    no_cuda("exl3_fat_gemm_scatter");
}
