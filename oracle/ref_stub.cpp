// Test infrastructure: link stub for building the reference's CPU binding.
//
// The reference's pybind module (csrc/bindings.cpp:169-200) references six CUDA
// entry points.  Only its CPU path (dequant_cpu, csrc/bindings.cpp:15-100, and
// the CPU branch of exl3_gemv, :134-147) is used here, so the CUDA symbols are
// defined to raise.  This file is ours; the reference sources are compiled in
// place from the read-only reference tree by oracle/build_ref.py.
#include <torch/extension.h>

at::Tensor exl3_gemv_cuda(const at::Tensor&, const at::Tensor&, const at::Tensor&,
                          const at::Tensor&, int64_t, bool, int64_t) {
    TORCH_CHECK(false, "reference CUDA path is not part of the CPU oracle build");
}
at::Tensor exl3_gemm_cuda(const at::Tensor&, const at::Tensor&, const at::Tensor&,
                          const at::Tensor&, int64_t, bool) {
    TORCH_CHECK(false, "reference CUDA path is not part of the CPU oracle build");
}
at::Tensor p2b_gemv_batched_cuda(const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                 const at::Tensor&, const at::Tensor&, int64_t, bool, int64_t) {
    TORCH_CHECK(false, "reference CUDA path is not part of the CPU oracle build");
}
at::Tensor p2b_fused_moe_cuda(const at::Tensor&, at::Tensor&, const at::Tensor&, const at::Tensor&,
                              const at::Tensor&, const at::Tensor&, const at::Tensor&,
                              const at::Tensor&, const at::Tensor&, const at::Tensor&,
                              const at::Tensor&, const at::Tensor&, const at::Tensor&,
                              int64_t, int64_t, int64_t, bool, int64_t, float) {
    TORCH_CHECK(false, "reference CUDA path is not part of the CPU oracle build");
}
void exl3_fat_gemm(at::Tensor, at::Tensor, at::Tensor, at::Tensor, int64_t, bool, bool) {
    TORCH_CHECK(false, "reference CUDA path is not part of the CPU oracle build");
}
void exl3_fat_gemm_scatter(at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor,
                           at::Tensor, int64_t, bool, bool) {
    TORCH_CHECK(false, "reference CUDA path is not part of the CPU oracle build");
}
