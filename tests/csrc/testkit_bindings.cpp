// Test-only native module `moet_testkit`: kernels that validate hardware paths
// but serve no model (built beside the product library, never imported by it).
#include <torch/extension.h>

void tc_gemm_test(torch::Tensor a, torch::Tensor sa, torch::Tensor b, torch::Tensor sb, torch::Tensor out,
                  torch::Tensor status, int64_t stage);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("tc_gemm_test", &tc_gemm_test, "one-CTA tcgen05 block-scaled e4m3 GEMM through TMEM (validation)");
}
