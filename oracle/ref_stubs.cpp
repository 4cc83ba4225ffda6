// Stand-ins for the two reference operators whose sources need CUTLASS or are
// outside this path (mla_decode, cutlass_gemm): the reference's pybind table
// (basic_ops.cu) binds them, so the checker build links these instead.  They
// only raise; nothing calls them.
#include <torch/extension.h>

torch::Tensor mla_decode(torch::Tensor, torch::Tensor) {
  TORCH_CHECK(false, "mla_decode is not part of the checker build");
  return torch::Tensor();
}

torch::Tensor cutlass_gemm(torch::Tensor, torch::Tensor) {
  TORCH_CHECK(false, "cutlass_gemm is not part of the checker build");
  return torch::Tensor();
}
