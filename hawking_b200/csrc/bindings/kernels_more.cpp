// torch bindings for kernel groups beyond the decode core (quantisers, tensor-core GEMM, MoE,
// DeltaNet, MLA, fused collectives).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "../kernels/kernels_api.h"
#include "../kernels/api.h"

namespace py = pybind11;
using at::Tensor;

namespace {
cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void quantize(int64_t fmt, const Tensor& x, const std::vector<Tensor>& planes) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kFloat && x.is_contiguous(), "quantize: x must be contiguous fp32 CUDA");
  void* p[4] = {nullptr, nullptr, nullptr, nullptr};
  for (size_t i = 0; i < planes.size() && i < 4; ++i) {
    TORCH_CHECK(planes[i].is_contiguous(), "quantize: planes must be contiguous");
    p[i] = planes[i].data_ptr();
  }
  const c10::cuda::CUDAGuard g(x.device());
  hk::quantize_launch((int)fmt, x.data_ptr<float>(), x.numel(), p[0], p[1], p[2], p[3], cur_stream());
}
}  // namespace

namespace hk {
void register_more_kernels(py::module_& m) {
  m.def("quantize", &quantize, py::arg("fmt"), py::arg("x"), py::arg("planes"));
}
}  // namespace hk
