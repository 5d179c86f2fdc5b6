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
void tc_gemm(int64_t fmt, const Tensor& w, int64_t N, int64_t K, const Tensor& x, const Tensor& y, bool atomic,
             bool y_zeroed, int64_t k_splits, int64_t bn, const Tensor& status, bool pdl) {
  TORCH_CHECK(w.is_cuda() && x.is_cuda() && y.is_cuda(), "tc_gemm: CUDA tensors required");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.stride(-1) == 1, "tc_gemm: x must be bf16 rows");
  TORCH_CHECK(y.scalar_type() == at::kFloat && y.stride(-1) == 1, "tc_gemm: y must be fp32 rows");
  TORCH_CHECK(w.dim() == 2 && w.stride(-1) == 1, "tc_gemm: w must be [N, row_bytes]");
  TORCH_CHECK(status.scalar_type() == at::kInt, "tc_gemm: status must be int32");
  hk::TcGemmArgs g{};
  g.fmt = (int)fmt;
  g.w = reinterpret_cast<const uint8_t*>(w.data_ptr());
  g.w_row_bytes = w.stride(0);
  g.N = (int)N;
  g.K = (int)K;
  g.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  g.x_stride = x.stride(0);
  g.M = (int)x.size(0);
  g.y = y.data_ptr<float>();
  g.y_stride = y.stride(0);
  g.atomic = atomic;
  g.y_zeroed = y_zeroed;
  g.k_splits = (int)k_splits;
  g.bn = (int)bn;
  g.status = status.data_ptr<int>();
  g.pdl = pdl;
  const c10::cuda::CUDAGuard guard(x.device());
  hk::tc_gemm_launch(g, cur_stream());
}

void swiglu_bf16(const Tensor& gu, int64_t F, const Tensor& h, bool clear, bool pdl) {
  const c10::cuda::CUDAGuard guard(gu.device());
  hk::swiglu_bf16_launch(gu.data_ptr<float>(), gu.stride(0), (int)gu.size(0), (int)F,
                         reinterpret_cast<__nv_bfloat16*>(h.data_ptr()), h.stride(0), clear, cur_stream(), pdl);
}
}  // namespace

namespace hk {
void register_more_kernels(py::module_& m) {
  m.def("quantize", &quantize, py::arg("fmt"), py::arg("x"), py::arg("planes"));
  m.def("tc_gemm", &tc_gemm, py::arg("fmt"), py::arg("w"), py::arg("N"), py::arg("K"), py::arg("x"), py::arg("y"),
        py::arg("atomic"), py::arg("y_zeroed"), py::arg("k_splits"), py::arg("bn"), py::arg("status"),
        py::arg("pdl") = false);
  m.def("tc_gemm_splits", &hk::tc_gemm_splits);
  m.def("swiglu_bf16", &swiglu_bf16, py::arg("gu"), py::arg("F"), py::arg("h"), py::arg("clear") = true,
        py::arg("pdl") = false);
}
}  // namespace hk
