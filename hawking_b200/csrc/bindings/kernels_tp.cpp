// torch bindings for the tensor-parallel plumbing: CUDA IPC buffers shared between the ranks of one
// node (no multicast objects) and the fused collective kernels of tp.cu.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <cstring>
#include <stdexcept>
#include <string>

#include "../kernels/api.h"
#include "../kernels/kernels_api.h"

#define HK_CUDA_CHECK(expr)                                                                 \
  do {                                                                                      \
    cudaError_t _e = (expr);                                                                \
    if (_e != cudaSuccess) throw std::runtime_error(std::string("CUDA error ") + cudaGetErrorString(_e)); \
  } while (0)

namespace py = pybind11;
using at::Tensor;

namespace {
cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

template <typename T>
T* as_ptr(int64_t p) { return reinterpret_cast<T*>(static_cast<uintptr_t>(p)); }

// Device memory shareable with the other processes of this node; zero-filled.
int64_t ipc_malloc(int64_t bytes) {
  void* p = nullptr;
  HK_CUDA_CHECK(cudaMalloc(&p, (size_t)bytes));
  HK_CUDA_CHECK(cudaMemset(p, 0, (size_t)bytes));
  return (int64_t)reinterpret_cast<uintptr_t>(p);
}
py::bytes ipc_handle(int64_t ptr) {
  cudaIpcMemHandle_t h;
  HK_CUDA_CHECK(cudaIpcGetMemHandle(&h, as_ptr<void>(ptr)));
  return py::bytes(reinterpret_cast<const char*>(&h), sizeof h);
}
int64_t ipc_open(const std::string& handle) {
  TORCH_CHECK(handle.size() == sizeof(cudaIpcMemHandle_t), "ipc_open: bad handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data(), sizeof h);
  void* p = nullptr;
  HK_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return (int64_t)reinterpret_cast<uintptr_t>(p);
}
void ipc_close(int64_t ptr) { HK_CUDA_CHECK(cudaIpcCloseMemHandle(as_ptr<void>(ptr))); }
void ipc_free(int64_t ptr) { HK_CUDA_CHECK(cudaFree(as_ptr<void>(ptr))); }

void tp_begin(const Tensor& epoch, bool pdl) {
  TORCH_CHECK(epoch.is_cuda() && epoch.scalar_type() == at::kInt, "tp_begin: int32 CUDA epoch");
  const c10::cuda::CUDAGuard g(epoch.device());
  hk::tp_begin_launch(epoch.data_ptr<int>(), cur_stream(), pdl);
}

void tp_allreduce_rmsnorm_q8(const Tensor& x_in, const Tensor& x_out, int64_t recv, int64_t rank_stride, int64_t n,
                             const Tensor& epoch, const c10::optional<Tensor>& w,
                             double eps, const c10::optional<Tensor>& xq, const c10::optional<Tensor>& xd,
                             const c10::optional<Tensor>& xs, const Tensor& status, bool pdl,
                             const c10::optional<Tensor>& yb, int64_t wait_ns) {
  TORCH_CHECK(x_in.is_cuda() && x_in.scalar_type() == at::kFloat && x_out.scalar_type() == at::kFloat,
              "tp norm: fp32 residual rows");
  TORCH_CHECK(x_in.stride(0) == x_out.stride(0), "tp norm: x_in / x_out strides differ");
  hk::TpReduceArgs a{};
  a.x_in = x_in.data_ptr<float>();
  a.x_out = x_out.data_ptr<float>();
  a.x_stride = x_in.stride(0);
  a.recv = as_ptr<const unsigned long long>(recv);
  a.rank_stride = rank_stride;
  a.n = (int)n;
  a.epoch = epoch.data_ptr<int>();
  a.w = w.has_value() ? w->data_ptr<float>() : nullptr;
  a.eps = (float)eps;
  a.K = (int)x_in.size(1);
  if (xq.has_value()) {
    TORCH_CHECK(xd.has_value() && xs.has_value(), "tp norm: q8 output needs q, d and s");
    a.xq = xq->data_ptr<int8_t>();
    a.xd = xd->data_ptr<float>();
    a.xs = xs->data_ptr<float>();
  } else {
    TORCH_CHECK(yb.has_value() && yb->scalar_type() == at::kBFloat16 && yb->stride(-1) == 1,
                "tp norm: a q8 or a bf16 output is required");
    a.yb = reinterpret_cast<__nv_bfloat16*>(yb->data_ptr());
    a.yb_stride = yb->stride(0);
  }
  a.status = status.data_ptr<int>();
  a.wait_ns = (unsigned long long)(wait_ns > 0 ? wait_ns : 0);
  const c10::cuda::CUDAGuard g(x_in.device());
  hk::tp_allreduce_rmsnorm_q8_launch(a, (int)x_in.size(0), cur_stream(), pdl);
}

void tp_argmax(const Tensor& slots, int64_t rows, int64_t max_rows, const Tensor& keys_table, int64_t keys_local,
               const Tensor& uses, int64_t me, const Tensor& out, const Tensor& status, bool pdl, int64_t wait_ns) {
  TORCH_CHECK(slots.is_cuda() && slots.scalar_type() == at::kLong, "tp_argmax: int64 slots");
  TORCH_CHECK(keys_table.scalar_type() == at::kLong, "tp_argmax: int64 pointer table");
  TORCH_CHECK(rows <= max_rows, "tp_argmax: rows exceed the key region");
  hk::TpArgmaxArgs a{};
  a.slots = reinterpret_cast<unsigned long long*>(slots.data_ptr<int64_t>());
  a.rows = (int)rows;
  a.max_rows = (int)max_rows;
  a.keys = reinterpret_cast<unsigned long long* const*>(keys_table.data_ptr<int64_t>());
  a.keys_local = as_ptr<const unsigned long long>(keys_local);
  a.uses = uses.data_ptr<int>();
  a.me = (int)me;
  a.n = (int)keys_table.numel();
  a.out = out.data_ptr<int>();
  a.status = status.data_ptr<int>();
  a.wait_ns = (unsigned long long)(wait_ns > 0 ? wait_ns : 0);
  const c10::cuda::CUDAGuard g(slots.device());
  hk::tp_argmax_launch(a, cur_stream(), pdl);
}
}  // namespace

namespace hk {
// Non-owning tensor over raw device memory (an IPC allocation) of `numel` fp32 elements.
Tensor wrap_f32(int64_t ptr, int64_t numel, int64_t device) {
  return at::from_blob(as_ptr<void>(ptr), {numel}, at::TensorOptions().dtype(at::kFloat).device(at::kCUDA, device));
}

void tp_p2p_allreduce_rmsnorm(const Tensor& x_in, const Tensor& x_out, const Tensor& parts, int64_t flags_local,
                              const Tensor& flag_ptrs, int64_t n, int64_t me, const Tensor& epoch,
                              const c10::optional<Tensor>& w, double eps, const c10::optional<Tensor>& xq,
                              const c10::optional<Tensor>& xd, const c10::optional<Tensor>& xs,
                              const c10::optional<Tensor>& yb, const Tensor& status, bool pdl, int64_t wait_ns) {
  TORCH_CHECK(x_in.is_cuda() && x_in.scalar_type() == at::kFloat && x_out.scalar_type() == at::kFloat &&
                  x_in.stride(0) == x_out.stride(0),
              "tp p2p norm: fp32 residual rows with equal strides");
  TORCH_CHECK(parts.scalar_type() == at::kLong && parts.numel() == n && flag_ptrs.scalar_type() == at::kLong &&
                  flag_ptrs.numel() == n,
              "tp p2p norm: int64 address tables of n ranks");
  hk::TpP2PArgs a{};
  a.x_in = x_in.data_ptr<float>();
  a.x_out = x_out.data_ptr<float>();
  a.x_stride = x_in.stride(0);
  a.parts = reinterpret_cast<const unsigned long long*>(parts.data_ptr<int64_t>());
  a.flags_local = as_ptr<unsigned int>(flags_local);
  a.flag_ptrs = reinterpret_cast<const unsigned long long*>(flag_ptrs.data_ptr<int64_t>());
  a.n = (int)n;
  a.me = (int)me;
  a.epoch = epoch.data_ptr<int>();
  a.w = w.has_value() ? w->data_ptr<float>() : nullptr;
  a.eps = (float)eps;
  a.K = (int)x_in.size(1);
  if (xq.has_value()) {
    TORCH_CHECK(xd.has_value() && xs.has_value(), "tp p2p norm: q8 output needs q, d and s");
    a.xq = xq->data_ptr<int8_t>();
    a.xd = xd->data_ptr<float>();
    a.xs = xs->data_ptr<float>();
  } else {
    TORCH_CHECK(yb.has_value() && yb->scalar_type() == at::kBFloat16 && yb->stride(-1) == 1,
                "tp p2p norm: a q8 or a bf16 output is required");
    a.yb = reinterpret_cast<__nv_bfloat16*>(yb->data_ptr());
    a.yb_stride = yb->stride(0);
  }
  a.status = status.data_ptr<int>();
  a.wait_ns = (unsigned long long)(wait_ns > 0 ? wait_ns : 0);
  const c10::cuda::CUDAGuard g(x_in.device());
  hk::tp_p2p_allreduce_rmsnorm_launch(a, (int)x_in.size(0), cur_stream(), pdl);
}

void register_tp_kernels(py::module_& m) {
  m.def("wrap_f32", &wrap_f32, py::arg("ptr"), py::arg("numel"), py::arg("device"));
  m.def("tp_p2p_allreduce_rmsnorm", &tp_p2p_allreduce_rmsnorm, py::arg("x_in"), py::arg("x_out"), py::arg("parts"),
        py::arg("flags_local"), py::arg("flag_ptrs"), py::arg("n"), py::arg("me"), py::arg("epoch"), py::arg("w"),
        py::arg("eps"), py::arg("xq") = py::none(), py::arg("xd") = py::none(), py::arg("xs") = py::none(),
        py::arg("yb") = py::none(), py::arg("status"), py::arg("pdl") = false, py::arg("wait_ns") = 0);
  m.def("ipc_malloc", &ipc_malloc, py::arg("bytes"));
  m.def("ipc_handle", &ipc_handle, py::arg("ptr"));
  m.def("ipc_open", &ipc_open, py::arg("handle"));
  m.def("ipc_close", &ipc_close, py::arg("ptr"));
  m.def("ipc_free", &ipc_free, py::arg("ptr"));
  m.def("tp_begin", &tp_begin, py::arg("epoch"), py::arg("pdl") = false);
  m.def("tp_allreduce_rmsnorm_q8", &tp_allreduce_rmsnorm_q8, py::arg("x_in"), py::arg("x_out"), py::arg("recv"),
        py::arg("rank_stride"), py::arg("n"), py::arg("epoch"), py::arg("w"), py::arg("eps"), py::arg("xq"), py::arg("xd"), py::arg("xs"), py::arg("status"),
        py::arg("pdl") = false, py::arg("yb") = py::none(), py::arg("wait_ns") = 0);
  m.def("tp_argmax", &tp_argmax, py::arg("slots"), py::arg("rows"), py::arg("max_rows"), py::arg("keys_table"),
        py::arg("keys_local"), py::arg("uses"), py::arg("me"), py::arg("out"), py::arg("status"), py::arg("pdl") = false,
        py::arg("wait_ns") = 0);
}
}  // namespace hk
