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
void tc_gemm(int64_t fmt, const std::vector<Tensor>& planes, int64_t N, int64_t K, const Tensor& x, const Tensor& y,
             bool atomic, bool y_zeroed, int64_t k_splits, int64_t bn, const Tensor& status, bool pdl,
             const c10::optional<Tensor>& h, bool persistent, bool stream_k) {
  TORCH_CHECK(planes.size() == 2, "tc_gemm: Q4_K expects [quants, headers] planes");
  const Tensor& w = planes[0];
  const Tensor& wh = planes[1];
  TORCH_CHECK(w.is_cuda() && x.is_cuda() && y.is_cuda(), "tc_gemm: CUDA tensors required");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.stride(-1) == 1, "tc_gemm: x must be bf16 rows");
  TORCH_CHECK(h.has_value() || (y.scalar_type() == at::kFloat && y.stride(-1) == 1), "tc_gemm: y must be fp32 rows");
  TORCH_CHECK(w.dim() == 2 && w.stride(-1) == 1, "tc_gemm: w must be [N, row_bytes]");
  TORCH_CHECK(status.scalar_type() == at::kInt, "tc_gemm: status must be int32");
  hk::TcGemmArgs g{};
  g.fmt = (int)fmt;
  g.w = reinterpret_cast<const uint8_t*>(w.data_ptr());
  g.w_row_bytes = w.stride(0);
  g.w_hdr = reinterpret_cast<const uint8_t*>(wh.data_ptr());
  g.w_hdr_row_bytes = wh.stride(0);
  g.N = (int)N;
  g.K = (int)K;
  g.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  g.x_stride = x.stride(0);
  g.M = (int)x.size(0);
  g.y = h.has_value() ? nullptr : y.data_ptr<float>();
  g.y_stride = y.stride(0);
  g.atomic = atomic;
  g.y_zeroed = y_zeroed;
  g.k_splits = (int)k_splits;
  g.bn = (int)bn;
  g.status = status.data_ptr<int>();
  g.pdl = pdl;
  g.persistent = stream_k ? 2 : (persistent ? 1 : 0);
  if (h.has_value()) {
    TORCH_CHECK(h->scalar_type() == at::kBFloat16 && h->stride(-1) == 1 && h->size(0) >= g.M && h->size(1) >= N / 2,
                "tc_gemm swiglu: h must be bf16 [M, >= N / 2]");
    g.h = reinterpret_cast<__nv_bfloat16*>(h->data_ptr());
    g.h_stride = h->stride(0);
  }
  const c10::cuda::CUDAGuard guard(x.device());
  hk::tc_gemm_launch(g, cur_stream());
}

void swiglu_bf16(const Tensor& gu, int64_t F, const Tensor& h, bool clear, bool pdl) {
  const c10::cuda::CUDAGuard guard(gu.device());
  hk::swiglu_bf16_launch(gu.data_ptr<float>(), gu.stride(0), (int)gu.size(0), (int)F,
                         reinterpret_cast<__nv_bfloat16*>(h.data_ptr()), h.stride(0), clear, cur_stream(), pdl);
}
hk::WPlanes planes_of(const std::vector<Tensor>& ps) {
  hk::WPlanes w{};
  const uint8_t** p[4] = {&w.p0, &w.p1, &w.p2, &w.p3};
  int64_t* rb[4] = {&w.rb0, &w.rb1, &w.rb2, &w.rb3};
  for (size_t i = 0; i < ps.size() && i < 4; ++i) {
    TORCH_CHECK(ps[i].is_cuda() && ps[i].stride(-1) == 1, "weight planes must be CUDA rows");
    *p[i] = reinterpret_cast<const uint8_t*>(ps[i].data_ptr());
    *rb[i] = ps[i].stride(0) * ps[i].element_size();
  }
  return w;
}

void router_logits(const Tensor& w, const Tensor& xq, const Tensor& xd, const Tensor& logits, bool pdl) {
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous(), "router weights must be contiguous fp32 [E, K]");
  const c10::cuda::CUDAGuard g(w.device());
  hk::router_logits_launch(w.data_ptr<float>(), (int)w.size(0), (int)w.size(1), xq.data_ptr<int8_t>(),
                           xd.data_ptr<float>(), xq.stride(0), xd.stride(0), logits.data_ptr<float>(),
                           (int)xq.size(0), cur_stream(), pdl);
}

void moe_topk(const Tensor& logits, const c10::optional<Tensor>& bias, int64_t k, int64_t scoring,
              int64_t n_groups, int64_t topk_groups, bool renorm, double scale, const Tensor& ids,
              const Tensor& weights, bool pdl) {
  hk::MoeTopkArgs a{};
  a.logits = logits.data_ptr<float>();
  a.bias = bias.has_value() ? bias->data_ptr<float>() : nullptr;
  a.T = (int)logits.size(0);
  a.E = (int)logits.size(1);
  a.k = (int)k;
  a.scoring = (int)scoring;
  a.n_groups = (int)n_groups;
  a.topk_groups = (int)topk_groups;
  a.renorm = renorm;
  a.scale = (float)scale;
  a.ids = ids.data_ptr<int>();
  a.weights = weights.data_ptr<float>();
  const c10::cuda::CUDAGuard g(logits.device());
  hk::moe_topk_launch(a, cur_stream(), pdl);
}

void moe_route(const Tensor& router, const Tensor& xq, const Tensor& xd, int64_t k, int64_t scoring,
               const c10::optional<Tensor>& bias, int64_t n_groups, int64_t topk_groups, bool renorm, double scale,
               const Tensor& logits, const Tensor& ids, const Tensor& weights, const Tensor& counts,
               const Tensor& offsets, const Tensor& sorted, const Tensor& active, const Tensor& n_active, bool shared,
               const Tensor& counter, bool pdl, int64_t e_lo, int64_t e_hi) {
  TORCH_CHECK(router.scalar_type() == at::kFloat && router.dim() == 2, "moe_route: fp32 router [E, K]");
  hk::MoeRouteArgs a{};
  a.e_lo = (int)e_lo;
  a.e_hi = (int)e_hi;
  a.router = router.data_ptr<float>();
  a.E = (int)router.size(0);
  a.K = (int)router.size(1);
  a.T = (int)xq.size(0);
  TORCH_CHECK(xq.size(1) >= a.K, "moe_route: activation width");
  a.xq = xq.data_ptr<int8_t>();
  a.xd = xd.data_ptr<float>();
  a.x_stride_q = xq.stride(0);
  a.x_stride_s = xd.stride(0);
  a.k = (int)k;
  a.bias = bias.has_value() ? bias->data_ptr<float>() : nullptr;
  a.scoring = (int)scoring;
  a.n_groups = (int)n_groups;
  a.topk_groups = (int)topk_groups;
  a.renorm = renorm;
  a.scale = (float)scale;
  TORCH_CHECK(logits.numel() >= (int64_t)a.T * a.E && ids.numel() >= (int64_t)a.T * a.k &&
                  weights.numel() >= (int64_t)a.T * a.k, "moe_route: logits / ids / weights too small");
  TORCH_CHECK(counts.numel() >= a.E + (shared ? 1 : 0) && offsets.numel() >= a.E + (shared ? 1 : 0) &&
                  active.numel() >= a.E + (shared ? 1 : 0) && sorted.numel() >= (int64_t)a.T * a.k + (shared ? a.T : 0),
              "moe_route: routing buffers too small");
  a.logits = logits.data_ptr<float>();
  a.ids = ids.data_ptr<int>();
  a.weights = weights.data_ptr<float>();
  a.counts = counts.data_ptr<int>();
  a.offsets = offsets.data_ptr<int>();
  a.sorted = sorted.data_ptr<int>();
  a.active = active.data_ptr<int>();
  a.n_active = n_active.data_ptr<int>();
  a.shared = shared ? 1 : 0;
  a.counter = counter.data_ptr<int>();
  const c10::cuda::CUDAGuard g(xq.device());
  hk::moe_route_launch(a, cur_stream(), pdl);
}

void moe_align(const Tensor& ids, int64_t E, const Tensor& xq, const Tensor& xd, const Tensor& xs,
               const Tensor& counts, const Tensor& offsets, const Tensor& sorted, const Tensor& gq,
               const Tensor& gd, const Tensor& gs, bool pdl, bool shared) {
  hk::MoeAlignArgs a{};
  a.shared = shared ? 1 : 0;
  a.ids = ids.data_ptr<int>();
  a.T = (int)ids.size(0);
  a.k = (int)ids.size(1);
  a.E = (int)E;
  a.K = (int)xq.size(1);
  a.xq = xq.data_ptr<int8_t>();
  a.xd = xd.data_ptr<float>();
  a.xs = xs.data_ptr<float>();
  a.x_stride_q = xq.stride(0);
  a.x_stride_s = xd.stride(0);
  a.counts = counts.data_ptr<int>();
  a.offsets = offsets.data_ptr<int>();
  a.sorted = sorted.data_ptr<int>();
  // empty gathered tensors: the counting sort only (the caller gathers its own rows)
  a.gq = gq.numel() ? gq.data_ptr<int8_t>() : nullptr;
  a.gd = gq.numel() ? gd.data_ptr<float>() : nullptr;
  a.gs = gq.numel() ? gs.data_ptr<float>() : nullptr;
  const c10::cuda::CUDAGuard g(ids.device());
  hk::moe_align_launch(a, cur_stream(), pdl);
}

void moe_gemv(int64_t fmt, int64_t epi, const std::vector<Tensor>& w0, const std::vector<Tensor>& w1, int64_t N,
              int64_t K, int64_t E, int64_t k, const Tensor& counts, const Tensor& offsets, const Tensor& sorted,
              const Tensor& xq, const Tensor& xd, const Tensor& xs, const c10::optional<Tensor>& oq,
              const c10::optional<Tensor>& od, const c10::optional<Tensor>& os, const c10::optional<Tensor>& y,
              const c10::optional<Tensor>& route_w, bool pdl, int64_t e_lo, int64_t T,
              const c10::optional<Tensor>& push_table, const c10::optional<Tensor>& push_epoch,
              const c10::optional<Tensor>& base) {
  hk::MoeGemvArgs a{};
  if (base.has_value()) {
    TORCH_CHECK(base->scalar_type() == at::kFloat && base->stride(-1) == 1, "moe_gemv: fp32 base rows");
    a.base = base->data_ptr<float>();
    a.base_stride = base->stride(0);
  }
  a.e_lo = (int)e_lo;
  a.T = (int)T;
  if (push_table.has_value()) {
    TORCH_CHECK(push_table->scalar_type() == at::kLong && push_epoch.has_value(), "moe_gemv push: int64 table + epoch");
    a.push_recv = reinterpret_cast<unsigned long long* const*>(push_table->data_ptr<int64_t>());
    a.push_n = (int)push_table->numel();
    a.push_epoch = push_epoch->data_ptr<int>();
  }
  a.w0 = planes_of(w0);
  if (!w1.empty()) a.w1 = planes_of(w1);
  a.N = (int)N;
  a.K = (int)K;
  a.E = (int)E;
  a.k = (int)k;
  a.counts = counts.data_ptr<int>();
  a.offsets = offsets.data_ptr<int>();
  a.sorted = sorted.data_ptr<int>();
  a.xq = xq.data_ptr<int8_t>();
  a.xd = xd.data_ptr<float>();
  a.xs = xs.data_ptr<float>();
  if (epi == 0) {
    TORCH_CHECK(oq.has_value() && od.has_value() && os.has_value() && !w1.empty(), "moe_gemv swiglu: outputs");
    a.oq = oq->data_ptr<int8_t>();
    a.od = od->data_ptr<float>();
    a.os = os->data_ptr<float>();
  } else if (epi == 2) {
    TORCH_CHECK(route_w.has_value() && a.push_recv, "moe_gemv combine push: route weights and push table required");
    a.route_w = route_w->data_ptr<float>();
  } else {
    TORCH_CHECK(y.has_value() && route_w.has_value(), "moe_gemv down: y and route weights required");
    a.y = y->data_ptr<float>();
    a.y_stride = y->stride(0);
    a.route_w = route_w->data_ptr<float>();
  }
  const c10::cuda::CUDAGuard g(xq.device());
  hk::moe_gemv_launch((int)fmt, (int)epi, a, cur_stream(), pdl);
}
}  // namespace

namespace hk {
void register_more_kernels(py::module_& m) {
  m.def("quantize", &quantize, py::arg("fmt"), py::arg("x"), py::arg("planes"));
  m.def("tc_gemm", &tc_gemm, py::arg("fmt"), py::arg("planes"), py::arg("N"), py::arg("K"), py::arg("x"), py::arg("y"),
        py::arg("atomic"), py::arg("y_zeroed"), py::arg("k_splits"), py::arg("bn"), py::arg("status"),
        py::arg("pdl") = false, py::arg("h") = py::none(), py::arg("persistent") = false,
        py::arg("stream_k") = false);
  m.def("tc_gemm_splits", &hk::tc_gemm_splits);
  m.def("router_logits", &router_logits, py::arg("w"), py::arg("xq"), py::arg("xd"), py::arg("logits"),
        py::arg("pdl") = false);
  m.def("moe_topk", &moe_topk, py::arg("logits"), py::arg("bias"), py::arg("k"), py::arg("scoring"),
        py::arg("n_groups"), py::arg("topk_groups"), py::arg("renorm"), py::arg("scale"), py::arg("ids"),
        py::arg("weights"), py::arg("pdl") = false);
  m.def("moe_route", &moe_route, py::arg("router"), py::arg("xq"), py::arg("xd"), py::arg("k"), py::arg("scoring"),
        py::arg("bias"), py::arg("n_groups"), py::arg("topk_groups"), py::arg("renorm"), py::arg("scale"),
        py::arg("logits"), py::arg("ids"), py::arg("weights"), py::arg("counts"), py::arg("offsets"),
        py::arg("sorted"), py::arg("active"), py::arg("n_active"), py::arg("shared"), py::arg("counter"),
        py::arg("pdl") = false, py::arg("e_lo") = 0, py::arg("e_hi") = 0);
  m.def("moe_align", &moe_align, py::arg("ids"), py::arg("E"), py::arg("xq"), py::arg("xd"), py::arg("xs"),
        py::arg("counts"), py::arg("offsets"), py::arg("sorted"), py::arg("gq"), py::arg("gd"), py::arg("gs"),
        py::arg("pdl") = false,
        py::arg("shared") = false);
  m.def("moe_gemv", &moe_gemv, py::arg("fmt"), py::arg("epi"), py::arg("w0"), py::arg("w1"), py::arg("N"),
        py::arg("K"), py::arg("E"), py::arg("k"), py::arg("counts"), py::arg("offsets"), py::arg("sorted"),
        py::arg("xq"), py::arg("xd"), py::arg("xs"), py::arg("oq") = py::none(), py::arg("od") = py::none(),
        py::arg("os") = py::none(), py::arg("y") = py::none(), py::arg("route_w") = py::none(),
        py::arg("pdl") = false, py::arg("e_lo") = 0, py::arg("T") = 0, py::arg("push_table") = py::none(),
        py::arg("push_epoch") = py::none(), py::arg("base") = py::none());
  m.def("swiglu_bf16", &swiglu_bf16, py::arg("gu"), py::arg("F"), py::arg("h"), py::arg("clear") = true,
        py::arg("pdl") = false);
}
}  // namespace hk
