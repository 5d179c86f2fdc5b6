// torch bindings of the sm_100a kernels (`hawking_b200._kernels`). Every op launches on the
// current torch CUDA stream, so the callers can capture whole decode steps in CUDA graphs.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "../kernels/api.h"
#include "../kernels/kernels_api.h"

namespace py = pybind11;
using at::Tensor;
using c10::optional;

namespace {

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check_cuda(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}

template <typename T> T* ptr(const Tensor& t) { return reinterpret_cast<T*>(t.data_ptr()); }
template <typename T> T* optr(const optional<Tensor>& t) { return t.has_value() ? ptr<T>(*t) : nullptr; }

hk::WPlanes planes(const std::vector<Tensor>& ps) {
  hk::WPlanes w{};
  const uint8_t** p[4] = {&w.p0, &w.p1, &w.p2, &w.p3};
  int64_t* rb[4] = {&w.rb0, &w.rb1, &w.rb2, &w.rb3};
  TORCH_CHECK(ps.size() >= 1 && ps.size() <= 4, "weight planes: 1..4 tensors");
  for (size_t i = 0; i < ps.size(); ++i) {
    check_cuda(ps[i], "weight plane");
    TORCH_CHECK(ps[i].dim() >= 2 && ps[i].stride(-1) == 1, "weight plane must be [rows, bytes] with unit inner stride");
    *p[i] = reinterpret_cast<const uint8_t*>(ps[i].data_ptr());
    *rb[i] = ps[i].stride(0) * ps[i].element_size();
  }
  return w;
}

void gemv(int64_t fmt, int64_t epi, const std::vector<Tensor>& w0, const std::vector<Tensor>& w1, int64_t N,
          int64_t K, const optional<Tensor>& xq_, const optional<Tensor>& xd_, const optional<Tensor>& xs_,
          const optional<Tensor>& y, const optional<Tensor>& bias, const optional<Tensor>& oq,
          const optional<Tensor>& od, const optional<Tensor>& os, const optional<Tensor>& x_f32,
          const optional<Tensor>& norm_w, double eps, bool pdl, const optional<Tensor>& argmax_slots,
          int64_t argmax_offset, const optional<Tensor>& push_recv, const optional<Tensor>& push_epoch,
          const std::vector<Tensor>& prefetch) {
  hk::GemvArgs a{};
  TORCH_CHECK(prefetch.size() <= 8, "gemv: at most 8 prefetch ranges");
  for (const Tensor& t : prefetch) {
    TORCH_CHECK(t.is_cuda() && t.is_contiguous(), "gemv: prefetch ranges must be contiguous CUDA tensors");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, "gemv: prefetch ranges must be 16-byte aligned");
    a.pf_ptr[a.pf_n] = reinterpret_cast<const uint8_t*>(t.data_ptr());
    a.pf_bytes[a.pf_n] = (int64_t)t.numel() * t.element_size();
    ++a.pf_n;
  }
  int nb;
  if (x_f32.has_value()) {
    check_cuda(*x_f32, "x_f32");
    TORCH_CHECK(x_f32->scalar_type() == at::kFloat && x_f32->stride(-1) == 1 && x_f32->size(1) >= K,
                "gemv: x_f32 must be fp32 [nb, K]");
    nb = (int)x_f32->size(0);
    a.x_f32 = x_f32->data_ptr<float>();
    a.x_f32_stride = x_f32->stride(0);
    a.norm_w = optr<float>(norm_w);
    a.eps = (float)eps;
    a.norm = eps >= 0.0 ? 1 : 0;
  } else {
    TORCH_CHECK(xq_.has_value() && xd_.has_value() && xs_.has_value(), "gemv: q8 activations required");
    const Tensor& xq = *xq_;
    const Tensor& xd = *xd_;
    const Tensor& xs = *xs_;
    check_cuda(xq, "xq");
    TORCH_CHECK(xq.scalar_type() == at::kChar && xd.scalar_type() == at::kFloat && xs.scalar_type() == at::kFloat,
                "gemv: activations must be int8 q / fp32 d / fp32 s");
    TORCH_CHECK(xq.dim() == 2 && xq.size(1) >= K && xq.stride(1) == 1, "gemv: xq must be [nb, K]");
    nb = (int)xq.size(0);
    a.xq = ptr<int8_t>(xq);
    a.xd = ptr<float>(xd);
    a.xs = ptr<float>(xs);
    a.x_stride_q = xq.stride(0);
    a.x_stride_s = xd.stride(0);
  }
  a.w0 = planes(w0);
  if (!w1.empty()) a.w1 = planes(w1);
  a.N = (int)N;
  a.K = (int)K;
  if (y.has_value()) {
    TORCH_CHECK(y->scalar_type() == at::kFloat && y->stride(-1) == 1 && y->size(0) >= nb && y->size(-1) >= N,
                "gemv: y must be fp32 [nb, >=N]");
    a.y = ptr<float>(*y);
    a.y_stride = y->stride(0);
  }
  a.bias = optr<float>(bias);
  if (argmax_slots.has_value()) {
    TORCH_CHECK(epi == hk::EPI_STORE, "gemv: argmax fusion needs the STORE epilogue");
    TORCH_CHECK(argmax_slots->scalar_type() == at::kLong && argmax_slots->numel() >= (int64_t)nb * hk::kArgmaxSlots,
                "gemv: argmax slots must be int64 [nb, 256]");
    a.argmax_slots = reinterpret_cast<unsigned long long*>(argmax_slots->data_ptr<int64_t>());
    a.argmax_offset = argmax_offset;
  }
  if (epi == hk::EPI_PUSH) {
    TORCH_CHECK(push_recv.has_value() && push_epoch.has_value(), "gemv push: peer pointer table and epoch required");
    TORCH_CHECK(push_recv->is_cuda() && push_recv->scalar_type() == at::kLong && push_epoch->is_cuda() &&
                    push_epoch->scalar_type() == at::kInt,
                "gemv push: int64 device pointer table and int32 epoch");
    a.push_recv = reinterpret_cast<unsigned long long* const*>(push_recv->data_ptr<int64_t>());
    a.push_epoch = push_epoch->data_ptr<int>();
    a.push_n = (int)push_recv->numel();
  }
  if (epi == hk::EPI_SWIGLU_Q8) {
    TORCH_CHECK(oq.has_value() && od.has_value() && os.has_value(), "gemv swiglu: q8 outputs required");
    TORCH_CHECK(!w1.empty(), "gemv swiglu: up-projection planes required");
    a.oq = ptr<int8_t>(*oq);
    a.od = ptr<float>(*od);
    a.os = ptr<float>(*os);
    a.o_stride_q = oq->stride(0);
    a.o_stride_s = od->stride(0);
  } else {
    TORCH_CHECK(a.y || epi == hk::EPI_PUSH, "gemv: output y required");
  }
  const c10::cuda::CUDAGuard g(w0[0].device());
  hk::gemv_launch((int)fmt, (int)epi, a, nb, cur_stream(), pdl);
}

void rmsnorm_q8(const Tensor& x, const optional<Tensor>& w, double eps, bool norm, const Tensor& xq,
                const Tensor& xd, const Tensor& xs, const optional<Tensor>& y, bool pdl) {
  check_cuda(x, "x");
  TORCH_CHECK(x.scalar_type() == at::kFloat && x.stride(-1) == 1, "rmsnorm_q8: x must be fp32 rows");
  const int rows = (int)x.size(0), K = (int)x.size(1);
  const c10::cuda::CUDAGuard g(x.device());
  hk::rmsnorm_q8_launch(ptr<float>(x), x.stride(0), optr<float>(w), (float)eps, norm, rows, K, ptr<int8_t>(xq),
                        ptr<float>(xd), ptr<float>(xs), optr<float>(y), cur_stream(), pdl);
}

void rmsnorm(const Tensor& x, const optional<Tensor>& w, double eps, const optional<Tensor>& yf,
             const optional<Tensor>& yb, bool pdl) {
  check_cuda(x, "x");
  const int rows = (int)x.size(0), K = (int)x.size(1);
  int64_t ys = yf.has_value() ? yf->stride(0) : yb->stride(0);
  const c10::cuda::CUDAGuard g(x.device());
  hk::rmsnorm_launch(ptr<float>(x), x.stride(0), optr<float>(w), (float)eps, rows, K, optr<float>(yf),
                     optr<__nv_bfloat16>(yb), ys, cur_stream(), pdl);
}

void rope_append(const Tensor& qkv, const optional<Tensor>& bias, const optional<Tensor>& q_norm,
                 const optional<Tensor>& k_norm, double eps, const Tensor& positions, const optional<Tensor>& slots,
                 const Tensor& rope, int64_t rot_dim, int64_t style, const Tensor& q_out, const Tensor& k_cache,
                 const Tensor& v_cache, int64_t nh, int64_t nkv, int64_t hd, int64_t block_size,
                 const optional<Tensor>& block_tables, const optional<Tensor>& row_seq, bool pdl) {
  check_cuda(qkv, "qkv");
  TORCH_CHECK(positions.scalar_type() == at::kInt, "positions must be int32");
  TORCH_CHECK(!slots.has_value() || slots->scalar_type() == at::kInt, "slots must be int32");
  TORCH_CHECK(k_cache.scalar_type() == at::kBFloat16, "kv cache must be bf16");
  hk::RopeAppendArgs a{};
  a.qkv = ptr<float>(qkv);
  a.qkv_stride = qkv.stride(0);
  a.bias = optr<float>(bias);
  a.q_norm = optr<float>(q_norm);
  a.k_norm = optr<float>(k_norm);
  a.eps = (float)eps;
  a.positions = ptr<int>(positions);
  a.slots = optr<int>(slots);
  a.rope = ptr<float>(rope);
  a.rot_dim = (int)rot_dim;
  a.rope_style = (int)style;
  a.q_out = ptr<float>(q_out);
  a.k_cache = ptr<__nv_bfloat16>(k_cache);
  a.v_cache = ptr<__nv_bfloat16>(v_cache);
  a.R = (int)qkv.size(0);
  a.nh = (int)nh;
  a.nkv = (int)nkv;
  a.hd = (int)hd;
  a.block_size = (int)block_size;
  a.block_tables = optr<int>(block_tables);
  a.row_seq = optr<int>(row_seq);
  a.max_blocks = block_tables.has_value() ? (int)block_tables->size(1) : 0;
  a.cache_blocks = k_cache.size(0);
  TORCH_CHECK(a.slots || (a.block_tables && a.row_seq), "rope_append: slots or block tables required");
  const c10::cuda::CUDAGuard g(qkv.device());
  hk::rope_append_launch(a, cur_stream(), pdl);
}

void attention_decode(const Tensor& q, const Tensor& k_cache, const Tensor& v_cache, const Tensor& block_tables,
                      const Tensor& row_seq, const Tensor& row_ctx, double scale, int64_t num_splits,
                      const Tensor& part_o, const Tensor& part_lse, const optional<Tensor>& out,
                      const optional<Tensor>& oq, const optional<Tensor>& od, const optional<Tensor>& os,
                      const optional<Tensor>& sinks, const optional<Tensor>& out_bf16,
                      const optional<Tensor>& counters, bool pdl, bool cluster, bool tc, const optional<Tensor>& status) {
  check_cuda(q, "q");
  TORCH_CHECK(q.dim() == 3 && q.scalar_type() == at::kFloat, "q must be fp32 [R, nh, hd]");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.scalar_type() == at::kBFloat16, "k_cache must be bf16 [blocks, nkv, bs, hd]");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && row_seq.scalar_type() == at::kInt &&
                  row_ctx.scalar_type() == at::kInt, "block tables / rows must be int32");
  const int R = (int)q.size(0), nh = (int)q.size(1), hd = (int)q.size(2);
  TORCH_CHECK(cluster || (part_o.numel() >= (int64_t)R * nh * num_splits * hd &&
                          part_lse.numel() >= (int64_t)R * nh * num_splits),
              "attention: scratch too small");
  hk::AttnDecodeArgs a{};
  a.q = ptr<float>(q);
  a.k_cache = ptr<__nv_bfloat16>(k_cache);
  a.v_cache = ptr<__nv_bfloat16>(v_cache);
  a.block_tables = ptr<int>(block_tables);
  a.max_blocks = (int)block_tables.size(1);
  a.row_seq = ptr<int>(row_seq);
  a.row_ctx = ptr<int>(row_ctx);
  a.scale = (float)scale;
  a.R = R;
  a.nh = nh;
  a.nkv = (int)k_cache.size(1);
  a.hd = hd;
  a.block_size = (int)k_cache.size(2);
  a.num_splits = (int)num_splits;
  a.part_o = ptr<float>(part_o);
  a.part_lse = ptr<float>(part_lse);
  a.out = optr<float>(out);
  a.oq = optr<int8_t>(oq);
  a.od = optr<float>(od);
  a.os = optr<float>(os);
  a.sinks = optr<float>(sinks);
  a.out_bf16 = optr<__nv_bfloat16>(out_bf16);
  a.counters = optr<int>(counters);
  TORCH_CHECK(!counters.has_value() || counters->numel() >= (int64_t)R * a.nkv, "attention: counters too small");
  a.status = optr<int>(status);
  a.table_rows = (int)block_tables.size(0);
  const c10::cuda::CUDAGuard g(q.device());
  if (tc && hk::attention_decode_tc_supported(a)) {
    TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous(), "attention (tensor cores): contiguous caches");
    hk::attention_decode_tc_launch(a, k_cache.numel() / hd, cur_stream(), pdl);
  } else if (cluster) {
    hk::attention_decode_cluster_launch(a, cur_stream(), pdl);
  } else {
    hk::attention_decode_launch(a, cur_stream(), pdl);
  }
}

void attention_prefill(const Tensor& q, const Tensor& k_cache, const Tensor& v_cache, const Tensor& block_tables,
                       const Tensor& row_seq, const Tensor& row_ctx, double scale, const optional<Tensor>& out,
                       const optional<Tensor>& oq, const optional<Tensor>& od, const optional<Tensor>& os,
                       const optional<Tensor>& sinks, const optional<Tensor>& out_bf16, bool pdl) {
  check_cuda(q, "q");
  TORCH_CHECK(q.dim() == 3 && q.scalar_type() == at::kFloat && q.is_contiguous(), "q must be contiguous fp32 [R, nh, hd]");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.scalar_type() == at::kBFloat16 && v_cache.sizes() == k_cache.sizes(),
              "k_cache / v_cache must be bf16 [blocks, nkv, bs, hd]");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && row_seq.scalar_type() == at::kInt &&
                  row_ctx.scalar_type() == at::kInt, "block tables / rows must be int32");
  hk::AttnDecodeArgs a{};
  a.q = ptr<float>(q);
  a.k_cache = ptr<__nv_bfloat16>(k_cache);
  a.v_cache = ptr<__nv_bfloat16>(v_cache);
  a.block_tables = ptr<int>(block_tables);
  a.max_blocks = (int)block_tables.size(1);
  a.row_seq = ptr<int>(row_seq);
  a.row_ctx = ptr<int>(row_ctx);
  a.scale = (float)scale;
  a.R = (int)q.size(0);
  a.nh = (int)q.size(1);
  a.hd = (int)q.size(2);
  a.nkv = (int)k_cache.size(1);
  a.block_size = (int)k_cache.size(2);
  TORCH_CHECK(k_cache.size(3) == a.hd, "attention prefill: head_dim mismatch");
  a.out = optr<float>(out);
  a.oq = optr<int8_t>(oq);
  a.od = optr<float>(od);
  a.os = optr<float>(os);
  a.sinks = optr<float>(sinks);
  a.out_bf16 = optr<__nv_bfloat16>(out_bf16);
  TORCH_CHECK(!a.oq || (a.od && a.os), "attention prefill: q8 output needs d and s");
  const c10::cuda::CUDAGuard g(q.device());
  hk::attention_prefill_launch(a, cur_stream(), pdl);
}

void argmax(const Tensor& logits, const Tensor& out, bool pdl) {
  check_cuda(logits, "logits");
  TORCH_CHECK(logits.scalar_type() == at::kFloat && out.scalar_type() == at::kInt, "argmax: fp32 logits, int32 out");
  const c10::cuda::CUDAGuard g(logits.device());
  hk::argmax_launch(ptr<float>(logits), logits.stride(0), (int)logits.size(0), (int)logits.size(1), ptr<int>(out),
                    cur_stream(), pdl);
}

void sample(const Tensor& logits, const Tensor& temperature, const optional<Tensor>& top_k,
            const optional<Tensor>& top_p, const optional<Tensor>& rep_penalty, const optional<Tensor>& recent,
            const Tensor& uniforms, const Tensor& out, bool pdl) {
  check_cuda(logits, "logits");
  hk::SampleArgs a{};
  a.logits = ptr<float>(logits);
  a.stride = logits.stride(0);
  a.R = (int)logits.size(0);
  a.V = (int)logits.size(1);
  a.temperature = ptr<float>(temperature);
  a.top_k = optr<int>(top_k);
  a.top_p = optr<float>(top_p);
  a.rep_penalty = optr<float>(rep_penalty);
  a.recent = optr<int>(recent);
  a.recent_n = recent.has_value() ? (int)recent->size(1) : 0;
  a.uniforms = ptr<float>(uniforms);
  a.out = ptr<int>(out);
  const c10::cuda::CUDAGuard g(logits.device());
  hk::sample_launch(a, cur_stream(), pdl);
}

void embed(int64_t fmt, const std::vector<Tensor>& table, const Tensor& ids, const Tensor& out, bool pdl) {
  check_cuda(ids, "ids");
  TORCH_CHECK(ids.scalar_type() == at::kInt, "ids must be int32");
  const c10::cuda::CUDAGuard g(ids.device());
  hk::embed_launch((int)fmt, planes(table), ptr<int>(ids), (int)ids.numel(), (int)out.size(1), ptr<float>(out),
                   out.stride(0), cur_stream(), pdl);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "hawking_b200 sm_100a kernels";
  m.def("gemv", &gemv, py::arg("fmt"), py::arg("epi"), py::arg("w0"), py::arg("w1"), py::arg("N"), py::arg("K"),
        py::arg("xq"), py::arg("xd"), py::arg("xs"), py::arg("y") = py::none(), py::arg("bias") = py::none(),
        py::arg("oq") = py::none(), py::arg("od") = py::none(), py::arg("os") = py::none(),
        py::arg("x_f32") = py::none(), py::arg("norm_w") = py::none(), py::arg("eps") = -1.0,
        py::arg("pdl") = false, py::arg("argmax_slots") = py::none(), py::arg("argmax_offset") = 0,
        py::arg("push_recv") = py::none(), py::arg("push_epoch") = py::none(),
        py::arg("prefetch") = std::vector<Tensor>{});
  m.def("rmsnorm_q8", &rmsnorm_q8, py::arg("x"), py::arg("w"), py::arg("eps"), py::arg("norm"), py::arg("xq"),
        py::arg("xd"), py::arg("xs"), py::arg("y") = py::none(), py::arg("pdl") = false);
  m.def("rmsnorm", &rmsnorm, py::arg("x"), py::arg("w"), py::arg("eps"), py::arg("yf") = py::none(),
        py::arg("yb") = py::none(), py::arg("pdl") = false);
  m.def("rope_append", &rope_append, py::arg("qkv"), py::arg("bias"), py::arg("q_norm"), py::arg("k_norm"),
        py::arg("eps"), py::arg("positions"), py::arg("slots"), py::arg("rope"), py::arg("rot_dim"),
        py::arg("style"), py::arg("q_out"), py::arg("k_cache"), py::arg("v_cache"), py::arg("nh"), py::arg("nkv"),
        py::arg("hd"), py::arg("block_size"), py::arg("block_tables") = py::none(), py::arg("row_seq") = py::none(),
        py::arg("pdl") = false);
  m.def("advance", [](const Tensor& ids, const Tensor& next_ids, const Tensor& positions, const Tensor& row_ctx,
                      int64_t R, bool pdl) {
    const c10::cuda::CUDAGuard g(ids.device());
    hk::advance_launch(ptr<int>(ids), ptr<int>(next_ids), ptr<int>(positions), ptr<int>(row_ctx), (int)R,
                       cur_stream(), pdl);
  }, py::arg("ids"), py::arg("next_ids"), py::arg("positions"), py::arg("row_ctx"), py::arg("R"),
        py::arg("pdl") = false);
  m.def("attention_prefill", &attention_prefill, py::arg("q"), py::arg("k_cache"), py::arg("v_cache"),
        py::arg("block_tables"), py::arg("row_seq"), py::arg("row_ctx"), py::arg("scale"), py::arg("out"),
        py::arg("oq"), py::arg("od"), py::arg("os"), py::arg("sinks"), py::arg("out_bf16"), py::arg("pdl") = false);
  m.def("attention_decode", &attention_decode, py::arg("q"), py::arg("k_cache"), py::arg("v_cache"),
        py::arg("block_tables"), py::arg("row_seq"), py::arg("row_ctx"), py::arg("scale"), py::arg("num_splits"),
        py::arg("part_o"), py::arg("part_lse"), py::arg("out") = py::none(), py::arg("oq") = py::none(),
        py::arg("od") = py::none(), py::arg("os") = py::none(), py::arg("sinks") = py::none(),
        py::arg("out_bf16") = py::none(), py::arg("counters") = py::none(), py::arg("pdl") = false,
        py::arg("cluster") = false, py::arg("tc") = false, py::arg("status") = py::none());
  m.def("argmax", &argmax, py::arg("logits"), py::arg("out"), py::arg("pdl") = false);
  m.def(
      "argmax_finalize",
      [](const Tensor& slots, int64_t rows, const Tensor& out, bool pdl) {
        check_cuda(slots, "slots");
        TORCH_CHECK(slots.scalar_type() == at::kLong && slots.numel() >= rows * hk::kArgmaxSlots,
                    "argmax_finalize: slots must be int64 [rows, 256]");
        TORCH_CHECK(out.scalar_type() == at::kInt && out.numel() >= rows, "argmax_finalize: int32 out");
        const c10::cuda::CUDAGuard g(slots.device());
        hk::argmax_finalize_launch(reinterpret_cast<unsigned long long*>(slots.data_ptr<int64_t>()), (int)rows,
                                   ptr<int>(out), cur_stream(), pdl);
      },
      py::arg("slots"), py::arg("rows"), py::arg("out"), py::arg("pdl") = false);
  m.def("sample", &sample, py::arg("logits"), py::arg("temperature"), py::arg("top_k"), py::arg("top_p"),
        py::arg("rep_penalty"), py::arg("recent"), py::arg("uniforms"), py::arg("out"), py::arg("pdl") = false);
  m.def("embed", &embed, py::arg("fmt"), py::arg("table"), py::arg("ids"), py::arg("out"), py::arg("pdl") = false);
  hk::register_more_kernels(m);
  hk::register_tp_kernels(m);
  hk::register_model_kernels(m);
  hk::register_mg_kernels(m);
  hk::register_ds_kernels(m);
}
