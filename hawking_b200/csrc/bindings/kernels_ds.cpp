// torch bindings of the persistent decode step (decode_step.cu): the per-layer pointer table and the
// one-launch step.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstring>

#include "../kernels/api.h"
#include "../kernels/kernels_api.h"

namespace py = pybind11;
using at::Tensor;
using c10::optional;

namespace {
template <typename T> T* ptr(const Tensor& t) { return reinterpret_cast<T*>(t.data_ptr()); }
template <typename T> T* optr(const optional<Tensor>& t) { return t.has_value() ? ptr<T>(*t) : nullptr; }

// Layer i: (qkv tiles, o tiles, gate/up tiles, down tiles, attn_norm, ffn_norm, qkv_bias or None).
// Returns the DsLayer array as a uint8 tensor on `device`.
Tensor ds_layer_table(const std::vector<std::vector<optional<Tensor>>>& layers, const at::Device& device) {
  std::vector<hk::DsLayer> rows(layers.size());
  for (size_t i = 0; i < layers.size(); ++i) {
    const auto& t = layers[i];
    TORCH_CHECK(t.size() == 7, "ds_layer_table: each layer is (qkv, o, gu, down, attn_norm, ffn_norm, qkv_bias)");
    for (int k = 0; k < 6; ++k)
      TORCH_CHECK(t[k].has_value() && t[k]->is_cuda() && t[k]->is_contiguous(), "ds_layer_table: tensor ", k,
                  " of layer ", i, " must be a contiguous CUDA tensor");
    for (int k = 4; k < 7; ++k)
      if (t[k].has_value()) TORCH_CHECK(t[k]->scalar_type() == at::kFloat, "ds_layer_table: norms / bias are fp32");
    rows[i] = hk::DsLayer{ptr<const uint8_t>(*t[0]), ptr<const uint8_t>(*t[1]), ptr<const uint8_t>(*t[2]),
                          ptr<const uint8_t>(*t[3]), ptr<const float>(*t[4]), ptr<const float>(*t[5]),
                          optr<const float>(t[6])};
  }
  Tensor host = torch::empty({(int64_t)(rows.size() * sizeof(hk::DsLayer))}, torch::kUInt8);
  std::memcpy(host.data_ptr(), rows.data(), rows.size() * sizeof(hk::DsLayer));
  return host.to(device);
}

// dims: H, F, nh, nkv, hd, rot, rope_style, block_size, max_blocks, num_cache_blocks, nb, splits, V, L
hk::DsArgs args_from_dims(const std::vector<int64_t>& d, double eps, double scale) {
  TORCH_CHECK(d.size() == 14, "decode step: 14 dims expected");
  hk::DsArgs a{};
  a.H = (int)d[0];
  a.F = (int)d[1];
  a.nh = (int)d[2];
  a.nkv = (int)d[3];
  a.hd = (int)d[4];
  a.rot = (int)d[5];
  a.rope_style = (int)d[6];
  a.block_size = (int)d[7];
  a.max_blocks = (int)d[8];
  a.num_cache_blocks = (int)d[9];
  a.nb = (int)d[10];
  a.splits = (int)d[11];
  a.V = (int)d[12];
  a.L = (int)d[13];
  a.eps = (float)eps;
  a.scale = (float)scale;
  return a;
}

bool ds_supported_dims(const std::vector<int64_t>& dims) { return hk::ds_supported(args_from_dims(dims, 1e-5, 1.0)); }

void ds_step(const Tensor& table, const std::vector<int64_t>& dims, double eps, double scale, const Tensor& positions,
             const Tensor& row_seq, const Tensor& row_ctx, const Tensor& block_tables, const Tensor& rope,
             const Tensor& x, const Tensor& q, const Tensor& k_cache, const Tensor& v_cache, const Tensor& att_o,
             const Tensor& att_ml, const Tensor& att_cnt, const Tensor& a_limbs, const Tensor& a_info,
             const Tensor& hf, const Tensor& h_limbs, const Tensor& h_info, const Tensor& h_cnt, const Tensor& part,
             const Tensor& counters, const Tensor& head, const Tensor& out_norm, const optional<Tensor>& logits,
             const optional<Tensor>& argmax_slots, const Tensor& bar, const Tensor& status, int64_t wait_ns,
             const optional<Tensor>& trace, const optional<Tensor>& tstamp) {
  hk::DsArgs a = args_from_dims(dims, eps, scale);
  const int Ka = a.nh * a.hd, G = a.nh / a.nkv, nb = a.nb;
  TORCH_CHECK(table.is_cuda() && table.numel() == (int64_t)(a.L * sizeof(hk::DsLayer)), "ds_step: layer table size");
  TORCH_CHECK(x.scalar_type() == at::kFloat && x.is_contiguous() && x.numel() >= (int64_t)nb * a.H, "ds_step: x");
  TORCH_CHECK(q.scalar_type() == at::kFloat && q.numel() >= (int64_t)nb * Ka, "ds_step: q");
  TORCH_CHECK(k_cache.scalar_type() == at::kBFloat16 && k_cache.is_contiguous() && v_cache.is_contiguous() &&
                  k_cache.numel() == (int64_t)a.L * a.num_cache_blocks * a.nkv * a.block_size * a.hd &&
                  v_cache.numel() == k_cache.numel(),
              "ds_step: caches must be contiguous bf16 [L, blocks, nkv, block_size, hd]");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && block_tables.size(1) == a.max_blocks, "ds_step: block tables");
  TORCH_CHECK(att_o.numel() >= (int64_t)nb * a.nkv * a.splits * G * a.hd && att_ml.numel() >= (int64_t)nb * a.nkv * a.splits * G * 2 &&
                  att_cnt.numel() >= (int64_t)nb * a.nkv,
              "ds_step: attention scratch too small");
  TORCH_CHECK(a_limbs.numel() * a_limbs.element_size() >= (int64_t)nb * Ka * 2 && a_info.numel() >= (int64_t)nb * Ka / 16,
              "ds_step: attention limbs too small");
  TORCH_CHECK(hf.numel() >= (int64_t)nb * a.F && h_limbs.numel() * h_limbs.element_size() >= (int64_t)nb * a.F * 2 &&
                  h_info.numel() >= (int64_t)nb * a.F / 16 && h_cnt.numel() >= a.F / 32,
              "ds_step: SwiGLU scratch too small");
  TORCH_CHECK(head.is_cuda() && head.numel() == (int64_t)((a.V + 15) / 16) * (a.H / 256) * hk::mg_tile_bytes(12),
              "ds_step: LM head tiles");
  TORCH_CHECK(bar.scalar_type() == at::kInt && bar.numel() >= 2 && status.scalar_type() == at::kInt, "ds_step: bar / status");
  if (logits.has_value()) TORCH_CHECK(logits->numel() >= (int64_t)nb * a.V && logits->is_contiguous(), "ds_step: logits");
  a.layers = reinterpret_cast<const hk::DsLayer*>(table.data_ptr());
  a.positions = positions.data_ptr<int>();
  a.row_seq = row_seq.data_ptr<int>();
  a.row_ctx = row_ctx.data_ptr<int>();
  a.block_tables = block_tables.data_ptr<int>();
  a.rope = rope.data_ptr<float>();
  a.x = x.data_ptr<float>();
  a.q = q.data_ptr<float>();
  a.k_cache = ptr<__nv_bfloat16>(k_cache);
  a.v_cache = ptr<__nv_bfloat16>(v_cache);
  a.att_o = att_o.data_ptr<float>();
  a.att_ml = reinterpret_cast<float2*>(att_ml.data_ptr<float>());
  a.att_cnt = att_cnt.data_ptr<int>();
  a.a_limbs = ptr<uint4>(a_limbs);
  a.a_info = reinterpret_cast<float2*>(a_info.data_ptr<float>());
  a.hf = hf.data_ptr<float>();
  a.h_limbs = ptr<uint4>(h_limbs);
  a.h_info = reinterpret_cast<float2*>(h_info.data_ptr<float>());
  a.h_cnt = h_cnt.data_ptr<int>();
  a.part = reinterpret_cast<float4*>(part.data_ptr<float>());
  a.counters = counters.data_ptr<int>();
  a.head = ptr<const uint8_t>(head);
  a.out_norm = out_norm.data_ptr<float>();
  a.logits = logits.has_value() ? logits->data_ptr<float>() : nullptr;
  a.argmax_slots = argmax_slots.has_value() ? reinterpret_cast<unsigned long long*>(argmax_slots->data_ptr()) : nullptr;
  a.bar = reinterpret_cast<unsigned int*>(bar.data_ptr<int>());
  a.status = status.data_ptr<int>();
  a.wait_ns = wait_ns > 0 ? wait_ns : 1000000000ll;
  if (trace.has_value()) {
    TORCH_CHECK(trace->scalar_type() == at::kInt && trace->is_cuda() && trace->numel() >= hk::ds_grid(x.device().index()) * 4,
                "ds_step: trace must be int32 [grid, 4]");
    a.trace = trace->data_ptr<int>();
  }
  if (tstamp.has_value()) {
    TORCH_CHECK(tstamp->scalar_type() == at::kLong && tstamp->is_cuda() && tstamp->numel() >= (5 * a.L + 2) * 4,
                "ds_step: tstamp must be int64 [5 L + 2, 4]");
    a.tstamp = reinterpret_cast<long long*>(tstamp->data_ptr<int64_t>());
  }
  const c10::cuda::CUDAGuard g(x.device());
  hk::ds_launch(a, at::cuda::getCurrentCUDAStream().stream());
}
}  // namespace

namespace hk {
void register_ds_kernels(py::module_& m) {
  m.def("ds_layer_table", &ds_layer_table, py::arg("layers"), py::arg("device"));
  m.def("ds_supported", &ds_supported_dims, py::arg("dims"));
  m.def("ds_grid", [](int64_t dev) { return hk::ds_grid((int)dev); });
  m.def("ds_step", &ds_step, py::arg("table"), py::arg("dims"), py::arg("eps"), py::arg("scale"),
        py::arg("positions"), py::arg("row_seq"), py::arg("row_ctx"), py::arg("block_tables"), py::arg("rope"),
        py::arg("x"), py::arg("q"), py::arg("k_cache"), py::arg("v_cache"), py::arg("att_o"), py::arg("att_ml"),
        py::arg("att_cnt"), py::arg("a_limbs"), py::arg("a_info"), py::arg("hf"), py::arg("h_limbs"),
        py::arg("h_info"), py::arg("h_cnt"), py::arg("part"), py::arg("counters"), py::arg("head"),
        py::arg("out_norm"), py::arg("logits") = py::none(), py::arg("argmax_slots") = py::none(), py::arg("bar"),
        py::arg("status"), py::arg("wait_ns") = 0, py::arg("trace") = py::none(), py::arg("tstamp") = py::none());
}
}  // namespace hk
