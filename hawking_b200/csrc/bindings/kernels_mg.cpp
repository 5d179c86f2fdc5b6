// torch bindings of the full-precision small-batch GEMV (mma_gemv.cu): weight packing into
// fragment-ordered tiles and the GEMV launch with its input / epilogue modes.
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
template <typename T> T* ptr(const Tensor& t) { return reinterpret_cast<T*>(t.data_ptr()); }
template <typename T> T* optr(const optional<Tensor>& t) { return t.has_value() ? ptr<T>(*t) : nullptr; }

int num_sms(int dev) {
  static int cached[64] = {0};
  if (dev < 0 || dev >= 64) dev = 0;
  if (!cached[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

// Pack Q4_K planes [quants (N, K/2), headers (N, K/16)] into tiles; rowmap int32 [G * 16].
void mg_pack(int64_t fmt, const std::vector<Tensor>& planes, const Tensor& rowmap, int64_t G, int64_t KT,
             const Tensor& out, int64_t math) {
  TORCH_CHECK(planes.size() == 2, "mg_pack: Q4_K expects [quants, headers] planes");
  TORCH_CHECK(rowmap.is_cuda() && rowmap.scalar_type() == at::kInt && rowmap.numel() == G * 16,
              "mg_pack: rowmap must be int32 [G * 16] on the device");
  TORCH_CHECK(out.is_cuda() && out.is_contiguous() && out.numel() == G * KT * hk::mg_tile_bytes((int)fmt),
              "mg_pack: output size mismatch");
  TORCH_CHECK(planes[0].size(1) * 2 == KT * 256 && planes[1].size(1) * 16 == KT * 256, "mg_pack: plane widths vs K");
  hk::WPlanes w{};
  w.p0 = ptr<const uint8_t>(planes[0]);
  w.rb0 = planes[0].stride(0);
  w.p1 = ptr<const uint8_t>(planes[1]);
  w.rb1 = planes[1].stride(0);
  const c10::cuda::CUDAGuard g(out.device());
  hk::mg_pack_launch((int)fmt, (int)math, w, rowmap.data_ptr<int>(), (int)G, (int)KT, ptr<uint8_t>(out), cur_stream());
}

void mg_gemv(int64_t fmt, int64_t xin, int64_t epi, const Tensor& tiles, int64_t G, int64_t KT, int64_t N, int64_t K,
             int64_t nb, const optional<Tensor>& x_f32, const optional<Tensor>& norm_w, double eps,
             const optional<Tensor>& xb, const optional<Tensor>& xfrag, int64_t xfrag_cstride,
             const optional<Tensor>& y, const optional<Tensor>& bias, int64_t F, const optional<Tensor>& hfrag,
             int64_t hfrag_cstride, const optional<Tensor>& hb, const optional<Tensor>& argmax_slots,
             int64_t argmax_offset, const optional<Tensor>& push_recv, const optional<Tensor>& push_epoch,
             const Tensor& part, const Tensor& counters, const Tensor& status, bool pdl, int64_t math,
             const optional<Tensor>& xinfo, const std::vector<int64_t>& rope_order,
             const std::vector<optional<Tensor>>& rope_epi, const std::vector<int64_t>& rope_dims) {
  TORCH_CHECK(tiles.is_cuda() && tiles.is_contiguous(), "mg_gemv: tiles must be a contiguous CUDA tensor");
  TORCH_CHECK(tiles.numel() == G * KT * hk::mg_tile_bytes((int)fmt) && KT * 256 == K, "mg_gemv: tile shape mismatch");
  TORCH_CHECK(nb >= 1 && nb <= 8, "mg_gemv: batch columns must be 1..8");
  const int dev = tiles.device().index();
  const int sms = num_sms(dev);
  TORCH_CHECK(part.is_cuda() && part.scalar_type() == at::kFloat && part.numel() >= (int64_t)sms * 3 * 8 * 2 * 32 * 4,
              "mg_gemv: partial scratch too small");
  TORCH_CHECK(counters.is_cuda() && counters.scalar_type() == at::kInt && counters.numel() >= G,
              "mg_gemv: counters too small");
  hk::MgArgs a{};
  a.tiles = ptr<const uint8_t>(tiles);
  a.G = (int)G;
  a.KT = (int)KT;
  a.N = (int)N;
  a.K = (int)K;
  a.nb = (int)nb;
  if (xin == hk::MG_X_NORM) {
    TORCH_CHECK(x_f32.has_value() && x_f32->scalar_type() == at::kFloat && x_f32->stride(-1) == 1 &&
                    x_f32->size(0) >= nb && x_f32->size(1) >= K,
                "mg_gemv: x_f32 must be fp32 [nb, K]");
    TORCH_CHECK(x_f32->stride(0) % 4 == 0 && reinterpret_cast<uintptr_t>(x_f32->data_ptr()) % 16 == 0,
                "mg_gemv: x_f32 rows must be 16-byte aligned");
    a.x_f32 = x_f32->data_ptr<float>();
    a.x_f32_stride = x_f32->stride(0);
    a.norm_w = optr<const float>(norm_w);
    a.eps = (float)eps;
  } else if (xin == hk::MG_X_BF16) {
    TORCH_CHECK(xb.has_value() && xb->scalar_type() == at::kBFloat16 && xb->stride(-1) == 1 && xb->size(0) >= nb &&
                    xb->size(1) >= K && xb->stride(0) % 2 == 0 &&
                    reinterpret_cast<uintptr_t>(xb->data_ptr()) % 4 == 0,
                "mg_gemv: xb must be bf16 [nb, K] with even row stride");
    TORCH_CHECK(math != hk::MG_MATH_INT ||
                    (xb->stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(xb->data_ptr()) % 16 == 0),
                "mg_gemv: integer math reads xb rows with 16-byte loads (16-byte aligned rows required)");
    a.xb = ptr<const __nv_bfloat16>(*xb);
    a.xb_stride = xb->stride(0);
  } else if (xin == hk::MG_X_FRAG) {
    TORCH_CHECK(xfrag.has_value() && xfrag->is_cuda() &&
                    xfrag->numel() * xfrag->element_size() >= (nb - 1) * xfrag_cstride * 16 + K * 2,
                "mg_gemv: fragment-order input too small");
    a.xfrag = ptr<const uint4>(*xfrag);
    a.xfrag_cstride = xfrag_cstride;
    if (math == hk::MG_MATH_INT) {
      TORCH_CHECK(xinfo.has_value() && xinfo->is_cuda() && xinfo->scalar_type() == at::kFloat &&
                      xinfo->numel() >= nb * (K / 32) * 2,
                  "mg_gemv: integer fragment input needs its block info (fp32 [nb, K/32, 2])");
      a.xinfo = reinterpret_cast<const float2*>(xinfo->data_ptr<float>());
    }
  } else {
    TORCH_CHECK(false, "mg_gemv: bad input mode");
  }
  if (y.has_value()) {
    TORCH_CHECK(y->scalar_type() == at::kFloat && y->stride(-1) == 1 && y->size(0) >= nb && y->size(-1) >= N,
                "mg_gemv: y must be fp32 [nb, >= N]");
    a.y = ptr<float>(*y);
    a.y_stride = y->stride(0);
  }
  a.bias = optr<const float>(bias);
  a.F = (int)F;
  if (hfrag.has_value()) {
    a.hfrag = ptr<__nv_bfloat16>(*hfrag);
    a.hfrag_cstride = hfrag_cstride;
  }
  if (hb.has_value()) {
    TORCH_CHECK(hb->scalar_type() == at::kBFloat16 && hb->stride(-1) == 1, "mg_gemv: hb must be bf16 rows");
    a.hb = ptr<__nv_bfloat16>(*hb);
    a.hb_stride = hb->stride(0);
  }
  if (argmax_slots.has_value()) {
    TORCH_CHECK(epi == hk::MG_STORE && argmax_slots->scalar_type() == at::kLong &&
                    argmax_slots->numel() >= nb * hk::kArgmaxSlots,
                "mg_gemv: argmax slots must be int64 [nb, 256] with the STORE epilogue");
    a.argmax_slots = reinterpret_cast<unsigned long long*>(argmax_slots->data_ptr<int64_t>());
    a.argmax_offset = argmax_offset;
  }
  if (epi == hk::MG_PUSH) {
    TORCH_CHECK(push_recv.has_value() && push_epoch.has_value() && push_recv->scalar_type() == at::kLong &&
                    push_epoch->scalar_type() == at::kInt,
                "mg_gemv push: int64 device pointer table and int32 epoch required");
    a.push_recv = reinterpret_cast<unsigned long long* const*>(push_recv->data_ptr<int64_t>());
    a.push_epoch = push_epoch->data_ptr<int>();
    a.push_n = (int)push_recv->numel();
  }
  if (!rope_order.empty()) {  // (heads, hd, rot, style): tiles packed in RoPE-pair order
    TORCH_CHECK(rope_order.size() == 4 && (epi == hk::MG_STORE || epi == hk::MG_ROPE),
                "mg_gemv: rope_order is (heads, hd, rot, style), STORE / ROPE epilogues");
    TORCH_CHECK(rope_order[1] % 16 == 0 && rope_order[2] % 16 == 0 && rope_order[2] <= rope_order[1],
                "mg_gemv: rope_order needs hd and rot multiples of 16");
    a.rp_heads = (int)rope_order[0];
    a.rp_hd = (int)rope_order[1];
    a.rp_rot = (int)rope_order[2];
    a.rp_style = (int)rope_order[3];
  }
  if (epi == hk::MG_ROPE) {
    // rope_epi: (rope table, positions, row_seq, block_tables, k_cache, v_cache, q_out)
    // rope_dims: (nh, nkv, block_size)
    TORCH_CHECK(!rope_order.empty() && rope_epi.size() == 7 && rope_dims.size() == 3,
                "mg_gemv rope: RoPE-ordered tiles, 7 tensors and (nh, nkv, block_size) required");
    for (int i = 0; i < 7; ++i) TORCH_CHECK(rope_epi[i].has_value() && rope_epi[i]->is_cuda(), "mg_gemv rope: tensor ", i);
    const Tensor& kc = *rope_epi[4];
    const Tensor& vc = *rope_epi[5];
    TORCH_CHECK(kc.scalar_type() == at::kBFloat16 && kc.is_contiguous() && vc.is_contiguous() &&
                    kc.size(-1) == rope_order[1] && kc.size(-2) == rope_dims[2] && kc.size(-3) == rope_dims[1],
                "mg_gemv rope: caches must be contiguous bf16 [blocks, nkv, block_size, hd]");
    TORCH_CHECK(rope_epi[6]->scalar_type() == at::kFloat && rope_epi[6]->numel() >= nb * rope_dims[0] * rope_order[1],
                "mg_gemv rope: q_out must be fp32 [nb, nh, hd]");
    TORCH_CHECK(rope_order[0] == rope_dims[0] + rope_dims[1] && N == (rope_dims[0] + 2 * rope_dims[1]) * rope_order[1],
                "mg_gemv rope: head counts do not match the matrix");
    a.rope = rope_epi[0]->data_ptr<float>();
    a.positions = rope_epi[1]->data_ptr<int>();
    a.row_seq = rope_epi[2]->data_ptr<int>();
    a.block_tables = rope_epi[3]->data_ptr<int>();
    a.max_blocks = (int)rope_epi[3]->size(1);
    a.block_size = (int)rope_dims[2];
    a.k_cache = ptr<__nv_bfloat16>(kc);
    a.v_cache = ptr<__nv_bfloat16>(vc);
    a.cache_blocks = kc.size(0);
    a.q_out = rope_epi[6]->data_ptr<float>();
    a.nh = (int)rope_dims[0];
    a.nkv = (int)rope_dims[1];
  }
  a.part = reinterpret_cast<float4*>(part.data_ptr<float>());
  a.counters = counters.data_ptr<int>();
  a.status = status.data_ptr<int>();
  a.math = (int)math;
  const c10::cuda::CUDAGuard g(tiles.device());
  hk::mg_gemv_launch((int)fmt, (int)xin, (int)epi, a, sms, cur_stream(), pdl);
}
void mg_quant(const Tensor& x, int64_t nb, int64_t K, const Tensor& xfrag, int64_t cstride, const Tensor& xinfo,
              bool pdl) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.stride(-1) == 1 && x.size(0) >= nb &&
                  x.size(1) >= K && x.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
              "mg_quant: x must be bf16 [nb, K] with 16-byte aligned rows");
  TORCH_CHECK(xfrag.is_cuda() && xfrag.numel() * xfrag.element_size() >= nb * cstride * 16, "mg_quant: xfrag too small");
  TORCH_CHECK(xinfo.is_cuda() && xinfo.scalar_type() == at::kFloat && xinfo.numel() >= nb * (K / 32) * 2,
              "mg_quant: xinfo too small");
  const c10::cuda::CUDAGuard g(x.device());
  hk::mg_quant_launch(ptr<const __nv_bfloat16>(x), x.stride(0), (int)nb, (int)K, ptr<uint4>(xfrag), cstride,
                      reinterpret_cast<float2*>(xinfo.data_ptr<float>()), cur_stream(), pdl);
}
}  // namespace

namespace hk {
void register_mg_kernels(py::module_& m) {
  m.def("mg_pack", &mg_pack, py::arg("fmt"), py::arg("planes"), py::arg("rowmap"), py::arg("G"), py::arg("KT"),
        py::arg("out"), py::arg("math") = 0);
  m.def("mg_quant", &mg_quant, py::arg("x"), py::arg("nb"), py::arg("K"), py::arg("xfrag"), py::arg("cstride"),
        py::arg("xinfo"), py::arg("pdl") = false);
  m.def("mg_tile_bytes", &hk::mg_tile_bytes);
  m.def("mg_num_sms", [](int64_t dev) { return num_sms((int)dev); });
  m.def("mg_gemv", &mg_gemv, py::arg("fmt"), py::arg("xin"), py::arg("epi"), py::arg("tiles"), py::arg("G"),
        py::arg("KT"), py::arg("N"), py::arg("K"), py::arg("nb"), py::arg("x_f32") = py::none(),
        py::arg("norm_w") = py::none(), py::arg("eps") = 1e-5, py::arg("xb") = py::none(),
        py::arg("xfrag") = py::none(), py::arg("xfrag_cstride") = 0, py::arg("y") = py::none(),
        py::arg("bias") = py::none(), py::arg("F") = 0, py::arg("hfrag") = py::none(),
        py::arg("hfrag_cstride") = 0, py::arg("hb") = py::none(), py::arg("argmax_slots") = py::none(),
        py::arg("argmax_offset") = 0, py::arg("push_recv") = py::none(), py::arg("push_epoch") = py::none(),
        py::arg("part"), py::arg("counters"), py::arg("status"), py::arg("pdl") = false, py::arg("math") = 0,
        py::arg("xinfo") = py::none(), py::arg("rope_order") = std::vector<int64_t>{},
        py::arg("rope_epi") = std::vector<optional<Tensor>>{}, py::arg("rope_dims") = std::vector<int64_t>{});
}
}  // namespace hk
