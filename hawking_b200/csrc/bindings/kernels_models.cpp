// torch bindings for the hybrid-model kernels: `.gravity` mixed-codec GEMVs (dense and routed
// experts) and gated DeltaNet.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <climits>

#include <stdexcept>
#include <string>

#include "../kernels/api.h"
#include "../kernels/kernels_api.h"

namespace py = pybind11;
using at::Tensor;
using c10::optional;

namespace {
cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }
template <typename T> T* ptr(const Tensor& t) { return reinterpret_cast<T*>(t.data_ptr()); }
template <typename T> T* optr(const optional<Tensor>& t) { return t.has_value() ? ptr<T>(*t) : nullptr; }

// Pack descriptors (codes / scales tensors + codec fields) into a device byte tensor.
Tensor mixed_descs(const std::vector<Tensor>& codes, const std::vector<Tensor>& scales, const std::vector<int64_t>& kind,
                   const std::vector<int64_t>& bits, const std::vector<int64_t>& group,
                   const std::vector<int64_t>& zeros) {
  const size_t n = codes.size();
  TORCH_CHECK(scales.size() == n && kind.size() == n && bits.size() == n && group.size() == n, "mixed_descs: lengths");
  std::vector<hk::MixedDesc> h(n);
  for (size_t i = 0; i < n; ++i) {
    TORCH_CHECK(codes[i].is_cuda() && codes[i].scalar_type() == at::kByte && codes[i].dim() == 2, "codes: uint8 [rows, bytes]");
    const bool fp8 = kind[i] == hk::MIXED_FP8 || kind[i] == hk::MIXED_FP4;  // fp32 scales
    TORCH_CHECK(scales[i].is_cuda() && scales[i].scalar_type() == (fp8 ? at::kFloat : at::kHalf) && scales[i].dim() == 2,
                "scales: fp16 (fp32 for fp8 / fp4) [rows, groups]");
    TORCH_CHECK((reinterpret_cast<uintptr_t>(codes[i].data_ptr()) & 15) == 0 && codes[i].stride(0) % 16 == 0,
                "codes rows must be 16-byte aligned");
    h[i].codes = ptr<uint8_t>(codes[i]);
    h[i].scales = fp8 ? nullptr : ptr<__half>(scales[i]);
    h[i].scales_f32 = fp8 ? ptr<float>(scales[i]) : nullptr;
    h[i].code_row_bytes = codes[i].stride(0);
    h[i].scale_row_elems = scales[i].stride(0);
    h[i].kind = (int)kind[i];
    h[i].bits = (int)bits[i];
    h[i].group = (int)group[i];
    // the code's zero point: 2^(bits-1) - 1 for HGRAVU01; HQ30UQ4 stores q + 8 (zero 8)
    h[i].bound = kind[i] == hk::MIXED_UNIFORM ? (i < zeros.size() && zeros[i] >= 0 ? (int)zeros[i]
                                                                                    : (1 << (bits[i] - 1)) - 1)
                                              : 0;
    TORCH_CHECK(kind[i] == hk::MIXED_BINARY ? bits[i] == 1
                                            : (kind[i] == hk::MIXED_FP8 || kind[i] == hk::MIXED_Q4K || kind[i] == hk::MIXED_FP4
                                                   ? bits[i] == (kind[i] == hk::MIXED_FP8 ? 8 : 4)
                                                   : (bits[i] == 2 || bits[i] == 4 || bits[i] == 8)),
                "mixed codec: binary (1 bit), uniform 2/4/8 bits, fp8 (8 bits), Q4_K or fp4 (4 bits)");
    TORCH_CHECK(kind[i] != hk::MIXED_FP4 || group[i] == 32, "mixed fp4: one scale per 32 columns");
    TORCH_CHECK(group[i] % 32 == 0, "mixed codec: group must be a multiple of 32");
    TORCH_CHECK(kind[i] != hk::MIXED_Q4K || (group[i] == 256 && scales[i].stride(0) % 8 == 0 &&
                                             (reinterpret_cast<uintptr_t>(scales[i].data_ptr()) & 15) == 0),
                "mixed Q4_K: 256-element super-blocks, 16-byte aligned header rows");
  }
  Tensor out = torch::empty({(int64_t)(n * sizeof(hk::MixedDesc))},
                            torch::TensorOptions().dtype(torch::kUInt8).device(codes.empty() ? torch::kCPU : codes[0].device()));
  if (n) {
    const c10::cuda::CUDAGuard g(codes[0].device());
    C10_CUDA_CHECK(cudaMemcpyAsync(out.data_ptr(), h.data(), n * sizeof(hk::MixedDesc), cudaMemcpyHostToDevice,
                                   cur_stream()));
    C10_CUDA_CHECK(cudaStreamSynchronize(cur_stream()));
  }
  return out;
}

void mixed_gemv(int64_t epi, const Tensor& descs, int64_t d0, int64_t d1, int64_t N, int64_t K, const Tensor& xq,
                const Tensor& xd, const Tensor& xs, const optional<Tensor>& y, double alpha, const optional<Tensor>& oq,
                const optional<Tensor>& od, const optional<Tensor>& os, bool pdl, const optional<Tensor>& gate_logit,
                const optional<Tensor>& push_table, const optional<Tensor>& push_epoch,
                const optional<Tensor>& argmax_slots, int64_t argmax_offset) {
  hk::MixedGemvArgs a{};
  if (argmax_slots.has_value()) {
    TORCH_CHECK(argmax_slots->scalar_type() == at::kLong && argmax_slots->size(0) >= xq.size(0) &&
                    argmax_slots->size(1) == hk::kArgmaxSlots, "mixed_gemv: argmax slots [rows, 256] int64");
    a.argmax_slots = reinterpret_cast<unsigned long long*>(argmax_slots->data_ptr<int64_t>());
    a.argmax_offset = argmax_offset;
  }
  if (push_table.has_value()) {
    TORCH_CHECK(push_table->scalar_type() == at::kLong && push_epoch.has_value(), "mixed_gemv push: int64 table + epoch");
    a.push_recv = reinterpret_cast<unsigned long long* const*>(push_table->data_ptr<int64_t>());
    a.push_n = (int)push_table->numel();
    a.push_epoch = push_epoch->data_ptr<int>();
  }
  a.desc = reinterpret_cast<const hk::MixedDesc*>(descs.data_ptr());
  a.d0 = (int)d0;
  a.d1 = (int)d1;
  a.N = (int)N;
  a.K = (int)K;
  a.nb = (int)xq.size(0);
  a.xq = ptr<int8_t>(xq);
  a.xd = ptr<float>(xd);
  a.xs = ptr<float>(xs);
  a.x_stride_q = xq.stride(0);
  a.x_stride_s = xd.stride(0);
  a.alpha = (float)alpha;
  if (gate_logit.has_value()) {
    a.gate_logit = ptr<float>(*gate_logit);
    a.gate_stride = gate_logit->stride(0);
  }
  if (y.has_value()) {
    a.y = ptr<float>(*y);
    a.y_stride = y->stride(0);
  }
  if (oq.has_value()) {
    a.oq = ptr<int8_t>(*oq);
    a.od = ptr<float>(*od);
    a.os = ptr<float>(*os);
    a.o_stride_q = oq->stride(0);
    a.o_stride_s = od->stride(0);
  }
  TORCH_CHECK(epi == hk::EPI_SWIGLU_Q8 ? a.oq != nullptr : (epi == hk::EPI_PUSH ? a.push_recv != nullptr : a.y != nullptr),
              "mixed_gemv: output missing");
  const c10::cuda::CUDAGuard g(xq.device());
  hk::mixed_gemv_launch((int)epi, a, cur_stream(), pdl);
}

void moe_active(const Tensor& counts, const Tensor& active, const Tensor& n_active, bool pdl) {
  const c10::cuda::CUDAGuard g(counts.device());
  hk::moe_active_launch(ptr<int>(counts), (int)counts.numel(), ptr<int>(active), ptr<int>(n_active), cur_stream(), pdl);
}

using bf16_t = __nv_bfloat16;
static const bf16_t* bfp(const Tensor& t) { return reinterpret_cast<const bf16_t*>(t.data_ptr()); }
static bf16_t* bfpm(const Tensor& t) { return reinterpret_cast<bf16_t*>(t.data_ptr()); }

void mixed_dequant_bf16(const Tensor& descs, const Tensor& didx, const Tensor& drow, int64_t rows, int64_t K,
                        const Tensor& out, bool pdl) {
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.stride(-1) == 1, "mixed_dequant_bf16: bf16 rows");
  TORCH_CHECK(didx.scalar_type() == at::kInt && drow.scalar_type() == at::kInt && didx.numel() == drow.numel(),
              "mixed_dequant_bf16: int32 index / row lists of one length");
  const c10::cuda::CUDAGuard g(out.device());
  hk::mixed_dequant_bf16_launch(reinterpret_cast<const hk::MixedDesc*>(descs.data_ptr()), didx.data_ptr<int>(),
                                drow.data_ptr<int>(), (int)didx.numel(), (int)rows, (int)K, bfpm(out), out.stride(0),
                                cur_stream(), pdl);
}

void tc_gemm_bf16(const Tensor& w, const Tensor& x, int64_t N, int64_t M, const optional<Tensor>& y,
                  const optional<Tensor>& h, bool atomic, bool y_zeroed, int64_t k_splits, int64_t bn,
                  const Tensor& status, bool pdl, const optional<Tensor>& tiles, const optional<Tensor>& n_tiles,
                  int64_t max_tiles, int64_t group_rows) {
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && x.scalar_type() == at::kBFloat16 && w.stride(-1) == 1 &&
              x.stride(-1) == 1 && w.size(1) == x.size(1), "tc_gemm_bf16: bf16 rows, same K");
  hk::TcBf16Args g{};
  g.w = bfp(w);
  g.w_stride = w.stride(0);
  g.w_rows = (int)w.size(0);
  g.N = (int)N;
  g.K = (int)w.size(1);
  g.x = bfp(x);
  g.x_stride = x.stride(0);
  g.x_rows = (int)x.size(0);
  g.M = (int)M;
  if (y.has_value()) {
    TORCH_CHECK(y->scalar_type() == at::kFloat && y->stride(-1) == 1, "tc_gemm_bf16: fp32 rows out");
    g.y = y->data_ptr<float>();
    g.y_stride = y->stride(0);
  }
  if (h.has_value()) {
    TORCH_CHECK(h->scalar_type() == at::kBFloat16 && h->stride(-1) == 1, "tc_gemm_bf16: bf16 SwiGLU rows out");
    g.h = bfpm(*h);
    g.h_stride = h->stride(0);
  }
  TORCH_CHECK(g.y || g.h, "tc_gemm_bf16: an output");
  g.atomic = atomic;
  g.y_zeroed = y_zeroed;
  g.k_splits = (int)k_splits;
  g.bn = (int)bn;
  g.status = status.data_ptr<int>();
  g.pdl = pdl;
  if (tiles.has_value()) {
    TORCH_CHECK(n_tiles.has_value() && tiles->scalar_type() == at::kInt, "tc_gemm_bf16: int32 tile list + count");
    g.tiles = tiles->data_ptr<int>();
    g.n_tiles = n_tiles->data_ptr<int>();
    g.max_tiles = (int)max_tiles;
    g.group_rows = (int)group_rows;
  }
  const c10::cuda::CUDAGuard guard(x.device());
  hk::tc_gemm_bf16_launch(g, cur_stream());
}

void moe_tiles(const Tensor& counts, const Tensor& offsets, int64_t E1, int64_t bn, const Tensor& tiles,
               const Tensor& n_tiles, bool pdl, int64_t e_lo, int64_t e_hi, int64_t shared_e) {
  const c10::cuda::CUDAGuard g(counts.device());
  hk::moe_tiles_launch(counts.data_ptr<int>(), offsets.data_ptr<int>(), (int)E1, (int)bn, tiles.data_ptr<int>(),
                       n_tiles.data_ptr<int>(), (int)e_lo, (int)e_hi, (int)shared_e, cur_stream(), pdl);
}

void moe_gather_bf16(const Tensor& sorted, int64_t PS, int64_t P, int64_t k, const Tensor& x, const Tensor& xg,
                     const Tensor& pos, bool pdl) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && xg.scalar_type() == at::kBFloat16, "moe_gather_bf16: bf16 rows");
  const c10::cuda::CUDAGuard g(x.device());
  hk::moe_gather_bf16_launch(sorted.data_ptr<int>(), (int)PS, (int)P, (int)k, bfp(x), x.stride(0), (int)x.size(1),
                             bfpm(xg), xg.stride(0), pos.data_ptr<int>(), cur_stream(), pdl);
}

void moe_combine(const Tensor& y, const Tensor& pos, const Tensor& w, int64_t T, int64_t k, bool shared,
                 const optional<Tensor>& shared_gate, const Tensor& x, bool pdl, const optional<Tensor>& ids,
                 int64_t e_lo, int64_t e_hi) {
  TORCH_CHECK(y.scalar_type() == at::kFloat && x.scalar_type() == at::kFloat, "moe_combine: fp32 rows");
  const c10::cuda::CUDAGuard g(x.device());
  hk::moe_combine_launch(y.data_ptr<float>(), y.stride(0), pos.data_ptr<int>(), w.data_ptr<float>(), (int)T, (int)k,
                         shared, shared_gate.has_value() ? shared_gate->data_ptr<float>() : nullptr,
                         shared_gate.has_value() ? (shared_gate->dim() > 1 ? shared_gate->stride(0) : 1) : 0,
                         x.data_ptr<float>(), x.stride(0), (int)x.size(1),
                         ids.has_value() ? ids->data_ptr<int>() : nullptr, (int)e_lo, (int)e_hi, cur_stream(), pdl);
}

void qweight_dequant_bf16(int64_t fmt, const std::vector<Tensor>& planes, int64_t K, int64_t group_rows,
                          int64_t dst_group_rows, int64_t dst_off, const Tensor& out, bool pdl) {
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.stride(-1) == 1, "qweight_dequant_bf16: bf16 rows");
  TORCH_CHECK(!planes.empty() && planes.size() <= 4, "qweight_dequant_bf16: 1-4 planes");
  hk::WPlanes w{};
  const uint8_t** p[4] = {&w.p0, &w.p1, &w.p2, &w.p3};
  int64_t* rb[4] = {&w.rb0, &w.rb1, &w.rb2, &w.rb3};
  for (size_t i = 0; i < planes.size(); ++i) {
    *p[i] = reinterpret_cast<const uint8_t*>(planes[i].data_ptr());
    *rb[i] = planes[i].stride(0);
  }
  const c10::cuda::CUDAGuard g(out.device());
  hk::qweight_dequant_bf16_launch((int)fmt, w, (int)planes[0].size(0), (int)K, (int)group_rows, (int)dst_group_rows,
                                  (int)dst_off, bfpm(out), out.stride(0), cur_stream(), pdl);
}

void q8_to_bf16(const Tensor& q, const Tensor& d, const Tensor& out, bool pdl) {
  const c10::cuda::CUDAGuard g(q.device());
  hk::q8_to_bf16_launch(q.data_ptr<int8_t>(), d.data_ptr<float>(), q.stride(0), d.stride(0), (int)q.size(0),
                        (int)q.size(1), bfpm(out), out.stride(0), cur_stream(), pdl);
}

void moe_mixed_gemv(int64_t epi, const Tensor& descs, int64_t base0, int64_t base1, int64_t N, int64_t K, int64_t k,
                    const Tensor& counts, const Tensor& offsets, const Tensor& sorted, const Tensor& active,
                    const Tensor& n_active, int64_t max_active, const Tensor& xq, const Tensor& xd, const Tensor& xs,
                    const optional<Tensor>& oq, const optional<Tensor>& od, const optional<Tensor>& os,
                    const optional<Tensor>& y, const optional<Tensor>& route_w, bool pdl, int64_t routed_pairs,
                    bool direct, int64_t e_lo, int64_t e_count, int64_t T, const optional<Tensor>& push_table,
                    const optional<Tensor>& push_epoch, const optional<Tensor>& shared_gate) {
  hk::MoeMixedArgs a{};
  if (shared_gate.has_value()) {
    TORCH_CHECK(shared_gate->is_cuda() && shared_gate->scalar_type() == at::kFloat, "moe_mixed_gemv: fp32 shared gate logits");
    a.shared_gate = shared_gate->data_ptr<float>();
    a.shared_gate_stride = shared_gate->dim() > 1 ? shared_gate->stride(0) : 1;
  }
  a.e_lo = (int)e_lo;
  a.e_count = (int)e_count;
  a.T = (int)T;
  if (push_table.has_value()) {
    TORCH_CHECK(push_table->scalar_type() == at::kLong && push_epoch.has_value(), "moe_mixed_gemv push: int64 table + epoch");
    a.push_recv = reinterpret_cast<unsigned long long* const*>(push_table->data_ptr<int64_t>());
    a.push_n = (int)push_table->numel();
    a.push_epoch = push_epoch->data_ptr<int>();
  }
  a.routed_pairs = routed_pairs < 0 ? INT_MAX : (int)routed_pairs;
  a.direct = direct ? 1 : 0;
  a.x_stride_q = xq.stride(0);
  a.x_stride_s = xd.stride(0);
  TORCH_CHECK(!direct || routed_pairs >= 0, "moe_mixed_gemv: direct input needs routed_pairs");
  a.desc = reinterpret_cast<const hk::MixedDesc*>(descs.data_ptr());
  a.desc_base0 = (int)base0;
  a.desc_base1 = (int)base1;
  a.N = (int)N;
  a.K = (int)K;
  a.k = (int)k;
  a.counts = ptr<int>(counts);
  a.offsets = ptr<int>(offsets);
  a.sorted = ptr<int>(sorted);
  a.active = ptr<int>(active);
  a.n_active = ptr<int>(n_active);
  a.xq = ptr<int8_t>(xq);
  a.xd = ptr<float>(xd);
  a.xs = ptr<float>(xs);
  a.oq = optr<int8_t>(oq);
  a.od = optr<float>(od);
  a.os = optr<float>(os);
  if (y.has_value()) {
    a.y = ptr<float>(*y);
    a.y_stride = y->stride(0);
  }
  a.route_w = optr<float>(route_w);
  TORCH_CHECK(epi == 0 ? a.oq != nullptr : (epi == 2 ? (a.push_recv != nullptr && a.route_w != nullptr)
                                                      : (a.y != nullptr && a.route_w != nullptr)),
              "moe_mixed_gemv: outputs");
  const c10::cuda::CUDAGuard g(xq.device());
  hk::moe_mixed_gemv_launch((int)epi, a, (int)max_active, cur_stream(), pdl);
}

void codebook_gemv(const Tensor& codebooks, const Tensor& codes, int64_t rows, int64_t nchunk, int64_t nsub,
                   int64_t card, int64_t width, int64_t d, int64_t sub_stride, int64_t bits, const Tensor& xq,
                   const Tensor& xd, const Tensor& lut, const Tensor& y, double alpha, bool accumulate, bool pdl) {
  TORCH_CHECK(codebooks.is_cuda() && codebooks.scalar_type() == at::kHalf, "codebook gemv: fp16 codebooks");
  TORCH_CHECK(codes.is_cuda() && codes.scalar_type() == at::kByte, "codebook gemv: uint8 code stream");
  const int64_t need_bits = rows * nchunk * nsub * bits;
  TORCH_CHECK(codes.numel() >= (need_bits + 7) / 8 + 4, "codebook gemv: code stream too short (needs 4 bytes padding)");
  TORCH_CHECK(codebooks.numel() == nsub * card * width, "codebook gemv: codebook size");
  const int nb = (int)xq.size(0);
  TORCH_CHECK(lut.scalar_type() == at::kFloat && lut.numel() >= nb * nchunk * nsub * card, "codebook gemv: LUT scratch");
  TORCH_CHECK(y.scalar_type() == at::kFloat && y.size(0) >= nb && y.size(1) >= rows && y.stride(1) == 1, "codebook gemv: y");
  TORCH_CHECK(xq.size(1) >= (nchunk - 1) * d + (nsub - 1) * sub_stride + width, "codebook gemv: activation width");
  hk::CodebookArgs a{};
  a.codebooks = ptr<__half>(codebooks);
  a.codes = ptr<uint8_t>(codes);
  a.rows = (int)rows; a.nchunk = (int)nchunk; a.nsub = (int)nsub; a.card = (int)card; a.width = (int)width;
  a.d = (int)d; a.sub_stride = (int)sub_stride; a.bits = (int)bits;
  a.xq = ptr<int8_t>(xq); a.xd = ptr<float>(xd);
  a.x_stride_q = xq.stride(0); a.x_stride_s = xd.stride(0);
  a.nb = nb;
  a.lut = ptr<float>(lut);
  a.y = ptr<float>(y); a.y_stride = y.stride(0);
  a.alpha = (float)alpha;
  a.accumulate = accumulate ? 1 : 0;
  const c10::cuda::CUDAGuard g(xq.device());
  hk::codebook_gemv_launch(a, cur_stream(), pdl);
}

void aap_gemv(const Tensor& in_proj, const Tensor& out_proj, int64_t rows, int64_t cols, int64_t rank, int64_t side,
              const Tensor& xq, const Tensor& xd, const Tensor& latent, const Tensor& y, double alpha, bool accumulate,
              bool pdl) {
  TORCH_CHECK(in_proj.scalar_type() == at::kHalf && out_proj.scalar_type() == at::kHalf, "aap gemv: fp16 factors");
  TORCH_CHECK(in_proj.numel() == cols * rank && out_proj.numel() == rows * rank, "aap gemv: factor sizes");
  TORCH_CHECK(side == 1 || side == 2, "aap gemv: side 1 (input) or 2 (output)");
  const int nb = (int)xq.size(0);
  TORCH_CHECK(latent.scalar_type() == at::kFloat && latent.numel() >= nb * rank, "aap gemv: latent scratch");
  TORCH_CHECK(y.scalar_type() == at::kFloat && y.size(0) >= nb && y.size(1) >= rows && y.stride(1) == 1, "aap gemv: y");
  hk::AapArgs a{};
  a.in_proj = ptr<__half>(in_proj); a.out_proj = ptr<__half>(out_proj);
  a.rows = (int)rows; a.cols = (int)cols; a.rank = (int)rank; a.side = (int)side;
  a.xq = ptr<int8_t>(xq); a.xd = ptr<float>(xd);
  a.x_stride_q = xq.stride(0); a.x_stride_s = xd.stride(0);
  a.nb = nb;
  a.latent = ptr<float>(latent);
  a.y = ptr<float>(y); a.y_stride = y.stride(0);
  a.alpha = (float)alpha;
  a.accumulate = accumulate ? 1 : 0;
  const c10::cuda::CUDAGuard g(xq.device());
  hk::aap_gemv_launch(a, cur_stream(), pdl);
}

void sparse_rows(const Tensor& row_ptr, const Tensor& col, const Tensor& val, const Tensor& xq, const Tensor& xd,
                 const Tensor& y, double alpha, bool pdl) {
  TORCH_CHECK(row_ptr.scalar_type() == at::kInt && col.scalar_type() == at::kInt && val.scalar_type() == at::kHalf,
              "sparse rows: int32 row_ptr / col, fp16 values");
  hk::SparseArgs a{};
  a.row_ptr = ptr<int>(row_ptr); a.col = ptr<int>(col); a.val = ptr<__half>(val);
  a.rows = (int)row_ptr.numel() - 1;
  a.xq = ptr<int8_t>(xq); a.xd = ptr<float>(xd);
  a.x_stride_q = xq.stride(0); a.x_stride_s = xd.stride(0);
  a.nb = (int)xq.size(0);
  a.y = ptr<float>(y); a.y_stride = y.stride(0);
  a.alpha = (float)alpha;
  const c10::cuda::CUDAGuard g(xq.device());
  hk::sparse_rows_launch(a, cur_stream(), pdl);
}

void deltanet_conv(const Tensor& qkvz, const Tensor& conv_w, const Tensor& conv_state, const optional<Tensor>& slot,
                   int64_t kh, int64_t r, int64_t dk, int64_t dv, int64_t kc, double eps, const Tensor& q,
                   const Tensor& k, const Tensor& v, const Tensor& z, bool pdl) {
  hk::DeltaConvArgs a{};
  a.qkvz = ptr<float>(qkvz);
  a.qkvz_stride = qkvz.stride(0);
  a.conv_w = ptr<float>(conv_w);
  a.conv_state = ptr<float>(conv_state);
  a.state_slot = optr<int>(slot);
  a.kh = (int)kh;
  a.r = (int)r;
  a.dk = (int)dk;
  a.dv = (int)dv;
  a.kc = (int)kc;
  a.eps = (float)eps;
  a.q = ptr<float>(q);
  a.k = ptr<float>(k);
  a.v = ptr<float>(v);
  a.z = ptr<float>(z);
  const c10::cuda::CUDAGuard g(qkvz.device());
  hk::deltanet_conv_launch(a, (int)qkvz.size(0), cur_stream(), pdl);
}

void deltanet_recurrent(const Tensor& state, const optional<Tensor>& slot, const Tensor& q, const Tensor& k,
                        const Tensor& v, const Tensor& z, const Tensor& ba, const Tensor& a_log, const Tensor& dt_bias,
                        int64_t r, int64_t dk, int64_t dv, const Tensor& norm_w, double eps, const optional<Tensor>& out,
                        const Tensor& oq, const Tensor& od, const Tensor& os, bool pdl) {
  hk::DeltaRecArgs a{};
  a.state = ptr<float>(state);
  a.state_slot = optr<int>(slot);
  a.q = ptr<float>(q);
  a.k = ptr<float>(k);
  a.v = ptr<float>(v);
  a.z = ptr<float>(z);
  a.ba = ptr<float>(ba);
  a.ba_stride = ba.stride(0);
  a.a_log = ptr<float>(a_log);
  a.dt_bias = ptr<float>(dt_bias);
  a.r = (int)r;
  a.dk = (int)dk;
  a.dv = (int)dv;
  a.norm_w = ptr<float>(norm_w);
  a.eps = (float)eps;
  a.out = optr<float>(out);
  a.oq = ptr<int8_t>(oq);
  a.od = ptr<float>(od);
  a.os = ptr<float>(os);
  const int nvh = (int)a_log.numel();
  const c10::cuda::CUDAGuard g(q.device());
  hk::deltanet_recurrent_launch(a, nvh, (int)q.size(0), cur_stream(), pdl);
}

void sigmoid_gate_q8(const Tensor& o, const Tensor& gate, const Tensor& oq, const Tensor& od, const Tensor& os, bool pdl) {
  const c10::cuda::CUDAGuard g(o.device());
  hk::sigmoid_gate_q8_launch(ptr<float>(o), ptr<float>(gate), gate.stride(0), (int)o.size(0), (int)o.size(1),
                             ptr<int8_t>(oq), ptr<float>(od), ptr<float>(os), cur_stream(), pdl);
}
void mla_kv_append(const Tensor& kv_a, const Tensor& norm_w, double eps, const Tensor& positions,
                   const Tensor& block_tables, const Tensor& row_seq, const Tensor& rope, const Tensor& cache, bool pdl) {
  hk::MlaAppendArgs a{};
  a.kv_a = ptr<float>(kv_a);
  a.kv_a_stride = kv_a.stride(0);
  a.norm_w = ptr<float>(norm_w);
  a.eps = (float)eps;
  a.positions = ptr<int>(positions);
  a.block_tables = ptr<int>(block_tables);
  a.row_seq = ptr<int>(row_seq);
  a.max_blocks = (int)block_tables.size(1);
  a.block_size = (int)cache.size(1);
  a.rope = ptr<float>(rope);
  a.cache = ptr<__nv_bfloat16>(cache);
  TORCH_CHECK(cache.scalar_type() == at::kBFloat16 && cache.size(2) == 576, "mla cache: bf16 [blocks, bs, 576]");
  const c10::cuda::CUDAGuard g(kv_a.device());
  hk::mla_kv_append_launch(a, (int)kv_a.size(0), cur_stream(), pdl);
}

void mla_absorb_q(const Tensor& q, const Tensor& w_uk, const Tensor& positions, const Tensor& rope, const Tensor& q_lat,
                  const Tensor& q_pe, bool pdl) {
  hk::MlaAbsorbArgs a{};
  a.q = ptr<float>(q);
  a.w_uk = ptr<__nv_bfloat16>(w_uk);
  a.positions = ptr<int>(positions);
  a.rope = ptr<float>(rope);
  a.nh = (int)w_uk.size(0);
  a.nope = (int)w_uk.size(1);
  a.q_lat = ptr<float>(q_lat);
  a.q_pe = ptr<float>(q_pe);
  const c10::cuda::CUDAGuard g(q.device());
  hk::mla_absorb_q_launch(a, (int)q.size(0), cur_stream(), pdl);
}

void mla_decode(const Tensor& q_lat, const Tensor& q_pe, const Tensor& cache, const Tensor& block_tables,
                const Tensor& row_seq, const Tensor& row_ctx, double scale, int64_t num_splits, const Tensor& o_lat,
                const Tensor& status, bool pdl) {
  hk::MlaDecodeArgs a{};
  a.q_lat = ptr<float>(q_lat);
  a.q_pe = ptr<float>(q_pe);
  a.cache = ptr<__nv_bfloat16>(cache);
  a.block_tables = ptr<int>(block_tables);
  a.max_blocks = (int)block_tables.size(1);
  a.row_seq = ptr<int>(row_seq);
  a.row_ctx = ptr<int>(row_ctx);
  a.scale = (float)scale;
  a.R = (int)q_lat.size(0);
  a.nh = (int)q_lat.size(1);
  a.block_size = (int)cache.size(1);
  a.num_splits = (int)num_splits;
  a.o_lat = ptr<float>(o_lat);
  a.status = ptr<int>(status);
  const c10::cuda::CUDAGuard g(q_lat.device());
  if (num_splits <= 0) hk::mla_flash_decode_launch(a, cur_stream(), pdl);  // tensor-core kernel
  else hk::mla_decode_launch(a, cur_stream(), pdl);
}

void mla_out(const Tensor& o_lat, const Tensor& w_uv, const Tensor& oq, const Tensor& od, const Tensor& os, bool pdl) {
  hk::MlaOutArgs a{};
  a.o_lat = ptr<float>(o_lat);
  a.w_uv = ptr<__nv_bfloat16>(w_uv);
  a.nh = (int)w_uv.size(0);
  a.vdim = (int)w_uv.size(1);
  a.oq = ptr<int8_t>(oq);
  a.od = ptr<float>(od);
  a.os = ptr<float>(os);
  const c10::cuda::CUDAGuard g(o_lat.device());
  hk::mla_out_launch(a, (int)o_lat.size(0), cur_stream(), pdl);
}
}  // namespace

namespace {
void sparse_residual(const Tensor& row_ptr, const Tensor& cols, const Tensor& signs, double scale, int64_t N,
                     const Tensor& xq, const Tensor& xd, int64_t K, int64_t nb, const Tensor& y, bool pdl) {
  TORCH_CHECK(row_ptr.is_cuda() && row_ptr.scalar_type() == at::kInt && row_ptr.numel() == N + 1,
              "sparse_residual: row_ptr int32 [N + 1]");
  TORCH_CHECK(cols.scalar_type() == at::kInt && signs.scalar_type() == at::kChar && cols.numel() == signs.numel(),
              "sparse_residual: cols int32 / signs int8 [nnz]");
  TORCH_CHECK(xq.scalar_type() == at::kChar && xq.is_contiguous() && xq.numel() >= nb * K && xd.numel() >= nb * K / 32,
              "sparse_residual: q8 activations [nb, K]");
  TORCH_CHECK(y.scalar_type() == at::kFloat && y.stride(-1) == 1 && y.size(0) >= nb && y.size(-1) >= N,
              "sparse_residual: y fp32 [nb, >= N]");
  const c10::cuda::CUDAGuard g(y.device());
  hk::sparse_residual_launch(row_ptr.data_ptr<int>(), cols.data_ptr<int>(), signs.data_ptr<int8_t>(), (float)scale,
                             (int)N, xq.data_ptr<int8_t>(), xd.data_ptr<float>(), (int)K, (int)nb, y.data_ptr<float>(),
                             y.stride(0), at::cuda::getCurrentCUDAStream().stream(), pdl);
}
}  // namespace

namespace hk {
void register_model_kernels(py::module_& m) {
  m.def("sparse_residual", &sparse_residual, py::arg("row_ptr"), py::arg("cols"), py::arg("signs"), py::arg("scale"),
        py::arg("N"), py::arg("xq"), py::arg("xd"), py::arg("K"), py::arg("nb"), py::arg("y"), py::arg("pdl") = false);
  m.def("mla_kv_append", &mla_kv_append, py::arg("kv_a"), py::arg("norm_w"), py::arg("eps"), py::arg("positions"),
        py::arg("block_tables"), py::arg("row_seq"), py::arg("rope"), py::arg("cache"), py::arg("pdl") = false);
  m.def("mla_absorb_q", &mla_absorb_q, py::arg("q"), py::arg("w_uk"), py::arg("positions"), py::arg("rope"),
        py::arg("q_lat"), py::arg("q_pe"), py::arg("pdl") = false);
  m.def("mla_heads_per_cta", &hk::mla_heads_per_cta, py::arg("nh"), py::arg("rows"));
  m.def("mla_decode", &mla_decode, py::arg("q_lat"), py::arg("q_pe"), py::arg("cache"), py::arg("block_tables"),
        py::arg("row_seq"), py::arg("row_ctx"), py::arg("scale"), py::arg("num_splits"), py::arg("o_lat"),
        py::arg("status"), py::arg("pdl") = false);
  m.def("mla_out", &mla_out, py::arg("o_lat"), py::arg("w_uv"), py::arg("oq"), py::arg("od"), py::arg("os"),
        py::arg("pdl") = false);
  m.def("mixed_dequant_bf16", &mixed_dequant_bf16, py::arg("descs"), py::arg("didx"), py::arg("drow"),
        py::arg("rows"), py::arg("K"), py::arg("out"), py::arg("pdl") = false);
  m.def("tc_gemm_bf16", &tc_gemm_bf16, py::arg("w"), py::arg("x"), py::arg("N"), py::arg("M"),
        py::arg("y") = py::none(), py::arg("h") = py::none(), py::arg("atomic") = false, py::arg("y_zeroed") = false,
        py::arg("k_splits") = 1, py::arg("bn") = 128, py::arg("status"), py::arg("pdl") = false,
        py::arg("tiles") = py::none(), py::arg("n_tiles") = py::none(), py::arg("max_tiles") = 0,
        py::arg("group_rows") = 0);
  m.def("moe_tiles", &moe_tiles, py::arg("counts"), py::arg("offsets"), py::arg("E1"), py::arg("bn"),
        py::arg("tiles"), py::arg("n_tiles"), py::arg("pdl") = false, py::arg("e_lo") = 0, py::arg("e_hi") = 0,
        py::arg("shared_e") = -1);
  m.def("moe_gather_bf16", &moe_gather_bf16, py::arg("sorted"), py::arg("PS"), py::arg("P"), py::arg("k"),
        py::arg("x"), py::arg("xg"), py::arg("pos"), py::arg("pdl") = false);
  m.def("moe_combine", &moe_combine, py::arg("y"), py::arg("pos"), py::arg("w"), py::arg("T"), py::arg("k"),
        py::arg("shared"), py::arg("shared_gate"), py::arg("x"), py::arg("pdl") = false, py::arg("ids") = py::none(),
        py::arg("e_lo") = 0, py::arg("e_hi") = 0);
  m.def("qweight_dequant_bf16", &qweight_dequant_bf16, py::arg("fmt"), py::arg("planes"), py::arg("K"),
        py::arg("group_rows"), py::arg("dst_group_rows"), py::arg("dst_off"), py::arg("out"), py::arg("pdl") = false);
  m.def("q8_to_bf16", &q8_to_bf16, py::arg("q"), py::arg("d"), py::arg("out"), py::arg("pdl") = false);
  m.def("mixed_descs", &mixed_descs, py::arg("codes"), py::arg("scales"), py::arg("kind"), py::arg("bits"),
        py::arg("group"), py::arg("zeros") = std::vector<int64_t>{});
  m.def("codebook_gemv", &codebook_gemv, py::arg("codebooks"), py::arg("codes"), py::arg("rows"), py::arg("nchunk"),
        py::arg("nsub"), py::arg("card"), py::arg("width"), py::arg("d"), py::arg("sub_stride"), py::arg("bits"),
        py::arg("xq"), py::arg("xd"), py::arg("lut"), py::arg("y"), py::arg("alpha") = 1.0,
        py::arg("accumulate") = false, py::arg("pdl") = false);
  m.def("aap_gemv", &aap_gemv, py::arg("in_proj"), py::arg("out_proj"), py::arg("rows"), py::arg("cols"),
        py::arg("rank"), py::arg("side"), py::arg("xq"), py::arg("xd"), py::arg("latent"), py::arg("y"),
        py::arg("alpha") = 1.0, py::arg("accumulate") = false, py::arg("pdl") = false);
  m.def("sparse_rows", &sparse_rows, py::arg("row_ptr"), py::arg("col"), py::arg("val"), py::arg("xq"),
        py::arg("xd"), py::arg("y"), py::arg("alpha") = 1.0, py::arg("pdl") = false);
  m.def("mixed_gemv", &mixed_gemv, py::arg("epi"), py::arg("descs"), py::arg("d0"), py::arg("d1"), py::arg("N"),
        py::arg("K"), py::arg("xq"), py::arg("xd"), py::arg("xs"), py::arg("y") = py::none(), py::arg("alpha") = 1.0,
        py::arg("oq") = py::none(), py::arg("od") = py::none(), py::arg("os") = py::none(), py::arg("pdl") = false,
        py::arg("gate_logit") = py::none(), py::arg("push_table") = py::none(), py::arg("push_epoch") = py::none(),
        py::arg("argmax_slots") = py::none(), py::arg("argmax_offset") = 0);
  m.def("moe_active", &moe_active, py::arg("counts"), py::arg("active"), py::arg("n_active"), py::arg("pdl") = false);
  m.def("moe_mixed_gemv", &moe_mixed_gemv, py::arg("epi"), py::arg("descs"), py::arg("base0"), py::arg("base1"),
        py::arg("N"), py::arg("K"), py::arg("k"), py::arg("counts"), py::arg("offsets"), py::arg("sorted"),
        py::arg("active"), py::arg("n_active"), py::arg("max_active"), py::arg("xq"), py::arg("xd"), py::arg("xs"),
        py::arg("oq") = py::none(), py::arg("od") = py::none(), py::arg("os") = py::none(), py::arg("y") = py::none(),
        py::arg("route_w") = py::none(), py::arg("pdl") = false,
        py::arg("routed_pairs") = -1,
        py::arg("direct") = false, py::arg("e_lo") = 0, py::arg("e_count") = 0, py::arg("T") = 0,
        py::arg("push_table") = py::none(), py::arg("push_epoch") = py::none(), py::arg("shared_gate") = py::none());
  m.def("deltanet_conv", &deltanet_conv, py::arg("qkvz"), py::arg("conv_w"), py::arg("conv_state"), py::arg("slot"),
        py::arg("kh"), py::arg("r"), py::arg("dk"), py::arg("dv"), py::arg("kc"), py::arg("eps"), py::arg("q"),
        py::arg("k"), py::arg("v"), py::arg("z"), py::arg("pdl") = false);
  m.def("deltanet_recurrent", &deltanet_recurrent, py::arg("state"), py::arg("slot"), py::arg("q"), py::arg("k"),
        py::arg("v"), py::arg("z"), py::arg("ba"), py::arg("a_log"), py::arg("dt_bias"), py::arg("r"), py::arg("dk"),
        py::arg("dv"), py::arg("norm_w"), py::arg("eps"), py::arg("out"), py::arg("oq"), py::arg("od"), py::arg("os"),
        py::arg("pdl") = false);
  m.def("sigmoid_gate_q8", &sigmoid_gate_q8, py::arg("o"), py::arg("gate"), py::arg("oq"), py::arg("od"), py::arg("os"),
        py::arg("pdl") = false);
}
}  // namespace hk
