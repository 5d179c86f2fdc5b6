// pybind11 module `hawking_b200._native`: formats, CPU reference, engine host logic and server.
// Host-only C++ (no CUDA, no torch headers) so it builds and tests on a CPU box.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstring>

#include "../native/cpu_ref.h"
#include "../native/ggml_quant.h"
#include "../native/gguf.h"

namespace py = pybind11;
using namespace hk;

void bind_engine(py::module_& m);   // engine_bindings.cpp
void bind_formats(py::module_& m);  // formats_bindings.cpp
void bind_serve(py::module_& m);    // serve_bindings.cpp

namespace {

py::object gguf_value_to_py(const GgufValue& v) {
  switch (v.kind) {
    case GgufKind::F32:
    case GgufKind::F64: return py::float_(v.f);
    case GgufKind::BOOL: return py::bool_(v.i != 0);
    case GgufKind::STRING: return py::bytes(v.s).attr("decode")("utf-8", "replace");
    case GgufKind::U64: return py::int_((uint64_t)v.i);
    case GgufKind::ARRAY: {
      py::list l;
      if (v.arr)
        for (const auto& e : *v.arr) l.append(gguf_value_to_py(e));
      return l;
    }
    default: return py::int_(v.i);
  }
}

GgufValue py_to_gguf_value(py::handle o, int kind_hint) {
  GgufValue v;
  if (kind_hint >= 0) v.kind = (GgufKind)kind_hint;
  if (py::isinstance<py::bool_>(o)) {
    v.kind = GgufKind::BOOL;
    v.i = o.cast<bool>();
  } else if (py::isinstance<py::int_>(o)) {
    if (kind_hint < 0) v.kind = GgufKind::U32;
    v.i = o.cast<int64_t>();
    if (kind_hint < 0 && (v.i < 0 || v.i > 0xFFFFFFFFll)) v.kind = GgufKind::I64;
    if (v.kind == GgufKind::F32 || v.kind == GgufKind::F64) v.f = (double)v.i;
  } else if (py::isinstance<py::float_>(o)) {
    if (kind_hint < 0 || (v.kind != GgufKind::F32 && v.kind != GgufKind::F64)) v.kind = GgufKind::F32;
    v.f = o.cast<double>();
  } else if (py::isinstance<py::str>(o)) {
    v.kind = GgufKind::STRING;
    v.s = o.cast<std::string>();
  } else if (py::isinstance<py::list>(o) || py::isinstance<py::tuple>(o)) {
    v.kind = GgufKind::ARRAY;
    v.arr = std::make_shared<GgufArray>();
    py::sequence seq = o.cast<py::sequence>();
    GgufKind ek = GgufKind::U32;
    bool first = true;
    for (auto e : seq) {
      GgufValue ev = py_to_gguf_value(e, -1);
      if (first) { ek = ev.kind; first = false; }
      if (ev.kind == GgufKind::U32 && ek == GgufKind::I32) ev.kind = GgufKind::I32;
      if (ev.kind != ek) {
        if ((ek == GgufKind::U32 || ek == GgufKind::I32) && ev.kind == GgufKind::I64) ek = GgufKind::I64;
        ev.kind = ek;
      }
      v.arr->push_back(ev);
    }
    for (auto& e : *v.arr) e.kind = ek;
    v.arr_kind = ek;
  } else {
    throw std::runtime_error("gguf: unsupported metadata value type");
  }
  return v;
}

py::array_t<float> np_dequantize(uint32_t type, py::array_t<uint8_t, py::array::c_style> src, size_t n) {
  if ((size_t)src.size() < type_nbytes(type, n)) throw std::runtime_error("dequantize: source too small");
  py::array_t<float> out(n);
  {
    py::gil_scoped_release r;
    dequantize(type, src.data(), out.mutable_data(), n);
  }
  return out;
}

py::array_t<uint8_t> np_quantize_rows(uint32_t type, py::array_t<float, py::array::c_style | py::array::forcecast> src,
                                      int threads) {
  size_t rows, cols;
  if (src.ndim() == 1) { rows = 1; cols = src.shape(0); }
  else if (src.ndim() == 2) { rows = src.shape(0); cols = src.shape(1); }
  else throw std::runtime_error("quantize: expected 1-D or 2-D array");
  size_t rb = type_nbytes(type, cols);
  py::array_t<uint8_t> out({rows, rb});
  {
    py::gil_scoped_release r;
    quantize_rows(type, src.data(), out.mutable_data(), rows, cols, threads);
  }
  return out;
}

py::array_t<float> np_dequantize_rows(uint32_t type, py::array_t<uint8_t, py::array::c_style> src, size_t rows,
                                      size_t cols, int threads) {
  if ((size_t)src.size() < rows * type_nbytes(type, cols)) throw std::runtime_error("dequantize_rows: source too small");
  py::array_t<float> out({rows, cols});
  {
    py::gil_scoped_release r;
    dequantize_rows(type, src.data(), out.mutable_data(), rows, cols, threads);
  }
  return out;
}

}  // namespace

PYBIND11_MODULE(_native, m) {
  m.doc() = "hawking_b200 host-side native core (formats, CPU reference, engine, server)";

  m.def("type_info", [](uint32_t t) {
    const auto& tt = type_traits(t);
    return py::make_tuple(std::string(tt.name), tt.block_elems, tt.block_bytes, tt.supported);
  });
  m.def("type_nbytes", &type_nbytes);
  m.def("dequantize", &np_dequantize, py::arg("type"), py::arg("src"), py::arg("n"));
  m.def("dequantize_rows", &np_dequantize_rows, py::arg("type"), py::arg("src"), py::arg("rows"),
        py::arg("cols"), py::arg("threads") = 8);
  m.def("quantize_rows", &np_quantize_rows, py::arg("type"), py::arg("src"), py::arg("threads") = 8);
  m.def("fp16_to_f32", &fp16_to_f32);
  m.def("f32_to_fp16", &f32_to_fp16);

  py::class_<GgufFile, std::shared_ptr<GgufFile>>(m, "GgufFile")
      .def_static("open", [](const std::string& p) { return std::shared_ptr<GgufFile>(GgufFile::open(p)); })
      .def_property_readonly("version", &GgufFile::version)
      .def_property_readonly("alignment", &GgufFile::alignment)
      .def_property_readonly("data_offset", &GgufFile::data_offset)
      .def_property_readonly("path", &GgufFile::path)
      .def_property_readonly("size", &GgufFile::size)
      .def("metadata", [](const GgufFile& f) {
        py::dict d;
        for (const auto& kv : f.metadata()) d[py::str(kv.first)] = gguf_value_to_py(kv.second);
        return d;
      })
      .def("metadata_kinds", [](const GgufFile& f) {
        py::dict d;
        for (const auto& kv : f.metadata()) d[py::str(kv.first)] = (int)kv.second.kind;
        return d;
      })
      .def("tensors", [](const GgufFile& f) {
        py::list l;
        for (const auto& t : f.tensors())
          l.append(py::make_tuple(t.name, t.dims, t.type, t.offset, t.nbytes));
        return l;
      });

  py::class_<GgufWriter>(m, "GgufWriter")
      .def(py::init<uint64_t>(), py::arg("alignment") = 32)
      .def("set", [](GgufWriter& w, const std::string& k, py::handle v, int kind) {
        w.set(k, py_to_gguf_value(v, kind));
      }, py::arg("key"), py::arg("value"), py::arg("kind") = -1)
      .def("add_tensor", [](GgufWriter& w, const std::string& name, std::vector<uint64_t> dims, uint32_t type,
                            py::array_t<uint8_t, py::array::c_style> data) {
        w.add_tensor(name, dims, type, data.data(), data.size());
      })
      .def("write", &GgufWriter::write, py::call_guard<py::gil_scoped_release>());

  // ---- CPU reference ops ----
  m.def("ref_rmsnorm", [](py::array_t<float, py::array::c_style | py::array::forcecast> x,
                          py::array_t<float, py::array::c_style | py::array::forcecast> w, float eps) {
    int n = (int)x.shape(x.ndim() - 1);
    size_t rows = x.size() / n;
    py::array_t<float> y(x.request().shape);
    for (size_t r = 0; r < rows; ++r) ref_rmsnorm(x.data() + r * n, w.data(), y.mutable_data() + r * n, n, eps);
    return y;
  });
  m.def("ref_rope", [](py::array_t<float, py::array::c_style | py::array::forcecast> x, int pos, int rot_dim,
                       float theta, int style) {
    int hd = (int)x.shape(x.ndim() - 1);
    size_t rows = x.size() / hd;
    py::array_t<float> y(x.request().shape);
    std::memcpy(y.mutable_data(), x.data(), sizeof(float) * x.size());
    for (size_t r = 0; r < rows; ++r) ref_rope(y.mutable_data() + r * hd, hd, rot_dim, pos, theta, style, nullptr);
    return y;
  });
  m.def("ref_q8_roundtrip", [](py::array_t<float, py::array::c_style | py::array::forcecast> x) {
    py::array_t<float> y(x.request().shape);
    std::memcpy(y.mutable_data(), x.data(), sizeof(float) * x.size());
    ref_q8_roundtrip(y.mutable_data(), (int)y.size());
    return y;
  });
  m.def("ref_topk_gate", [](py::array_t<float, py::array::c_style | py::array::forcecast> logits, int k, bool renorm) {
    int n = (int)logits.size();
    std::vector<int> ids(k);
    std::vector<float> w(k);
    ref_topk_gate(logits.data(), n, k, renorm, ids.data(), w.data());
    return py::make_tuple(ids, w);
  });

  py::class_<SamplingParams>(m, "SamplingParams")
      .def(py::init<>())
      .def_readwrite("temperature", &SamplingParams::temperature)
      .def_readwrite("top_k", &SamplingParams::top_k)
      .def_readwrite("top_p", &SamplingParams::top_p)
      .def_readwrite("repetition_penalty", &SamplingParams::repetition_penalty)
      .def_readwrite("seed", &SamplingParams::seed);

  py::class_<Sampler>(m, "Sampler")
      .def(py::init<uint64_t, int>(), py::arg("seed"), py::arg("rep_window") = 64)
      .def("record", &Sampler::record)
      .def("sample", [](Sampler& s, py::array_t<float, py::array::c_style | py::array::forcecast> logits,
                        const SamplingParams& p) {
        std::vector<float> l(logits.data(), logits.data() + logits.size());
        return s.sample(l, p);
      });

  py::class_<Pcg64>(m, "Pcg64").def(py::init<uint64_t>()).def("next_u64", &Pcg64::next_u64).def("next_f32", &Pcg64::next_f32);

  py::class_<CpuLlama>(m, "CpuLlama")
      .def(py::init([](const std::string& path, int max_ctx, int threads, bool act_q8, bool bf16_kv) {
             return new CpuLlama(std::shared_ptr<GgufFile>(GgufFile::open(path)), max_ctx, threads, act_q8, bf16_kv);
           }),
           py::arg("path"), py::arg("max_ctx") = 2048, py::arg("threads") = 8, py::arg("act_q8") = false,
           py::arg("bf16_kv") = false)
      .def("forward", [](CpuLlama& m, int tok, int pos) {
        std::vector<float> l;
        {
          py::gil_scoped_release r;
          l = m.forward(tok, pos);
        }
        return py::array_t<float>(l.size(), l.data());
      })
      .def("reset", &CpuLlama::reset)
      .def("last_hidden", [](const CpuLlama& m) {
        const auto& h = m.last_hidden();
        return py::array_t<float>(h.size(), h.data());
      })
      .def("generate_greedy", &CpuLlama::generate_greedy, py::call_guard<py::gil_scoped_release>())
      .def("generate", &CpuLlama::generate, py::call_guard<py::gil_scoped_release>())
      .def_property_readonly("config", [](const CpuLlama& m) {
        const auto& c = m.config();
        py::dict d;
        d["arch"] = c.arch; d["vocab"] = c.vocab; d["hidden"] = c.hidden; d["layers"] = c.layers;
        d["n_heads"] = c.n_heads; d["n_kv_heads"] = c.n_kv_heads; d["head_dim"] = c.head_dim;
        d["ffn"] = c.ffn; d["rope_style"] = c.rope_style; d["theta"] = c.theta; d["eps"] = c.eps;
        d["n_experts"] = c.n_experts; d["top_k"] = c.top_k;
        return d;
      });

  bind_formats(m);
  bind_engine(m);
  bind_serve(m);
}
