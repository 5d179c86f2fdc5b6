// Bindings for the artifact formats (.gravity shards, HGRAV* mixed codecs, HQ80M15 catalog,
// sha256, canonical JSON).
#include <cstring>

#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "../native/codecs.h"
#include "../native/ggml_quant.h"
#include "../native/gravity.h"
#include "../native/json.h"
#include "../native/mixed.h"
#include "../native/sha256.h"

namespace py = pybind11;
using namespace hk;

namespace {
// JSON <-> Python through the json module (text), keeping one canonical encoder in C++.
Json from_py(py::handle o) {
  py::object dumps = py::module_::import("json").attr("dumps");
  return Json::parse(dumps(o).cast<std::string>());
}
py::object to_py(const Json& j) {
  return py::module_::import("json").attr("loads")(j.dump());
}
py::array_t<uint8_t> bytes_view(const uint8_t* p, size_t n, py::handle owner) {
  return py::array_t<uint8_t>({(py::ssize_t)n}, {1}, p, owner);
}
py::array_t<uint8_t> to_np(const std::vector<uint8_t>& v) {
  py::array_t<uint8_t> a(v.size());
  std::memcpy(a.mutable_data(), v.data(), v.size());
  return a;
}
}  // namespace

void bind_formats(py::module_& m) {
  m.def("sha256_hex", [](py::array_t<uint8_t, py::array::c_style> a) {
    const uint8_t* p = a.data();
    const size_t n = (size_t)a.size();
    py::gil_scoped_release unlocked;  // callers hash several files on threads
    return Sha256::hex_of(p, n);
  });
  m.def("sha256_hex_portable", [](py::array_t<uint8_t, py::array::c_style> a) {
    Sha256 h(true);
    h.update(a.data(), (size_t)a.size());
    return h.hex();
  });
  m.def("canonical_json", [](py::handle o) { return from_py(o).canonical(); });
  m.def("json_number", &json_number);

  py::class_<GravityShard, std::shared_ptr<GravityShard>>(m, "GravityShard")
      .def_static("open", [](const std::string& p) { return std::shared_ptr<GravityShard>(GravityShard::open(p)); })
      .def_property_readonly("path", &GravityShard::path)
      .def_property_readonly("format_version", &GravityShard::format_version)
      .def_property_readonly("body_offset", &GravityShard::body_offset)
      .def("header", [](const GravityShard& s) { return to_py(s.header()); })
      .def("tensors", [](const GravityShard& s) {
        py::list l;
        for (const auto& t : s.tensors())
          l.append(py::make_tuple(t.name, t.codec, t.offset, t.bytes, t.sha256, t.shape, t.elements));
        return l;
      })
      .def("descriptor", [](const GravityShard& s, const std::string& n) {
        const auto* t = s.find(n);
        if (!t) throw std::runtime_error("gravity: no tensor " + n);
        return to_py(t->extra);
      })
      .def("raw", [](std::shared_ptr<GravityShard> s, const std::string& n) {
        const auto* t = s->find(n);
        if (!t) throw std::runtime_error("gravity: no tensor " + n);
        return bytes_view(s->data(*t), t->bytes, py::cast(s));
      })
      .def("verify", [](const GravityShard& s) { return to_py(s.verify()); })
      .def("verify_tensor", &GravityShard::verify_tensor);

  py::class_<GravityWriter>(m, "GravityWriter")
      .def(py::init([](py::handle meta) { return new GravityWriter(meta.is_none() ? Json::object() : from_py(meta)); }),
           py::arg("meta") = py::none())
      .def("add", [](GravityWriter& w, py::handle desc, py::array_t<uint8_t, py::array::c_style> data) {
        w.add(from_py(desc), data.data(), data.size());
      })
      .def("write", [](const GravityWriter& w, const std::string& p) { return to_py(w.write(p)); });
  m.def("gravity_codec_to_ggml", &gravity_codec_to_ggml);

  // mixed codecs
  // fixed-header codecs (PQ, residual PQ, AAP, HQ30 family) and the .hawking sidecar
  using U8 = py::array_t<uint8_t, py::array::c_style>;
  using F32 = py::array_t<float, py::array::c_style | py::array::forcecast>;
  auto f32_np = [](const std::vector<float>& v, py::ssize_t rows, py::ssize_t cols) {
    py::array_t<float> out({rows, cols});
    std::memcpy(out.mutable_data(), v.data(), v.size() * 4);
    return out;
  };
  auto f64_np = [](const std::vector<double>& v) {
    py::array_t<double> out((py::ssize_t)v.size());
    std::memcpy(out.mutable_data(), v.data(), v.size() * 8);
    return out;
  };
  m.def("pq_header", [](U8 a) {
    auto h = pq_parse(a.data(), a.size());
    py::dict d;
    d["d"] = h.d; d["s"] = h.s; d["sub"] = h.sub; d["card"] = h.card; d["rows"] = h.rows; d["cols"] = h.cols;
    d["nchunk"] = h.nchunk; d["seed"] = h.seed; d["bits"] = h.bits; d["rotate"] = h.rotate;
    d["n_codebooks"] = h.n_codebooks;
    return d;
  });
  m.def("pq_parts", [](U8 a) {  // codebooks [s, card, sub] f32 and indices [rows, nchunk, s]
    PqHeader h;
    std::vector<float> cb;
    std::vector<uint16_t> idx;
    pq_sections(a.data(), a.size(), h, cb, idx);
    py::array_t<float> c({(py::ssize_t)h.s, (py::ssize_t)h.card, (py::ssize_t)h.sub});
    std::memcpy(c.mutable_data(), cb.data(), cb.size() * 4);
    py::array_t<int16_t> i({(py::ssize_t)h.rows, (py::ssize_t)h.nchunk, (py::ssize_t)h.s});
    std::memcpy(i.mutable_data(), idx.data(), idx.size() * 2);
    return py::make_tuple(c, i);
  });
  m.def("pq_decode", [f32_np](U8 a) {
    auto h = pq_parse(a.data(), a.size());
    return f32_np(pq_decode(a.data(), a.size()), h.rows, h.cols);
  });
  m.def("pq_matvec_f64", [f64_np](U8 a, F32 x) { return f64_np(pq_matvec_f64(a.data(), a.size(), x.data())); });
  m.def("pq_encode", [](int d, int s, int sub, int card, int rows, int cols, int nchunk, int seed, int bits,
                        py::array_t<uint16_t, py::array::c_style | py::array::forcecast> cb,
                        py::array_t<uint32_t, py::array::c_style | py::array::forcecast> idx) {
    PqHeader h;
    h.d = d; h.s = s; h.sub = sub; h.card = card; h.rows = rows; h.cols = cols; h.nchunk = nchunk; h.seed = seed;
    h.bits = bits; h.rotate = 0; h.n_codebooks = (uint8_t)s;
    return to_np(pq_encode(h, std::vector<uint16_t>(cb.data(), cb.data() + cb.size()),
                           std::vector<uint32_t>(idx.data(), idx.data() + idx.size())));
  });
  m.def("rpq_header", [](U8 a) {
    auto h = rpq_parse(a.data(), a.size());
    py::dict d;
    d["d"] = h.d; d["stages"] = h.stages; d["card"] = h.card; d["rows"] = h.rows; d["cols"] = h.cols;
    d["nchunk"] = h.nchunk; d["seed"] = h.seed; d["bits"] = h.bits;
    return d;
  });
  m.def("rpq_parts", [](U8 a) {  // codebooks [stages, card, d] f32 and indices [rows, nchunk, stages]
    RpqHeader h;
    std::vector<float> cb;
    std::vector<uint16_t> idx;
    rpq_sections(a.data(), a.size(), h, cb, idx);
    py::array_t<float> c({(py::ssize_t)h.stages, (py::ssize_t)h.card, (py::ssize_t)h.d});
    std::memcpy(c.mutable_data(), cb.data(), cb.size() * 4);
    py::array_t<int16_t> i({(py::ssize_t)h.rows, (py::ssize_t)h.nchunk, (py::ssize_t)h.stages});
    std::memcpy(i.mutable_data(), idx.data(), idx.size() * 2);
    return py::make_tuple(c, i);
  });
  m.def("rpq_decode", [f32_np](U8 a) {
    auto h = rpq_parse(a.data(), a.size());
    return f32_np(rpq_decode(a.data(), a.size()), h.rows, h.cols);
  });
  m.def("rpq_matvec_f64", [f64_np](U8 a, F32 x) { return f64_np(rpq_matvec_f64(a.data(), a.size(), x.data())); });
  m.def("rpq_encode", [](int d, int stages, int card, int rows, int cols, int nchunk, int seed, int bits,
                         py::array_t<uint16_t, py::array::c_style | py::array::forcecast> cb,
                         py::array_t<uint32_t, py::array::c_style | py::array::forcecast> idx) {
    RpqHeader h;
    h.d = d; h.stages = stages; h.card = card; h.rows = rows; h.cols = cols; h.nchunk = nchunk; h.seed = seed;
    h.bits = bits;
    return to_np(rpq_encode(h, std::vector<uint16_t>(cb.data(), cb.data() + cb.size()),
                            std::vector<uint32_t>(idx.data(), idx.data() + idx.size())));
  });
  m.def("aap_header", [](U8 a) {
    auto h = aap_parse(a.data(), a.size());
    py::dict d;
    d["rows"] = h.rows; d["cols"] = h.cols; d["rank"] = h.rank; d["basis_layer"] = h.basis_layer;
    d["side"] = h.side == 1 ? "input" : "output"; d["has_basis"] = h.has_basis;
    return d;
  });
  m.def("aap_decode", [f32_np](U8 a) {
    auto h = aap_parse(a.data(), a.size());
    return f32_np(aap_decode(a.data(), a.size()), h.rows, h.cols);
  });
  m.def("aap_matvec_f64", [f64_np](U8 a, F32 x) { return f64_np(aap_matvec_f64(a.data(), a.size(), x.data())); });
  m.def("aap_encode", [](int rows, int cols, int rank, int basis_layer, int side,
                         py::array_t<uint16_t, py::array::c_style | py::array::forcecast> coeff,
                         py::array_t<uint16_t, py::array::c_style | py::array::forcecast> basis) {
    AapHeader h;
    h.rows = rows; h.cols = cols; h.rank = rank; h.basis_layer = basis_layer; h.side = side; h.has_basis = true;
    return to_np(aap_encode(h, std::vector<uint16_t>(coeff.data(), coeff.data() + coeff.size()),
                            std::vector<uint16_t>(basis.data(), basis.data() + basis.size())));
  });
  auto hq30_dict = [](const Hq30Header& h) {
    py::dict d;
    d["version"] = h.version; d["group_size"] = h.group_size; d["shape"] = h.shape; d["elements"] = h.elements;
    d["groups"] = h.groups; d["scale_offset"] = h.scale_offset; d["code_offset"] = h.code_offset;
    d["payload_bytes"] = h.payload_bytes;
    return d;
  };
  m.def("hq30_binary_header", [hq30_dict](U8 a) { return hq30_dict(hq30_binary_parse(a.data(), a.size())); });
  m.def("hq30_uq4_header", [hq30_dict](U8 a) { return hq30_dict(hq30_uq4_parse(a.data(), a.size())); });
  m.def("hq30_residual_header", [hq30_dict](U8 a) {
    auto r = hq30_residual_parse(a.data(), a.size());
    py::dict d = hq30_dict(r.base);
    d["base_offset"] = r.base_offset; d["base_bytes"] = r.base_bytes; d["indices"] = r.indices;
    std::vector<float> vals;
    for (uint16_t v : r.values) vals.push_back(fp16_to_f32(v));
    d["values"] = vals;
    return d;
  });
  auto flat_np = [](const std::vector<float>& v) {
    py::array_t<float> out((py::ssize_t)v.size());
    std::memcpy(out.mutable_data(), v.data(), v.size() * 4);
    return out;
  };
  m.def("hq30_binary_decode", [flat_np](U8 a) { return flat_np(hq30_binary_decode(a.data(), a.size())); });
  m.def("hq30_uq4_decode", [flat_np](U8 a) { return flat_np(hq30_uq4_decode(a.data(), a.size())); });
  m.def("hq30_residual_decode", [flat_np](U8 a) { return flat_np(hq30_residual_decode(a.data(), a.size())); });
  m.def("hq30_binary_encode", [](std::vector<uint32_t> shape, F32 w, int group) {
    return to_np(hq30_binary_encode(shape, w.data(), group));
  });
  m.def("hq30_uq4_encode", [](std::vector<uint32_t> shape, F32 w, int group) {
    return to_np(hq30_uq4_encode(shape, w.data(), group));
  });
  m.def("hq30_residual_encode", [](std::vector<uint32_t> shape, F32 w, int group, size_t keep) {
    return to_np(hq30_residual_encode(shape, w.data(), group, keep));
  });
  m.def("predecode_q4k_scales", [flat_np](U8 a) { return flat_np(predecode_q4k_scales(a.data(), a.size())); });
  m.def("sidecar_write", [](const std::string& path, const std::string& header_json, py::list entries) {
    std::vector<SidecarEntry> es;
    for (auto item : entries) {
      auto t = item.cast<py::tuple>();
      SidecarEntry e;
      e.offset = t[0].cast<uint64_t>();
      auto arr = t[1].cast<py::array_t<float, py::array::c_style | py::array::forcecast>>();
      e.scales.assign(arr.data(), arr.data() + arr.size());
      es.push_back(std::move(e));
    }
    sidecar_write(path, header_json, es);
  });
  m.def("sidecar_read", [flat_np](const std::string& path) {
    std::string hj;
    std::vector<SidecarEntry> es;
    sidecar_read(path, hj, es);
    py::list out;
    for (auto& e : es) out.append(py::make_tuple(e.offset, flat_np(e.scales)));
    return py::make_tuple(hj, out);
  });

  m.def("mixed_header", [](py::array_t<uint8_t, py::array::c_style> a) {
    auto e = mixed_split(a.data(), a.size());
    return py::make_tuple(py::bytes(e.magic), to_py(e.header), (size_t)(e.body - a.data()), e.body_bytes);
  });
  m.def("mixed_decode", [](py::array_t<uint8_t, py::array::c_style> a) {
    int r = 0, c = 0;
    auto w = decode_mixed(a.data(), a.size(), &r, &c);
    py::array_t<float> out({(py::ssize_t)r, (py::ssize_t)c});
    std::memcpy(out.mutable_data(), w.data(), w.size() * 4);
    return out;
  });
  m.def("rice_indices", [](py::array_t<uint8_t, py::array::c_style> a) { return parse_hgravr02(a.data(), a.size()).indices; });
  m.def("encode_hgravb01", [](py::array_t<float, py::array::c_style | py::array::forcecast> w, int group) {
    return to_np(encode_hgravb01(w.data(), (int)w.shape(0), (int)w.shape(1), group));
  });
  m.def("encode_hgravu01", [](py::array_t<float, py::array::c_style | py::array::forcecast> w, int group, int bits) {
    return to_np(encode_hgravu01(w.data(), (int)w.shape(0), (int)w.shape(1), group, bits));
  });
  // Planes of the residual / low-rank codecs for the device GEMVs (ops/mixed.py).
  m.def("hgravr02_parts", [](py::array_t<uint8_t, py::array::c_style> a) {
    auto r = parse_hgravr02(a.data(), a.size());
    py::dict d;
    d["rows"] = r.base.rows;
    d["cols"] = r.base.cols;
    d["group"] = r.base.group;
    std::vector<uint8_t> sc(r.base.scales.size() * 2);
    std::memcpy(sc.data(), r.base.scales.data(), sc.size());
    d["scales"] = to_np(sc);
    d["signs"] = to_np(r.base.signs);
    py::array_t<uint32_t> idx(r.indices.size());
    std::memcpy(idx.mutable_data(), r.indices.data(), r.indices.size() * 4);
    d["indices"] = idx;
    d["residual_scale"] = fp16_to_f32(r.residual_scale);
    d["residual_signs"] = to_np(r.residual_signs);
    return d;
  });
  m.def("hgravs01_parts", [](py::array_t<uint8_t, py::array::c_style> a) {
    auto lr = parse_hgravs01(a.data(), a.size());
    auto factor = [](const UniformGroup& u) {
      py::dict f;
      f["rows"] = u.rows;
      f["cols"] = u.cols;
      f["group"] = u.group;
      f["bits"] = u.bits;
      std::vector<uint8_t> sc(u.scales.size() * 2);
      std::memcpy(sc.data(), u.scales.data(), sc.size());
      f["scales"] = to_np(sc);
      f["codes"] = to_np(u.codes);
      return f;
    };
    py::dict d;
    d["rank"] = lr.rank;
    d["left"] = factor(lr.left);
    d["right"] = factor(lr.right);
    return d;
  });
  m.def("wrap_hgravb01", [](int rows, int cols, int group, py::array_t<uint8_t, py::array::c_style> scales,
                            py::array_t<uint8_t, py::array::c_style> signs) {
    return to_np(wrap_hgravb01(rows, cols, group, scales.data(), (size_t)scales.size(), signs.data(), (size_t)signs.size()));
  });
  m.def("wrap_hgravu01", [](int rows, int cols, int group, int bits, py::array_t<uint8_t, py::array::c_style> scales,
                            py::array_t<uint8_t, py::array::c_style> codes) {
    return to_np(wrap_hgravu01(rows, cols, group, bits, scales.data(), (size_t)scales.size(), codes.data(),
                               (size_t)codes.size()));
  });
  m.def("encode_hgravr02", [](py::array_t<float, py::array::c_style | py::array::forcecast> w, int group, double ratio,
                              uint32_t k) {
    return to_np(encode_hgravr02(w.data(), (int)w.shape(0), (int)w.shape(1), group, ratio, k));
  });
  m.def("encode_hgravs01", [](py::array_t<float, py::array::c_style | py::array::forcecast> l,
                              py::array_t<float, py::array::c_style | py::array::forcecast> r, int group, int bits) {
    return to_np(encode_hgravs01(l.data(), r.data(), (int)l.shape(0), (int)l.shape(1), (int)r.shape(1), group, bits));
  });

  py::class_<CatalogTensor>(m, "CatalogTensor")
      .def(py::init<>())
      .def_readwrite("name", &CatalogTensor::name)
      .def_readwrite("codec", &CatalogTensor::codec)
      .def_readwrite("organ", &CatalogTensor::organ)
      .def_readwrite("ndim", &CatalogTensor::ndim)
      .def_property("dims", [](const CatalogTensor& t) { return std::vector<uint32_t>(t.dims, t.dims + 4); },
                    [](CatalogTensor& t, std::vector<uint32_t> d) { for (int i = 0; i < 4; ++i) t.dims[i] = i < (int)d.size() ? d[i] : 0; })
      .def_readwrite("elements", &CatalogTensor::elements)
      .def_readwrite("segment", &CatalogTensor::segment)
      .def_readwrite("rank", &CatalogTensor::rank)
      .def_readwrite("offset", &CatalogTensor::offset)
      .def_readwrite("nbytes", &CatalogTensor::nbytes)
      .def_readwrite("sha256", &CatalogTensor::sha256)
      .def_readwrite("flags", &CatalogTensor::flags)
      .def_readwrite("n_fit_rows", &CatalogTensor::n_fit_rows)
      .def_readwrite("codec_bpw", &CatalogTensor::codec_bpw);
  py::class_<CatalogSegment>(m, "CatalogSegment")
      .def(py::init<>())
      .def_readwrite("id", &CatalogSegment::id)
      .def_readwrite("name", &CatalogSegment::name)
      .def_readwrite("bytes", &CatalogSegment::bytes)
      .def_readwrite("sha256", &CatalogSegment::sha256);
  py::class_<Catalog>(m, "Catalog")
      .def(py::init<>())
      .def_readwrite("version", &Catalog::version)
      .def_readwrite("flags", &Catalog::flags)
      .def_readwrite("segments", &Catalog::segments)
      .def_readwrite("tensors", &Catalog::tensors);
  m.def("read_catalog", &read_catalog);
  m.def("write_catalog", &write_catalog);
}
