// Bindings for the artifact formats (.gravity shards, HGRAV* mixed codecs, HQ80M15 catalog,
// sha256, canonical JSON).
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

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
  m.def("sha256_hex", [](py::array_t<uint8_t, py::array::c_style> a) { return Sha256::hex_of(a.data(), a.size()); });
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
