// Bindings for the serving host logic: tokenizer, streaming detokeniser.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "../native/gguf.h"
#include "../native/tokenizer.h"

namespace py = pybind11;
using namespace hk;

void bind_serve(py::module_& m) {
  py::class_<TokenizerSpec>(m, "TokenizerSpec")
      .def(py::init<>())
      .def_readwrite("model", &TokenizerSpec::model)
      .def_readwrite("pre", &TokenizerSpec::pre)
      .def_readwrite("tokens", &TokenizerSpec::tokens)
      .def_readwrite("merges", &TokenizerSpec::merges)
      .def_readwrite("scores", &TokenizerSpec::scores)
      .def_readwrite("token_types", &TokenizerSpec::token_types)
      .def_readwrite("bos", &TokenizerSpec::bos)
      .def_readwrite("eos", &TokenizerSpec::eos)
      .def_readwrite("unk", &TokenizerSpec::unk)
      .def_readwrite("pad", &TokenizerSpec::pad)
      .def_readwrite("add_bos", &TokenizerSpec::add_bos)
      .def_readwrite("add_eos", &TokenizerSpec::add_eos);

  py::class_<Tokenizer, std::shared_ptr<Tokenizer>>(m, "Tokenizer")
      .def_static("from_spec", [](const TokenizerSpec& s) { return std::shared_ptr<Tokenizer>(Tokenizer::from_spec(s)); })
      .def_static("from_gguf",
                  [](const GgufFile& f) { return std::shared_ptr<Tokenizer>(Tokenizer::from_gguf(f)); })
      .def("encode", &Tokenizer::encode, py::arg("text"), py::arg("add_special") = true,
           py::call_guard<py::gil_scoped_release>())
      .def("decode", &Tokenizer::decode, py::arg("ids"), py::arg("skip_special") = true)
      .def("token_bytes", [](const Tokenizer& t, int32_t id) { return py::bytes(t.token_bytes(id)); })
      .def("is_special", &Tokenizer::is_special)
      .def("is_eog", &Tokenizer::is_eog)
      .def("eog_ids", &Tokenizer::eog_ids)
      .def("find", &Tokenizer::find)
      .def("token", &Tokenizer::token)
      .def_property_readonly("bos", &Tokenizer::bos)
      .def_property_readonly("eos", &Tokenizer::eos)
      .def_property_readonly("pad", &Tokenizer::pad)
      .def_property_readonly("add_bos", &Tokenizer::add_bos)
      .def_property_readonly("vocab_size", &Tokenizer::vocab_size)
      .def_property_readonly("is_spm", &Tokenizer::is_spm);

  py::class_<StreamDecoder>(m, "StreamDecoder")
      .def(py::init<const Tokenizer*, bool>(), py::arg("tokenizer"), py::arg("skip_special") = true,
           py::keep_alive<1, 2>())
      .def("push", [](StreamDecoder& d, int32_t id) { return py::bytes(d.push(id)); })
      .def("flush", [](StreamDecoder& d) { return py::bytes(d.flush()); });

  m.def("pretokenize", &pretokenize, py::arg("text"), py::arg("pre") = "default");
}
