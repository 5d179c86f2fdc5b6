// Bindings for the serving host logic: tokenizer, streaming detokeniser, HTTP server.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "../native/gguf.h"
#include "../native/http_server.h"
#include "../native/json.h"
#include "../native/json_constrain.h"
#include "../native/tokenizer.h"
#include "../native/tool_calls.h"
#include "../native/trace.h"

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
      .def_static("from_json",
                  [](const std::string& path, const std::string& config) {
                    return std::shared_ptr<Tokenizer>(Tokenizer::from_json(path, config));
                  },
                  py::arg("path"), py::arg("config") = "")
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

  py::class_<ServeOptions>(m, "ServeOptions")
      .def(py::init<>())
      .def_readwrite("host", &ServeOptions::host)
      .def_readwrite("port", &ServeOptions::port)
      .def_readwrite("model_id", &ServeOptions::model_id)
      .def_readwrite("chat_template", &ServeOptions::chat_template)
      .def_readwrite("max_queue", &ServeOptions::max_queue)
      .def_readwrite("max_connections", &ServeOptions::max_connections)
      .def_readwrite("default_max_tokens", &ServeOptions::default_max_tokens)
      .def_readwrite("max_context", &ServeOptions::max_context)
      .def_readwrite("request_timeout_s", &ServeOptions::request_timeout_s)
      .def_readwrite("max_batch", &ServeOptions::max_batch)
      .def_readwrite("architecture", &ServeOptions::architecture)
      .def_readwrite("recurrent_state_bytes", &ServeOptions::recurrent_state_bytes);

  py::class_<ServeRequest>(m, "ServeRequest")
      .def_readonly("id", &ServeRequest::id)
      .def_readonly("kind", &ServeRequest::kind)
      .def_readonly("prompt", &ServeRequest::prompt)
      .def_readonly("inputs", &ServeRequest::inputs)
      .def_readonly("max_tokens", &ServeRequest::max_tokens)
      .def_readonly("temperature", &ServeRequest::temperature)
      .def_readonly("top_p", &ServeRequest::top_p)
      .def_readonly("top_k", &ServeRequest::top_k)
      .def_readonly("repetition_penalty", &ServeRequest::repetition_penalty)
      .def_readonly("seed", &ServeRequest::seed)
      .def_readonly("stream", &ServeRequest::stream)
      .def_readonly("json_mode", &ServeRequest::json_mode)
      .def_readonly("stop_ids", &ServeRequest::stop_ids);

  py::class_<JsonConstraint>(m, "JsonConstraint")
      .def(py::init<bool>(), py::arg("lenient_whitespace") = false)
      .def("accepts", [](const JsonConstraint& c, const py::bytes& b) { return c.accepts(std::string(b)); })
      .def("advance", [](JsonConstraint& c, const py::bytes& b) { return c.advance(std::string(b)); })
      .def_property_readonly("done", &JsonConstraint::done)
      .def("pick", [](const JsonConstraint& c, const Tokenizer& tok, py::buffer logits) {
        py::buffer_info bi = logits.request();
        if (bi.format != py::format_descriptor<float>::format() || bi.ndim != 1)
          throw std::runtime_error("pick: 1-D float32 logits");
        return c.pick(tok, static_cast<const float*>(bi.ptr), (int64_t)bi.shape[0]);
      })
      .def("mask", [](const JsonConstraint& c, const Tokenizer& tok, py::buffer logits) {
        py::buffer_info bi = logits.request(true);
        if (bi.format != py::format_descriptor<float>::format() || bi.ndim != 1)
          throw std::runtime_error("mask: 1-D float32 logits");
        c.mask(tok, static_cast<float*>(bi.ptr), (int64_t)bi.shape[0]);
      })
      .def_static("validate", &JsonConstraint::validate);

  m.def("trace_available", &trace_available);
  m.def("trace_push", &trace_push, py::arg("name"));
  m.def("trace_pop", &trace_pop);

  m.def("render_tools_preamble", [](const std::string& tools_json) {
    return render_tools_preamble(Json::parse(tools_json));
  });
  m.def("extract_tool_calls", [](const std::string& text, const std::vector<std::string>& known) {
    py::list out;
    for (const auto& c : extract_tool_calls(text, known)) out.append(py::make_tuple(c.id, c.name, c.arguments));
    return out;
  }, py::arg("text"), py::arg("known_tools"));

  py::class_<HttpServer, std::shared_ptr<HttpServer>>(m, "HttpServer")
      .def(py::init<ServeOptions, std::shared_ptr<Tokenizer>>(), py::arg("options"), py::arg("tokenizer"))
      .def("start", &HttpServer::start)
      .def("stop", &HttpServer::stop, py::call_guard<py::gil_scoped_release>())
      .def_property_readonly("port", &HttpServer::port)
      .def("poll", &HttpServer::poll, py::arg("timeout_ms") = 0, py::call_guard<py::gil_scoped_release>())
      .def("push", &HttpServer::push, py::arg("id"), py::arg("tokens"), py::arg("finish") = 0,
           py::call_guard<py::gil_scoped_release>())
      .def("push_embeddings", &HttpServer::push_embeddings, py::call_guard<py::gil_scoped_release>())
      .def("fail", &HttpServer::fail)
      .def("take_cancelled", &HttpServer::take_cancelled)
      .def("set_metric", &HttpServer::set_metric, py::arg("name"), py::arg("value"), py::arg("help") = "",
           py::arg("counter") = false)
      .def("set_health", &HttpServer::set_health, py::arg("ok"), py::arg("reason") = "")
      .def("stats", [](const HttpServer& s) { return s.stats().dump(); })
      .def("render_chat", [](const HttpServer& s, const std::string& messages_json, const std::string& tmpl) {
        return s.render_chat(Json::parse(messages_json), tmpl.empty() ? s.resolve_template() : tmpl);
      }, py::arg("messages_json"), py::arg("template") = "");
}
