// OpenAI-compatible HTTP/1.1 + SSE server; see http_server.h.
#include "http_server.h"
#include "tool_calls.h"

#include <arpa/inet.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <sys/socket.h>
#include <sys/time.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <stdexcept>

namespace hk {

struct HttpServer::Pending {
  uint64_t id = 0;
  std::mutex mu;
  std::condition_variable cv;
  std::deque<int32_t> tokens;
  int finish = 0;
  bool done = false;
  std::vector<std::vector<float>> emb;
  bool emb_ready = false;
  int err_status = 0;
  std::string err_msg;
};

namespace {

using Clock = std::chrono::steady_clock;

const char* status_text(int s) {
  switch (s) {
    case 200: return "OK";
    case 400: return "Bad Request";
    case 404: return "Not Found";
    case 405: return "Method Not Allowed";
    case 413: return "Payload Too Large";
    case 500: return "Internal Server Error";
    case 501: return "Not Implemented";
    case 503: return "Service Unavailable";
    case 504: return "Gateway Timeout";
    default: return "Error";
  }
}

bool write_all(int fd, const std::string& s) {
  size_t off = 0;
  while (off < s.size()) {
    const ssize_t n = ::send(fd, s.data() + off, s.size() - off, MSG_NOSIGNAL);
    if (n <= 0) return false;
    off += (size_t)n;
  }
  return true;
}

// (No iostreams in this file: the module may carry its own static C++ runtime, whose stream
// locale is not set up when no stream object is constructed at load time.)
bool respond(int fd, int status, const std::string& ctype, const std::string& body, bool keep_alive) {
  std::string h = "HTTP/1.1 " + std::to_string(status) + " " + status_text(status) + "\r\n";
  h += "Content-Type: " + ctype + "\r\n";
  h += "Content-Length: " + std::to_string(body.size()) + "\r\n";
  h += std::string("Connection: ") + (keep_alive ? "keep-alive" : "close") + "\r\n\r\n";
  return write_all(fd, h + body);
}

std::string error_body(const std::string& message, const std::string& type, const std::string& code) {
  Json e = Json::object();
  e.set("message", Json::string(message));
  e.set("type", Json::string(type));
  e.set("code", Json::string(code));
  Json o = Json::object();
  o.set("error", e);
  return o.dump();
}

bool respond_error(int fd, int status, const std::string& message, const std::string& code, bool keep_alive) {
  const std::string type = status >= 500 ? (status == 501 ? "not_implemented" : "internal_error")
                                         : "invalid_request_error";
  return respond(fd, status, "application/json", error_body(message, type, code), keep_alive);
}

std::string lower(std::string s) {
  for (auto& c : s) c = (char)std::tolower((unsigned char)c);
  return s;
}

// Text of an OpenAI message "content": a string, or an array of {"type":"text","text":...} parts.
std::string content_text(const Json& c) {
  if (c.is_string()) return c.as_string();
  std::string out;
  if (c.is_array())
    for (const auto& p : c.items())
      if (p.is_object() && p["text"].is_string()) out += p["text"].as_string();
  return out;
}

double num_or(const Json& o, const char* k, double d) { return o.has(k) && o[k].is_number() ? o[k].as_double() : d; }

// Longest suffix of `text` that is a proper prefix of some stop string (held back while streaming).
size_t stop_holdback(const std::string& text, const std::vector<std::string>& stops) {
  size_t hold = 0;
  for (const auto& s : stops)
    for (size_t k = std::min(s.size() - 1, text.size()); k > hold; --k)
      if (text.compare(text.size() - k, k, s, 0, k) == 0) { hold = k; break; }
  return hold;
}

std::string random_hex_id(uint64_t id) {
  char buf[40];
  snprintf(buf, sizeof buf, "%016llx", (unsigned long long)(id * 0x9E3779B97F4A7C15ull));
  return buf;
}

}  // namespace

HttpServer::HttpServer(ServeOptions opts, std::shared_ptr<Tokenizer> tok) : opts_(std::move(opts)), tok_(std::move(tok)) {
  if (!tok_) throw std::runtime_error("http server: a tokenizer is required");
}

HttpServer::~HttpServer() { stop(); }

void HttpServer::start() {
  if (running_) return;
  listen_fd_ = ::socket(AF_INET, SOCK_STREAM, 0);
  if (listen_fd_ < 0) throw std::runtime_error("http server: socket() failed");
  int one = 1;
  setsockopt(listen_fd_, SOL_SOCKET, SO_REUSEADDR, &one, sizeof one);
  sockaddr_in addr{};
  addr.sin_family = AF_INET;
  addr.sin_port = htons((uint16_t)opts_.port);
  if (inet_pton(AF_INET, opts_.host.c_str(), &addr.sin_addr) != 1) {
    ::close(listen_fd_);
    throw std::runtime_error("http server: bad host " + opts_.host);
  }
  if (::bind(listen_fd_, (sockaddr*)&addr, sizeof addr) != 0 || ::listen(listen_fd_, 128) != 0) {
    ::close(listen_fd_);
    throw std::runtime_error("http server: cannot listen on " + opts_.host + ":" + std::to_string(opts_.port));
  }
  socklen_t len = sizeof addr;
  getsockname(listen_fd_, (sockaddr*)&addr, &len);
  bound_port_ = ntohs(addr.sin_port);
  running_ = true;
  accept_thread_ = std::thread([this] { accept_loop(); });
}

void HttpServer::stop() {
  if (!running_.exchange(false)) return;
  ::shutdown(listen_fd_, SHUT_RDWR);
  ::close(listen_fd_);
  if (accept_thread_.joinable()) accept_thread_.join();
  std::vector<std::shared_ptr<Pending>> ps;
  {
    std::lock_guard<std::mutex> g(mu_);
    for (auto& kv : pending_) ps.push_back(kv.second);
    queue_.clear();
  }
  for (auto& p : ps) {
    std::lock_guard<std::mutex> g(p->mu);
    p->err_status = 503;
    p->err_msg = "server shutting down";
    p->done = true;
    p->cv.notify_all();
  }
  cv_.notify_all();
  // connection threads are detached; wait (bounded) for them to leave
  for (int i = 0; i < 500 && connections_.load() > 0; ++i) std::this_thread::sleep_for(std::chrono::milliseconds(10));
}

void HttpServer::accept_loop() {
  while (running_) {
    pollfd p{listen_fd_, POLLIN, 0};
    if (::poll(&p, 1, 100) <= 0) continue;
    const int fd = ::accept(listen_fd_, nullptr, nullptr);
    if (fd < 0) continue;
    if (connections_.load() >= opts_.max_connections) {
      respond_error(fd, 503, "too many connections", "overloaded", false);
      ::close(fd);
      continue;
    }
    int one = 1;
    setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof one);
    timeval tv{30, 0};
    setsockopt(fd, SOL_SOCKET, SO_RCVTIMEO, &tv, sizeof tv);
    connections_++;
    std::thread([this, fd] {
      try {
        serve_connection(fd);
      } catch (...) {
      }
      ::close(fd);
      connections_--;
    }).detach();
  }
}

void HttpServer::serve_connection(int fd) {
  std::string buf;
  char tmp[8192];
  while (running_) {
    // ---- read the header block ----
    size_t hend;
    while ((hend = buf.find("\r\n\r\n")) == std::string::npos) {
      if (buf.size() > (1 << 16)) { respond_error(fd, 413, "header too large", "header_too_large", false); return; }
      const ssize_t n = ::recv(fd, tmp, sizeof tmp, 0);
      if (n <= 0) return;
      buf.append(tmp, (size_t)n);
    }
    const std::string head = buf.substr(0, hend);
    buf.erase(0, hend + 4);
    std::vector<std::string> lines;
    for (size_t a = 0; a <= head.size();) {
      size_t e = head.find("\r\n", a);
      if (e == std::string::npos) e = head.size();
      lines.push_back(head.substr(a, e - a));
      a = e + 2;
    }
    std::string method, target, version;
    {
      const std::string& rl = lines[0];
      const size_t s1 = rl.find(' '), s2 = s1 == std::string::npos ? s1 : rl.find(' ', s1 + 1);
      if (s1 == std::string::npos || s2 == std::string::npos) {
        respond_error(fd, 400, "malformed request line", "bad_request", false);
        return;
      }
      method = rl.substr(0, s1);
      target = rl.substr(s1 + 1, s2 - s1 - 1);
      version = rl.substr(s2 + 1);
    }
    size_t clen = 0;
    bool keep_alive = version == "HTTP/1.1";
    for (size_t li = 1; li < lines.size(); ++li) {
      const std::string& line = lines[li];
      const size_t c = line.find(':');
      if (c == std::string::npos) continue;
      const std::string k = lower(line.substr(0, c));
      std::string v = line.substr(c + 1);
      v.erase(0, v.find_first_not_of(" \t"));
      if (k == "content-length") clen = (size_t)std::strtoull(v.c_str(), nullptr, 10);
      else if (k == "connection") keep_alive = lower(v) != "close";
    }
    if (clen > (64u << 20)) { respond_error(fd, 413, "body too large", "body_too_large", false); return; }
    while (buf.size() < clen) {
      const ssize_t n = ::recv(fd, tmp, sizeof tmp, 0);
      if (n <= 0) return;
      buf.append(tmp, (size_t)n);
    }
    const std::string body = buf.substr(0, clen);
    buf.erase(0, clen);
    const size_t q = target.find('?');
    const std::string path = q == std::string::npos ? target : target.substr(0, q);
    if (!handle(fd, method, path, body, keep_alive) || !keep_alive) return;
  }
}

bool HttpServer::handle(int fd, const std::string& method, const std::string& path, const std::string& body,
                        bool keep_alive) {
  if (path == "/healthz" || path == "/health") {
    if (method != "GET") return respond_error(fd, 405, "use GET", "method_not_allowed", keep_alive);
    if (!healthy_) {
      Json h = Json::object();
      h.set("status", Json::string("unhealthy"));
      {
        std::lock_guard<std::mutex> g(mu_);
        h.set("reason", Json::string(health_reason_));
      }
      return respond(fd, 503, "application/json", h.dump(), keep_alive);
    }
    return respond(fd, 200, "text/plain", "ok", keep_alive);
  }
  if (path == "/metrics") return respond(fd, 200, "text/plain; version=0.0.4", metrics_text(), keep_alive);
  if (path == "/v1/models") {
    Json m = Json::object();
    m.set("id", Json::string(opts_.model_id));
    m.set("object", Json::string("model"));
    m.set("owned_by", Json::string("hawking-b200"));
    Json d = Json::array();
    d.push(m);
    Json o = Json::object();
    o.set("object", Json::string("list"));
    o.set("data", d);
    return respond(fd, 200, "application/json", o.dump(), keep_alive);
  }
  if (path == "/v1/responses" || path == "/v1/messages") {
    requests_rejected_++;
    return respond(fd, 501, "application/json",
                   error_body("POST " + path + " is not implemented by this server", "not_implemented",
                              "not_implemented"),
                   keep_alive);
  }
  if (path == "/v1/hawking/context") {
    Json c = Json::object();
    size_t active = 0;
    {
      std::lock_guard<std::mutex> g(mu_);
      active = pending_.size();
    }
    c.set("model_id", Json::string(opts_.model_id));
    c.set("arch", Json::string(opts_.architecture));
    c.set("ctx_len_native", Json::integer(opts_.max_context));
    c.set("ctx_len_effective", Json::integer(opts_.max_context));
    c.set("tq_multiplier", Json::number(1.0));
    c.set("tq_estimated", Json::boolean(false));
    c.set("recurrent_state_bytes",
          opts_.recurrent_state_bytes > 0 ? Json::integer(opts_.recurrent_state_bytes) : Json::null());
    c.set("active_slots", Json::integer((int64_t)active));
    c.set("free_slots", Json::integer(std::max<int64_t>(0, (int64_t)opts_.max_batch - (int64_t)active)));
    c.set("max_batch", Json::integer(opts_.max_batch));
    return respond(fd, 200, "application/json", c.dump(), keep_alive);
  }
  if (path == "/v1/hawking/surface") {
    Json o = Json::object();
    o.set("server", Json::string("hawking-b200"));
    Json routes = Json::array();
    for (const char* r : {"GET /healthz", "GET /metrics", "GET /v1/models", "POST /v1/chat/completions",
                          "POST /v1/completions", "POST /v1/embeddings", "POST /v1/hawking/generate",
                          "POST /v1/hawking/tokens", "GET /v1/hawking/context", "GET /v1/hawking/surface"})
      routes.push(Json::string(r));
    o.set("routes", routes);
    Json ni = Json::array();
    ni.push(Json::string("POST /v1/responses"));
    ni.push(Json::string("POST /v1/messages"));
    o.set("not_implemented", ni);
    Json f = Json::object();
    for (const char* k : {"streaming", "tool_calls", "json_mode", "embeddings", "continuous_batching",
                          "prefix_reuse", "speculative_decoding"})
      f.set(k, Json::boolean(true));
    o.set("features", f);
    Json fam = Json::object();
    for (const char* a : {"llama", "qwen2", "qwen3", "mixtral", "qwen2moe", "qwen3moe", "qwen3next", "deepseek2"})
      fam.set(a, Json::string("served"));
    o.set("architectures", fam);
    o.set("model_id", Json::string(opts_.model_id));
    o.set("arch", Json::string(opts_.architecture));
    return respond(fd, 200, "application/json", o.dump(), keep_alive);
  }
  const bool chat = path == "/v1/chat/completions", comp = path == "/v1/completions", emb = path == "/v1/embeddings";
  const bool hgen = path == "/v1/hawking/generate", htok = path == "/v1/hawking/tokens";
  if (!chat && !comp && !emb && !hgen && !htok) return respond_error(fd, 404, "no route for " + path, "not_found", keep_alive);
  if (method != "POST") return respond_error(fd, 405, "use POST", "method_not_allowed", keep_alive);
  Json j;
  try {
    j = Json::parse(body);
  } catch (const std::exception& e) {
    return respond_error(fd, 400, std::string("request body is not valid JSON: ") + e.what(), "invalid_json",
                         keep_alive);
  }
  if (!j.is_object()) return respond_error(fd, 400, "request body must be a JSON object", "invalid_json", keep_alive);
  if (emb) return handle_embeddings(fd, j, keep_alive);
  if (hgen || htok) {
    if (!j["prompt"].is_string() || j["prompt"].as_string().empty())
      return respond_error(fd, 400, "'prompt' must not be empty", "missing_required_parameter", keep_alive);
    return handle_generate(fd, j, false, keep_alive, hgen ? "generate" : "tokens");
  }
  return handle_generate(fd, j, chat, keep_alive);
}

std::string HttpServer::resolve_template() const {
  if (opts_.chat_template != "auto") return opts_.chat_template;
  if (tok_->find("<|start_header_id|>") >= 0) return "llama3";
  if (tok_->find("<|im_start|>") >= 0) return "chatml";
  return "generic";
}

std::string HttpServer::render_chat(const Json& messages, const std::string& tmpl) const {
  std::string out;
  for (const auto& m : messages.items()) {
    std::string role = m["role"].is_string() ? m["role"].as_string() : "user";
    std::string text = content_text(m["content"]);
    if (role == "tool") {  // a tool result goes back to the model as a user turn
      role = "user";
      text = "<tool_response>\n" + text + "\n</tool_response>";
    }
    if (m["tool_calls"].is_array())  // the assistant's earlier calls, in the format it was taught
      for (const auto& tc : m["tool_calls"].items()) {
        const Json& f = tc["function"];
        std::string args = f["arguments"].is_string() ? f["arguments"].as_string() : f["arguments"].dump();
        text += "<tool_call>\n{\"name\": " + Json::string(f["name"].is_string() ? f["name"].as_string() : "").dump() +
                ", \"arguments\": " + args + "}\n</tool_call>";
      }
    if (tmpl == "llama3") out += "<|start_header_id|>" + role + "<|end_header_id|>\n\n" + text + "<|eot_id|>";
    else if (tmpl == "chatml") out += "<|im_start|>" + role + "\n" + text + "<|im_end|>\n";
    else if (tmpl == "deepseek") {
      if (role == "system") out += text + "\n\n";
      else if (role == "assistant") out += "Assistant: " + text + "\n\n";
      else out += "User: " + text + "\n\n";
    } else out += role + ": " + text + "\n";
  }
  if (tmpl == "llama3") out += "<|start_header_id|>assistant<|end_header_id|>\n\n";
  else if (tmpl == "chatml") out += "<|im_start|>assistant\n";
  else if (tmpl == "deepseek") out += "Assistant:";
  else out += "assistant:";
  return out;
}

std::shared_ptr<HttpServer::Pending> HttpServer::admit(ServeRequest req) {
  auto p = std::make_shared<Pending>();
  std::lock_guard<std::mutex> g(mu_);
  if ((int)queue_.size() >= opts_.max_queue) return nullptr;
  req.id = next_id_++;
  p->id = req.id;
  pending_[req.id] = p;
  prompt_tokens_ += req.prompt.size();
  for (const auto& in : req.inputs) prompt_tokens_ += in.size();
  queue_.push_back(std::move(req));
  requests_admitted_++;
  cv_.notify_one();
  return p;
}

void HttpServer::forget(uint64_t id) {
  std::lock_guard<std::mutex> g(mu_);
  pending_.erase(id);
}

void HttpServer::set_health(bool ok, const std::string& reason) {
  {
    std::lock_guard<std::mutex> g(mu_);
    health_reason_ = reason;
  }
  healthy_ = ok;
}

bool HttpServer::handle_generate(int fd, const Json& j, bool chat, bool keep_alive, const std::string& native) {
  if (!healthy_) {
    requests_rejected_++;
    std::string why;
    {
      std::lock_guard<std::mutex> g(mu_);
      why = health_reason_;
    }
    return respond_error(fd, 503, "engine unavailable: " + why, "unavailable", keep_alive);
  }
  ServeRequest r;
  r.kind = chat ? "chat" : "completion";
  std::string prompt_text;
  std::vector<std::string> known_tools;
  const bool tools_on = chat && j["tools"].is_array() && j["tools"].size() > 0 &&
                        !(j["tool_choice"].is_string() && j["tool_choice"].as_string() == "none");
  if (chat) {
    if (!j["messages"].is_array()) return respond_error(fd, 400, "'messages' must be an array", "invalid_json", keep_alive);
    if (j["messages"].size() == 0)
      return respond_error(fd, 400, "'messages' must not be empty", "missing_required_parameter", keep_alive);
    if (tools_on) {  // the tools preamble leads the system turn
      known_tools = tool_names(j["tools"]);
      Json msgs = Json::array();
      const std::string pre = render_tools_preamble(j["tools"]);
      bool merged = false;
      for (const auto& m : j["messages"].items()) {
        if (!merged && m["role"].is_string() && m["role"].as_string() == "system") {
          Json sys = Json::object();
          sys.set("role", Json::string("system"));
          sys.set("content", Json::string(content_text(m["content"]) + "\n\n" + pre));
          msgs.push(sys);
          merged = true;
        } else {
          msgs.push(m);
        }
      }
      if (!merged) {
        Json all = Json::array(), sys = Json::object();
        sys.set("role", Json::string("system"));
        sys.set("content", Json::string(pre));
        all.push(sys);
        for (const auto& m : msgs.items()) all.push(m);
        msgs = all;
      }
      prompt_text = render_chat(msgs, resolve_template());
    } else {
      prompt_text = render_chat(j["messages"], resolve_template());
    }
  } else {
    const Json& p = j["prompt"];
    if (p.is_string()) prompt_text = p.as_string();
    else if (p.is_array() && p.size() > 0 && p.at(0).is_string()) prompt_text = p.at(0).as_string();
    else if (!(p.is_array() && p.size() > 0 && p.at(0).is_number()))
      return respond_error(fd, 400, "'prompt' must be a string or a token-id array", "missing_required_parameter",
                           keep_alive);
    if (p.is_array() && p.size() > 0 && p.at(0).is_number())
      for (const auto& t : p.items()) r.prompt.push_back((int32_t)t.as_int());
  }
  if (r.prompt.empty()) r.prompt = tok_->encode(prompt_text, true);
  if (r.prompt.empty()) return respond_error(fd, 400, "prompt tokenizes to nothing", "missing_required_parameter", keep_alive);
  for (int32_t t : r.prompt)
    if (t < 0 || (size_t)t >= tok_->vocab_size())
      return respond_error(fd, 400, "token id out of range", "invalid_json", keep_alive);
  r.max_tokens = (int)num_or(j, "max_completion_tokens", num_or(j, "max_tokens", opts_.default_max_tokens));
  if (r.max_tokens <= 0) return respond_error(fd, 400, "'max_tokens' must be positive", "invalid_json", keep_alive);
  if ((int)r.prompt.size() + r.max_tokens > opts_.max_context)
    r.max_tokens = std::max(1, opts_.max_context - (int)r.prompt.size());
  if ((int)r.prompt.size() >= opts_.max_context)
    return respond_error(fd, 400, "prompt longer than the context window", "context_length_exceeded", keep_alive);
  r.temperature = (float)num_or(j, "temperature", native.empty() ? 1.0 : 0.0);
  r.top_p = (float)num_or(j, "top_p", native == "generate" && r.temperature > 0.f ? 0.9 : 1.0);
  r.top_k = (int)num_or(j, "top_k", native == "generate" && r.temperature > 0.f ? 40 : 0);
  if (native == "tokens") r.temperature = 0.f;  // greedy token stream
  r.json_mode = j["response_format"].is_object() && j["response_format"]["type"].is_string() &&
                j["response_format"]["type"].as_string() == "json_object";
  r.repetition_penalty = (float)num_or(j, "repetition_penalty", 1.0);
  r.seed = (uint64_t)num_or(j, "seed", 42);
  r.stream = native == "tokens" || (native.empty() && j["stream"].type() == Json::Type::Bool && j["stream"].as_bool());
  r.stop_ids = tok_->eog_ids();
  std::vector<std::string> stops;
  if (j["stop"].is_string()) stops.push_back(j["stop"].as_string());
  else if (j["stop"].is_array())
    for (const auto& s : j["stop"].items())
      if (s.is_string() && !s.as_string().empty()) stops.push_back(s.as_string());
  const size_t n_prompt = r.prompt.size();
  const bool stream = r.stream;
  auto p = admit(std::move(r));
  if (!p) {
    requests_rejected_++;
    return respond_error(fd, 503, "request queue is full", "overloaded", keep_alive);
  }
  const uint64_t id = p->id;
  const std::string oid = (chat ? "chatcmpl-" : "cmpl-") + random_hex_id(id);
  const int64_t created = (int64_t)std::chrono::duration_cast<std::chrono::seconds>(
                              std::chrono::system_clock::now().time_since_epoch()).count();
  StreamDecoder dec(tok_.get());
  std::string text, sent_upto_text;
  size_t sent = 0, n_gen = 0;
  std::string finish_reason;
  bool stopped_by_string = false, client_gone = false;

  auto chunk_json = [&](const std::string& delta, const std::string& fin, bool first) {
    Json c = Json::object();
    c.set("id", Json::string(oid));
    c.set("object", Json::string(chat ? "chat.completion.chunk" : "text_completion"));
    c.set("created", Json::integer(created));
    c.set("model", Json::string(opts_.model_id));
    Json ch = Json::object();
    ch.set("index", Json::integer(0));
    if (chat) {
      Json d = Json::object();
      if (first) d.set("role", Json::string("assistant"));
      if (!delta.empty() || fin.empty()) d.set("content", Json::string(delta));
      ch.set("delta", d);
    } else {
      ch.set("text", Json::string(delta));
    }
    ch.set("finish_reason", fin.empty() ? Json::null() : Json::string(fin));
    Json arr = Json::array();
    arr.push(ch);
    c.set("choices", arr);
    return "data: " + c.dump() + "\n\n";
  };

  if (stream) {
    const std::string h =
        "HTTP/1.1 200 OK\r\nContent-Type: text/event-stream\r\nCache-Control: no-cache\r\nConnection: close\r\n\r\n";
    if (!write_all(fd, h)) client_gone = true;
  }
  const auto t_start = Clock::now();
  auto t_first = t_start;
  bool first = true;
  const auto deadline = Clock::now() + std::chrono::milliseconds((int64_t)(opts_.request_timeout_s * 1000));
  while (!client_gone) {
    std::deque<int32_t> toks;
    int fin = 0;
    bool done = false;
    int err = 0;
    std::string err_msg;
    {
      std::unique_lock<std::mutex> g(p->mu);
      p->cv.wait_until(g, deadline, [&] { return !p->tokens.empty() || p->done; });
      toks.swap(p->tokens);
      fin = p->finish;
      done = p->done;
      err = p->err_status;
      err_msg = p->err_msg;
    }
    if (err) {
      forget(id);
      if (stream) {
        write_all(fd, "data: " + error_body(err_msg, "internal_error", "internal_error") + "\n\ndata: [DONE]\n\n");
        return false;
      }
      return respond_error(fd, err, err_msg, err == 503 ? "overloaded" : "internal_error", keep_alive);
    }
    if (toks.empty() && !done) {  // timed out
      forget(id);
      {
        std::lock_guard<std::mutex> g(mu_);
        cancelled_.push_back(id);
      }
      if (stream) return false;
      return respond_error(fd, 504, "generation timed out", "timeout", keep_alive);
    }
    for (int32_t t : toks) {
      if (n_gen == 0) t_first = Clock::now();
      n_gen++;
      tokens_generated_++;
      if (native == "tokens" && !client_gone) {  // token ids as they come
        Json e = Json::object();
        e.set("token", Json::integer(t));
        if (!write_all(fd, "data: " + e.dump() + "\n\n")) client_gone = true;
      }
      if (tok_->is_eog(t)) continue;
      text += dec.push(t);
    }
    if (done) text += dec.flush();
    // stop strings
    for (const auto& s : stops) {
      const size_t at = text.find(s, sent > s.size() ? sent - s.size() : 0);
      if (at != std::string::npos) {
        text.resize(at);
        stopped_by_string = true;
      }
    }
    if (stopped_by_string) {
      done = true;
      fin = 2;
    }
    if (done) finish_reason = fin == 1 ? "length" : "stop";
    if (native == "tokens") {
      if (done && !client_gone) write_all(fd, "data: [DONE]\n\n");
      if (done) break;
      continue;
    }
    if (stream) {
      const size_t hold = done ? 0 : stop_holdback(text, stops);
      const size_t upto = text.size() - std::min(hold, text.size() - sent);
      if (upto > sent || first) {
        const std::string delta = text.substr(sent, upto - sent);
        if ((!delta.empty() || first) && !write_all(fd, chunk_json(delta, "", first))) client_gone = true;
        first = false;
        sent = upto;
      }
      if (done && !client_gone) {
        const auto calls = tools_on ? extract_tool_calls(text, known_tools) : std::vector<ToolCall>{};
        if (!calls.empty()) {  // the calls as one final delta
          Json c = Json::object();
          c.set("id", Json::string(oid));
          c.set("object", Json::string("chat.completion.chunk"));
          c.set("created", Json::integer(created));
          c.set("model", Json::string(opts_.model_id));
          Json ch = Json::object(), d = Json::object(), arr = Json::array(), tcs = Json::array();
          for (size_t i = 0; i < calls.size(); ++i) {
            Json tc = Json::object(), f = Json::object();
            tc.set("index", Json::integer((int64_t)i));
            tc.set("id", Json::string(calls[i].id));
            tc.set("type", Json::string("function"));
            f.set("name", Json::string(calls[i].name));
            f.set("arguments", Json::string(calls[i].arguments));
            tc.set("function", f);
            tcs.push(tc);
          }
          d.set("tool_calls", tcs);
          ch.set("index", Json::integer(0));
          ch.set("delta", d);
          ch.set("finish_reason", Json::string("tool_calls"));
          arr.push(ch);
          c.set("choices", arr);
          write_all(fd, "data: " + c.dump() + "\n\n");
        } else {
          write_all(fd, chunk_json("", finish_reason, false));
        }
        write_all(fd, "data: [DONE]\n\n");
      }
    }
    if (done) break;
  }
  forget(id);
  if (client_gone || stopped_by_string) {
    std::lock_guard<std::mutex> g(mu_);
    cancelled_.push_back(id);
  }
  requests_finished_++;
  if (stream || client_gone) return false;
  if (native == "generate") {
    const double total_ms = std::chrono::duration<double, std::milli>(Clock::now() - t_start).count();
    const double decode_ms = std::chrono::duration<double, std::milli>(Clock::now() - t_first).count();
    Json st = Json::object();
    st.set("prompt_tokens", Json::integer((int64_t)n_prompt));
    st.set("completion_tokens", Json::integer((int64_t)n_gen));
    st.set("decode_ms", Json::number(decode_ms));
    st.set("dec_tps", Json::number(n_gen > 1 ? (double)(n_gen - 1) / std::max(decode_ms / 1000.0, 1e-6) : 0.0));
    st.set("ttft_ms", Json::number(total_ms - decode_ms));
    Json o = Json::object();
    o.set("text", Json::string(text));
    o.set("finish_reason", Json::string(finish_reason));
    o.set("stats", st);
    return respond(fd, 200, "application/json", o.dump(), keep_alive);
  }
  Json o = Json::object();
  o.set("id", Json::string(oid));
  o.set("object", Json::string(chat ? "chat.completion" : "text_completion"));
  o.set("created", Json::integer(created));
  o.set("model", Json::string(opts_.model_id));
  Json ch = Json::object();
  ch.set("index", Json::integer(0));
  if (chat) {
    Json msg = Json::object();
    msg.set("role", Json::string("assistant"));
    const auto calls = tools_on ? extract_tool_calls(text, known_tools) : std::vector<ToolCall>{};
    if (!calls.empty()) {
      Json tcs = Json::array();
      for (const auto& c : calls) {
        Json tc = Json::object(), f = Json::object();
        tc.set("id", Json::string(c.id));
        tc.set("type", Json::string("function"));
        f.set("name", Json::string(c.name));
        f.set("arguments", Json::string(c.arguments));
        tc.set("function", f);
        tcs.push(tc);
      }
      msg.set("content", Json::null());
      msg.set("tool_calls", tcs);
      finish_reason = "tool_calls";
    } else {
      msg.set("content", Json::string(text));
    }
    ch.set("message", msg);
  } else {
    ch.set("text", Json::string(text));
  }
  ch.set("finish_reason", Json::string(finish_reason));
  Json arr = Json::array();
  arr.push(ch);
  o.set("choices", arr);
  Json u = Json::object();
  u.set("prompt_tokens", Json::integer((int64_t)n_prompt));
  u.set("completion_tokens", Json::integer((int64_t)n_gen));
  u.set("total_tokens", Json::integer((int64_t)(n_prompt + n_gen)));
  o.set("usage", u);
  return respond(fd, 200, "application/json", o.dump(), keep_alive);
}

bool HttpServer::handle_embeddings(int fd, const Json& j, bool keep_alive) {
  ServeRequest r;
  r.kind = "embedding";
  std::vector<std::string> inputs;
  if (j["input"].is_string()) inputs.push_back(j["input"].as_string());
  else if (j["input"].is_array())
    for (const auto& s : j["input"].items())
      if (s.is_string()) inputs.push_back(s.as_string());
  if (inputs.empty()) return respond_error(fd, 400, "'input' must not be empty", "missing_required_parameter", keep_alive);
  if (j.has("encoding_format") && j["encoding_format"].is_string() && j["encoding_format"].as_string() != "float")
    return respond_error(fd, 400, "only encoding_format=float is supported", "invalid_json", keep_alive);
  size_t n_tok = 0;
  for (const auto& s : inputs) {
    r.inputs.push_back(tok_->encode(s, true));
    if (r.inputs.back().empty()) return respond_error(fd, 400, "input tokenizes to nothing", "missing_required_parameter", keep_alive);
    if ((int)r.inputs.back().size() >= opts_.max_context)
      return respond_error(fd, 400, "input longer than the context window", "context_length_exceeded", keep_alive);
    n_tok += r.inputs.back().size();
  }
  auto p = admit(std::move(r));
  if (!p) return respond_error(fd, 503, "request queue is full", "overloaded", keep_alive);
  std::vector<std::vector<float>> vecs;
  {
    std::unique_lock<std::mutex> g(p->mu);
    const bool ok = p->cv.wait_for(g, std::chrono::milliseconds((int64_t)(opts_.request_timeout_s * 1000)),
                                   [&] { return p->emb_ready || p->done; });
    if (!ok || p->err_status || !p->emb_ready) {
      const int st = p->err_status ? p->err_status : 504;
      const std::string msg = p->err_status ? p->err_msg : "embedding timed out";
      g.unlock();
      forget(p->id);
      return respond_error(fd, st, msg, "internal_error", keep_alive);
    }
    vecs.swap(p->emb);
  }
  forget(p->id);
  requests_finished_++;
  Json data = Json::array();
  for (size_t i = 0; i < vecs.size(); ++i) {
    Json e = Json::object();
    e.set("object", Json::string("embedding"));
    e.set("index", Json::integer((int64_t)i));
    Json v = Json::array();
    for (float x : vecs[i]) v.push(Json::number(x));
    e.set("embedding", v);
    data.push(e);
  }
  Json o = Json::object();
  o.set("object", Json::string("list"));
  o.set("data", data);
  o.set("model", Json::string(opts_.model_id));
  Json u = Json::object();
  u.set("prompt_tokens", Json::integer((int64_t)n_tok));
  u.set("total_tokens", Json::integer((int64_t)n_tok));
  o.set("usage", u);
  return respond(fd, 200, "application/json", o.dump(), keep_alive);
}

std::vector<ServeRequest> HttpServer::poll(int timeout_ms) {
  std::unique_lock<std::mutex> g(mu_);
  if (queue_.empty() && timeout_ms > 0)
    cv_.wait_for(g, std::chrono::milliseconds(timeout_ms), [&] { return !queue_.empty() || !running_; });
  std::vector<ServeRequest> out(std::make_move_iterator(queue_.begin()), std::make_move_iterator(queue_.end()));
  queue_.clear();
  return out;
}

void HttpServer::push(uint64_t id, const std::vector<int32_t>& tokens, int finish) {
  std::shared_ptr<Pending> p;
  {
    std::lock_guard<std::mutex> g(mu_);
    auto it = pending_.find(id);
    if (it == pending_.end()) return;
    p = it->second;
  }
  std::lock_guard<std::mutex> g(p->mu);
  p->tokens.insert(p->tokens.end(), tokens.begin(), tokens.end());
  if (finish) {
    p->finish = finish;
    p->done = true;
  }
  p->cv.notify_all();
}

void HttpServer::push_embeddings(uint64_t id, const std::vector<std::vector<float>>& vecs) {
  std::shared_ptr<Pending> p;
  {
    std::lock_guard<std::mutex> g(mu_);
    auto it = pending_.find(id);
    if (it == pending_.end()) return;
    p = it->second;
  }
  std::lock_guard<std::mutex> g(p->mu);
  p->emb = vecs;
  p->emb_ready = true;
  p->cv.notify_all();
}

void HttpServer::fail(uint64_t id, int status, const std::string& message) {
  std::shared_ptr<Pending> p;
  {
    std::lock_guard<std::mutex> g(mu_);
    auto it = pending_.find(id);
    if (it == pending_.end()) return;
    p = it->second;
  }
  std::lock_guard<std::mutex> g(p->mu);
  p->err_status = status;
  p->err_msg = message;
  p->done = true;
  p->cv.notify_all();
}

std::vector<uint64_t> HttpServer::take_cancelled() {
  std::lock_guard<std::mutex> g(mu_);
  std::vector<uint64_t> out;
  out.swap(cancelled_);
  return out;
}

void HttpServer::set_metric(const std::string& name, double value, const std::string& help, bool counter) {
  std::lock_guard<std::mutex> g(mu_);
  metrics_[name] = {value, {help, counter}};
}

std::string HttpServer::metrics_text() const {
  std::string o;
  auto emit = [&](const std::string& name, double v, const std::string& help, bool counter) {
    o += "# HELP " + name + " " + help + "\n# TYPE " + name + " " + (counter ? "counter" : "gauge") + "\n" + name +
         " " + json_number(v) + "\n";
  };
  size_t queued, active;
  std::map<std::string, std::pair<double, std::pair<std::string, bool>>> extra;
  {
    std::lock_guard<std::mutex> g(mu_);
    queued = queue_.size();
    active = pending_.size() - std::min(pending_.size(), queued);
    extra = metrics_;
  }
  emit("hawking_requests_admitted_total", (double)requests_admitted_, "Requests admitted to the engine queue", true);
  emit("hawking_requests_finished_total", (double)requests_finished_, "Requests answered", true);
  emit("hawking_requests_rejected_total", (double)requests_rejected_, "Requests refused (queue full or 501)", true);
  emit("hawking_tokens_generated_total", (double)tokens_generated_, "Tokens generated across all requests", true);
  emit("hawking_prompt_tokens_total", (double)prompt_tokens_, "Prompt tokens admitted", true);
  emit("hawking_active_slots", (double)active, "Requests being generated", false);
  emit("hawking_queued_requests", (double)queued, "Requests waiting for the engine loop", false);
  for (const auto& kv : extra) emit(kv.first, kv.second.first, kv.second.second.first, kv.second.second.second);
  return o;
}

Json HttpServer::stats() const {
  Json o = Json::object();
  o.set("requests_admitted", Json::uinteger(requests_admitted_));
  o.set("requests_finished", Json::uinteger(requests_finished_));
  o.set("tokens_generated", Json::uinteger(tokens_generated_));
  o.set("connections", Json::integer(connections_.load()));
  return o;
}

}  // namespace hk
