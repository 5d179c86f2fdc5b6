// OpenAI-compatible HTTP/1.1 + SSE front end, written from scratch on POSIX sockets.
//
// The server owns the network side: it accepts connections (one thread per connection, capped),
// parses requests, validates the JSON bodies, renders chat templates, tokenizes, and streams or
// returns the responses (detokenisation, stop strings, SSE framing, usage accounting). Generation
// itself is driven by the engine loop, which pulls admitted requests with poll() and pushes
// sampled tokens back with push(); every network wait happens on the server's own threads, so
// the engine loop never blocks on a client.
//
// Routes: GET /healthz, GET /metrics (Prometheus text), GET /v1/models,
// POST /v1/chat/completions, POST /v1/completions (both with "stream": true -> SSE ending in
// "data: [DONE]"), POST /v1/embeddings, and 501 bodies for POST /v1/responses and /v1/messages.
// Chat requests with "tools" get the tools preamble in the prompt and their completion parsed for
// tool calls (message.tool_calls, finish_reason "tool_calls"); "response_format":
// {"type": "json_object"} marks the request JSON-constrained (the engine masks its sampling).
// Native routes: POST /v1/hawking/generate (lean generate with decode statistics),
// POST /v1/hawking/tokens (greedy token ids as SSE), GET /v1/hawking/context (context and slot
// status), GET /v1/hawking/surface (routes, features and model families served).
// Errors use the OpenAI shape {"error": {"message", "type", "code"}}.
//
// Parity: crates/hawking-serve/src/http.rs:265-281 (routes), :307 (healthz), :329-365 (metrics
// names), :610 / :673 (chat / completions), :828 (SSE [DONE]), :1410 (embeddings), :290-305
// (501 stubs), :43-91 (error body), :871 (wait queue bounded at max_batch * 8), :272-276 and
// :971-1140 (/v1/hawking routes), :389-420 (context status), :650 (json_mode from response_format).
#pragma once
#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <deque>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "json.h"
#include "tokenizer.h"

namespace hk {

struct ServeOptions {
  std::string host = "127.0.0.1";
  int port = 8000;                 // 0 picks a free port (see HttpServer::port)
  std::string model_id = "hawking-b200";
  std::string chat_template = "auto";  // auto | llama3 | chatml | deepseek | generic
  int max_queue = 512;             // admitted-but-not-started requests beyond this get 503
  int max_connections = 256;
  int default_max_tokens = 256;
  int max_context = 8192;
  double request_timeout_s = 600.0;
  int max_batch = 8;               // engine decode slots (reported by /v1/hawking/context)
  std::string architecture = "llama";
  int64_t recurrent_state_bytes = 0;  // per sequence (hybrid models)
};

// One admitted request, handed to the engine loop by poll().
struct ServeRequest {
  uint64_t id = 0;
  std::string kind;  // "chat" | "completion" | "embedding"
  std::vector<int32_t> prompt;
  std::vector<std::vector<int32_t>> inputs;  // embeddings: one token list per input
  int max_tokens = 256;
  float temperature = 1.0f, top_p = 1.0f, repetition_penalty = 1.0f;
  int top_k = 0;
  uint64_t seed = 42;
  bool stream = false;
  bool json_mode = false;         // constrain sampling to a JSON object
  std::vector<int32_t> stop_ids;  // end-of-generation token ids
};

class HttpServer {
 public:
  HttpServer(ServeOptions opts, std::shared_ptr<Tokenizer> tok);
  ~HttpServer();
  void start();  // binds and starts the accept thread; throws on bind failure
  void stop();   // closes the listener and fails every pending request
  int port() const { return bound_port_; }

  // Engine side.
  std::vector<ServeRequest> poll(int timeout_ms);
  // finish: 0 = running, 1 = length, 2 = stop (end-of-generation token), 3 = aborted.
  void push(uint64_t id, const std::vector<int32_t>& tokens, int finish);
  void push_embeddings(uint64_t id, const std::vector<std::vector<float>>& vecs);
  void fail(uint64_t id, int status, const std::string& message);
  std::vector<uint64_t> take_cancelled();  // requests whose client left or hit a stop string
  void set_metric(const std::string& name, double value, const std::string& help, bool counter);
  // Unhealthy: /healthz answers 503 with the reason and new generation requests are refused.
  void set_health(bool ok, const std::string& reason);
  Json stats() const;

  // Chat template rendering (exposed for tests). messages: [{"role", "content"}].
  std::string render_chat(const Json& messages, const std::string& tmpl) const;
  std::string resolve_template() const;

  struct Pending;  // per-request channel between the engine loop and a connection thread

 private:
  void accept_loop();
  void serve_connection(int fd);
  bool handle(int fd, const std::string& method, const std::string& path, const std::string& body, bool keep_alive);
  // native: "" (OpenAI shape), "generate" (/v1/hawking/generate), "tokens" (/v1/hawking/tokens)
  bool handle_generate(int fd, const Json& body, bool chat, bool keep_alive, const std::string& native = "");
  bool handle_embeddings(int fd, const Json& body, bool keep_alive);
  std::string metrics_text() const;
  std::shared_ptr<Pending> admit(ServeRequest req);
  void forget(uint64_t id);

  ServeOptions opts_;
  std::shared_ptr<Tokenizer> tok_;
  int listen_fd_ = -1;
  int bound_port_ = 0;
  std::atomic<bool> running_{false};
  std::thread accept_thread_;
  std::atomic<int> connections_{0};

  mutable std::mutex mu_;
  std::condition_variable cv_;  // new requests for poll()
  std::deque<ServeRequest> queue_;
  std::map<uint64_t, std::shared_ptr<Pending>> pending_;
  std::vector<uint64_t> cancelled_;
  uint64_t next_id_ = 1;
  std::map<std::string, std::pair<double, std::pair<std::string, bool>>> metrics_;

  std::atomic<bool> healthy_{true};
  std::string health_reason_;  // guarded by mu_
  std::atomic<uint64_t> requests_admitted_{0}, requests_finished_{0}, requests_rejected_{0},
      tokens_generated_{0}, prompt_tokens_{0};
};

}  // namespace hk
