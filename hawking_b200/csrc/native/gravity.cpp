// `.gravity` container; see gravity.h.
#include "gravity.h"

#include <atomic>
#include <thread>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <set>
#include <stdexcept>

#include "ggml_quant.h"
#include "sha256.h"

namespace hk {

namespace {
constexpr char kMagic[8] = {'G', 'R', 'A', 'V', 'I', 'T', 'Y', '\0'};
constexpr uint32_t kMaxVersion = 1;
constexpr size_t kPrefix = 20;
const char* kSchema = "hawking.gravity.shard_header.v1";

template <typename T> T rd(const uint8_t* p) { T v; std::memcpy(&v, p, sizeof(T)); return v; }
}  // namespace

int gravity_codec_to_ggml(const std::string& c) {
  static const std::map<std::string, int> m = {
      {"native.f32", 0}, {"native.f16", 1}, {"native.bf16", 30}, {"ggml.q3_k", 11}, {"ggml.q4_k", 12},
      {"ggml.q5_k", 13}, {"ggml.q6_k", 14}, {"ggml.q8_0", 8},    {"ggml.q5_0", 6},  {"ggml.q4_0", 2}};
  auto it = m.find(c);
  return it == m.end() ? -1 : it->second;
}

std::unique_ptr<GravityShard> GravityShard::open(const std::string& path) {
  int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) throw std::runtime_error("gravity: cannot open " + path);
  struct stat st;
  if (fstat(fd, &st) != 0) { ::close(fd); throw std::runtime_error("gravity: cannot stat " + path); }
  size_t size = (size_t)st.st_size;
  void* m = size ? mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0) : MAP_FAILED;
  ::close(fd);
  if (m == MAP_FAILED) throw std::runtime_error("gravity: mmap failed for " + path);
  std::unique_ptr<GravityShard> s(new GravityShard());
  s->path_ = path;
  s->base_ = static_cast<const uint8_t*>(m);
  s->size_ = size;
  if (size < kPrefix) throw std::runtime_error("gravity: prefix short: " + std::to_string(size));
  if (std::memcmp(s->base_, kMagic, 8) != 0) throw std::runtime_error("gravity: bad magic");
  s->version_ = rd<uint32_t>(s->base_ + 8);
  if (s->version_ > kMaxVersion) throw std::runtime_error("gravity: bad version " + std::to_string(s->version_));
  uint64_t hlen = rd<uint64_t>(s->base_ + 12);
  if (hlen > size - kPrefix) throw std::runtime_error("gravity: header runs past end of file");
  s->header_ = Json::parse(reinterpret_cast<const char*>(s->base_ + kPrefix), hlen);
  s->body_off_ = kPrefix + hlen;
  const Json& ts = s->header_["tensors"];
  if (!ts.is_array()) throw std::runtime_error("gravity: header has no tensors array");
  for (const auto& d : ts.items()) {
    GravityTensor t;
    t.name = d["name"].as_string();
    t.codec = d["codec"].is_string() ? d["codec"].as_string() : "";
    t.offset = d["offset"].as_uint();
    t.bytes = d["bytes"].as_uint();
    t.sha256 = d["sha256"].is_string() ? d["sha256"].as_string() : "";
    if (d["shape"].is_array())
      for (const auto& x : d["shape"].items()) t.shape.push_back(x.as_uint());
    t.elements = d["elements"].is_number() ? d["elements"].as_uint() : 0;
    t.extra = d;
    if (s->index_.count(t.name)) throw std::runtime_error("gravity: duplicate tensor " + t.name);
    if (s->body_off_ + t.offset + t.bytes > size) throw std::runtime_error("gravity: tensor " + t.name + " runs past end");
    s->index_[t.name] = s->tensors_.size();
    s->tensors_.push_back(std::move(t));
  }
  return s;
}

GravityShard::~GravityShard() {
  if (base_) munmap(const_cast<uint8_t*>(base_), size_);
}

const GravityTensor* GravityShard::find(const std::string& name) const {
  auto it = index_.find(name);
  return it == index_.end() ? nullptr : &tensors_[it->second];
}

namespace {
// Runs f(i) for i in [0, n) on up to hardware_concurrency threads (payload hashing).
template <typename F>
void parallel_for(size_t n, F f) {
  const size_t nt = std::max<size_t>(1, std::min<size_t>(n, std::thread::hardware_concurrency()));
  if (nt <= 1) {
    for (size_t i = 0; i < n; ++i) f(i);
    return;
  }
  std::atomic<size_t> next{0};
  std::vector<std::thread> ts;
  for (size_t t = 0; t < nt; ++t)
    ts.emplace_back([&]() {
      for (size_t i = next++; i < n; i = next++) f(i);
    });
  for (auto& t : ts) t.join();
}
}  // namespace

bool GravityShard::verify_tensor(const std::string& name) const {
  const auto* t = find(name);
  if (!t) throw std::runtime_error("gravity: no tensor " + name);
  return Sha256::hex_of(data(*t), t->bytes) == t->sha256;
}

Json GravityShard::verify() const {
  std::vector<const GravityTensor*> ord;
  for (const auto& t : tensors_) ord.push_back(&t);
  std::sort(ord.begin(), ord.end(), [](const GravityTensor* a, const GravityTensor* b) {
    return a->offset != b->offset ? a->offset < b->offset : a->name < b->name;
  });
  Json rep = Json::object();
  rep.set("path", Json::string(path_));
  rep.set("format_version", Json::uinteger(version_));
  const uint64_t phys = size_ - body_off_;
  uint64_t cursor = 0;
  std::string layout_err;
  for (const auto* t : ord) {
    if (t->offset != cursor && layout_err.empty())
      layout_err = std::string(t->offset < cursor ? "overlap" : "gap") + " at tensor " + t->name;
    cursor = t->offset + t->bytes;
  }
  if (layout_err.empty() && cursor != phys)
    layout_err = "trailing or undeclared body bytes: declared " + std::to_string(cursor) + ", physical " +
                 std::to_string(phys);
  std::string body_hex;
  std::vector<char> tensor_ok(ord.size(), 0);
  std::thread body_thread([&]() { body_hex = Sha256::hex_of(base_ + body_off_, phys); });
  parallel_for(ord.size(), [&](size_t i) { tensor_ok[i] = Sha256::hex_of(data(*ord[i]), ord[i]->bytes) == ord[i]->sha256; });
  body_thread.join();
  const bool body_ok = body_hex == header_.pointer("/integrity/body_sha256").as_string();
  Json bad = Json::array(), empty = Json::array();
  uint64_t el_all = 0, by_all = 0, el_cmp = 0, by_cmp = 0;
  for (size_t i = 0; i < ord.size(); ++i) {
    const auto* t = ord[i];
    if (!tensor_ok[i]) bad.push(Json::string(t->name));
    if (t->bytes == 0) empty.push(Json::string(t->name));
    if (t->elements) {
      el_all += t->elements;
      by_all += t->bytes;
      if (t->codec.rfind("native.", 0) != 0) { el_cmp += t->elements; by_cmp += t->bytes; }
    }
  }
  const double packed = el_cmp ? by_cmp * 8.0 / el_cmp : 0.0;
  const double complete = el_all ? by_all * 8.0 / el_all : 0.0;
  const Json& comp = header_["compression"];
  const double claim_p = comp["packed_bpw"].is_number() ? comp["packed_bpw"].as_double() : packed;
  const double claim_c = comp["complete_bpw"].is_number() ? comp["complete_bpw"].as_double() : complete;
  const bool bpw_ok = std::fabs(packed - claim_p) < 1e-6 && std::fabs(complete - claim_c) < 1e-6;
  rep.set("body_sha256_ok", Json::boolean(body_ok));
  rep.set("layout_error", Json::string(layout_err));
  rep.set("bad_tensors", bad);
  rep.set("empty_tensors", empty);
  rep.set("observed_packed_bpw", Json::number(packed));
  rep.set("observed_complete_bpw", Json::number(complete));
  rep.set("bpw_claims_ok", Json::boolean(bpw_ok));
  rep.set("tensor_count", Json::uinteger(tensors_.size()));
  rep.set("ok", Json::boolean(body_ok && layout_err.empty() && bad.size() == 0 && empty.size() == 0 && bpw_ok));
  return rep;
}

void GravityWriter::add(Json d, const uint8_t* data, size_t n) {
  if (!d.is_object() || !d["name"].is_string()) throw std::runtime_error("gravity writer: descriptor needs a name");
  items_.emplace_back(std::move(d), std::vector<uint8_t>(data, data + n));
}

Json GravityWriter::write(const std::string& path) const {
  Json tensors = Json::array();
  std::set<std::string> seen;
  // the body digest (one stream) on its own thread, the payload digests in parallel
  std::string body_hex;
  std::thread body_thread([&]() {
    Sha256 body;
    for (const auto& it : items_) body.update(it.second.data(), it.second.size());
    body_hex = body.hex();
  });
  std::vector<std::string> digests(items_.size());
  parallel_for(items_.size(), [&](size_t i) {
    digests[i] = Sha256::hex_of(items_[i].second.data(), items_[i].second.size());
  });
  body_thread.join();
  uint64_t off = 0;
  for (size_t i = 0; i < items_.size(); ++i) {
    const auto& it = items_[i];
    Json e = it.first;
    const std::string name = e["name"].as_string();
    if (!name.empty() && !seen.insert(name).second) throw std::runtime_error("gravity writer: duplicate tensor " + name);
    e.set("offset", Json::uinteger(off));
    e.set("bytes", Json::uinteger(it.second.size()));
    e.set("sha256", Json::string(digests[i]));
    tensors.push(std::move(e));
    off += it.second.size();
  }
  auto meta_or = [&](const char* k) { return meta_.has(k) ? meta_[k] : Json::object(); };
  Json h = Json::object();
  h.set("schema", Json::string(kSchema));
  h.set("format_version", Json::uinteger(1));
  for (const char* k : {"model", "architecture", "tokenizer", "compression", "shard", "gguf_metadata"})
    h.set(k, meta_or(k));
  Json integ = Json::object();
  integ.set("body_sha256", Json::string(body_hex));
  integ.set("tensor_count", Json::uinteger(items_.size()));
  h.set("integrity", integ);
  h.set("tensors", tensors);
  const std::string enc = h.canonical();
  const std::string tmp = path + ".tmp";
  FILE* f = std::fopen(tmp.c_str(), "wb");
  if (!f) throw std::runtime_error("gravity writer: cannot create " + tmp);
  const uint32_t ver = 1;
  const uint64_t hl = enc.size();
  bool ok = std::fwrite(kMagic, 1, 8, f) == 8 && std::fwrite(&ver, 4, 1, f) == 1 && std::fwrite(&hl, 8, 1, f) == 1 &&
            std::fwrite(enc.data(), 1, enc.size(), f) == enc.size();
  for (const auto& it : items_)
    ok = ok && std::fwrite(it.second.data(), 1, it.second.size(), f) == it.second.size();
  ok = (std::fclose(f) == 0) && ok;
  if (!ok) {
    std::remove(tmp.c_str());
    throw std::runtime_error("gravity writer: write failed for " + tmp);
  }
  if (std::rename(tmp.c_str(), path.c_str()) != 0) {
    std::remove(tmp.c_str());
    throw std::runtime_error("gravity writer: rename failed for " + path);
  }
  return h;
}

}  // namespace hk
