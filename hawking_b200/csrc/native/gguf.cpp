// GGUF reader/writer; see gguf.h.
#include "gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <cstring>
#include <stdexcept>

#include "ggml_quant.h"

namespace hk {

namespace {
constexpr uint32_t kMagic = 0x46554747u;  // "GGUF" little endian

struct Cursor {
  const uint8_t* p;
  size_t n, off = 0;
  void need(size_t k) const {
    if (off + k > n) throw std::runtime_error("gguf: truncated at byte " + std::to_string(off));
  }
  template <typename T> T get() {
    need(sizeof(T));
    T v; std::memcpy(&v, p + off, sizeof(T)); off += sizeof(T);
    return v;
  }
  std::string str() {
    uint64_t len = get<uint64_t>();
    if (len > (1ull << 32)) throw std::runtime_error("gguf: implausible string length");
    need(len);
    std::string s(reinterpret_cast<const char*>(p + off), len);
    off += len;
    return s;
  }
};

GgufValue read_value(Cursor& c, GgufKind k, int depth) {
  GgufValue v;
  v.kind = k;
  switch (k) {
    case GgufKind::U8: v.i = c.get<uint8_t>(); break;
    case GgufKind::I8: v.i = c.get<int8_t>(); break;
    case GgufKind::U16: v.i = c.get<uint16_t>(); break;
    case GgufKind::I16: v.i = c.get<int16_t>(); break;
    case GgufKind::U32: v.i = c.get<uint32_t>(); break;
    case GgufKind::I32: v.i = c.get<int32_t>(); break;
    case GgufKind::U64: v.i = (int64_t)c.get<uint64_t>(); break;
    case GgufKind::I64: v.i = c.get<int64_t>(); break;
    case GgufKind::F32: v.f = c.get<float>(); break;
    case GgufKind::F64: v.f = c.get<double>(); break;
    case GgufKind::BOOL: v.i = c.get<uint8_t>() ? 1 : 0; break;
    case GgufKind::STRING: v.s = c.str(); break;
    case GgufKind::ARRAY: {
      if (depth > 4) throw std::runtime_error("gguf: nested arrays too deep");
      auto ek = static_cast<GgufKind>(c.get<uint32_t>());
      uint64_t n = c.get<uint64_t>();
      if (n > c.n) throw std::runtime_error("gguf: implausible array length");
      v.arr_kind = ek;
      v.arr = std::make_shared<GgufArray>();
      v.arr->reserve(n);
      for (uint64_t i = 0; i < n; ++i) v.arr->push_back(read_value(c, ek, depth + 1));
      break;
    }
    default: throw std::runtime_error("gguf: unknown metadata kind " + std::to_string((uint32_t)k));
  }
  return v;
}

void put(std::vector<uint8_t>& o, const void* p, size_t n) {
  const uint8_t* b = static_cast<const uint8_t*>(p);
  o.insert(o.end(), b, b + n);
}
template <typename T> void put(std::vector<uint8_t>& o, T v) { put(o, &v, sizeof(T)); }
void put_str(std::vector<uint8_t>& o, const std::string& s) { put<uint64_t>(o, s.size()); put(o, s.data(), s.size()); }

void write_value(std::vector<uint8_t>& o, const GgufValue& v, bool with_kind) {
  if (with_kind) put<uint32_t>(o, (uint32_t)v.kind);
  switch (v.kind) {
    case GgufKind::U8: put<uint8_t>(o, (uint8_t)v.i); break;
    case GgufKind::I8: put<int8_t>(o, (int8_t)v.i); break;
    case GgufKind::U16: put<uint16_t>(o, (uint16_t)v.i); break;
    case GgufKind::I16: put<int16_t>(o, (int16_t)v.i); break;
    case GgufKind::U32: put<uint32_t>(o, (uint32_t)v.i); break;
    case GgufKind::I32: put<int32_t>(o, (int32_t)v.i); break;
    case GgufKind::U64: put<uint64_t>(o, (uint64_t)v.i); break;
    case GgufKind::I64: put<int64_t>(o, v.i); break;
    case GgufKind::F32: put<float>(o, (float)v.f); break;
    case GgufKind::F64: put<double>(o, v.f); break;
    case GgufKind::BOOL: put<uint8_t>(o, v.i ? 1 : 0); break;
    case GgufKind::STRING: put_str(o, v.s); break;
    case GgufKind::ARRAY: {
      put<uint32_t>(o, (uint32_t)v.arr_kind);
      uint64_t n = v.arr ? v.arr->size() : 0;
      put<uint64_t>(o, n);
      for (uint64_t i = 0; i < n; ++i) write_value(o, (*v.arr)[i], false);
      break;
    }
  }
}
uint64_t align_up(uint64_t x, uint64_t a) { return (x + a - 1) / a * a; }
}  // namespace

uint64_t GgufTensorInfo::n_elements() const {
  uint64_t n = 1;
  for (auto d : dims) n *= d;
  return n;
}

std::unique_ptr<GgufFile> GgufFile::open(const std::string& path) {
  int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) throw std::runtime_error("gguf: cannot open " + path);
  struct stat st;
  if (fstat(fd, &st) != 0) { ::close(fd); throw std::runtime_error("gguf: cannot stat " + path); }
  size_t size = (size_t)st.st_size;
  void* m = size ? mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0) : MAP_FAILED;
  ::close(fd);
  if (m == MAP_FAILED) throw std::runtime_error("gguf: mmap failed for " + path);
  std::unique_ptr<GgufFile> f(new GgufFile());
  f->path_ = path;
  f->base_ = static_cast<const uint8_t*>(m);
  f->size_ = size;
  f->mapped_ = true;
  f->parse();
  return f;
}

std::unique_ptr<GgufFile> GgufFile::from_memory(const uint8_t* data, size_t size) {
  std::unique_ptr<GgufFile> f(new GgufFile());
  f->base_ = data;
  f->size_ = size;
  f->parse();
  return f;
}

GgufFile::~GgufFile() {
  if (mapped_ && base_) munmap(const_cast<uint8_t*>(base_), size_);
}

void GgufFile::parse() {
  Cursor c{base_, size_};
  uint32_t magic = c.get<uint32_t>();
  if (magic != kMagic) throw std::runtime_error("gguf: bad magic");
  version_ = c.get<uint32_t>();
  if (version_ < 2 || version_ > 3) throw std::runtime_error("gguf: unsupported version " + std::to_string(version_));
  uint64_t n_tensors = c.get<uint64_t>();
  uint64_t n_kv = c.get<uint64_t>();
  if (n_tensors > (1u << 24) || n_kv > (1u << 24)) throw std::runtime_error("gguf: implausible table sizes");
  for (uint64_t i = 0; i < n_kv; ++i) {
    std::string key = c.str();
    auto kind = static_cast<GgufKind>(c.get<uint32_t>());
    kv_[key] = read_value(c, kind, 0);
  }
  auto it = kv_.find("general.alignment");
  if (it != kv_.end()) {
    alignment_ = (uint64_t)it->second.i;
    if (alignment_ == 0 || (alignment_ & (alignment_ - 1))) throw std::runtime_error("gguf: bad alignment");
  }
  tensors_.reserve(n_tensors);
  for (uint64_t i = 0; i < n_tensors; ++i) {
    GgufTensorInfo t;
    t.name = c.str();
    uint32_t nd = c.get<uint32_t>();
    if (nd == 0 || nd > 4) throw std::runtime_error("gguf: bad n_dims for " + t.name);
    for (uint32_t d = 0; d < nd; ++d) t.dims.push_back(c.get<uint64_t>());
    t.type = c.get<uint32_t>();
    t.offset = c.get<uint64_t>();
    if (!type_known(t.type)) throw std::runtime_error("gguf: unknown ggml type for " + t.name);
    t.nbytes = type_nbytes(t.type, t.n_elements());
    if (t.offset % alignment_) throw std::runtime_error("gguf: misaligned tensor " + t.name);
    index_[t.name] = tensors_.size();
    tensors_.push_back(std::move(t));
  }
  data_offset_ = align_up(c.off, alignment_);
  for (const auto& t : tensors_)
    if (data_offset_ + t.offset + t.nbytes > size_)
      throw std::runtime_error("gguf: tensor " + t.name + " runs past end of file");
}

const GgufTensorInfo* GgufFile::find(const std::string& name) const {
  auto it = index_.find(name);
  return it == index_.end() ? nullptr : &tensors_[it->second];
}

void GgufWriter::add_tensor(const std::string& name, const std::vector<uint64_t>& dims, uint32_t type,
                            const uint8_t* data, size_t nbytes) {
  Pending p;
  p.info.name = name;
  p.info.dims = dims;
  p.info.type = type;
  p.info.nbytes = type_nbytes(type, p.info.n_elements());
  if (p.info.nbytes != nbytes) throw std::runtime_error("gguf writer: size mismatch for " + name);
  p.bytes.assign(data, data + nbytes);
  tensors_.push_back(std::move(p));
}

void GgufWriter::write(const std::string& path) const {
  std::vector<uint8_t> h;
  put<uint32_t>(h, kMagic);
  put<uint32_t>(h, 3);
  put<uint64_t>(h, tensors_.size());
  bool has_align = false;
  for (auto& kv : kv_) has_align |= kv.first == "general.alignment";
  put<uint64_t>(h, kv_.size() + (has_align ? 0 : 1));
  if (!has_align) {
    put_str(h, "general.alignment");
    GgufValue a; a.kind = GgufKind::U32; a.i = (int64_t)alignment_;
    write_value(h, a, true);
  }
  for (auto& kv : kv_) { put_str(h, kv.first); write_value(h, kv.second, true); }
  uint64_t off = 0;
  std::vector<uint64_t> offs;
  for (auto& t : tensors_) {
    put_str(h, t.info.name);
    put<uint32_t>(h, (uint32_t)t.info.dims.size());
    for (auto d : t.info.dims) put<uint64_t>(h, d);
    put<uint32_t>(h, t.info.type);
    put<uint64_t>(h, off);
    offs.push_back(off);
    off = align_up(off + t.bytes.size(), alignment_);
  }
  std::string tmp = path + ".tmp";
  FILE* f = std::fopen(tmp.c_str(), "wb");
  if (!f) throw std::runtime_error("gguf writer: cannot create " + tmp);
  std::fwrite(h.data(), 1, h.size(), f);
  std::vector<uint8_t> pad(alignment_, 0);
  uint64_t pos = h.size(), data0 = align_up(pos, alignment_);
  std::fwrite(pad.data(), 1, data0 - pos, f);
  pos = data0;
  for (size_t i = 0; i < tensors_.size(); ++i) {
    uint64_t want = data0 + offs[i];
    std::fwrite(pad.data(), 1, want - pos, f);
    std::fwrite(tensors_[i].bytes.data(), 1, tensors_[i].bytes.size(), f);
    pos = want + tensors_[i].bytes.size();
  }
  uint64_t end = align_up(pos, alignment_);
  std::fwrite(pad.data(), 1, end - pos, f);
  if (std::fclose(f) != 0) throw std::runtime_error("gguf writer: write failed");
  if (std::rename(tmp.c_str(), path.c_str()) != 0) throw std::runtime_error("gguf writer: rename failed");
}

}  // namespace hk
