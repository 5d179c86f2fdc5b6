// Paged KV block manager; see block_manager.h.
#include "block_manager.h"

#include <stdexcept>
#include <string>

namespace hk {

BlockManager::BlockManager(int num_blocks, int block_size, bool prefix_cache)
    : bs_(block_size), prefix_cache_(prefix_cache), ref_(num_blocks, 0) {
  if (num_blocks <= 0 || block_size <= 0) throw std::runtime_error("block manager: bad geometry");
  free_.reserve(num_blocks);
  for (int b = num_blocks - 1; b >= 0; --b) free_.push_back(b);
}

uint64_t BlockManager::mix(uint64_t h, const int* t, int n) {
  // FNV-1a over the token ids, seeded by the parent block's hash (chaining).
  for (int i = 0; i < n; ++i) {
    uint32_t v = (uint32_t)t[i];
    for (int k = 0; k < 4; ++k) {
      h ^= (v >> (8 * k)) & 0xFF;
      h *= 1099511628211ull;
    }
  }
  return h;
}

int BlockManager::num_tokens(int64_t seq) const {
  auto it = seqs_.find(seq);
  return it == seqs_.end() ? 0 : it->second.tokens;
}

int BlockManager::take_block() {
  int b;
  if (!free_.empty()) {
    b = free_.back();
    free_.pop_back();
  } else if (!lru_.empty()) {  // evict the oldest cached block
    b = lru_.front();
    lru_.pop_front();
    lru_pos_.erase(b);
    auto bi = block_info_.find(b);
    if (bi != block_info_.end()) {
      auto ix = index_.find(bi->second.hash);
      if (ix != index_.end() && ix->second == b) index_.erase(ix);
      block_info_.erase(bi);
    }
  } else {
    throw std::runtime_error("block manager: out of blocks");
  }
  ref_[b] = 1;
  return b;
}

void BlockManager::put_block(int b) {
  if (--ref_[b] > 0) return;
  if (ref_[b] < 0) throw std::runtime_error("block manager: double free of block " + std::to_string(b));
  if (prefix_cache_ && block_info_.count(b)) {
    lru_.push_back(b);
    lru_pos_[b] = std::prev(lru_.end());
  } else {
    block_info_.erase(b);
    free_.push_back(b);
  }
}

int BlockManager::blocks_needed(int64_t seq, int n_tokens) const {
  auto it = seqs_.find(seq);
  int have = it == seqs_.end() ? 0 : (int)it->second.blocks.size();
  int need = (n_tokens + bs_ - 1) / bs_;
  return need > have ? need - have : 0;
}

bool BlockManager::reserve(int64_t seq, int n_tokens) {
  int extra = blocks_needed(seq, n_tokens);
  if (extra > num_free()) return false;
  auto& s = seqs_[seq];
  for (int i = 0; i < extra; ++i) s.blocks.push_back(take_block());
  if (n_tokens > s.tokens) s.tokens = n_tokens;
  return true;
}

void BlockManager::release(int64_t seq) {
  auto it = seqs_.find(seq);
  if (it == seqs_.end()) return;
  // Release in reverse so a prefix's deeper blocks are evicted before its roots.
  for (auto b = it->second.blocks.rbegin(); b != it->second.blocks.rend(); ++b) put_block(*b);
  seqs_.erase(it);
}

const std::vector<int>& BlockManager::table(int64_t seq) const {
  auto it = seqs_.find(seq);
  if (it == seqs_.end()) throw std::runtime_error("block manager: unknown sequence " + std::to_string(seq));
  return it->second.blocks;
}

std::vector<int64_t> BlockManager::slots(int64_t seq, int p0, int p1) const {
  const auto& t = table(seq);
  std::vector<int64_t> out;
  out.reserve(p1 - p0);
  for (int p = p0; p < p1; ++p) {
    int bi = p / bs_;
    if (bi >= (int)t.size()) throw std::runtime_error("block manager: position beyond reserved blocks");
    out.push_back((int64_t)t[bi] * bs_ + p % bs_);
  }
  return out;
}

int BlockManager::attach_prefix(int64_t seq, const std::vector<int>& tokens) {
  if (seqs_.count(seq)) throw std::runtime_error("attach_prefix: sequence already exists");
  auto& s = seqs_[seq];
  if (!prefix_cache_) return 0;
  int max_full = ((int)tokens.size() - 1) / bs_;  // keep at least one token to compute
  uint64_t h = 1469598103934665603ull;
  for (int i = 0; i < max_full; ++i) {
    h = mix(h, tokens.data() + i * bs_, bs_);
    auto ix = index_.find(h);
    if (ix == index_.end()) break;
    int b = ix->second;
    const auto& info = block_info_.at(b);
    bool same = true;
    for (int k = 0; k < bs_ && same; ++k) same = info.toks[k] == tokens[i * bs_ + k];
    if (!same) break;
    if (ref_[b] == 0) {  // revive from the LRU
      auto p = lru_pos_.find(b);
      if (p != lru_pos_.end()) { lru_.erase(p->second); lru_pos_.erase(p); }
    }
    ++ref_[b];
    s.blocks.push_back(b);
  }
  s.tokens = (int)s.blocks.size() * bs_;
  if (s.tokens) { ++hits_; hit_tokens_ += s.tokens; }
  return s.tokens;
}

int BlockManager::cached_prefix(const std::vector<int>& tokens) const {
  if (!prefix_cache_) return 0;
  const int max_full = ((int)tokens.size() - 1) / bs_;
  uint64_t h = 1469598103934665603ull;
  int n = 0;
  for (int i = 0; i < max_full; ++i) {
    h = mix(h, tokens.data() + i * bs_, bs_);
    auto ix = index_.find(h);
    if (ix == index_.end()) break;
    const auto& info = block_info_.at(ix->second);
    bool same = true;
    for (int k = 0; k < bs_ && same; ++k) same = info.toks[k] == tokens[i * bs_ + k];
    if (!same) break;
    n += bs_;
  }
  return n;
}

void BlockManager::commit_prefix(int64_t seq, const std::vector<int>& tokens, int n_valid) {
  if (!prefix_cache_) return;
  const auto& t = table(seq);
  int full = std::min<int>(n_valid, (int)tokens.size()) / bs_;
  uint64_t h = 1469598103934665603ull;
  for (int i = 0; i < full && i < (int)t.size(); ++i) {
    h = mix(h, tokens.data() + i * bs_, bs_);
    int b = t[i];
    auto bi = block_info_.find(b);
    if (bi != block_info_.end()) continue;  // already indexed (shared prefix)
    if (index_.count(h)) continue;           // another block holds the same prefix
    index_[h] = b;
    block_info_[b] = Cached{h, std::vector<int>(tokens.begin() + i * bs_, tokens.begin() + (i + 1) * bs_)};
  }
}

std::vector<std::pair<int, int>> BlockManager::fork(int64_t src, int64_t dst) {
  const auto& st = table(src);
  if (seqs_.count(dst)) throw std::runtime_error("fork: destination exists");
  int tokens = seqs_.at(src).tokens;
  int full = tokens / bs_;
  bool partial = tokens % bs_ != 0;
  if (partial && num_free() < 1) throw std::runtime_error("fork: out of blocks");
  Seq d;
  std::vector<std::pair<int, int>> copies;
  for (int i = 0; i < full; ++i) { ++ref_[st[i]]; d.blocks.push_back(st[i]); }
  if (partial) {
    int nb = take_block();
    d.blocks.push_back(nb);
    copies.emplace_back(st[full], nb);
  }
  d.tokens = tokens;
  seqs_[dst] = std::move(d);
  return copies;
}

void BlockManager::truncate(int64_t seq, int n_tokens) {
  auto& s = seqs_.at(seq);
  int keep = (n_tokens + bs_ - 1) / bs_;
  while ((int)s.blocks.size() > keep) {
    put_block(s.blocks.back());
    s.blocks.pop_back();
  }
  if (n_tokens < s.tokens) s.tokens = n_tokens;
}

}  // namespace hk
