// Paged KV-cache block manager: fixed-size token blocks, per-sequence block tables, reference
// counts, exact prefix reuse over full blocks (chained hash + stored token ids, so a hit is never
// a collision), copy-on-write fork and tail truncation (speculative-decode rollback).
//
// Parity: the reference has no paged KV; its nearest behaviour is the 8-slot multiseq arena with
// per-sequence regions (crates/hawking-core/src/model/qwen_dense.rs:481-488) plus
// copy_kv_prefix_to_slot prefix sharing (crates/hawking-core/src/engine.rs:600) and the serve-side
// SystemPromptKvBank (crates/hawking-serve/src/system_kv_bank.rs:93-280). Paged blocks with a
// prefix index subsume both: a shared prefix is shared blocks, not a copy.
#pragma once
#include <cstdint>
#include <list>
#include <unordered_map>
#include <utility>
#include <vector>

namespace hk {

class BlockManager {
 public:
  BlockManager(int num_blocks, int block_size, bool prefix_cache = true);

  int block_size() const { return bs_; }
  int num_blocks() const { return (int)ref_.size(); }
  // Blocks that can be handed out now (free list plus evictable cached blocks).
  int num_free() const { return (int)free_.size() + (int)lru_.size(); }
  bool has(int64_t seq) const { return seqs_.count(seq) != 0; }
  int num_tokens(int64_t seq) const;

  // Make room for n_tokens in total; false (and no change) if the pool cannot supply the blocks.
  bool reserve(int64_t seq, int n_tokens);
  // Blocks needed to grow seq to n_tokens.
  int blocks_needed(int64_t seq, int n_tokens) const;
  void release(int64_t seq);
  const std::vector<int>& table(int64_t seq) const;
  // Slot ids (block * block_size + offset) of positions [p0, p1).
  std::vector<int64_t> slots(int64_t seq, int p0, int p1) const;

  // Attach the longest cached prefix of full blocks of `tokens` to a new sequence; returns the
  // number of tokens covered (a multiple of block_size, at most tokens.size() - 1 so at least
  // one token is always computed).
  int attach_prefix(int64_t seq, const std::vector<int>& tokens);
  // Tokens of `tokens` that attach_prefix would find cached (whole blocks, at least one token left
  // to compute), without attaching anything.
  int cached_prefix(const std::vector<int>& tokens) const;
  // Register the full blocks of seq holding tokens[0:n_valid] in the prefix index.
  void commit_prefix(int64_t seq, const std::vector<int>& tokens, int n_valid);
  // Share src's blocks with dst. Full blocks are shared; a partial last block is copied: the
  // returned (src_block, dst_block) pairs must be copied on the device by the caller.
  std::vector<std::pair<int, int>> fork(int64_t src, int64_t dst);
  // Shrink seq to n_tokens, returning freed tail blocks to the pool.
  void truncate(int64_t seq, int n_tokens);

  int64_t prefix_hits() const { return hits_; }
  int64_t prefix_hit_tokens() const { return hit_tokens_; }

 private:
  struct Seq { std::vector<int> blocks; int tokens = 0; };
  struct Cached { uint64_t hash; std::vector<int> toks; };
  int take_block();
  void put_block(int b);
  static uint64_t mix(uint64_t h, const int* t, int n);

  int bs_;
  bool prefix_cache_;
  std::vector<int> ref_;
  std::vector<int> free_;
  std::list<int> lru_;  // ref==0 blocks still indexed (evictable, oldest first)
  std::unordered_map<int, std::list<int>::iterator> lru_pos_;
  std::unordered_map<int64_t, Seq> seqs_;
  std::unordered_map<uint64_t, int> index_;      // chained hash -> block
  std::unordered_map<int, Cached> block_info_;   // block -> its hash and tokens
  int64_t hits_ = 0, hit_tokens_ = 0;
};

}  // namespace hk
