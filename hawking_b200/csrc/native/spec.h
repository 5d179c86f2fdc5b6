// Speculative decoding host logic: the online n-gram draft, the exact-verify acceptance rule and
// the acceptance governor. The model verifies every draft, so output is identical to greedy.
//
//   NgramDraft   (prev, cur) -> successor counts with a cur -> successor backoff, grown from the
//                emitted stream; propose() chains the most frequent successor (smallest id on a
//                count tie), stops at the first context with no successor, and stops a run of the
//                same token at 3 repeats.
//   accept_draft longest prefix of the draft that equals the verifier's argmax at each position,
//                plus the verifier's token after it (the correction, or the bonus token when the
//                whole draft is accepted).
//   SpecGovernor rolling accept rate over a window with hysteresis: disable after N consecutive
//                zero-accept cycles or when the full-window rate <= disable_below; re-enable only
//                after a cooldown of recorded cycles and a rate >= enable_above.
//
// Parity: crates/hawking-speculate/src/user_ngram.rs:1-60, :96 (note_token), :154 (propose),
// crates/hawking-speculate/src/shared.rs:66 (verify_draft_ids_until_mismatch),
// crates/hawking-speculate/src/governor.rs:1-233, crates/hawking-speculate/src/router.rs
// (MAX_VERIFY_BATCH = 8).
#pragma once
#include <cstdint>
#include <deque>
#include <unordered_map>
#include <vector>

namespace hk {

constexpr int kMaxVerifyBatch = 8;

class NgramDraft {
 public:
  void note_token(int32_t t);
  void warm_start(const std::vector<int32_t>& history);
  void reset_context() { has_prev_ = has_cur_ = false; }
  std::vector<int32_t> propose(const std::vector<int32_t>& ctx, int k) const;
  uint64_t transitions() const { return transitions_; }

 private:
  bool best(bool has_prev, int32_t prev, int32_t cur, int32_t* out) const;
  static uint64_t key(int32_t a, int32_t b) { return ((uint64_t)(uint32_t)a << 32) | (uint32_t)b; }
  std::unordered_map<uint64_t, std::unordered_map<int32_t, uint32_t>> bigram_;
  std::unordered_map<int32_t, std::unordered_map<int32_t, uint32_t>> unigram_;
  bool has_prev_ = false, has_cur_ = false;
  int32_t prev_ = 0, cur_ = 0;
  uint64_t transitions_ = 0;
};

// verifier[i] = argmax after consuming draft[0..i) (verifier has draft.size() + 1 entries).
// Returns the tokens to emit: draft[0..a) + verifier[a], a = accepted count.
std::vector<int32_t> accept_draft(const std::vector<int32_t>& draft, const std::vector<int32_t>& verifier, int* accepted);

class SpecGovernor {
 public:
  explicit SpecGovernor(int window = 16, float min_accept_rate = 0.2f, int max_consecutive_rejections = 5,
                        int cooldown = -1);
  bool step(bool accepted);  // record one cycle; returns whether spec stays enabled
  bool tick_disabled();      // a cycle with spec off (cooldown dwell only)
  bool enabled() const { return cooldown_left_ < 0; }
  float accept_rate() const { return hist_.empty() ? 0.f : (float)n_true_ / (float)hist_.size(); }

 private:
  int window_, max_rej_, cooldown_;
  float enable_above_, disable_below_;
  std::deque<bool> hist_;
  int n_true_ = 0, consec_rej_ = 0;
  int cooldown_left_ = -1;  // -1: enabled
};

}  // namespace hk
