// Speculative decoding host logic; see spec.h.
#include "spec.h"

#include <algorithm>

namespace hk {

void NgramDraft::note_token(int32_t t) {
  if (has_cur_) {
    unigram_[cur_][t]++;
    if (has_prev_) bigram_[key(prev_, cur_)][t]++;
    transitions_++;
  }
  prev_ = cur_;
  has_prev_ = has_cur_;
  cur_ = t;
  has_cur_ = true;
}

void NgramDraft::warm_start(const std::vector<int32_t>& history) {
  for (int32_t t : history) note_token(t);
  reset_context();
}

static bool most_frequent(const std::unordered_map<int32_t, uint32_t>& m, int32_t* out) {
  bool found = false;
  uint32_t bc = 0;
  int32_t bt = 0;
  for (const auto& kv : m) {
    if (!found || kv.second > bc || (kv.second == bc && kv.first < bt)) {
      bc = kv.second;
      bt = kv.first;
      found = true;
    }
  }
  if (found) *out = bt;
  return found;
}

bool NgramDraft::best(bool has_prev, int32_t prev, int32_t cur, int32_t* out) const {
  if (has_prev) {
    auto it = bigram_.find(key(prev, cur));
    if (it != bigram_.end() && most_frequent(it->second, out)) return true;
  }
  auto jt = unigram_.find(cur);
  return jt != unigram_.end() && most_frequent(jt->second, out);
}

std::vector<int32_t> NgramDraft::propose(const std::vector<int32_t>& ctx, int k) const {
  std::vector<int32_t> out;
  if (k <= 0 || ctx.empty()) return out;
  bool has_prev = ctx.size() >= 2;
  int32_t prev = has_prev ? ctx[ctx.size() - 2] : 0, cur = ctx.back();
  int run = 0;
  for (int i = 0; i < k; ++i) {
    int32_t next;
    if (!best(has_prev, prev, cur, &next)) break;
    if (!out.empty() && out.back() == next) {
      if (++run >= 3) break;
    } else {
      run = 0;
    }
    out.push_back(next);
    prev = cur;
    has_prev = true;
    cur = next;
  }
  return out;
}

std::vector<int32_t> accept_draft(const std::vector<int32_t>& draft, const std::vector<int32_t>& verifier,
                                  int* accepted) {
  size_t a = 0;
  while (a < draft.size() && a < verifier.size() && draft[a] == verifier[a]) ++a;
  std::vector<int32_t> out(draft.begin(), draft.begin() + a);
  if (a < verifier.size()) out.push_back(verifier[a]);
  if (accepted) *accepted = (int)a;
  return out;
}

SpecGovernor::SpecGovernor(int window, float min_accept_rate, int max_consecutive_rejections, int cooldown)
    : window_(std::max(1, window)),
      max_rej_(std::max(1, max_consecutive_rejections)),
      cooldown_(cooldown < 0 ? std::max(1, window) : cooldown) {
  disable_below_ = std::min(1.f, std::max(0.f, min_accept_rate));
  enable_above_ = std::max(disable_below_, std::min(1.f, min_accept_rate + 0.10f));
}

bool SpecGovernor::step(bool accepted) {
  if ((int)hist_.size() >= window_) {
    if (hist_.front()) n_true_--;
    hist_.pop_front();
  }
  hist_.push_back(accepted);
  if (accepted) {
    n_true_++;
    consec_rej_ = 0;
  } else {
    consec_rej_++;
  }
  if (enabled()) {
    const bool full = (int)hist_.size() >= window_;
    if (consec_rej_ >= max_rej_ || (full && accept_rate() <= disable_below_)) cooldown_left_ = cooldown_;
  } else {
    cooldown_left_ = std::max(0, cooldown_left_ - 1);
    if (cooldown_left_ == 0 && accept_rate() >= enable_above_) {
      cooldown_left_ = -1;
      consec_rej_ = 0;
    }
  }
  return enabled();
}

bool SpecGovernor::tick_disabled() {
  if (!enabled()) cooldown_left_ = std::max(0, cooldown_left_ - 1);
  return enabled();
}

}  // namespace hk
