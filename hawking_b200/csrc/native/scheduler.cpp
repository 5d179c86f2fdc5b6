// Continuous-batching scheduler; see scheduler.h.
#include "scheduler.h"

#include <algorithm>
#include <stdexcept>

namespace hk {

Scheduler::Scheduler(BlockManager& bm, int max_batch, int max_prefill_tokens, BatchPolicy policy)
    : bm_(bm), max_batch_(max_batch), max_prefill_(max_prefill_tokens), policy_(policy) {
  if (max_batch <= 0 || max_prefill_tokens <= 0) throw std::runtime_error("scheduler: bad limits");
}

void Scheduler::add(int64_t id, const std::vector<int>& prompt, int max_new, bool greedy,
                    const std::vector<int>& stop_ids, int max_context) {
  if (reqs_.count(id)) throw std::runtime_error("scheduler: duplicate request id");
  if (prompt.empty()) throw std::runtime_error("scheduler: empty prompt");
  if ((int)prompt.size() >= max_context) throw std::runtime_error("scheduler: prompt exceeds the context window");
  Req r;
  r.id = id;
  r.tokens = prompt;
  r.prompt_len = (int)prompt.size();
  r.max_new = max_new;
  r.max_context = max_context;
  r.greedy = greedy;
  r.arrival = clock_++;
  r.stop = stop_ids;
  reqs_.emplace(id, std::move(r));
  order_.push_back(id);
}

bool Scheduler::abort(int64_t id) {
  auto it = reqs_.find(id);
  if (it == reqs_.end()) return false;
  bm_.release(id);
  reqs_.erase(it);
  order_.erase(std::remove(order_.begin(), order_.end(), id), order_.end());
  return true;
}

bool Scheduler::preempt_one(int64_t keep) {
  // Newest running request (other than `keep`) goes back to the queue for recompute.
  for (auto it = order_.rbegin(); it != order_.rend(); ++it) {
    auto& r = reqs_.at(*it);
    if (r.id == keep || r.state == ReqState::Waiting) continue;
    bm_.release(r.id);
    r.state = ReqState::Waiting;
    r.computed = 0;
    ++preemptions_;
    return true;
  }
  return false;
}

StepPlan Scheduler::schedule() {
  StepPlan plan;
  // 1) decode rows, in arrival order (GreedyFirst: greedy rows first).
  std::vector<int64_t> dec;
  for (int64_t id : order_)
    if (reqs_.at(id).state == ReqState::Decoding) dec.push_back(id);
  if (policy_ == BatchPolicy::GreedyFirst)
    std::stable_sort(dec.begin(), dec.end(), [&](int64_t a, int64_t b) { return reqs_.at(a).greedy > reqs_.at(b).greedy; });
  for (int64_t id : dec) {
    if ((int)plan.items.size() >= max_batch_) break;
    auto& r = reqs_.at(id);
    if (r.state != ReqState::Decoding) continue;  // preempted below
    while (!bm_.reserve(id, r.computed + 1)) {
      if (!preempt_one(id)) throw std::runtime_error("scheduler: KV pool too small for a single sequence");
      plan.preempted.push_back(-1);
    }
    plan.items.push_back(StepItem{id, r.computed, r.computed + 1, true, r.greedy});
  }
  // drop items whose request got preempted while later rows reserved
  plan.items.erase(std::remove_if(plan.items.begin(), plan.items.end(),
                                  [&](const StepItem& it) { return reqs_.at(it.id).state != ReqState::Decoding; }),
                   plan.items.end());
  plan.preempted.clear();
  // 2) prefill chunks under the token budget.
  int budget = max_prefill_;
  std::vector<int64_t> pre;
  for (int64_t id : order_) {
    auto st = reqs_.at(id).state;
    if (st == ReqState::Prefilling) pre.push_back(id);
  }
  std::vector<int64_t> wait;
  for (int64_t id : order_)
    if (reqs_.at(id).state == ReqState::Waiting) wait.push_back(id);
  if (policy_ == BatchPolicy::PrefixGrouped) {
    // Requests sharing their first tokens are admitted together (maximises prefix reuse).
    auto key = [&](int64_t id) {
      const auto& t = reqs_.at(id).tokens;
      uint64_t h = 1469598103934665603ull;
      for (int i = 0; i < std::min<int>(bm_.block_size(), (int)t.size()); ++i) h = (h ^ (uint32_t)t[i]) * 1099511628211ull;
      return h;
    };
    std::stable_sort(wait.begin(), wait.end(), [&](int64_t a, int64_t b) { return key(a) < key(b); });
  }
  pre.insert(pre.end(), wait.begin(), wait.end());
  for (int64_t id : pre) {
    if (budget <= 0 || (int)plan.items.size() >= max_batch_) break;
    auto& r = reqs_.at(id);
    if (r.state == ReqState::Waiting) {
      if (!bm_.has(id)) r.computed = bm_.attach_prefix(id, r.tokens);
      r.state = ReqState::Prefilling;
    }
    // After a preemption the generated tokens are recomputed along with the prompt.
    int target = (int)r.tokens.size();
    int chunk = std::min(budget, target - r.computed);
    if (chunk <= 0) continue;
    if (!bm_.reserve(id, r.computed + chunk)) {
      // Shrink the chunk to what the free blocks can hold.
      const int cur_blocks = bm_.has(id) ? (int)bm_.table(id).size() : 0;
      const int cap = (cur_blocks + bm_.num_free()) * bm_.block_size() - r.computed;
      chunk = std::min(chunk, cap);
      if (chunk <= 0 || !bm_.reserve(id, r.computed + chunk)) break;
    }
    bool done = r.computed + chunk == target;
    plan.items.push_back(StepItem{id, r.computed, r.computed + chunk, done, r.greedy});
    budget -= chunk;
  }
  return plan;
}

void Scheduler::finish(Req& r) {
  bm_.commit_prefix(r.id, r.tokens, r.computed);
  bm_.release(r.id);
  r.state = ReqState::Finished;
}

std::vector<StepEvent> Scheduler::commit(const StepPlan& plan, const std::vector<int>& sampled) {
  std::vector<StepEvent> ev;
  size_t si = 0;
  for (const auto& it : plan.items) {
    auto rit = reqs_.find(it.id);
    if (rit == reqs_.end()) {  // aborted during the step
      if (it.sample) ++si;
      continue;
    }
    auto& r = rit->second;
    r.computed = std::max(r.computed, it.p1);
    if (r.state == ReqState::Prefilling && r.computed >= r.prompt_len) {
      bm_.commit_prefix(r.id, r.tokens, r.prompt_len);
    }
    if (!it.sample) {
      ev.push_back(StepEvent{it.id, -1, 0});
      continue;
    }
    if (si >= sampled.size()) throw std::runtime_error("scheduler commit: missing sampled tokens");
    int tok = sampled[si++];
    r.tokens.push_back(tok);
    r.generated += 1;
    r.state = ReqState::Decoding;
    int fin = 0;
    if (std::find(r.stop.begin(), r.stop.end(), tok) != r.stop.end()) fin = (int)FinishReason::Stop;
    else if (r.generated >= r.max_new || (int)r.tokens.size() >= r.max_context) fin = (int)FinishReason::Length;
    ev.push_back(StepEvent{it.id, tok, fin});
    if (fin) finish(r);
  }
  // Retire finished requests.
  for (auto it = order_.begin(); it != order_.end();) {
    auto r = reqs_.find(*it);
    if (r != reqs_.end() && r->second.state == ReqState::Finished) {
      reqs_.erase(r);
      it = order_.erase(it);
    } else {
      ++it;
    }
  }
  return ev;
}

std::vector<StepEvent> Scheduler::commit_run(int64_t id, const std::vector<int>& toks, int computed) {
  std::vector<StepEvent> ev;
  auto rit = reqs_.find(id);
  if (rit == reqs_.end()) return ev;
  auto& r = rit->second;
  if (r.state != ReqState::Decoding) throw std::runtime_error("scheduler commit_run: request is not decoding");
  r.computed = std::max(r.computed, computed);
  for (int tok : toks) {
    r.tokens.push_back(tok);
    r.generated += 1;
    int fin = 0;
    if (std::find(r.stop.begin(), r.stop.end(), tok) != r.stop.end()) fin = (int)FinishReason::Stop;
    else if (r.generated >= r.max_new || (int)r.tokens.size() >= r.max_context) fin = (int)FinishReason::Length;
    ev.push_back(StepEvent{id, tok, fin});
    if (fin) {
      finish(r);
      break;
    }
  }
  if (r.state == ReqState::Finished) {
    reqs_.erase(rit);
    order_.erase(std::remove(order_.begin(), order_.end(), id), order_.end());
  }
  return ev;
}

int Scheduler::num_waiting() const {
  int n = 0;
  for (const auto& kv : reqs_) n += kv.second.state == ReqState::Waiting;
  return n;
}
int Scheduler::num_running() const {
  int n = 0;
  for (const auto& kv : reqs_) n += kv.second.state == ReqState::Prefilling || kv.second.state == ReqState::Decoding;
  return n;
}
const std::vector<int>& Scheduler::tokens(int64_t id) const { return reqs_.at(id).tokens; }
int Scheduler::prompt_len(int64_t id) const { return reqs_.at(id).prompt_len; }
int Scheduler::state(int64_t id) const {
  auto it = reqs_.find(id);
  return it == reqs_.end() ? (int)ReqState::Finished : (int)it->second.state;
}

}  // namespace hk
