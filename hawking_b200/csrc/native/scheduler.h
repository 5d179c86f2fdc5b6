// Continuous-batching scheduler over the paged KV block manager.
//
// Each step carries every decoding sequence (one token each) plus prefill chunks that fit a
// token budget (chunked prefill), so long prompts never stall running decodes. When the KV pool
// runs dry the newest running request is preempted (its blocks are released and it is requeued
// for recompute). Prompts are matched against the block manager's prefix index when they are
// first admitted, so a shared system prompt is prefilled once.
//
// Parity: crates/hawking-serve/src/batch/scheduler.rs:258 (Scheduler), :18-32 (BatchPolicy
// Default / GreedyFirst / PrefixGrouped), :504 (prefill_chunks_token_budgeted), :546
// (commit_prefill_chunk), :634 (apply_decode_tokens); slot states Idle/Prefilling/Decoding/
// Finishing (crates/hawking-serve/src/batch/mod.rs:14-19).
#pragma once
#include <cstdint>
#include <deque>
#include <map>
#include <string>
#include <vector>

#include "block_manager.h"

namespace hk {

enum class ReqState : int { Waiting = 0, Prefilling = 1, Decoding = 2, Finished = 3 };
enum class BatchPolicy : int { Default = 0, GreedyFirst = 1, PrefixGrouped = 2 };
enum class FinishReason : int { None = 0, Length = 1, Stop = 2, Aborted = 3 };

struct StepItem {
  int64_t id;
  int p0, p1;        // compute KV for tokens[p0:p1)
  bool sample;       // sample the next token from the row at p1-1
  bool greedy;
};

struct StepPlan {
  std::vector<StepItem> items;
  std::vector<int64_t> preempted;
  int rows() const {
    int r = 0;
    for (const auto& i : items) r += i.p1 - i.p0;
    return r;
  }
};

struct StepEvent {
  int64_t id;
  int token;          // -1 when the item did not sample
  int finish;         // FinishReason
};

class Scheduler {
 public:
  Scheduler(BlockManager& bm, int max_batch, int max_prefill_tokens, BatchPolicy policy = BatchPolicy::Default);

  void add(int64_t id, const std::vector<int>& prompt, int max_new, bool greedy, const std::vector<int>& stop_ids,
           int max_context);
  bool abort(int64_t id);
  StepPlan schedule();
  std::vector<StepEvent> commit(const StepPlan& plan, const std::vector<int>& sampled);
  // Speculative decoding: the decoding request `id` emitted `toks` (accepted drafts plus the
  // verifier's token) and its KV now covers `computed` tokens. Stop ids and length end the run
  // early; one event per emitted token.
  std::vector<StepEvent> commit_run(int64_t id, const std::vector<int>& toks, int computed);

  int num_waiting() const;
  int num_running() const;
  bool idle() const { return reqs_.empty(); }
  const std::vector<int>& tokens(int64_t id) const;
  int prompt_len(int64_t id) const;
  int state(int64_t id) const;
  int64_t total_preemptions() const { return preemptions_; }

 private:
  struct Req {
    int64_t id;
    std::vector<int> tokens;
    int prompt_len;
    int max_new;
    int max_context;
    int computed = 0;
    int generated = 0;
    bool greedy;
    ReqState state = ReqState::Waiting;
    int64_t arrival;
    std::vector<int> stop;
  };
  bool preempt_one(int64_t keep);
  void finish(Req& r);

  BlockManager& bm_;
  int max_batch_, max_prefill_;
  BatchPolicy policy_;
  std::map<int64_t, Req> reqs_;
  std::deque<int64_t> order_;  // arrival order
  int64_t clock_ = 0, preemptions_ = 0;
};

}  // namespace hk
