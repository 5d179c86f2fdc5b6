// Bindings for the engine host logic (paged-KV block manager, scheduler, n-gram drafter).
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "../native/block_manager.h"
#include "../native/scheduler.h"
#include "../native/spec.h"

namespace py = pybind11;
using namespace hk;

void bind_engine(py::module_& m) {
  py::class_<BlockManager>(m, "BlockManager")
      .def(py::init<int, int, bool>(), py::arg("num_blocks"), py::arg("block_size"), py::arg("prefix_cache") = true)
      .def_property_readonly("block_size", &BlockManager::block_size)
      .def_property_readonly("num_blocks", &BlockManager::num_blocks)
      .def_property_readonly("num_free", &BlockManager::num_free)
      .def("has", &BlockManager::has)
      .def("num_tokens", &BlockManager::num_tokens)
      .def("reserve", &BlockManager::reserve)
      .def("blocks_needed", &BlockManager::blocks_needed)
      .def("release", &BlockManager::release)
      .def("table", &BlockManager::table)
      .def("slots", &BlockManager::slots)
      .def("attach_prefix", &BlockManager::attach_prefix)
      .def("cached_prefix", &BlockManager::cached_prefix)
      .def("commit_prefix", &BlockManager::commit_prefix)
      .def("fork", &BlockManager::fork)
      .def("truncate", &BlockManager::truncate)
      .def_property_readonly("prefix_hits", &BlockManager::prefix_hits)
      .def_property_readonly("prefix_hit_tokens", &BlockManager::prefix_hit_tokens);

  py::class_<StepItem>(m, "StepItem")
      .def_readonly("id", &StepItem::id)
      .def_readonly("p0", &StepItem::p0)
      .def_readonly("p1", &StepItem::p1)
      .def_readonly("sample", &StepItem::sample)
      .def_readonly("greedy", &StepItem::greedy)
      .def("__repr__", [](const StepItem& i) {
        return "StepItem(id=" + std::to_string(i.id) + ", p0=" + std::to_string(i.p0) + ", p1=" + std::to_string(i.p1) +
               ", sample=" + (i.sample ? "True" : "False") + ")";
      });
  py::class_<StepPlan>(m, "StepPlan")
      .def_readonly("items", &StepPlan::items)
      .def_property_readonly("rows", &StepPlan::rows);
  py::class_<StepEvent>(m, "StepEvent")
      .def_readonly("id", &StepEvent::id)
      .def_readonly("token", &StepEvent::token)
      .def_readonly("finish", &StepEvent::finish);

  py::class_<Scheduler>(m, "Scheduler")
      .def(py::init([](BlockManager& bm, int max_batch, int max_prefill, int policy) {
             return new Scheduler(bm, max_batch, max_prefill, (BatchPolicy)policy);
           }),
           py::arg("block_manager"), py::arg("max_batch"), py::arg("max_prefill_tokens"), py::arg("policy") = 0,
           py::keep_alive<1, 2>())
      .def("add", &Scheduler::add, py::arg("id"), py::arg("prompt"), py::arg("max_new"), py::arg("greedy"),
           py::arg("stop_ids"), py::arg("max_context"))
      .def("abort", &Scheduler::abort)
      .def("schedule", &Scheduler::schedule)
      .def("commit", &Scheduler::commit)
      .def("commit_run", &Scheduler::commit_run, py::arg("id"), py::arg("toks"), py::arg("computed"))
      .def_property_readonly("num_waiting", &Scheduler::num_waiting)
      .def_property_readonly("num_running", &Scheduler::num_running)
      .def("idle", &Scheduler::idle)
      .def("tokens", &Scheduler::tokens)
      .def("prompt_len", &Scheduler::prompt_len)
      .def("state", &Scheduler::state)
      .def_property_readonly("total_preemptions", &Scheduler::total_preemptions);

  py::class_<NgramDraft>(m, "NgramDraft")
      .def(py::init<>())
      .def("note_token", &NgramDraft::note_token)
      .def("warm_start", &NgramDraft::warm_start)
      .def("reset_context", &NgramDraft::reset_context)
      .def("propose", &NgramDraft::propose, py::arg("ctx"), py::arg("k"))
      .def_property_readonly("transitions", &NgramDraft::transitions);
  m.def("accept_draft", [](const std::vector<int32_t>& draft, const std::vector<int32_t>& verifier) {
    int a = 0;
    auto out = accept_draft(draft, verifier, &a);
    return py::make_tuple(out, a);
  });
  m.attr("MAX_VERIFY_BATCH") = kMaxVerifyBatch;
  py::class_<SpecGovernor>(m, "SpecGovernor")
      .def(py::init<int, float, int, int>(), py::arg("window") = 16, py::arg("min_accept_rate") = 0.2f,
           py::arg("max_consecutive_rejections") = 5, py::arg("cooldown") = -1)
      .def("step", &SpecGovernor::step)
      .def("tick_disabled", &SpecGovernor::tick_disabled)
      .def_property_readonly("enabled", &SpecGovernor::enabled)
      .def_property_readonly("accept_rate", &SpecGovernor::accept_rate);
}
