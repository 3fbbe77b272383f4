// Python bindings of the C++ serving runtime (module _sp_core).
//
// Errors raised by the runtime (spc::StatusError) surface in Python as
// sparkpipe_rs_b200.core.StatusError subclasses of RuntimeError carrying the
// numeric status code in `.code` and its name in `.status`.
#include <torch/extension.h>

#include <cstring>

#include "memory.h"
#include "prefix_cache.h"
#include "registry.h"
#include "scheduler.h"

namespace py = pybind11;
using namespace spc;

namespace {

template <typename T>
py::array_t<T> to_np(const std::vector<T>& v) {
  py::array_t<T> a(v.size());
  if (!v.empty()) std::memcpy(a.mutable_data(), v.data(), v.size() * sizeof(T));
  return a;
}

void copy_into(const torch::Tensor& dst, const void* src, size_t bytes) {
  TORCH_CHECK(dst.is_contiguous() && !dst.is_cuda(), "destination must be a contiguous CPU tensor");
  TORCH_CHECK(size_t(dst.numel()) * dst.element_size() >= bytes, "destination tensor too small");
  if (bytes) std::memcpy(dst.data_ptr(), src, bytes);
}

}  // namespace

void bind_memory(py::module_& m) {
  py::class_<KvArenaConfig>(m, "KvArenaConfig")
      .def(py::init<>())
      .def_readwrite("physical_block_count", &KvArenaConfig::physical_block_count)
      .def_readwrite("block_token_count", &KvArenaConfig::block_token_count)
      .def_readwrite("resident_block_capacity", &KvArenaConfig::resident_block_capacity)
      .def_readwrite("layer_count", &KvArenaConfig::layer_count)
      .def_readwrite("kv_head_count", &KvArenaConfig::kv_head_count)
      .def_readwrite("head_dim", &KvArenaConfig::head_dim)
      .def_readwrite("bytes_per_scalar", &KvArenaConfig::bytes_per_scalar)
      .def_readwrite("key_block_stride_bytes", &KvArenaConfig::key_block_stride_bytes)
      .def_readwrite("value_block_stride_bytes", &KvArenaConfig::value_block_stride_bytes)
      .def_readwrite("key_device_base", &KvArenaConfig::key_device_base)
      .def_readwrite("value_device_base", &KvArenaConfig::value_device_base);
  py::class_<KvBlockView>(m, "KvBlockView")
      .def_readonly("physical_block_index", &KvBlockView::physical_block_index)
      .def_readonly("token_capacity", &KvBlockView::token_capacity)
      .def_readonly("generation", &KvBlockView::generation)
      .def_readonly("key_device_address", &KvBlockView::key_device_address)
      .def_readonly("value_device_address", &KvBlockView::value_device_address)
      .def_readonly("key_block_stride_bytes", &KvBlockView::key_block_stride_bytes)
      .def_readonly("value_block_stride_bytes", &KvBlockView::value_block_stride_bytes);
  py::class_<KvArena>(m, "KvArena")
      .def(py::init<const KvArenaConfig&>())
      .def("acquire_block", &KvArena::acquire_block)
      .def("recycle_block", &KvArena::recycle_block)
      .def("retain_block", &KvArena::retain_block)
      .def("release_block_reference", &KvArena::release_block_reference)
      .def("mark_block_resident", &KvArena::mark_block_resident)
      .def("mark_block_nonresident", &KvArena::mark_block_nonresident)
      .def("free_block", &KvArena::free_block)
      .def("resolve_block", &KvArena::resolve_block)
      .def("trim_resident_blocks", &KvArena::trim_resident_blocks)
      .def("evict_resident_blocks_to_limit", &KvArena::evict_resident_blocks_to_limit)
      .def("reset", &KvArena::reset)
      .def("is_allocated", &KvArena::is_allocated)
      .def("is_resident", &KvArena::is_resident)
      .def("reference_count", &KvArena::reference_count)
      .def("generation", &KvArena::generation)
      .def("last_used_epoch", &KvArena::last_used_epoch)
      .def("key_device_address", &KvArena::key_device_address)
      .def("value_device_address", &KvArena::value_device_address)
      .def("block_token_capacity", &KvArena::block_token_capacity)
      .def_property_readonly("block_token_count", &KvArena::block_token_count)
      .def_property_readonly("physical_block_count", &KvArena::physical_block_count)
      .def_property_readonly("free_block_count", &KvArena::free_block_count)
      .def_property_readonly("epoch", &KvArena::epoch)
      .def_property_readonly("allocated_block_count", &KvArena::allocated_block_count)
      .def_property_readonly("recycled_block_count", &KvArena::recycled_block_count)
      .def_property_readonly("resident_block_count", &KvArena::resident_block_count)
      .def_property_readonly("resident_evicted_block_count", &KvArena::resident_evicted_block_count)
      .def_property_readonly("resident_capacity_stall_count", &KvArena::resident_capacity_stall_count)
      .def_property_readonly("retained_block_count", &KvArena::retained_block_count)
      .def_property_readonly("released_reference_count", &KvArena::released_reference_count)
      .def_property_readonly("key_block_stride_bytes", &KvArena::key_block_stride_bytes)
      .def_property_readonly("value_block_stride_bytes", &KvArena::value_block_stride_bytes);

  py::class_<ArenaHandle>(m, "ArenaHandle")
      .def_readonly("class_index", &ArenaHandle::class_index)
      .def_readonly("slot_index", &ArenaHandle::slot_index)
      .def_readonly("generation", &ArenaHandle::generation)
      .def("__eq__", [](const ArenaHandle& a, const ArenaHandle& b) {
        return a.class_index == b.class_index && a.slot_index == b.slot_index && a.generation == b.generation;
      });
  py::class_<Arena>(m, "Arena")
      .def(py::init([](const std::vector<std::pair<uint32_t, uint32_t>>& cls) {
        std::vector<ArenaClass> c;
        for (auto& p : cls) c.push_back(ArenaClass{p.first, p.second});
        return new Arena(c);
      }))
      .def("acquire", &Arena::acquire)
      .def("release", &Arena::release)
      .def("write", [](Arena& a, const ArenaHandle& h, py::bytes data) {
        uint8_t* p = a.get(h);
        if (!p) fail(Status::NotFound, "Arena: stale handle");
        std::string s = data;
        if (s.size() > a.class_slot_bytes(h.class_index)) fail(Status::InvalidArgument, "Arena: write too large");
        std::memcpy(p, s.data(), s.size());
      })
      .def("read", [](Arena& a, const ArenaHandle& h, uint32_t n) {
        uint8_t* p = a.get(h);
        if (!p) fail(Status::NotFound, "Arena: stale handle");
        return py::bytes(reinterpret_cast<const char*>(p), std::min(n, a.class_slot_bytes(h.class_index)));
      })
      .def("is_live", [](Arena& a, const ArenaHandle& h) { return a.get(h) != nullptr; })
      .def_property_readonly("reserved_bytes", &Arena::reserved_bytes)
      .def("class_free_count", &Arena::class_free_count)
      .def("class_generation", &Arena::class_generation)
      .def("class_slot_bytes", &Arena::class_slot_bytes);

  py::class_<StatePool>(m, "StatePool")
      .def(py::init<uint32_t, uint64_t>())
      .def("acquire", &StatePool::acquire)
      .def("release", &StatePool::release)
      .def("in_use", &StatePool::in_use)
      .def_property_readonly("free_count", &StatePool::free_count)
      .def_property_readonly("slot_count", &StatePool::slot_count)
      .def_property_readonly("slot_bytes", &StatePool::slot_bytes);

  py::enum_<SeqState>(m, "SeqState")
      .value("FREE", SeqState::Free)
      .value("ACTIVE", SeqState::Active)
      .value("AWAITING_TOOL", SeqState::AwaitingTool)
      .value("COMPLETE", SeqState::Complete);
  py::class_<BatchSequence>(m, "BatchSequence")
      .def_readonly("sequence_id", &BatchSequence::sequence_id)
      .def_readonly("state", &BatchSequence::state)
      .def_readonly("lane_count", &BatchSequence::lane_count)
      .def_readonly("exchange_number", &BatchSequence::exchange_number)
      .def_readonly("context_tokens", &BatchSequence::context_tokens)
      .def_readonly("fragment_base", &BatchSequence::fragment_base)
      .def_readonly("fragment_count", &BatchSequence::fragment_count);
  py::class_<BatchSequenceTable>(m, "BatchSequenceTable")
      .def(py::init<uint32_t, uint32_t>())
      .def("admit", &BatchSequenceTable::admit)
      .def("begin_exchange", &BatchSequenceTable::begin_exchange)
      .def("pause_for_tool", &BatchSequenceTable::pause_for_tool)
      .def("complete", &BatchSequenceTable::complete)
      .def("sequence", &BatchSequenceTable::sequence, py::return_value_policy::copy)
      .def("firing_threshold", &BatchSequenceTable::firing_threshold)
      .def_property_readonly("active_count", &BatchSequenceTable::active_count)
      .def_property_readonly("awaiting_tool_count", &BatchSequenceTable::awaiting_tool_count)
      .def_property_readonly("complete_count", &BatchSequenceTable::complete_count)
      .def_property_readonly("exchange_count", &BatchSequenceTable::exchange_count)
      .def_property_readonly("capacity", &BatchSequenceTable::capacity);

  m.def("row_allocator_assign",
        [](const std::vector<std::tuple<uint32_t, uint32_t, uint32_t>>& slots, uint32_t cap, uint32_t cost) {
          std::vector<RowSlot> s;
          for (auto& t : slots) s.push_back(RowSlot{std::get<0>(t), std::get<1>(t), std::get<2>(t)});
          std::vector<uint32_t> budgets;
          const uint32_t total = row_allocator_assign(s, cap, cost, budgets);
          return py::make_tuple(total, budgets);
        });
}

void bind_prefix(py::module_& m) {
  m.attr("EMPTY_PARENT_HASH") = kEmptyParentHash;
  m.def("prefix_hash_block", [](const std::vector<uint32_t>& t, uint64_t parent) {
    return prefix_hash_block(t.data(), (uint32_t)t.size(), parent);
  });
  py::class_<PromptHash>(m, "PromptHash")
      .def_readonly("token_count", &PromptHash::token_count)
      .def_readonly("hashed_token_count", &PromptHash::hashed_token_count)
      .def_readonly("block_count", &PromptHash::block_count)
      .def_readonly("last_block_token_count", &PromptHash::last_block_token_count)
      .def_readonly("parent_hash", &PromptHash::parent_hash)
      .def_readonly("prompt_hash", &PromptHash::prompt_hash);
  m.def("prefix_hash_prompt", [](uint32_t bt, uint64_t parent, const std::vector<uint32_t>& t) {
    return prefix_hash_prompt(bt, parent, t.data(), (uint32_t)t.size());
  });
  py::class_<PrefixLookup>(m, "PrefixLookup")
      .def_readonly("requested_token_count", &PrefixLookup::requested_token_count)
      .def_readonly("matched_token_count", &PrefixLookup::matched_token_count)
      .def_readonly("matched_block_count", &PrefixLookup::matched_block_count)
      .def_readonly("host_block_count", &PrefixLookup::host_block_count)
      .def_readonly("next_token_index", &PrefixLookup::next_token_index)
      .def_readonly("last_block_hash", &PrefixLookup::last_block_hash);
  py::class_<PrefixReservation>(m, "PrefixReservation")
      .def_readonly("sequence_id", &PrefixReservation::sequence_id)
      .def_readonly("requested_token_count", &PrefixReservation::requested_token_count)
      .def_readonly("reusable_token_count", &PrefixReservation::reusable_token_count)
      .def_readonly("reserved_token_count", &PrefixReservation::reserved_token_count)
      .def_readonly("physical_blocks", &PrefixReservation::physical_blocks);
  py::class_<PrefixCacheStats>(m, "PrefixCacheStats")
      .def_readonly("lookups", &PrefixCacheStats::lookups)
      .def_readonly("hits", &PrefixCacheStats::hits)
      .def_readonly("hit_tokens", &PrefixCacheStats::hit_tokens)
      .def_readonly("missed_tokens", &PrefixCacheStats::missed_tokens)
      .def_readonly("committed_blocks", &PrefixCacheStats::committed_blocks)
      .def_readonly("evicted_blocks", &PrefixCacheStats::evicted_blocks)
      .def_readonly("reservations", &PrefixCacheStats::reservations)
      .def_readonly("cancellations", &PrefixCacheStats::cancellations)
      .def_readonly("released_sequences", &PrefixCacheStats::released_sequences)
      .def_readonly("lookahead_protections", &PrefixCacheStats::lookahead_protections)
      .def_readonly("protected_evictions", &PrefixCacheStats::protected_evictions)
      .def_readonly("trimmed_blocks", &PrefixCacheStats::trimmed_blocks)
      .def_readonly("demoted_blocks", &PrefixCacheStats::demoted_blocks)
      .def_readonly("promoted_blocks", &PrefixCacheStats::promoted_blocks)
      .def_readonly("host_dropped_blocks", &PrefixCacheStats::host_dropped_blocks);
  py::class_<PrefixCache>(m, "PrefixCache")
      .def(py::init<uint32_t, uint32_t, uint32_t>(), py::arg("block_tokens"), py::arg("physical_blocks"),
           py::arg("max_sequences"))
      .def("probe_prompt", [](const PrefixCache& c, const std::vector<uint32_t>& t) {
        return c.probe_prompt(t.data(), (uint32_t)t.size());
      })
      .def("reserve_prompt", [](PrefixCache& c, uint64_t id, const std::vector<uint32_t>& t) {
        return c.reserve_prompt(id, t.data(), (uint32_t)t.size());
      })
      .def("commit", &PrefixCache::commit)
      .def("cancel_reservation", &PrefixCache::cancel_reservation)
      .def("append_tokens", [](PrefixCache& c, uint64_t id, const std::vector<uint32_t>& t) {
        c.append_tokens(id, t.data(), (uint32_t)t.size());
      })
      .def("ensure_sequence_token_capacity", &PrefixCache::ensure_sequence_token_capacity)
      .def("can_allocate", &PrefixCache::can_allocate)
      .def("block_table", &PrefixCache::block_table)
      .def("sequence_token_count", &PrefixCache::sequence_token_count)
      .def("has_sequence", &PrefixCache::has_sequence)
      .def("release_sequence", &PrefixCache::release_sequence)
      .def("evict_to_free", &PrefixCache::evict_to_free)
      .def("reset_lookahead_protection", &PrefixCache::reset_lookahead_protection)
      .def("protect_prompt_lookahead", [](PrefixCache& c, const std::vector<uint32_t>& t, uint32_t weight) {
        return c.protect_prompt_lookahead(t.data(), (uint32_t)t.size(), weight);
      })
      .def_property_readonly("protected_warm_blocks", &PrefixCache::protected_warm_blocks)
      .def("trim_warm_blocks", &PrefixCache::trim_warm_blocks)
      .def("enable_host_tier", &PrefixCache::enable_host_tier)
      .def("take_tier_copies", [](PrefixCache& c) {
        std::vector<int32_t> o, i;
        c.take_tier_copies(o, i);
        return py::make_tuple(o, i);
      })
      .def("release_deferred_slots", &PrefixCache::release_deferred_slots)
      .def_property_readonly("host_entries", &PrefixCache::host_entries)
      .def("bind_committed_prefix_from_sequence", &PrefixCache::bind_committed_prefix_from_sequence)
      .def("reset", &PrefixCache::reset)
      .def("reference_count", [](const PrefixCache& c, uint32_t b) { return c.arena().reference_count(b); })
      .def_property_readonly("block_tokens", &PrefixCache::block_tokens)
      .def_property_readonly("free_blocks", &PrefixCache::free_blocks)
      .def_property_readonly("warm_blocks", &PrefixCache::warm_blocks)
      .def_property_readonly("entry_count", &PrefixCache::entry_count)
      .def_property_readonly("sequence_count", &PrefixCache::sequence_count)
      .def_property_readonly("stats", &PrefixCache::stats);
}

void bind_speculation(py::module_& m) {
  auto s = m.def_submodule("speculation", "speculative-decode policy: lane EMA, row allocator, utility");
  s.attr("EMA_INITIAL_MILLI") = spec::kEmaInitialMilli;
  s.attr("SUPPRESS_MILLI") = spec::kSuppressMilli;
  s.attr("REPROBE_INTERVAL") = spec::kReprobeInterval;
  s.attr("MAX_SPECULATIVE_TOKENS") = spec::kMaxSpeculativeTokens;
  s.def("alpha_milli", &spec::alpha_milli);
  s.def("row_allocator_assign",
        [](const std::vector<std::tuple<uint32_t, uint32_t, uint32_t>>& lanes, uint32_t cap, uint32_t cost) {
          std::vector<spec::SlotInput> in;
          for (const auto& t : lanes) in.push_back(spec::SlotInput{std::get<0>(t), std::get<1>(t), std::get<2>(t)});
          std::vector<uint32_t> out(in.size(), 0);
          const uint32_t total = spec::row_allocator_assign(in, cap, cost, out);
          return py::make_tuple(total, out);
        },
        py::arg("lanes"), py::arg("firing_row_cap"), py::arg("spec_row_relative_cost_milli") = 1000);
  s.def("observe",
        [](uint32_t ema, uint32_t budget, uint32_t countdown, const std::vector<std::pair<char, uint32_t>>& events,
           uint32_t full) {
          // replays ('v', committed) verify rounds and ('p', committed) plain steps on one lane
          spec::LaneState l;
          l.ema_milli = ema;
          l.budget = budget;
          l.countdown = countdown;
          py::list out;
          for (const auto& e : events) {
            if (e.first == 'v') spec::observe_verify(l, e.second, full);
            else spec::observe_plain(l, e.second, full);
            out.append(py::make_tuple(l.ema_milli, l.budget, l.countdown));
          }
          return out;
        });
  s.def("outranks_plain", &spec::outranks_plain);
}

void bind_scheduler(py::module_& m) {
  bind_speculation(m);
  py::enum_<SlotState>(m, "SlotState")
      .value("FREE", SlotState::Free)
      .value("QUEUED_PREFILL", SlotState::QueuedPrefill)
      .value("RUNNING_PREFILL", SlotState::RunningPrefill)
      .value("READY_DECODE", SlotState::ReadyDecode)
      .value("RUNNING_DECODE", SlotState::RunningDecode)
      .value("COMPLETED", SlotState::Completed)
      .value("CANCELLED", SlotState::Cancelled)
      .value("WAITING_PREFIX_COHORT", SlotState::WaitingPrefixCohort)
      .value("READY_SPECULATIVE_VERIFY", SlotState::ReadySpeculativeVerify)
      .value("RUNNING_SPECULATIVE_VERIFY", SlotState::RunningSpeculativeVerify)
      .value("SWAPPED", SlotState::Swapped);
  m.attr("SCHED_CHUNKED_PREFILL") = kSchedChunkedPrefill;
  m.attr("SCHED_PREFIX_CACHE") = kSchedPrefixCache;
  m.attr("SCHED_CUDAGRAPH_PADDING") = kSchedCudaGraphPadding;
  m.attr("SCHED_PREFILL_DECODE_INTERLEAVE") = kSchedPrefillDecodeInterleave;
  m.attr("SCHED_KV_CACHE_REQUIRED") = kSchedKvCacheRequired;
  m.attr("SCHED_CROSS_SEQUENCE_PREFIX_REUSE") = kSchedCrossSequencePrefixReuse;
  m.attr("SCHED_DEFAULT_FLAGS") = kSchedDefaultFlags;
  m.attr("DECISION_PREFILL_CHUNK") = kDecisionPrefillChunk;
  m.attr("DECISION_PREFILL_FINAL_CHUNK") = kDecisionPrefillFinalChunk;
  m.attr("DECISION_PREFIX_CACHE_USED") = kDecisionPrefixCacheUsed;
  m.attr("DECISION_CUDAGRAPH_PADDING") = kDecisionCudaGraphPadding;
  m.attr("DECISION_DECODE_STEP") = kDecisionDecodeStep;
  m.attr("DECISION_PREFILL_STEP") = kDecisionPrefillStep;
  m.attr("DECISION_SCHEDULED_AHEAD") = kDecisionScheduledAhead;
  m.attr("DECISION_PREEMPTED") = kDecisionPreempted;
  m.attr("DECISION_SPECULATIVE_VERIFY") = kDecisionSpeculativeVerify;
  m.attr("DECISION_MTP_TREE_VERIFY") = kDecisionMtpTreeVerify;
  m.attr("SCHED_MTP_FORCE_ENABLE") = kSchedMtpForceEnable;
  m.attr("SCHED_PREFIX_COHORTING") = kSchedPrefixCohorting;
  m.attr("SCHED_LOOKAHEAD_PROTECTION") = kSchedLookaheadProtection;
  m.attr("DECISION_PREFIX_FAMILY") = kDecisionPrefixFamily;
  m.attr("DECISION_SWAP") = kDecisionSwap;
  m.attr("SPEC_OFF") = uint32_t(SpecMode::Off);
  m.attr("SPEC_CHAIN") = uint32_t(SpecMode::Chain);
  m.attr("SPEC_MTP_TREE") = uint32_t(SpecMode::MtpTree);

  py::class_<SchedulerConfig>(m, "SchedulerConfig")
      .def(py::init<>())
      .def_readwrite("max_batch", &SchedulerConfig::max_batch)
      .def_readwrite("max_prefill_tokens", &SchedulerConfig::max_prefill_tokens)
      .def_readwrite("max_prefill_seqs", &SchedulerConfig::max_prefill_seqs)
      .def_readwrite("block_tokens", &SchedulerConfig::block_tokens)
      .def_readwrite("num_blocks", &SchedulerConfig::num_blocks)
      .def_readwrite("max_model_len", &SchedulerConfig::max_model_len)
      .def_readwrite("max_sequences", &SchedulerConfig::max_sequences)
      .def_readwrite("flags", &SchedulerConfig::flags)
      .def_readwrite("max_consecutive_prefills", &SchedulerConfig::max_consecutive_prefills)
      .def_readwrite("decode_buckets", &SchedulerConfig::decode_buckets)
      .def_readwrite("spec_mode", &SchedulerConfig::spec_mode)
      .def_readwrite("spec_draft_len", &SchedulerConfig::spec_draft_len)
      .def_readwrite("spec_row_cap", &SchedulerConfig::spec_row_cap)
      .def_readwrite("spec_row_cost_milli", &SchedulerConfig::spec_row_cost_milli)
      .def_readwrite("spec_shadow_slot_base", &SchedulerConfig::spec_shadow_slot_base)
      .def_readwrite("host_blocks", &SchedulerConfig::host_blocks)
      .def_readwrite("host_prefix_blocks", &SchedulerConfig::host_prefix_blocks)
      .def_readwrite("lookahead_requests", &SchedulerConfig::lookahead_requests);
  py::class_<RequestSpec>(m, "RequestSpec")
      .def(py::init<>())
      .def(py::init([](uint64_t id, const std::vector<uint32_t>& prompt, uint32_t max_new, uint32_t priority,
                       const std::vector<uint32_t>& stops, bool ignore_eos, float temperature, uint64_t seed) {
             RequestSpec r;
             r.id = id;
             r.prompt = prompt;
             r.max_new_tokens = max_new;
             r.priority = priority;
             r.stop_token_ids = stops;
             r.ignore_eos = ignore_eos;
             r.temperature = temperature;
             r.seed = seed;
             return r;
           }),
           py::arg("id"), py::arg("prompt"), py::arg("max_new_tokens") = 16, py::arg("priority") = 1000000,
           py::arg("stop_token_ids") = std::vector<uint32_t>{}, py::arg("ignore_eos") = false,
           py::arg("temperature") = 0.f, py::arg("seed") = 0)
      .def_readwrite("temperature", &RequestSpec::temperature)
      .def_readwrite("seed", &RequestSpec::seed)
      .def_readwrite("id", &RequestSpec::id)
      .def_readwrite("prompt", &RequestSpec::prompt)
      .def_readwrite("max_new_tokens", &RequestSpec::max_new_tokens)
      .def_readwrite("priority", &RequestSpec::priority)
      .def_readwrite("stop_token_ids", &RequestSpec::stop_token_ids)
      .def_readwrite("ignore_eos", &RequestSpec::ignore_eos)
      .def_readwrite("disable_speculation", &RequestSpec::disable_speculation);
  py::class_<StepPlan>(m, "StepPlan")
      .def_readonly("kind", &StepPlan::kind)
      .def_readonly("flags", &StepPlan::flags)
      .def_readonly("num_seqs", &StepPlan::num_seqs)
      .def_readonly("padded_seqs", &StepPlan::padded_seqs)
      .def_readonly("num_tokens", &StepPlan::num_tokens)
      .def_readonly("step_index", &StepPlan::step_index)
      .def_readonly("max_q", &StepPlan::max_q)
      .def_readonly("has_prefix", &StepPlan::has_prefix)
      .def_readonly("cached_prefix_tokens", &StepPlan::cached_prefix_tokens)
      .def_readonly("max_blocks", &StepPlan::max_blocks)
      .def_readonly("max_context", &StepPlan::max_context)
      .def_readonly("seq_ids", &StepPlan::seq_ids)
      .def_property_readonly("emits_token", [](const StepPlan& p) { return to_np(p.emits_token); })
      .def_property_readonly("token_ids", [](const StepPlan& p) { return to_np(p.token_ids); })
      .def_property_readonly("positions", [](const StepPlan& p) { return to_np(p.positions); })
      .def_property_readonly("slot_mapping", [](const StepPlan& p) { return to_np(p.slot_mapping); })
      .def_property_readonly("cu_q", [](const StepPlan& p) { return to_np(p.cu_q); })
      .def_property_readonly("cu_k", [](const StepPlan& p) { return to_np(p.cu_k); })
      .def_property_readonly("ctx_slots", [](const StepPlan& p) { return to_np(p.ctx_slots); })
      .def_property_readonly("logits_idx", [](const StepPlan& p) { return to_np(p.logits_idx); })
      .def_property_readonly("chunk_lens", [](const StepPlan& p) { return to_np(p.chunk_lens); })
      .def_property_readonly("block_table", [](const StepPlan& p) { return to_np(p.block_table); })
      .def_property_readonly("context_lens", [](const StepPlan& p) { return to_np(p.context_lens); })
      .def_property_readonly("src_rows", [](const StepPlan& p) { return to_np(p.src_rows); })
      .def_readonly("rows_per_seq", &StepPlan::rows_per_seq)
      .def_property_readonly("swap_out", [](const StepPlan& p) { return to_np(p.swap_out); })
      .def_property_readonly("swap_in", [](const StepPlan& p) { return to_np(p.swap_in); })
      .def_property_readonly("draft_budget", [](const StepPlan& p) { return to_np(p.draft_budget); })
      .def_property_readonly("accept_keys", [](const StepPlan& p) {
        py::array_t<int64_t> a((py::ssize_t)p.accept_keys.size());
        std::memcpy(a.mutable_data(), p.accept_keys.data(), p.accept_keys.size() * 8);
        return a;
      })
      .def_property_readonly("sync_token_ids", [](const StepPlan& p) { return to_np(p.sync_token_ids); })
      .def_property_readonly("sync_positions", [](const StepPlan& p) { return to_np(p.sync_positions); })
      .def_property_readonly("sync_slots", [](const StepPlan& p) { return to_np(p.sync_slots); })
      // Verify inputs into preallocated (pinned) CPU tensors: the row arrays
      // [rows x padded], the per-sequence block table, draft budgets and acceptance
      // keys, and (tree) the draft-sync rows. Returns the bytes written.
      .def("write_verify_inputs",
           [](const StepPlan& p, const torch::Tensor& ids, const torch::Tensor& pos, const torch::Tensor& slots,
              const torch::Tensor& ctx, const torch::Tensor& bt, const torch::Tensor& budget,
              const torch::Tensor& keys, const c10::optional<torch::Tensor>& sync) {
             TORCH_CHECK(p.kind == StepPlan::Verify, "not a verify plan");
             copy_into(ids, p.token_ids.data(), p.token_ids.size() * 4);
             copy_into(pos, p.positions.data(), p.positions.size() * 4);
             copy_into(slots, p.slot_mapping.data(), p.slot_mapping.size() * 4);
             copy_into(ctx, p.context_lens.data(), p.context_lens.size() * 4);
             copy_into(budget, p.draft_budget.data(), p.draft_budget.size() * 4);
             copy_into(keys, p.accept_keys.data(), p.accept_keys.size() * 8);
             const int64_t cols = bt.size(1);
             TORCH_CHECK(bt.size(0) >= p.padded_seqs, "block table tensor has too few rows");
             int32_t* dst = bt.data_ptr<int32_t>();
             for (uint32_t r = 0; r < p.padded_seqs; ++r)
               std::memcpy(dst + r * cols, p.block_table.data() + size_t(r) * p.max_blocks,
                           sizeof(int32_t) * std::min<int64_t>(cols, p.max_blocks));
             int64_t bytes = int64_t(p.token_ids.size() * 16 + p.draft_budget.size() * 12) +
                             int64_t(p.padded_seqs) * cols * 4;
             if (sync.has_value() && !p.sync_slots.empty()) {
               // [3][n] token ids, positions, slots
               const size_t n = p.sync_slots.size();
               TORCH_CHECK(sync->numel() >= int64_t(3 * n), "sync tensor too small");
               int32_t* d = sync->data_ptr<int32_t>();
               std::memcpy(d, p.sync_token_ids.data(), n * 4);
               std::memcpy(d + n, p.sync_positions.data(), n * 4);
               std::memcpy(d + 2 * n, p.sync_slots.data(), n * 4);
               bytes += int64_t(12 * n);
             }
             return bytes;
           })
      // Fast path: copy the decode inputs into preallocated (pinned) CPU tensors.
      .def("write_decode_inputs",
           [](const StepPlan& p, const torch::Tensor& ids, const torch::Tensor& pos, const torch::Tensor& slots,
              const torch::Tensor& ctx, const torch::Tensor& bt) {
             TORCH_CHECK(p.kind == StepPlan::Decode, "not a decode plan");
             copy_into(ids, p.token_ids.data(), p.token_ids.size() * 4);
             copy_into(pos, p.positions.data(), p.positions.size() * 4);
             copy_into(slots, p.slot_mapping.data(), p.slot_mapping.size() * 4);
             copy_into(ctx, p.context_lens.data(), p.context_lens.size() * 4);
             // the block table tensor may be narrower (fewer columns) than the plan's
             const int64_t cols = bt.size(1);
             TORCH_CHECK(bt.size(0) >= p.padded_seqs, "block table tensor has too few rows");
             int32_t* dst = bt.data_ptr<int32_t>();
             for (uint32_t r = 0; r < p.padded_seqs; ++r)
               std::memcpy(dst + r * cols, p.block_table.data() + size_t(r) * p.max_blocks,
                           sizeof(int32_t) * std::min<int64_t>(cols, p.max_blocks));
             return (int64_t)(p.token_ids.size() * 16 + size_t(p.padded_seqs) * cols * 4);
           });
  py::class_<SchedEvent>(m, "SchedEvent")
      .def_readonly("kind", &SchedEvent::kind)
      .def_readonly("id", &SchedEvent::id)
      .def_readonly("token", &SchedEvent::token)
      .def_readonly("reason", &SchedEvent::reason)
      .def_readonly("value", &SchedEvent::value);
  py::class_<SchedulerStats>(m, "SchedulerStats")
      .def_readonly("steps", &SchedulerStats::steps)
      .def_readonly("prefill_steps", &SchedulerStats::prefill_steps)
      .def_readonly("decode_steps", &SchedulerStats::decode_steps)
      .def_readonly("verify_steps", &SchedulerStats::verify_steps)
      .def_readonly("swapped_out", &SchedulerStats::swapped_out)
      .def_readonly("swapped_in", &SchedulerStats::swapped_in)
      .def_readonly("swap_out_blocks", &SchedulerStats::swap_out_blocks)
      .def_readonly("swap_in_blocks", &SchedulerStats::swap_in_blocks)
      .def_readonly("family_deferrals", &SchedulerStats::family_deferrals)
      .def_readonly("family_steps", &SchedulerStats::family_steps)
      .def_readonly("lookahead_protected_blocks", &SchedulerStats::lookahead_protected_blocks)
      .def_readonly("prefix_tier_out_blocks", &SchedulerStats::prefix_tier_out_blocks)
      .def_readonly("prefix_tier_in_blocks", &SchedulerStats::prefix_tier_in_blocks)
      .def_readonly("preemptions", &SchedulerStats::preemptions)
      .def_readonly("prefill_tokens", &SchedulerStats::prefill_tokens)
      .def_readonly("decode_tokens", &SchedulerStats::decode_tokens)
      .def_readonly("cached_prompt_tokens", &SchedulerStats::cached_prompt_tokens)
      .def_readonly("admitted", &SchedulerStats::admitted)
      .def_readonly("finished", &SchedulerStats::finished)
      .def_readonly("cancelled", &SchedulerStats::cancelled)
      .def_readonly("rejected", &SchedulerStats::rejected);
  py::class_<Scheduler>(m, "Scheduler")
      .def(py::init<const SchedulerConfig&>())
      .def("add_request", &Scheduler::add_request)
      .def("schedule", &Scheduler::schedule)
      .def("schedule_ahead", &Scheduler::schedule_ahead)
      .def("sampling_rows",
           [](const Scheduler& s, const StepPlan& p, const torch::Tensor& temp, const torch::Tensor& key) {
             TORCH_CHECK(!temp.is_cuda() && temp.scalar_type() == at::kFloat && temp.is_contiguous(),
                         "temperature rows: float32 CPU tensor");
             TORCH_CHECK(!key.is_cuda() && key.scalar_type() == at::kLong && key.is_contiguous(),
                         "key rows: int64 CPU tensor");
             TORCH_CHECK(temp.numel() == key.numel(), "sampling_rows: row counts differ");
             return s.sampling_rows(p, temp.data_ptr<float>(), reinterpret_cast<uint64_t*>(key.data_ptr<int64_t>()),
                                    (uint32_t)temp.numel());
           })
      .def("complete",
           [](Scheduler& s, const StepPlan& p, py::array_t<int32_t, py::array::c_style | py::array::forcecast> t) {
             return s.complete(p, t.data(), (uint32_t)t.size());
           })
      .def("complete_tensor",
           [](Scheduler& s, const StepPlan& p, const torch::Tensor& t) {
             TORCH_CHECK(!t.is_cuda() && t.scalar_type() == at::kInt && t.is_contiguous(), "int32 CPU tensor");
             return s.complete(p, t.data_ptr<int32_t>(), (uint32_t)t.numel());
           })
      .def("complete_verify",
           [](Scheduler& s, const StepPlan& p, py::array_t<int32_t, py::array::c_style | py::array::forcecast> committed,
              py::array_t<int32_t, py::array::c_style | py::array::forcecast> counts,
              py::object paths) {
             TORCH_CHECK(committed.ndim() == 2, "committed: [sequences, stride]");
             const int32_t* pp = nullptr;
             py::array_t<int32_t, py::array::c_style | py::array::forcecast> pa;
             if (!paths.is_none()) {
               pa = paths.cast<py::array_t<int32_t, py::array::c_style | py::array::forcecast>>();
               TORCH_CHECK(pa.size() >= counts.size(), "paths shorter than counts");
               pp = pa.data();
             }
             TORCH_CHECK(committed.shape(0) >= counts.size(), "committed rows shorter than counts");
             return s.complete_verify(p, committed.data(), (uint32_t)committed.shape(1), counts.data(), pp,
                                      (uint32_t)counts.size());
           },
           py::arg("plan"), py::arg("committed"), py::arg("counts"), py::arg("paths") = py::none())
      .def("set_step_cost", &Scheduler::set_step_cost, py::arg("kind"), py::arg("seqs"), py::arg("ns"))
      .def("estimate_step_ns", &Scheduler::estimate_step_ns)
      .def("lane_state",
           [](const Scheduler& s, uint64_t id) {
             const spec::LaneState l = s.lane_state(id);
             py::dict d;
             d["ema_milli"] = l.ema_milli;
             d["budget"] = l.budget;
             d["countdown"] = l.countdown;
             d["disabled"] = l.disabled;
             return d;
           })
      .def_property_readonly("spec_rows_per_seq", &Scheduler::spec_rows_per_seq)
      .def_property_readonly("spec_totals",
                             [](const Scheduler& s) {
                               const spec::Totals& t = s.spec_totals();
                               py::dict d;
                               d["rounds"] = t.rounds;
                               d["proposed"] = t.proposed;
                               d["accepted"] = t.accepted;
                               d["committed"] = t.committed;
                               d["verify_steps"] = t.verify_steps;
                               d["suppressed"] = t.suppressed;
                               d["reprobes"] = t.reprobes;
                               d["expected_committed_milli"] = spec::expected_committed_scaled(t);
                               return d;
                             })
      .def("cancel", &Scheduler::cancel)
      .def("fail_step", &Scheduler::fail_step)
      .def("has_work", &Scheduler::has_work)
      .def("state", &Scheduler::state)
      .def("output_tokens", &Scheduler::output_tokens)
      .def("bucket_for", &Scheduler::bucket_for)
      .def_property_readonly("waiting_count", &Scheduler::waiting_count)
      .def_property_readonly("running_count", &Scheduler::running_count)
      .def_property_readonly("swapped_count", &Scheduler::swapped_count)
      .def_property_readonly("free_host_blocks", &Scheduler::free_host_blocks)
      .def_property_readonly("max_blocks_per_seq", &Scheduler::max_blocks_per_seq)
      .def_property_readonly("stats", &Scheduler::stats)
      .def_property_readonly("prefix_cache", &Scheduler::prefix_cache, py::return_value_policy::reference_internal);
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "C++ serving runtime of sparkpipe_rs_b200";
  py::enum_<Status>(m, "Status")
      .value("OK", Status::Ok)
      .value("INVALID_ARGUMENT", Status::InvalidArgument)
      .value("CAPACITY_EXCEEDED", Status::CapacityExceeded)
      .value("NOT_FOUND", Status::NotFound)
      .value("IO_ERROR", Status::IoError)
      .value("PARSE_ERROR", Status::ParseError)
      .value("SCHEMA_ERROR", Status::SchemaError)
      .value("HASH_MISMATCH", Status::HashMismatch)
      .value("MODULE_NOT_VALIDATED", Status::ModuleNotValidated)
      .value("VALIDATION_FAILED", Status::ValidationFailed)
      .value("ABI_MISMATCH", Status::AbiMismatch)
      .value("TARGET_MISMATCH", Status::TargetMismatch)
      .value("COMPILER_ERROR", Status::CompilerError)
      .value("DRIVER_LOAD_ERROR", Status::DriverLoadError)
      .value("ROUTE_NOT_FOUND", Status::RouteNotFound)
      .value("BUSY", Status::Busy)
      .value("DUPLICATE", Status::Duplicate)
      .value("INTERNAL_ERROR", Status::InternalError)
      .value("PENDING", Status::Pending)
      .value("UNSUPPORTED", Status::Unsupported);
  static py::exception<StatusError> exc(m, "StatusError", PyExc_RuntimeError);
  py::register_exception_translator([](std::exception_ptr p) {
    try {
      if (p) std::rethrow_exception(p);
    } catch (const StatusError& e) {
      const std::string msg = std::string(status_name(e.status)) + ": " + e.what();
      py::object obj = py::reinterpret_steal<py::object>(PyObject_CallFunction(exc.ptr(), "s", msg.c_str()));
      obj.attr("code") = uint32_t(e.status);
      obj.attr("status") = status_name(e.status);
      PyErr_SetObject(exc.ptr(), obj.ptr());
    }
  });
  bind_memory(m);
  bind_prefix(m);
  bind_scheduler(m);
  for (auto& fn : registry()) fn(m);
}
