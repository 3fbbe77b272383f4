// Continuous-batching scheduler of the serving engine.
//
// Owns every request's slot state and its KV blocks (through the prefix
// cache), and turns the live set into one step plan per engine iteration:
// either a prefill step (chunked, prefix-cache aware, several prompts packed
// into one variable-length batch) or a decode step (all ready sequences, padded
// to a CUDA-graph batch bucket). The plan carries every host array the GPU
// step needs (token ids, positions, cache slots, cu_seqlens, block tables,
// context lengths), laid out for one pinned host->device copy each.
//
// Slot states and configuration / decision flag names follow the reference's
// request API and scheduler (crates/spark-serve/src/request_api/slot.rs:9-248,
// crates/spark-sched/src/scheduler.rs:73-170); the policy (prefill-first with
// an interleave cap, chunked prefill under a token budget, recompute preemption
// when KV blocks run out) is this engine's own single-box design.
#pragma once

#include <cstdint>
#include <deque>
#include <memory>
#include <unordered_map>
#include <vector>

#include "common.h"
#include "prefix_cache.h"
#include "speculation.h"

namespace spc {

enum class SlotState : uint32_t {
  Free = 0,
  QueuedPrefill = 1,
  RunningPrefill = 2,
  ReadyDecode = 3,
  RunningDecode = 4,
  Completed = 5,
  Cancelled = 6,
  WaitingPrefixCohort = 7,
  ReadySpeculativeVerify = 8,
  RunningSpeculativeVerify = 9,
  Swapped = 10,  // preempted with its KV copied to the host tier, waiting to be restored
};

// configuration flags
constexpr uint32_t kSchedChunkedPrefill = 0x01;
constexpr uint32_t kSchedPrefixCache = 0x02;
constexpr uint32_t kSchedCudaGraphPadding = 0x04;
constexpr uint32_t kSchedPrefillDecodeInterleave = 0x08;
constexpr uint32_t kSchedKvCacheRequired = 0x10;
constexpr uint32_t kSchedCrossSequencePrefixReuse = 0x40;
constexpr uint32_t kSchedPrefixCohorting = 0x80;     // prefill a prefix family's leader before its followers
constexpr uint32_t kSchedLookaheadProtection = 0x100;  // queued prompts protect the cached blocks they will reuse
constexpr uint32_t kSchedMtpForceEnable = 0x200;  // verify whenever the lanes qualify (no utility comparison)
constexpr uint32_t kSchedDefaultFlags = kSchedChunkedPrefill | kSchedPrefixCache | kSchedCudaGraphPadding |
                                        kSchedPrefillDecodeInterleave | kSchedKvCacheRequired |
                                        kSchedCrossSequencePrefixReuse | kSchedPrefixCohorting |
                                        kSchedLookaheadProtection;
// decision flags
constexpr uint32_t kDecisionPrefillChunk = 0x001;
constexpr uint32_t kDecisionPrefillFinalChunk = 0x002;
constexpr uint32_t kDecisionPrefixCacheUsed = 0x004;
constexpr uint32_t kDecisionCudaGraphPadding = 0x008;
constexpr uint32_t kDecisionDecodeStep = 0x010;
constexpr uint32_t kDecisionPrefillStep = 0x020;
constexpr uint32_t kDecisionScheduledAhead = 0x040;  // decode planned before the previous step's tokens were read
constexpr uint32_t kDecisionSpeculativeVerify = 0x080;
constexpr uint32_t kDecisionMtpTreeVerify = 0x100;
constexpr uint32_t kDecisionPrefixFamily = 0x200;   // followers of a prefix family wait for their leader
constexpr uint32_t kDecisionSwap = 0x400;           // the plan carries host-tier swap-out / swap-in copies
constexpr uint32_t kDecisionPreempted = 0x800;

// speculation modes: a draft chain of spec_draft_len tokens per lane, or the fixed
// MTP draft tree (5 candidates verified in 6 rows, work_control.h mtp::)
enum class SpecMode : uint32_t { Off = 0, Chain = 1, MtpTree = 2 };

// finish reasons
enum class FinishReason : uint32_t { None = 0, Length = 1, Stop = 2, Cancelled = 3, ContextLimit = 4, Error = 5 };

struct SchedulerConfig {
  uint32_t max_batch = 64;            // concurrently decoding sequences
  uint32_t max_prefill_tokens = 16384;  // token budget of one prefill step
  uint32_t max_prefill_seqs = 256;
  uint32_t block_tokens = 64;
  uint32_t num_blocks = 1024;
  uint32_t max_model_len = 8192;
  uint32_t max_sequences = 4096;      // admitted + queued
  uint32_t flags = kSchedDefaultFlags;
  uint32_t max_consecutive_prefills = 4;  // interleave cap while decodes wait
  std::vector<uint32_t> decode_buckets = {1, 2, 4, 8, 16, 32, 64, 128, 256};
  // speculation
  uint32_t spec_mode = 0;               // SpecMode
  uint32_t spec_draft_len = 3;          // chain: draft tokens per round (1..7)
  uint32_t spec_row_cap = 0;            // firing rows of a verify round (0: rows per lane x max_batch)
  uint32_t spec_row_cost_milli = 1000;  // a draft row's cost relative to a real row
  int64_t spec_shadow_slot_base = -1;   // tree: cache row of the first shadow slot (2 per batch row)
  // host KV tier: preemption copies a sequence's KV blocks to host slots and
  // restores them later instead of recomputing its context (0: recompute)
  uint32_t host_blocks = 0;
  // host slots (after the preemption slots) where warm prefix blocks evicted from the
  // device wait for a later prompt that reuses them (0: evicted blocks are dropped)
  uint32_t host_prefix_blocks = 0;
  uint32_t lookahead_requests = 64;     // queued prompts that protect their cached prefix
};

struct RequestSpec {
  uint64_t id = 0;
  std::vector<uint32_t> prompt;
  uint32_t max_new_tokens = 16;
  uint32_t priority = 1000000;        // higher runs first; ties by arrival
  std::vector<uint32_t> stop_token_ids;
  bool ignore_eos = false;
  float temperature = 0.f;            // <= 0: greedy
  uint64_t seed = 0;
  bool disable_speculation = false;   // sampled requests (temperature > 0) never speculate either
};

struct StepPlan {
  enum Kind : uint32_t { None = 0, Prefill = 1, Decode = 2, Verify = 3 };
  uint32_t kind = None;
  uint32_t flags = 0;
  uint32_t num_seqs = 0;      // real sequences
  uint32_t padded_seqs = 0;   // decode: CUDA-graph bucket size
  uint32_t num_tokens = 0;
  uint64_t step_index = 0;
  std::vector<uint64_t> seq_ids;
  std::vector<int32_t> token_ids, positions, slot_mapping;
  // prefill
  std::vector<int32_t> cu_q, cu_k, ctx_slots, logits_idx, chunk_lens;
  std::vector<uint8_t> emits_token;
  uint32_t max_q = 0;
  bool has_prefix = false;    // some sequence attends to previously cached tokens
  uint32_t cached_prefix_tokens = 0;
  // decode
  std::vector<int32_t> block_table, context_lens;
  // decode scheduled ahead: row i's input token is the previous step's sampled
  // token of row src_rows[i] (token_ids carries the same indices)
  std::vector<int32_t> src_rows;
  uint32_t max_blocks = 0;
  uint32_t max_context = 0;
  // verify: rows_per_seq rows per sequence, laid out row-major by draft depth / tree
  // row (row j * padded_seqs + b); block_table stays one row per sequence
  uint32_t rows_per_seq = 1;
  std::vector<int32_t> draft_budget;      // per sequence: drafts it may accept
  std::vector<uint64_t> accept_keys;      // per sequence: key of forced-acceptance draws
  // tree: the draft model's KV of the 3 positions before each lane's input token
  // (rewritten every round: accepted tree tokens may not be in the draft cache)
  std::vector<int32_t> sync_token_ids, sync_positions, sync_slots;  // [3 x padded_seqs], row k * padded + b
  // host tier, applied before the step in this order: (device block, host slot)
  // pairs to copy out, then (host slot, device block) pairs to copy in
  std::vector<int32_t> swap_out, swap_in;
};

struct SchedEvent {
  enum Kind : uint32_t { Token = 1, Finished = 2, Preempted = 3, PrefillProgress = 4 };
  uint32_t kind;
  uint64_t id;
  int32_t token;
  uint32_t reason;  // FinishReason for Finished
  uint32_t value;   // computed prompt tokens for PrefillProgress, generated count for Token
};

struct SchedulerStats {
  uint64_t steps = 0, prefill_steps = 0, decode_steps = 0, verify_steps = 0, preemptions = 0;
  uint64_t swapped_out = 0, swapped_in = 0, swap_out_blocks = 0, swap_in_blocks = 0;
  uint64_t family_deferrals = 0, family_steps = 0, lookahead_protected_blocks = 0;
  uint64_t prefix_tier_out_blocks = 0, prefix_tier_in_blocks = 0;
  uint64_t prefill_tokens = 0, decode_tokens = 0, cached_prompt_tokens = 0;
  uint64_t admitted = 0, finished = 0, cancelled = 0, rejected = 0;
};

class Scheduler {
 public:
  explicit Scheduler(const SchedulerConfig& cfg);
  void add_request(const RequestSpec& spec);
  StepPlan schedule();
  // The decode step that follows the in-flight decode step `inflight`, planned
  // before its tokens are known (every earlier step must be completed). Each of
  // its sequences is assumed to continue; one that stops at `inflight` gets one
  // discarded extra token. Returns an empty plan (kind None) when that is not
  // safe or not the policy's choice: a prefill may be due, the decode set
  // changed, or the KV blocks for one more token are not free.
  StepPlan schedule_ahead(const StepPlan& inflight);
  std::vector<SchedEvent> complete(const StepPlan& plan, const int32_t* sampled, uint32_t n_sampled);
  // Completes a verify plan: sequence b committed counts[b] tokens, committed[b *
  // stride ..]; paths[b] is the tree resolution (tree mode). Updates each lane's
  // speculation state and stops a sequence at its first stop token / length limit.
  std::vector<SchedEvent> complete_verify(const StepPlan& plan, const int32_t* committed, uint32_t stride,
                                          const int32_t* counts, const int32_t* paths, uint32_t n);
  // Measured device time of one plain decode step (kind 2) or verify round (kind 3)
  // of a padded batch; the speculation utility compares them.
  void set_step_cost(uint32_t kind, uint32_t seqs, uint64_t ns) { cost_.set(kind, seqs, ns); }
  uint64_t estimate_step_ns(uint32_t kind, uint32_t seqs) const;
  const spec::Totals& spec_totals() const { return spec_; }
  spec::LaneState lane_state(uint64_t id) const;
  uint32_t spec_rows_per_seq() const;
  // Per-row sampling parameters of a plan (rows beyond num_seqs are greedy):
  // temperature and a noise key derived from the request's seed and the position
  // of the token that is sampled, so a request draws the same tokens however it
  // is batched. Returns whether any row samples (temperature > 0).
  bool sampling_rows(const StepPlan& plan, float* temp, uint64_t* key, uint32_t rows) const;
  bool cancel(uint64_t id);  // false when unknown / already finished
  void fail_step(const StepPlan& plan);  // a dispatched step failed: cancel its sequences

  bool has_work() const { return !waiting_.empty() || running_count_ > 0 || !swapped_.empty(); }
  uint32_t swapped_count() const { return (uint32_t)swapped_.size(); }
  uint32_t free_host_blocks() const { return (uint32_t)host_free_.size(); }
  uint32_t waiting_count() const { return (uint32_t)waiting_.size(); }
  uint32_t running_count() const { return running_count_; }
  SlotState state(uint64_t id) const;
  std::vector<uint32_t> output_tokens(uint64_t id) const;
  uint32_t bucket_for(uint32_t n) const;
  const SchedulerConfig& config() const { return cfg_; }
  const SchedulerStats& stats() const { return stats_; }
  const PrefixCache& prefix_cache() const { return *cache_; }
  uint32_t max_blocks_per_seq() const { return max_blocks_; }

 private:
  struct Req {
    RequestSpec spec;
    std::vector<uint32_t> tokens;  // prompt + generated
    uint32_t prompt_len = 0;       // may grow on preemption (recompute the generated tail)
    uint32_t computed = 0;         // tokens with KV in the cache
    uint32_t generated = 0;
    SlotState state = SlotState::QueuedPrefill;
    spec::LaneState lane;
    std::vector<uint64_t> block_hashes;  // chain hashes of the prompt's full blocks (prefix families)
    std::vector<uint32_t> host_slots;    // swapped: host slot of each of its leading blocks
    bool reserved = false;
    uint64_t arrival = 0;
    FinishReason reason = FinishReason::None;
  };
  StepPlan build_prefill();
  StepPlan build_decode();
  // the verify form of a decode plan, or an empty plan when the policy keeps plain decode
  StepPlan try_build_verify(const StepPlan& decode);
  // per-lane draft budgets of a verify round over `ids`; false when the policy keeps plain decode
  bool spec_grants(const std::vector<uint64_t>& ids, std::vector<uint32_t>& grant) const;
  uint32_t full_budget() const;
  std::vector<SchedEvent> append_committed(Req& r, uint64_t id, const int32_t* toks, uint32_t n);
  void preempt_one(uint64_t keep);
  bool swap_out(uint64_t id);   // false when the host tier has no room
  void resume_swapped();         // restores swapped sequences while seats and blocks allow
  void attach_swaps(StepPlan& p);
  // prefix families among queued, unreserved prompts: the requests to hold back this step
  std::vector<uint64_t> family_followers();
  StepPlan schedule_step();
  const std::vector<uint64_t>& prompt_hashes(Req& r);
  void finish(Req& r, uint64_t id, FinishReason why, std::vector<SchedEvent>& ev);
  int32_t slot_of(const Req& r, uint64_t id, uint32_t pos) const;

  SchedulerConfig cfg_;
  std::unique_ptr<PrefixCache> cache_;
  std::unordered_map<uint64_t, Req> reqs_;
  std::deque<uint64_t> waiting_;   // queued for (more) prefill, in admission order
  std::vector<uint64_t> running_;  // ready to decode, in admission order
  std::deque<uint64_t> swapped_;   // swapped out, oldest first
  std::vector<uint32_t> host_free_;
  std::vector<int32_t> pending_out_, pending_in_;
  std::vector<uint32_t> host_release_;  // host slots free from the next plan on
  uint32_t running_count_ = 0;
  uint32_t consecutive_prefills_ = 0;
  uint32_t max_blocks_;
  uint64_t arrival_clock_ = 0;
  uint64_t step_clock_ = 0;
  SchedulerStats stats_;
  spec::Totals spec_;
  spec::StepCost cost_;
};

}  // namespace spc
