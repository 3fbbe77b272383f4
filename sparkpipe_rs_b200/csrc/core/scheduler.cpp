#include "scheduler.h"

#include <algorithm>

namespace spc {

Scheduler::Scheduler(const SchedulerConfig& cfg) : cfg_(cfg) {
  if (cfg.max_batch == 0 || cfg.max_prefill_tokens == 0 || cfg.block_tokens == 0 || cfg.num_blocks == 0 ||
      cfg.max_model_len < 2 || cfg.max_sequences == 0)
    fail(Status::InvalidArgument, "Scheduler: invalid configuration");
  std::sort(cfg_.decode_buckets.begin(), cfg_.decode_buckets.end());
  cache_ = std::make_unique<PrefixCache>(cfg.block_tokens, cfg.num_blocks, cfg.max_sequences);
  max_blocks_ = (cfg.max_model_len + cfg.block_tokens - 1) / cfg.block_tokens;
}

uint32_t Scheduler::bucket_for(uint32_t n) const {
  if (!(cfg_.flags & kSchedCudaGraphPadding)) return n;
  for (uint32_t b : cfg_.decode_buckets)
    if (b >= n) return b;
  return n;
}

void Scheduler::add_request(const RequestSpec& spec) {
  if (reqs_.count(spec.id)) fail(Status::Duplicate, "Scheduler: duplicate request id");
  if (spec.prompt.empty()) fail(Status::InvalidArgument, "Scheduler: empty prompt");
  if (spec.prompt.size() + 1 > cfg_.max_model_len) {
    ++stats_.rejected;
    fail(Status::CapacityExceeded, "Scheduler: prompt longer than the model context");
  }
  if (reqs_.size() >= cfg_.max_sequences) {
    ++stats_.rejected;
    fail(Status::CapacityExceeded, "Scheduler: request table full");
  }
  Req r;
  r.spec = spec;
  r.tokens = spec.prompt;
  r.prompt_len = (uint32_t)spec.prompt.size();
  r.arrival = ++arrival_clock_;
  r.state = SlotState::QueuedPrefill;
  // priority order (higher first), arrival order within a priority
  auto pos = waiting_.end();
  for (auto it = waiting_.begin(); it != waiting_.end(); ++it) {
    if (reqs_.at(*it).spec.priority < spec.priority) { pos = it; break; }
  }
  reqs_.emplace(spec.id, std::move(r));
  waiting_.insert(pos, spec.id);
  ++stats_.admitted;
}

SlotState Scheduler::state(uint64_t id) const {
  auto it = reqs_.find(id);
  return it == reqs_.end() ? SlotState::Free : it->second.state;
}

std::vector<uint32_t> Scheduler::output_tokens(uint64_t id) const {
  auto it = reqs_.find(id);
  if (it == reqs_.end()) return {};
  const Req& r = it->second;
  return std::vector<uint32_t>(r.tokens.begin() + r.spec.prompt.size(), r.tokens.end());
}

int32_t Scheduler::slot_of(const Req&, uint64_t id, uint32_t pos) const {
  const auto& blocks = cache_->block_list(id);
  const uint32_t b = pos / cfg_.block_tokens;
  return int32_t(blocks.at(b) * cfg_.block_tokens + pos % cfg_.block_tokens);
}

StepPlan Scheduler::schedule() {
  bool prefill = !waiting_.empty() && running_count_ < cfg_.max_batch;
  if (prefill && running_count_ > 0 && (cfg_.flags & kSchedPrefillDecodeInterleave) &&
      consecutive_prefills_ >= cfg_.max_consecutive_prefills)
    prefill = false;
  if (prefill) {
    StepPlan p = build_prefill();
    if (p.kind != StepPlan::None) {
      ++consecutive_prefills_;
      return p;
    }
  }
  if (running_count_ > 0) {
    consecutive_prefills_ = 0;
    return build_decode();
  }
  return StepPlan{};
}

StepPlan Scheduler::build_prefill() {
  StepPlan p;
  p.kind = StepPlan::Prefill;
  p.flags = kDecisionPrefillStep;
  p.step_index = ++step_clock_;
  p.cu_q.push_back(0);
  p.cu_k.push_back(0);
  uint32_t budget = cfg_.max_prefill_tokens;
  uint32_t held = 0;  // waiting sequences that already hold a decode seat
  for (uint64_t id : waiting_)
    if (reqs_.at(id).reserved) ++held;
  uint32_t seats = cfg_.max_batch > running_count_ + held ? cfg_.max_batch - running_count_ - held : 0;
  int32_t q_off = 0, k_off = 0;
  for (uint64_t id : waiting_) {
    if (budget == 0 || p.num_seqs >= cfg_.max_prefill_seqs) break;
    Req& r = reqs_.at(id);
    if (!r.reserved) {
      if (seats == 0) break;
      try {
        // without the prefix-cache flag nothing is ever committed, so nothing can hit
        PrefixReservation res = cache_->reserve_prompt(id, r.tokens.data(), r.prompt_len);
        r.computed = res.reusable_token_count;
        if (r.computed) {
          p.flags |= kDecisionPrefixCacheUsed;
          stats_.cached_prompt_tokens += r.computed;
          p.cached_prefix_tokens += r.computed;
        }
      } catch (const StatusError& e) {
        if (e.status == Status::CapacityExceeded) break;  // no KV room: wait for sequences to finish
        throw;
      }
      r.reserved = true;
      --seats;
    }
    const uint32_t remaining = r.prompt_len - r.computed;
    uint32_t chunk = std::min(remaining, budget);
    if (chunk < remaining && !(cfg_.flags & kSchedChunkedPrefill)) {
      if (p.num_seqs > 0) break;
      chunk = remaining;  // an unchunked prompt larger than the budget runs alone
    }
    if (chunk == 0) break;
    for (uint32_t t = r.computed; t < r.computed + chunk; ++t) {
      p.token_ids.push_back(int32_t(r.tokens[t]));
      p.positions.push_back(int32_t(t));
      p.slot_mapping.push_back(slot_of(r, id, t));
    }
    const uint32_t ctx = r.computed + chunk;
    for (uint32_t t = 0; t < ctx; ++t) p.ctx_slots.push_back(slot_of(r, id, t));
    if (r.computed > 0) p.has_prefix = true;
    q_off += int32_t(chunk);
    k_off += int32_t(ctx);
    p.cu_q.push_back(q_off);
    p.cu_k.push_back(k_off);
    p.logits_idx.push_back(q_off - 1);
    p.chunk_lens.push_back(int32_t(chunk));
    const bool final_chunk = ctx == r.prompt_len;
    p.emits_token.push_back(final_chunk ? 1 : 0);
    p.flags |= final_chunk ? kDecisionPrefillFinalChunk : kDecisionPrefillChunk;
    p.seq_ids.push_back(id);
    p.max_q = std::max(p.max_q, chunk);
    r.state = SlotState::RunningPrefill;
    ++p.num_seqs;
    budget -= chunk;
  }
  if (p.num_seqs == 0) return StepPlan{};
  p.num_tokens = (uint32_t)p.token_ids.size();
  p.padded_seqs = p.num_seqs;
  ++stats_.steps;
  ++stats_.prefill_steps;
  stats_.prefill_tokens += p.num_tokens;
  return p;
}

void Scheduler::preempt_one(uint64_t keep) {
  // the most recently admitted running sequence gives its blocks back and will
  // recompute its context through prefill
  uint64_t victim = 0;
  uint64_t newest = 0;
  for (uint64_t id : running_) {
    if (id == keep) continue;
    const Req& r = reqs_.at(id);
    if (r.arrival > newest) { newest = r.arrival; victim = id; }
  }
  if (newest == 0) victim = keep;
  Req& r = reqs_.at(victim);
  cache_->release_sequence(victim);
  r.reserved = false;
  r.computed = 0;
  r.prompt_len = (uint32_t)r.tokens.size();
  r.state = SlotState::QueuedPrefill;
  running_.erase(std::find(running_.begin(), running_.end(), victim));
  --running_count_;
  waiting_.push_front(victim);
  ++stats_.preemptions;
}

StepPlan Scheduler::build_decode() {
  StepPlan p;
  p.kind = StepPlan::Decode;
  p.flags = kDecisionDecodeStep;
  p.step_index = ++step_clock_;
  // make room for every running sequence's next token, preempting if needed
  for (size_t i = 0; i < running_.size();) {
    const uint64_t id = running_[i];
    Req& r = reqs_.at(id);
    try {
      cache_->ensure_sequence_token_capacity(id, (uint32_t)r.tokens.size());
      ++i;
    } catch (const StatusError& e) {
      if (e.status != Status::CapacityExceeded) throw;
      const size_t before = running_.size();
      preempt_one(id);
      p.flags |= kDecisionPreempted;
      if (running_.size() == before) break;
      if (std::find(running_.begin(), running_.end(), id) == running_.end()) continue;  // we were the victim
      i = 0;  // restart: indices shifted
    }
  }
  const uint32_t n = std::min<uint32_t>((uint32_t)running_.size(), cfg_.max_batch);
  if (n == 0) return StepPlan{};
  const uint32_t padded = bucket_for(n);
  if (padded != n) p.flags |= kDecisionCudaGraphPadding;
  p.num_seqs = n;
  p.padded_seqs = padded;
  p.max_blocks = max_blocks_;
  p.token_ids.assign(padded, 0);
  p.positions.assign(padded, 0);
  p.slot_mapping.assign(padded, -1);
  p.context_lens.assign(padded, 0);
  p.block_table.assign(size_t(padded) * max_blocks_, 0);
  for (uint32_t i = 0; i < n; ++i) {
    const uint64_t id = running_[i];
    Req& r = reqs_.at(id);
    const uint32_t len = (uint32_t)r.tokens.size();
    p.seq_ids.push_back(id);
    p.token_ids[i] = int32_t(r.tokens.back());
    p.positions[i] = int32_t(len - 1);
    p.slot_mapping[i] = slot_of(r, id, len - 1);
    p.context_lens[i] = int32_t(len);
    const auto& blocks = cache_->block_list(id);
    std::copy(blocks.begin(), blocks.end(), p.block_table.begin() + size_t(i) * max_blocks_);
    p.max_context = std::max(p.max_context, len);
    r.state = SlotState::RunningDecode;
  }
  p.num_tokens = n;
  ++stats_.steps;
  ++stats_.decode_steps;
  stats_.decode_tokens += n;
  return p;
}

StepPlan Scheduler::schedule_ahead(const StepPlan& inflight) {
  if (inflight.kind != StepPlan::Decode) return StepPlan{};
  // the policy would run a prefill next (a waiting prompt and a free seat)
  if (!waiting_.empty() && running_count_ < cfg_.max_batch) return StepPlan{};
  // the decode set must be the in-flight step's live sequences, in order
  std::vector<uint32_t> rows;
  rows.reserve(inflight.num_seqs);
  for (uint32_t i = 0; i < inflight.num_seqs; ++i)
    if (reqs_.count(inflight.seq_ids[i])) rows.push_back(i);
  if (rows.size() != running_.size()) return StepPlan{};
  for (size_t k = 0; k < rows.size(); ++k)
    if (running_[k] != inflight.seq_ids[rows[k]]) return StepPlan{};
  // keep the sequences that cannot end by length or context at the in-flight step
  std::vector<uint32_t> keep;
  for (uint32_t i : rows) {
    const uint64_t id = inflight.seq_ids[i];
    const Req& r = reqs_.at(id);
    const uint32_t len = (uint32_t)r.tokens.size();
    if (r.generated + 1 >= r.spec.max_new_tokens || len + 1 >= cfg_.max_model_len) continue;
    try {
      cache_->ensure_sequence_token_capacity(id, len + 1);
    } catch (const StatusError& e) {
      if (e.status == Status::CapacityExceeded) return StepPlan{};  // the synchronous path preempts
      throw;
    }
    keep.push_back(i);
  }
  const uint32_t n = (uint32_t)keep.size();
  if (n == 0) return StepPlan{};
  StepPlan p;
  p.kind = StepPlan::Decode;
  p.flags = kDecisionDecodeStep | kDecisionScheduledAhead;
  p.step_index = ++step_clock_;
  const uint32_t padded = bucket_for(n);
  if (padded != n) p.flags |= kDecisionCudaGraphPadding;
  p.num_seqs = n;
  p.padded_seqs = padded;
  p.max_blocks = max_blocks_;
  p.token_ids.assign(padded, 0);
  p.src_rows.assign(padded, -1);
  p.positions.assign(padded, 0);
  p.slot_mapping.assign(padded, -1);
  p.context_lens.assign(padded, 0);
  p.block_table.assign(size_t(padded) * max_blocks_, 0);
  for (uint32_t k = 0; k < n; ++k) {
    const uint64_t id = inflight.seq_ids[keep[k]];
    const Req& r = reqs_.at(id);
    const uint32_t pos = (uint32_t)r.tokens.size();  // the in-flight step's token lands here
    p.seq_ids.push_back(id);
    p.token_ids[k] = int32_t(keep[k]);
    p.src_rows[k] = int32_t(keep[k]);
    p.positions[k] = int32_t(pos);
    p.slot_mapping[k] = slot_of(r, id, pos);
    p.context_lens[k] = int32_t(pos + 1);
    const auto& blocks = cache_->block_list(id);
    std::copy(blocks.begin(), blocks.end(), p.block_table.begin() + size_t(k) * max_blocks_);
    p.max_context = std::max(p.max_context, pos + 1);
  }
  p.num_tokens = n;
  ++stats_.steps;
  ++stats_.decode_steps;
  stats_.decode_tokens += n;
  return p;
}

namespace {
uint64_t mix64(uint64_t z) {  // SplitMix64 finaliser (Steele, Lea & Flood, OOPSLA 2014)
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
}  // namespace

bool Scheduler::sampling_rows(const StepPlan& p, float* temp, uint64_t* key, uint32_t rows) const {
  bool any = false;
  for (uint32_t i = 0; i < rows; ++i) {
    temp[i] = 0.f;
    key[i] = 0;
    if (i >= p.num_seqs) continue;
    auto it = reqs_.find(p.seq_ids[i]);
    if (it == reqs_.end() || it->second.spec.temperature <= 0.f) continue;
    // position of the token whose successor this row samples
    int32_t pos = p.kind == StepPlan::Prefill ? p.positions[size_t(p.cu_q[i + 1]) - 1] : p.positions[i];
    temp[i] = it->second.spec.temperature;
    key[i] = mix64(it->second.spec.seed ^ mix64(uint64_t(uint32_t(pos)) + 1));
    any = true;
  }
  return any;
}

void Scheduler::finish(Req& r, uint64_t id, FinishReason why, std::vector<SchedEvent>& ev) {
  if (r.reserved) cache_->release_sequence(id);
  r.reserved = false;
  r.state = why == FinishReason::Cancelled ? SlotState::Cancelled : SlotState::Completed;
  auto it = std::find(running_.begin(), running_.end(), id);
  if (it != running_.end()) {
    running_.erase(it);
    --running_count_;
  }
  auto wt = std::find(waiting_.begin(), waiting_.end(), id);
  if (wt != waiting_.end()) waiting_.erase(wt);
  ev.push_back(SchedEvent{SchedEvent::Finished, id, -1, uint32_t(why), r.generated});
  if (why == FinishReason::Cancelled) ++stats_.cancelled;
  else ++stats_.finished;
  reqs_.erase(id);
}

std::vector<SchedEvent> Scheduler::complete(const StepPlan& p, const int32_t* sampled, uint32_t n_sampled) {
  std::vector<SchedEvent> ev;
  if (p.kind == StepPlan::None) return ev;
  if (n_sampled < p.num_seqs) fail(Status::InvalidArgument, "Scheduler: fewer sampled tokens than sequences");
  for (uint32_t i = 0; i < p.num_seqs; ++i) {
    const uint64_t id = p.seq_ids[i];
    auto it = reqs_.find(id);
    if (it == reqs_.end()) continue;  // cancelled while the step ran
    Req& r = it->second;
    bool emits;
    if (p.kind == StepPlan::Prefill) {
      r.computed += uint32_t(p.chunk_lens[i]);
      emits = p.emits_token[i] != 0;
      if (!emits) {
        r.state = SlotState::QueuedPrefill;
        if (cfg_.flags & kSchedPrefixCache) cache_->commit(id, r.computed);
        ev.push_back(SchedEvent{SchedEvent::PrefillProgress, id, -1, 0, r.computed});
        continue;
      }
      // the prompt is done: move from the prefill queue to the decode set
      auto wt = std::find(waiting_.begin(), waiting_.end(), id);
      if (wt != waiting_.end()) waiting_.erase(wt);
      running_.push_back(id);
      ++running_count_;
    } else {
      r.computed = (uint32_t)r.tokens.size();
      emits = true;
    }
    if (cfg_.flags & kSchedPrefixCache) cache_->commit(id, r.computed);
    const int32_t tok = sampled[i];
    r.tokens.push_back(uint32_t(tok));
    cache_->append_tokens(id, reinterpret_cast<const uint32_t*>(&tok), 1);
    ++r.generated;
    r.state = SlotState::ReadyDecode;
    ev.push_back(SchedEvent{SchedEvent::Token, id, tok, 0, r.generated});
    FinishReason why = FinishReason::None;
    if (!r.spec.ignore_eos && std::find(r.spec.stop_token_ids.begin(), r.spec.stop_token_ids.end(), uint32_t(tok)) !=
                                  r.spec.stop_token_ids.end())
      why = FinishReason::Stop;
    else if (r.generated >= r.spec.max_new_tokens)
      why = FinishReason::Length;
    else if (r.tokens.size() >= cfg_.max_model_len)
      why = FinishReason::ContextLimit;
    if (why != FinishReason::None) finish(r, id, why, ev);
  }
  return ev;
}

bool Scheduler::cancel(uint64_t id) {
  auto it = reqs_.find(id);
  if (it == reqs_.end()) return false;
  std::vector<SchedEvent> ev;
  finish(it->second, id, FinishReason::Cancelled, ev);
  return true;
}

void Scheduler::fail_step(const StepPlan& p) {
  for (uint32_t i = 0; i < p.num_seqs; ++i) cancel(p.seq_ids[i]);
}

}  // namespace spc
