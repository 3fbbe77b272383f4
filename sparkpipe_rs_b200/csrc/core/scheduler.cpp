#include "scheduler.h"

#include <algorithm>

#include "work_control.h"

namespace spc {

Scheduler::Scheduler(const SchedulerConfig& cfg) : cfg_(cfg) {
  if (cfg.max_batch == 0 || cfg.max_prefill_tokens == 0 || cfg.block_tokens == 0 || cfg.num_blocks == 0 ||
      cfg.max_model_len < 2 || cfg.max_sequences == 0)
    fail(Status::InvalidArgument, "Scheduler: invalid configuration");
  std::sort(cfg_.decode_buckets.begin(), cfg_.decode_buckets.end());
  if (cfg.spec_mode > uint32_t(SpecMode::MtpTree)) fail(Status::InvalidArgument, "Scheduler: unknown speculation mode");
  if (cfg.spec_mode == uint32_t(SpecMode::Chain) &&
      (cfg.spec_draft_len == 0 || cfg.spec_draft_len > spec::kMaxSpeculativeTokens))
    fail(Status::InvalidArgument, "Scheduler: chain draft length must be 1..7");
  if (cfg.spec_mode == uint32_t(SpecMode::MtpTree) && cfg.spec_shadow_slot_base < 0)
    fail(Status::InvalidArgument, "Scheduler: tree speculation needs shadow slots");
  cache_ = std::make_unique<PrefixCache>(cfg.block_tokens, cfg.num_blocks, cfg.max_sequences);
  max_blocks_ = (cfg.max_model_len + cfg.block_tokens - 1) / cfg.block_tokens;
  for (uint32_t i = cfg.host_blocks; i > 0; --i) host_free_.push_back(i - 1);
  if (cfg.host_prefix_blocks) cache_->enable_host_tier(cfg.host_blocks, cfg.host_prefix_blocks);
}

uint32_t Scheduler::full_budget() const {
  return cfg_.spec_mode == uint32_t(SpecMode::MtpTree) ? wc::mtp::kCandidates : cfg_.spec_draft_len;
}

uint32_t Scheduler::spec_rows_per_seq() const {
  if (cfg_.spec_mode == uint32_t(SpecMode::MtpTree)) return wc::mtp::kVerifierRows;
  if (cfg_.spec_mode == uint32_t(SpecMode::Chain)) return cfg_.spec_draft_len + 1;
  return 1;
}

uint64_t Scheduler::estimate_step_ns(uint32_t kind, uint32_t seqs) const {
  return cost_.estimate(kind, bucket_for(seqs), kind == StepPlan::Verify ? spec_rows_per_seq() : 1);
}

spec::LaneState Scheduler::lane_state(uint64_t id) const {
  auto it = reqs_.find(id);
  if (it == reqs_.end()) fail(Status::NotFound, "Scheduler: unknown request");
  return it->second.lane;
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
  r.lane.disabled = spec.disable_speculation || spec.temperature > 0.f || cfg_.spec_mode == 0;
  r.lane.budget = r.lane.disabled ? 0 : full_budget();
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

void Scheduler::attach_swaps(StepPlan& p) {
  // prefix blocks demoted to / promoted from the cache's host tier while planning
  const size_t o0 = pending_out_.size(), i0 = pending_in_.size();
  cache_->take_tier_copies(pending_out_, pending_in_);
  stats_.prefix_tier_out_blocks += (pending_out_.size() - o0) / 2;
  stats_.prefix_tier_in_blocks += (pending_in_.size() - i0) / 2;
  if (pending_out_.empty() && pending_in_.empty()) return;
  p.swap_out = std::move(pending_out_);
  p.swap_in = std::move(pending_in_);
  pending_out_.clear();
  pending_in_.clear();
  p.flags |= kDecisionSwap;
}

StepPlan Scheduler::schedule() {
  // host slots read by the previous plan's restores are ordered before any copy
  // this plan issues, so they can be handed out again
  host_free_.insert(host_free_.end(), host_release_.begin(), host_release_.end());
  host_release_.clear();
  cache_->release_deferred_slots();
  resume_swapped();
  StepPlan p = schedule_step();
  attach_swaps(p);
  return p;
}

StepPlan Scheduler::schedule_step() {
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
    StepPlan d = build_decode();
    if (cfg_.spec_mode && d.kind == StepPlan::Decode) {
      StepPlan v = try_build_verify(d);
      if (v.kind == StepPlan::Verify) return v;
    }
    return d;
  }
  return StepPlan{};
}

const std::vector<uint64_t>& Scheduler::prompt_hashes(Req& r) {
  // full blocks of the reusable part of the prompt (all but its last token)
  const uint32_t bt = cfg_.block_tokens, nb = r.prompt_len ? (r.prompt_len - 1) / bt : 0;
  if (r.block_hashes.size() != nb) {
    r.block_hashes.clear();
    uint64_t h = kEmptyParentHash;
    for (uint32_t b = 0; b < nb; ++b) {
      h = prefix_hash_block(r.tokens.data() + size_t(b) * bt, bt, h);
      r.block_hashes.push_back(h);
    }
  }
  return r.block_hashes;
}

std::vector<uint64_t> Scheduler::family_followers() {
  // Requests whose prompts share a block-aligned prefix that nobody has cached yet
  // form a family per shared prefix length; the best family (highest priority, then
  // most prompt tokens saved = shared x (members - 1), more members, longer prefix,
  // earlier leader) prefills its leader alone and holds its followers back until the
  // leader's KV for the shared prefix is in the cache, where they find it. A request
  // already in chunked prefill leads any family it is in.
  struct Group {
    uint32_t blocks = 0, count = 0, prio = 0;
    uint64_t leader = 0, leader_arrival = ~0ull;
    bool leader_running = false;
    std::vector<uint64_t> members;
  };
  std::unordered_map<uint64_t, Group> groups;
  uint32_t scanned = 0;
  for (uint64_t id : waiting_) {
    if (++scanned > 256) break;
    Req& r = reqs_.at(id);
    const auto& hs = prompt_hashes(r);
    const uint32_t from = r.reserved ? r.computed / cfg_.block_tokens : cache_->cached_prefix_blocks(hs);
    for (uint32_t k = from; k < hs.size(); ++k) {
      Group& g = groups[hs[k]];
      g.blocks = k + 1;
      ++g.count;
      g.prio = std::max(g.prio, r.spec.priority);
      g.members.push_back(id);
      const bool better = r.reserved != g.leader_running ? r.reserved
                          : g.leader == 0 || r.spec.priority > reqs_.at(g.leader).spec.priority ||
                                (r.spec.priority == reqs_.at(g.leader).spec.priority && r.arrival < g.leader_arrival);
      if (better) {
        g.leader = id;
        g.leader_arrival = r.arrival;
        g.leader_running = r.reserved;
      }
    }
  }
  const Group* best = nullptr;
  for (const auto& kv : groups) {
    const Group& g = kv.second;
    if (g.count < 2) continue;
    if (!best) { best = &g; continue; }
    const uint64_t sg = uint64_t(g.blocks) * (g.count - 1), sb = uint64_t(best->blocks) * (best->count - 1);
    if (g.prio != best->prio ? g.prio > best->prio
        : sg != sb           ? sg > sb
        : g.count != best->count ? g.count > best->count
        : g.blocks != best->blocks ? g.blocks > best->blocks
                                   : g.leader_arrival < best->leader_arrival)
      best = &g;
  }
  std::vector<uint64_t> hold;
  if (!best) return hold;
  for (uint64_t id : best->members)
    if (id != best->leader && !reqs_.at(id).reserved) hold.push_back(id);
  if (!hold.empty()) ++stats_.family_steps;
  return hold;
}

StepPlan Scheduler::build_prefill() {
  StepPlan p;
  p.kind = StepPlan::Prefill;
  p.flags = kDecisionPrefillStep;
  p.step_index = ++step_clock_;
  p.cu_q.push_back(0);
  p.cu_k.push_back(0);
  const bool caching = cfg_.flags & kSchedPrefixCache;
  if (caching && (cfg_.flags & kSchedLookaheadProtection)) {
    cache_->reset_lookahead_protection();
    uint32_t k = 0;
    for (uint64_t id : waiting_) {
      if (k++ >= cfg_.lookahead_requests) break;
      Req& r = reqs_.at(id);
      if (!r.reserved)
        stats_.lookahead_protected_blocks +=
            cache_->protect_prompt_lookahead(r.tokens.data(), r.prompt_len, r.spec.priority);
    }
  }
  std::vector<uint64_t> hold;
  if (caching && (cfg_.flags & kSchedPrefixCohorting)) hold = family_followers();
  for (uint64_t id : waiting_) {
    Req& r = reqs_.at(id);
    if (r.state == SlotState::WaitingPrefixCohort) r.state = SlotState::QueuedPrefill;
  }
  uint32_t budget = cfg_.max_prefill_tokens;
  uint32_t held = 0;  // waiting sequences that already hold a decode seat
  for (uint64_t id : waiting_)
    if (reqs_.at(id).reserved) ++held;
  uint32_t seats = cfg_.max_batch > running_count_ + held ? cfg_.max_batch - running_count_ - held : 0;
  int32_t q_off = 0, k_off = 0;
  for (uint64_t id : waiting_) {
    if (budget == 0 || p.num_seqs >= cfg_.max_prefill_seqs) break;
    Req& r = reqs_.at(id);
    if (!r.reserved && std::find(hold.begin(), hold.end(), id) != hold.end()) {
      r.state = SlotState::WaitingPrefixCohort;  // its prefix is being prefilled by the family's leader
      p.flags |= kDecisionPrefixFamily;
      ++stats_.family_deferrals;
      continue;
    }
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
  if (cfg_.host_blocks && swap_out(victim)) return;
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

bool Scheduler::swap_out(uint64_t id) {
  Req& r = reqs_.at(id);
  const uint32_t kv_blocks = (r.computed + cfg_.block_tokens - 1) / cfg_.block_tokens;
  if (kv_blocks > host_free_.size()) return false;
  const auto& blocks = cache_->block_list(id);
  r.host_slots.clear();
  for (uint32_t b = 0; b < kv_blocks; ++b) {
    const uint32_t slot = host_free_.back();
    host_free_.pop_back();
    r.host_slots.push_back(slot);
    pending_out_.push_back(int32_t(blocks[b]));
    pending_out_.push_back(int32_t(slot));
  }
  // the copies run before this plan's step, so the blocks may be reused by it
  cache_->release_sequence(id);
  r.reserved = false;
  r.state = SlotState::Swapped;
  running_.erase(std::find(running_.begin(), running_.end(), id));
  --running_count_;
  swapped_.push_back(id);
  ++stats_.swapped_out;
  ++stats_.preemptions;
  stats_.swap_out_blocks += kv_blocks;
  return true;
}

void Scheduler::resume_swapped() {
  while (!swapped_.empty() && running_count_ < cfg_.max_batch) {
    const uint64_t id = swapped_.front();
    Req& r = reqs_.at(id);
    const uint32_t len = (uint32_t)r.tokens.size();
    PrefixReservation res;
    try {
      // blocks for every token; a cached prefix is bound instead of restored
      res = cache_->reserve_prompt(id, r.tokens.data(), len);
    } catch (const StatusError& e) {
      if (e.status == Status::CapacityExceeded) break;
      throw;
    }
    const uint32_t bt = cfg_.block_tokens;
    const uint32_t hit = res.reusable_token_count / bt, kv_blocks = (r.computed + bt - 1) / bt;
    const auto& blocks = cache_->block_list(id);
    for (uint32_t b = hit; b < kv_blocks; ++b) {
      pending_in_.push_back(int32_t(r.host_slots[b]));
      pending_in_.push_back(int32_t(blocks[b]));
    }
    stats_.swap_in_blocks += kv_blocks > hit ? kv_blocks - hit : 0;
    host_release_.insert(host_release_.end(), r.host_slots.begin(), r.host_slots.end());
    r.host_slots.clear();
    r.reserved = true;
    r.state = r.lane.budget ? SlotState::ReadySpeculativeVerify : SlotState::ReadyDecode;
    running_.push_back(id);
    ++running_count_;
    swapped_.pop_front();
    ++stats_.swapped_in;
  }
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

namespace {
uint64_t mix64(uint64_t z) {  // SplitMix64 finaliser (Steele, Lea & Flood, OOPSLA 2014)
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
}  // namespace

bool Scheduler::spec_grants(const std::vector<uint64_t>& ids, std::vector<uint32_t>& grant) const {
  const bool tree = cfg_.spec_mode == uint32_t(SpecMode::MtpTree);
  const uint32_t n = (uint32_t)ids.size(), full = full_budget();
  if (!cfg_.spec_mode || n == 0) return false;
  std::vector<spec::SlotInput> in(n);
  for (uint32_t i = 0; i < n; ++i) {
    const Req& r = reqs_.at(ids[i]);
    const uint32_t len = (uint32_t)r.tokens.size();
    const uint32_t remaining = r.spec.max_new_tokens > r.generated ? r.spec.max_new_tokens - r.generated : 0;
    uint32_t depth = spec::max_depth(r.lane, full);
    // a round commits at most depth + 1 tokens, within the length budget and the context
    if (tree) {
      if (remaining < wc::mtp::kMaxCommitted + 1 || len + wc::mtp::kMaxCommitted > cfg_.max_model_len) depth = 0;
    } else {
      depth = std::min(depth, remaining ? remaining - 1 : 0);
      depth = std::min(depth, cfg_.max_model_len > len ? cfg_.max_model_len - len - 1 : 0);
    }
    in[i] = spec::SlotInput{r.lane.ema_milli, depth, 0};
  }
  const uint32_t rows = spec_rows_per_seq();
  const uint32_t cap = cfg_.spec_row_cap ? cfg_.spec_row_cap : rows * cfg_.max_batch;
  spec::row_allocator_assign(in, cap, cfg_.spec_row_cost_milli, grant);
  bool any = false, all = true;
  for (uint32_t g : grant) {
    any |= g > 0;
    all &= g == full;
  }
  // the tree verifies a batch only when every lane drafts the full tree
  if (tree ? !all : !any) return false;
  if (cfg_.flags & kSchedMtpForceEnable) return true;
  const uint64_t plain = estimate_step_ns(StepPlan::Decode, n), round = estimate_step_ns(StepPlan::Verify, n);
  return spec::outranks_plain(spec::expected_committed_scaled(spec_), n, n, plain, round);
}

StepPlan Scheduler::try_build_verify(const StepPlan& d) {
  const bool tree = cfg_.spec_mode == uint32_t(SpecMode::MtpTree);
  const uint32_t n = d.num_seqs, Bp = d.padded_seqs, rows = spec_rows_per_seq();
  std::vector<uint32_t> grant;
  if (!spec_grants(d.seq_ids, grant)) return StepPlan{};
  // KV blocks for every position a lane's rows write; without them this step decodes plainly
  for (uint32_t i = 0; i < n; ++i) {
    if (!grant[i]) continue;
    const Req& r = reqs_.at(d.seq_ids[i]);
    const uint32_t ext = tree ? wc::mtp::kContextExtension : grant[i];
    try {
      cache_->ensure_sequence_token_capacity(d.seq_ids[i], (uint32_t)r.tokens.size() + ext);
    } catch (const StatusError& e) {
      if (e.status == Status::CapacityExceeded) return StepPlan{};
      throw;
    }
  }
  StepPlan v;
  v.kind = StepPlan::Verify;
  v.flags = kDecisionDecodeStep | kDecisionSpeculativeVerify | (tree ? kDecisionMtpTreeVerify : 0u) |
            (d.flags & (kDecisionCudaGraphPadding | kDecisionPreempted));
  v.step_index = d.step_index;
  v.num_seqs = n;
  v.padded_seqs = Bp;
  v.max_blocks = max_blocks_;
  v.rows_per_seq = rows;
  v.seq_ids = d.seq_ids;
  v.block_table.assign(size_t(Bp) * max_blocks_, 0);
  const size_t R = size_t(rows) * Bp;
  v.token_ids.assign(R, 0);
  v.positions.assign(R, 0);
  v.slot_mapping.assign(R, -1);
  v.context_lens.assign(R, 0);
  v.draft_budget.assign(Bp, 0);
  v.accept_keys.assign(Bp, 0);
  if (tree) {
    v.sync_token_ids.assign(size_t(3) * Bp, 0);
    v.sync_positions.assign(size_t(3) * Bp, 0);
    v.sync_slots.assign(size_t(3) * Bp, -1);
  }
  for (uint32_t b = 0; b < n; ++b) {
    const uint64_t id = d.seq_ids[b];
    Req& r = reqs_.at(id);
    const uint32_t len = (uint32_t)r.tokens.size(), p = len - 1;
    const auto& blocks = cache_->block_list(id);
    std::copy(blocks.begin(), blocks.end(), v.block_table.begin() + size_t(b) * max_blocks_);
    v.draft_budget[b] = int32_t(grant[b]);
    v.accept_keys[b] = mix64(id);
    v.token_ids[b] = int32_t(r.tokens.back());
    for (uint32_t j = 0; j < rows; ++j) {
      if (!tree && j > grant[b]) break;  // rows past the lane's budget stay idle
      const uint32_t depth = tree ? wc::mtp::node_at(j)->depth : j;
      const uint32_t q = p + depth;
      const size_t row = size_t(j) * Bp + b;
      v.positions[row] = int32_t(q);
      v.context_lens[row] = int32_t(q + 1);
      // the tree's alternate leaves (rows 3 and 5) share a position with a primary
      // row: their KV goes to this batch row's shadow slots
      if (tree && (j == 3 || j == 5))
        v.slot_mapping[row] = int32_t(cfg_.spec_shadow_slot_base + 2 * int64_t(b) + (j == 5 ? 1 : 0));
      else
        v.slot_mapping[row] = slot_of(r, id, q);
    }
    if (tree) {
      for (uint32_t k = 0; k < 3; ++k) {
        if (p < 3 - k) continue;
        const uint32_t q = p - 3 + k;
        const size_t row = size_t(k) * Bp + b;
        v.sync_token_ids[row] = int32_t(r.tokens[q]);
        v.sync_positions[row] = int32_t(q);
        v.sync_slots[row] = slot_of(r, id, q);
      }
    }
    v.max_context = std::max(v.max_context, p + (tree ? wc::mtp::kContextExtension : grant[b]) + 1);
    r.state = SlotState::RunningSpeculativeVerify;
  }
  v.num_tokens = n;
  --stats_.decode_steps;
  ++stats_.verify_steps;
  return v;
}

StepPlan Scheduler::schedule_ahead(const StepPlan& inflight) {
  if (inflight.kind != StepPlan::Decode) return StepPlan{};
  if (!swapped_.empty() || !pending_out_.empty() || !pending_in_.empty()) return StepPlan{};
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
  if (cfg_.spec_mode) {  // the next step may be a verify round, which needs this step's tokens
    std::vector<uint32_t> grant;
    if (spec_grants(running_, grant)) return StepPlan{};
  }
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
  if (n == 0) {
    if (cache_->has_tier_copies()) {  // copies already planned must still reach the engine
      StepPlan none;
      attach_swaps(none);
      return none;
    }
    return StepPlan{};
  }
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
  cache_->release_deferred_slots();
  attach_swaps(p);
  return p;
}

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
  if (r.state == SlotState::Swapped) {
    host_release_.insert(host_release_.end(), r.host_slots.begin(), r.host_slots.end());
    r.host_slots.clear();
    swapped_.erase(std::find(swapped_.begin(), swapped_.end(), id));
  }
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
      if (cfg_.spec_mode && !r.lane.disabled) {
        const bool was = r.lane.budget == 0 && r.lane.countdown != 0;
        spec::observe_plain(r.lane, 1, full_budget());
        if (was && r.lane.budget) ++spec_.reprobes;
      }
    }
    if (cfg_.flags & kSchedPrefixCache) cache_->commit(id, r.computed);
    const int32_t tok = sampled[i];
    r.tokens.push_back(uint32_t(tok));
    cache_->append_tokens(id, reinterpret_cast<const uint32_t*>(&tok), 1);
    ++r.generated;
    r.state = r.lane.budget ? SlotState::ReadySpeculativeVerify : SlotState::ReadyDecode;
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

std::vector<SchedEvent> Scheduler::complete_verify(const StepPlan& p, const int32_t* committed, uint32_t stride,
                                                   const int32_t* counts, const int32_t* paths, uint32_t n) {
  std::vector<SchedEvent> ev;
  if (p.kind != StepPlan::Verify) fail(Status::InvalidArgument, "Scheduler: complete_verify needs a verify plan");
  if (n < p.num_seqs || stride < p.rows_per_seq) fail(Status::InvalidArgument, "Scheduler: verify results too short");
  const bool tree = p.flags & kDecisionMtpTreeVerify;
  if (tree && !paths) fail(Status::InvalidArgument, "Scheduler: tree verify needs resolution paths");
  const uint32_t full = full_budget();
  for (uint32_t i = 0; i < p.num_seqs; ++i) {  // validate every lane before applying any
    const uint32_t c = uint32_t(counts[i]), g = uint32_t(p.draft_budget[i]);
    if (counts[i] <= 0 || c > g + 1) fail(Status::InvalidArgument, "Scheduler: committed token count out of range");
    if (tree && (c > wc::mtp::kMaxCommitted ||
                 !wc::mtp::resolution_is_valid(wc::mtp::kCandidates, c - 1, uint32_t(paths[i]))))
      fail(Status::InvalidArgument, "Scheduler: invalid tree resolution");
  }
  ++spec_.verify_steps;
  for (uint32_t i = 0; i < p.num_seqs; ++i) {
    const uint64_t id = p.seq_ids[i];
    auto it = reqs_.find(id);
    if (it == reqs_.end()) continue;  // cancelled while the round ran
    Req& r = it->second;
    const uint32_t c = uint32_t(counts[i]), g = uint32_t(p.draft_budget[i]);
    if (g > 0) {
      spec::observe_verify(r.lane, c, full);
      if (r.lane.budget == 0) ++spec_.suppressed;
      ++spec_.rounds;
      spec_.proposed += g;
      spec_.accepted += c - 1;
      spec_.committed += c;
    } else {
      const bool was = r.lane.budget == 0 && r.lane.countdown != 0;
      spec::observe_plain(r.lane, c, full);
      if (was && r.lane.budget) ++spec_.reprobes;
    }
    auto e = append_committed(r, id, committed + size_t(i) * stride, c);
    ev.insert(ev.end(), e.begin(), e.end());
  }
  return ev;
}

std::vector<SchedEvent> Scheduler::append_committed(Req& r, uint64_t id, const int32_t* toks, uint32_t c) {
  std::vector<SchedEvent> ev;
  // the cache now holds the KV of the input token and of the accepted drafts
  const uint32_t len = (uint32_t)r.tokens.size();
  for (uint32_t k = 0; k < c; ++k) {
    const int32_t tok = toks[k];
    r.tokens.push_back(uint32_t(tok));
    cache_->append_tokens(id, reinterpret_cast<const uint32_t*>(&tok), 1);
    ++r.generated;
    ev.push_back(SchedEvent{SchedEvent::Token, id, tok, 0, r.generated});
    FinishReason why = FinishReason::None;
    if (!r.spec.ignore_eos &&
        std::find(r.spec.stop_token_ids.begin(), r.spec.stop_token_ids.end(), uint32_t(tok)) !=
            r.spec.stop_token_ids.end())
      why = FinishReason::Stop;
    else if (r.generated >= r.spec.max_new_tokens)
      why = FinishReason::Length;
    else if (r.tokens.size() >= cfg_.max_model_len)
      why = FinishReason::ContextLimit;
    if (why != FinishReason::None) {
      finish(r, id, why, ev);
      return ev;
    }
  }
  r.computed = len + c - 1;
  if (cfg_.flags & kSchedPrefixCache) cache_->commit(id, r.computed);
  r.state = r.lane.budget ? SlotState::ReadySpeculativeVerify : SlotState::ReadyDecode;
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
