#include "work_control.h"

#include <cstring>

#include <algorithm>

namespace spc {
namespace wc {

uint64_t fingerprint_bytes(const uint8_t* d, size_t n) {
  if (n == 0) return 0;
  const uint64_t h = fnv1a64(d, n, 14695981039346656037ull);
  return h == 0 ? 1 : h;
}

void validate_identity(const Identity& i) {
  if (!i.control_generation || !i.transaction_id || !i.dispatch_generation || !i.request_generation ||
      !i.step_generation || !i.step_chunk_count || i.step_chunk_index >= i.step_chunk_count ||
      i.transaction_phase < kPhasePrefill || i.transaction_phase > kPhaseCancel)
    fail(Status::InvalidArgument, "work control: invalid transaction identity");
}

// ----------------------------------------------------------------- MTP tree
namespace mtp {
// row: parent, depth, candidate, first child row, child count
static const Node kNodes[kVerifierRows] = {
    {0, 0, 0, 1, 1}, {0, 1, 0, 2, 2}, {1, 2, 1, 4, 2}, {1, 2, 2, 0, 0}, {2, 3, 3, 0, 0}, {2, 3, 4, 0, 0},
};
const Node* node_at(uint32_t r) { return r < kVerifierRows ? &kNodes[r] : nullptr; }
uint32_t accepted_token_count(uint32_t p) { return node_at(p) ? node_at(p)->depth : 0; }
uint32_t fallback_row_index(uint32_t p) { return node_at(p) ? p : 0; }
uint32_t tail_candidate_index(uint32_t p) { return node_at(p) ? node_at(p)->candidate_index : 0; }
uint32_t tail_parent_row_index(uint32_t p) { return node_at(p) ? node_at(p)->parent_row : 0; }
uint32_t tail_base_position_offset(uint32_t p) {
  const uint32_t a = accepted_token_count(p);
  return a ? a - 1 : 0;
}
bool resolution_is_valid(uint32_t proposed, uint32_t accepted, uint32_t path) {
  if (accepted > proposed) return false;
  if (proposed == 0) return accepted == 0 && path == kResolutionNone;
  if (proposed != kCandidates) return path == kResolutionNone;
  if (path >= kVerifierRows) return false;
  return accepted == accepted_token_count(path);
}
bool topology_is_valid() {
  if (kNodes[0].depth != 0 || kNodes[0].parent_row != 0) return false;
  uint32_t seen = 0, max_depth = 0;
  for (uint32_t r = 1; r < kVerifierRows; ++r) {
    const Node& n = kNodes[r];
    const Node& p = kNodes[n.parent_row];
    if (n.parent_row >= r || n.depth != p.depth + 1 || n.candidate_index >= kCandidates ||
        (seen & (1u << n.candidate_index)))
      return false;
    seen |= 1u << n.candidate_index;
    max_depth = std::max<uint32_t>(max_depth, n.depth);
  }
  if (seen != (1u << kCandidates) - 1 || max_depth != kContextExtension || max_depth + 1 != kMaxCommitted)
    return false;
  for (uint32_t r = 0; r < kVerifierRows; ++r) {
    const Node& n = kNodes[r];
    if (!n.child_count) continue;
    if (n.child_row_base <= r || n.child_row_base + n.child_count > kVerifierRows) return false;
    for (uint32_t c = 0; c < n.child_count; ++c)
      if (kNodes[n.child_row_base + c].parent_row != r) return false;
  }
  return true;
}
Resolution resolve(const uint32_t* cand, const uint32_t* ver, uint32_t vocab) {
  for (uint32_t i = 0; i < kCandidates; ++i)
    if (cand[i] >= vocab) fail(Status::InvalidArgument, "mtp resolve: candidate token out of range");
  for (uint32_t i = 0; i < kVerifierRows; ++i)
    if (ver[i] >= vocab) fail(Status::InvalidArgument, "mtp resolve: verifier token out of range");
  uint32_t row = 0, path = kResolutionNone;
  for (bool matched = true; matched;) {
    matched = false;
    const Node& n = kNodes[row];
    for (uint32_t c = 0; c < n.child_count; ++c) {
      const uint32_t child = n.child_row_base + c;
      if (ver[row] != cand[kNodes[child].candidate_index]) continue;
      row = path = child;
      matched = true;
      break;
    }
  }
  const uint32_t acc = accepted_token_count(path);
  return Resolution{path, acc, acc + 1, fallback_row_index(path)};
}
}  // namespace mtp

// ----------------------------------------------------------------- packets
void Config::validate() const {
  if (!mtp_draft_token_count || !max_speculative_token_count || !maximum_context_tokens || !kv_block_tokens ||
      !max_prefill_tokens_per_packet || !output_vocab_count || !max_lane_count || !cohort_capacity ||
      maximum_context_tokens % kv_block_tokens)
    fail(Status::InvalidArgument, "work control: invalid configuration");
}

uint32_t select_batch_bucket(uint32_t n) {
  if (n == 0) fail(Status::InvalidArgument, "select_batch_bucket: zero sequences");
  for (uint32_t b = 16; b <= 1024; b *= 2)
    if (n <= b) return b;
  fail(Status::CapacityExceeded, "select_batch_bucket: more than 1024 sequences");
}

std::pair<uint32_t, uint32_t> execution_chunk_shape(uint32_t seqs, uint32_t rows, uint32_t cap, uint32_t max_bucket) {
  if (!seqs || !rows || !cap) fail(Status::InvalidArgument, "execution_chunk_shape: zero input");
  cap = std::min(cap, max_bucket);
  uint32_t per = cap / rows;
  if (!per) fail(Status::CapacityExceeded, "execution_chunk_shape: one sequence exceeds the row capacity");
  per = std::min(per, seqs);
  return {per, (seqs + per - 1) / per};
}

namespace {
struct Writer {
  std::vector<uint8_t> b;
  void u8(uint8_t v) { b.push_back(v); }
  void u16(uint16_t v) { u8(uint8_t(v)); u8(uint8_t(v >> 8)); }
  void u32(uint32_t v) { size_t o = b.size(); b.resize(o + 4); put_u32(&b[o], v); }
  void u64(uint64_t v) { size_t o = b.size(); b.resize(o + 8); put_u64(&b[o], v); }
};
struct Reader {
  const uint8_t* p;
  size_t n, o = 0;
  void need(size_t k) {
    if (o + k > n) fail(Status::ParseError, "work packet truncated");
  }
  uint8_t u8() { need(1); return p[o++]; }
  uint16_t u16() { uint16_t v = u8(); return uint16_t(v | (uint16_t(u8()) << 8)); }
  uint32_t u32() { need(4); uint32_t v = get_u32(p + o); o += 4; return v; }
  uint64_t u64() { need(8); uint64_t v = get_u64(p + o); o += 8; return v; }
};
}  // namespace

std::vector<uint8_t> serialize(const Packet& p) {
  Writer w;
  w.u32(p.magic);
  w.u32(p.abi_version);
  w.u32(0);  // total bytes, patched below
  w.u32(p.flags);
  const Identity& i = p.identity;
  w.u64(i.control_generation); w.u64(i.transaction_id); w.u64(i.dispatch_generation);
  w.u64(i.request_generation); w.u64(i.step_generation);
  w.u32(i.step_chunk_index); w.u32(i.step_chunk_count); w.u32(i.transaction_phase);
  w.u64(p.request_id); w.u64(p.sequence_id); w.u64(p.sequence_position); w.u64(p.deadline_time_ns);
  w.u32(p.active_sequence_count); w.u32(p.new_token_count); w.u32(p.pipeline_slot); w.u32(p.priority);
  w.u32(p.block_token_count); w.u32(p.max_blocks_per_sequence); w.u32(p.mtp_draft_token_count);
  w.u32(p.rows_per_lane); w.u32(p.execution_row_count); w.u32(p.execution_batch_bucket);
  w.u32((uint32_t)p.prefill_token_ids.size());
  for (uint32_t t : p.prefill_token_ids) w.u32(t);
  w.u32((uint32_t)p.lanes.size());
  for (const Lane& l : p.lanes) {
    w.u64(l.request_id); w.u64(l.request_generation); w.u64(l.step_generation); w.u64(l.sequence_id);
    w.u64(l.sequence_position);
    w.u32(l.request_slot_index); w.u32(l.context_token_count); w.u32(l.input_token_id);
    w.u32(l.mtp_draft_token_count); w.u32(l.speculative_token_count);
    w.u8(l.mtp_proposed); w.u8(l.mtp_accepted); w.u16(l.mtp_path_id);
    w.u32((uint32_t)l.speculative_draft_token_ids.size());
    for (uint32_t t : l.speculative_draft_token_ids) w.u32(t);
  }
  if (p.flags & kFlagExecutionPayload) {
    const ExecPayload& e = p.exec;
    auto ints = [&](const std::vector<int32_t>& v) {
      w.u32((uint32_t)v.size());
      for (int32_t x : v) w.u32(uint32_t(x));
    };
    ints(e.positions); ints(e.slots); ints(e.block_table); ints(e.context_lens);
    w.u32(e.block_table_cols);
    ints(e.cu_q); ints(e.cu_k); ints(e.ctx_slots); ints(e.logits_rows);
    w.u32(e.max_q);
    w.u32((uint32_t)e.temperature.size());
    for (float t : e.temperature) {
      uint32_t bits;
      std::memcpy(&bits, &t, 4);
      w.u32(bits);
    }
    w.u32((uint32_t)e.sample_keys.size());
    for (uint64_t k : e.sample_keys) w.u64(k);
  }
  put_u32(&w.b[8], (uint32_t)w.b.size());
  return w.b;
}

Packet deserialize(const uint8_t* d, size_t n) {
  Reader r{d, n};
  Packet p;
  p.magic = r.u32();
  p.abi_version = r.u32();
  const uint32_t total = r.u32();
  if (p.magic != kPacketMagic) fail(Status::ParseError, "work packet: bad magic");
  if (p.abi_version != kAbiVersion) fail(Status::AbiMismatch, "work packet: ABI version mismatch");
  if (total != n) fail(Status::ParseError, "work packet: length mismatch");
  p.flags = r.u32();
  Identity& i = p.identity;
  i.control_generation = r.u64(); i.transaction_id = r.u64(); i.dispatch_generation = r.u64();
  i.request_generation = r.u64(); i.step_generation = r.u64();
  i.step_chunk_index = r.u32(); i.step_chunk_count = r.u32(); i.transaction_phase = r.u32();
  p.request_id = r.u64(); p.sequence_id = r.u64(); p.sequence_position = r.u64(); p.deadline_time_ns = r.u64();
  p.active_sequence_count = r.u32(); p.new_token_count = r.u32(); p.pipeline_slot = r.u32(); p.priority = r.u32();
  p.block_token_count = r.u32(); p.max_blocks_per_sequence = r.u32(); p.mtp_draft_token_count = r.u32();
  p.rows_per_lane = r.u32(); p.execution_row_count = r.u32(); p.execution_batch_bucket = r.u32();
  const uint32_t np = r.u32();
  if (np > n / 4) fail(Status::ParseError, "work packet: prefill count");
  p.prefill_token_ids.resize(np);
  for (auto& t : p.prefill_token_ids) t = r.u32();
  const uint32_t nl = r.u32();
  if (nl > n / 64) fail(Status::ParseError, "work packet: lane count");
  p.lanes.resize(nl);
  for (Lane& l : p.lanes) {
    l.request_id = r.u64(); l.request_generation = r.u64(); l.step_generation = r.u64(); l.sequence_id = r.u64();
    l.sequence_position = r.u64();
    l.request_slot_index = r.u32(); l.context_token_count = r.u32(); l.input_token_id = r.u32();
    l.mtp_draft_token_count = r.u32(); l.speculative_token_count = r.u32();
    l.mtp_proposed = r.u8(); l.mtp_accepted = r.u8(); l.mtp_path_id = r.u16();
    const uint32_t ns = r.u32();
    if (ns > 64) fail(Status::ParseError, "work packet: speculative count");
    l.speculative_draft_token_ids.resize(ns);
    for (auto& t : l.speculative_draft_token_ids) t = r.u32();
  }
  if (p.flags & kFlagExecutionPayload) {
    ExecPayload& e = p.exec;
    auto ints = [&](std::vector<int32_t>& v) {
      const uint32_t c = r.u32();
      if (c > n / 4) fail(Status::ParseError, "work packet: payload array length");
      v.resize(c);
      for (auto& x : v) x = int32_t(r.u32());
    };
    ints(e.positions); ints(e.slots); ints(e.block_table); ints(e.context_lens);
    e.block_table_cols = r.u32();
    ints(e.cu_q); ints(e.cu_k); ints(e.ctx_slots); ints(e.logits_rows);
    e.max_q = r.u32();
    const uint32_t nt = r.u32();
    if (nt > n / 4) fail(Status::ParseError, "work packet: payload temperature count");
    e.temperature.resize(nt);
    for (auto& t : e.temperature) {
      const uint32_t bits = r.u32();
      std::memcpy(&t, &bits, 4);
    }
    const uint32_t nk = r.u32();
    if (nk > n / 8) fail(Status::ParseError, "work packet: payload key count");
    e.sample_keys.resize(nk);
    for (auto& k : e.sample_keys) k = r.u64();
  }
  if (r.o != n) fail(Status::ParseError, "work packet: trailing bytes");
  return p;
}

uint64_t fingerprint(const Packet& p) {
  const auto b = serialize(p);
  return fingerprint_bytes(b.data(), b.size());
}

void validate_packet(const Packet& p, const Config& cfg) {
  cfg.validate();
  if (p.magic != kPacketMagic) fail(Status::InvalidArgument, "packet: magic");
  if (p.abi_version != kAbiVersion) fail(Status::AbiMismatch, "packet: ABI version");
  if (p.flags & ~kKnownFlags) fail(Status::InvalidArgument, "packet: unknown flags");
  validate_identity(p.identity);
  const bool prefill = p.flags & kFlagPrefill;
  if (prefill != (p.identity.transaction_phase == kPhasePrefill))
    fail(Status::InvalidArgument, "packet: prefill flag disagrees with the phase");
  if (p.block_token_count != cfg.kv_block_tokens) fail(Status::InvalidArgument, "packet: block size");
  if (p.active_sequence_count == 0 || p.active_sequence_count > cfg.max_lane_count)
    fail(Status::InvalidArgument, "packet: active sequence count");
  if (p.lanes.size() != p.active_sequence_count) fail(Status::InvalidArgument, "packet: lane count");
  if (prefill) {
    if (p.prefill_token_ids.empty() || p.prefill_token_ids.size() > cfg.max_prefill_tokens_per_packet)
      fail(Status::InvalidArgument, "packet: prefill token count");
    if (p.new_token_count != p.prefill_token_ids.size()) fail(Status::InvalidArgument, "packet: new token count");
  } else if (!p.prefill_token_ids.empty()) {
    fail(Status::InvalidArgument, "packet: decode packet carries prefill tokens");
  }
  for (uint32_t t : p.prefill_token_ids)
    if (t >= cfg.output_vocab_count) fail(Status::InvalidArgument, "packet: token id out of range");
  for (const Lane& l : p.lanes) {
    if (l.context_token_count == 0 || l.context_token_count > cfg.maximum_context_tokens)
      fail(Status::InvalidArgument, "lane: context length");
    if (l.input_token_id >= cfg.output_vocab_count) fail(Status::InvalidArgument, "lane: input token");
    if (l.speculative_token_count > cfg.max_speculative_token_count ||
        l.speculative_draft_token_ids.size() != l.speculative_token_count)
      fail(Status::InvalidArgument, "lane: speculative tokens");
    if (l.mtp_proposed && !mtp::resolution_is_valid(l.mtp_proposed, l.mtp_accepted, l.mtp_path_id))
      fail(Status::InvalidArgument, "lane: MTP resolution");
  }
  if (p.execution_row_count != p.active_sequence_count * p.rows_per_lane)
    fail(Status::InvalidArgument, "packet: execution rows");
  if (p.flags & kFlagExecutionPayload) {
    const ExecPayload& e = p.exec;
    const size_t lanes = p.lanes.size(), rows = prefill ? p.prefill_token_ids.size() : lanes;
    if (e.positions.size() != rows || e.slots.size() != rows)
      fail(Status::InvalidArgument, "payload: one position and slot per row");
    if (e.temperature.size() != lanes || e.sample_keys.size() != lanes)
      fail(Status::InvalidArgument, "payload: sampling parameters per lane");
    if (prefill) {
      if (e.cu_q.size() != lanes + 1 || e.cu_k.size() != lanes + 1 || e.logits_rows.size() != lanes ||
          e.cu_q.front() != 0 || uint32_t(e.cu_q.back()) != rows)
        fail(Status::InvalidArgument, "payload: prefill layout");
      if (!e.ctx_slots.empty() && e.ctx_slots.size() != size_t(e.cu_k.back()))
        fail(Status::InvalidArgument, "payload: context slots");
    } else if (e.context_lens.size() != lanes || !e.block_table_cols ||
               e.block_table.size() != lanes * size_t(e.block_table_cols)) {
      fail(Status::InvalidArgument, "payload: decode layout");
    }
  }
}

Packet build_step_packet(const StepPlan& plan, const Identity& id, const Config& cfg, uint32_t slot) {
  if (plan.kind == StepPlan::None) fail(Status::InvalidArgument, "build_step_packet: empty plan");
  Packet p;
  p.identity = id;
  p.flags = plan.kind == StepPlan::Prefill ? kFlagPrefill : 0;
  p.identity.transaction_phase = plan.kind == StepPlan::Prefill ? kPhasePrefill : kPhaseDecode;
  p.block_token_count = cfg.kv_block_tokens;
  p.max_blocks_per_sequence = cfg.kv_block_capacity();
  p.pipeline_slot = slot;
  p.active_sequence_count = plan.num_seqs;
  p.rows_per_lane = 1;
  p.execution_row_count = plan.num_seqs;
  p.execution_batch_bucket = plan.num_seqs ? select_batch_bucket(plan.num_seqs) : 0;
  if (plan.kind == StepPlan::Prefill) {
    p.prefill_token_ids.assign(plan.token_ids.begin(), plan.token_ids.end());
    p.new_token_count = (uint32_t)plan.token_ids.size();
  } else {
    p.new_token_count = plan.num_seqs;
  }
  for (uint32_t i = 0; i < plan.num_seqs; ++i) {
    Lane l;
    l.request_id = plan.seq_ids[i];
    l.sequence_id = plan.seq_ids[i];
    l.request_generation = id.request_generation;
    l.step_generation = id.step_generation;
    l.request_slot_index = i;
    if (plan.kind == StepPlan::Decode) {
      l.context_token_count = uint32_t(plan.context_lens[i]);
      l.input_token_id = uint32_t(plan.token_ids[i]);
      l.sequence_position = uint64_t(plan.positions[i]);
    } else {
      const int32_t q1 = plan.cu_q[i + 1], k1 = plan.cu_k[i + 1] - plan.cu_k[i];
      l.context_token_count = uint32_t(k1);
      l.input_token_id = uint32_t(plan.token_ids[q1 - 1]);
      l.sequence_position = uint64_t(plan.positions[q1 - 1]);
    }
    p.lanes.push_back(std::move(l));
  }
  if (!p.lanes.empty()) {
    p.request_id = p.lanes[0].request_id;
    p.sequence_id = p.lanes[0].sequence_id;
    p.sequence_position = p.lanes[0].sequence_position;
  }
  return p;
}

std::vector<Packet> build_stage_packets(const StepPlan& plan, const Identity& base, const Config& cfg,
                                        uint32_t chunks, const float* temps, const uint64_t* keys) {
  if (plan.kind != StepPlan::Prefill && plan.kind != StepPlan::Decode)
    fail(Status::InvalidArgument, "build_stage_packets: prefill or decode plans only");
  const uint32_t n = plan.num_seqs;
  if (!n || !chunks) fail(Status::InvalidArgument, "build_stage_packets: empty plan or zero chunks");
  chunks = std::min(chunks, n);
  const bool prefill = plan.kind == StepPlan::Prefill;
  std::vector<Packet> out;
  for (uint32_t k = 0; k < chunks; ++k) {
    const uint32_t s0 = uint32_t(uint64_t(n) * k / chunks), s1 = uint32_t(uint64_t(n) * (k + 1) / chunks);
    Packet p;
    p.identity = base;
    p.identity.transaction_id = base.transaction_id + k;
    p.identity.step_chunk_index = k;
    p.identity.step_chunk_count = chunks;
    p.identity.transaction_phase = prefill ? kPhasePrefill : kPhaseDecode;
    p.flags = (prefill ? kFlagPrefill : 0u) | kFlagExecutionPayload;
    p.block_token_count = cfg.kv_block_tokens;
    p.max_blocks_per_sequence = cfg.kv_block_capacity();
    p.pipeline_slot = k;
    p.active_sequence_count = s1 - s0;
    p.rows_per_lane = 1;
    p.execution_row_count = s1 - s0;
    p.execution_batch_bucket = select_batch_bucket(s1 - s0);
    ExecPayload& e = p.exec;
    const uint32_t r0 = prefill ? uint32_t(plan.cu_q[s0]) : s0, r1 = prefill ? uint32_t(plan.cu_q[s1]) : s1;
    e.positions.assign(plan.positions.begin() + r0, plan.positions.begin() + r1);
    e.slots.assign(plan.slot_mapping.begin() + r0, plan.slot_mapping.begin() + r1);
    if (prefill) {
      p.prefill_token_ids.assign(plan.token_ids.begin() + r0, plan.token_ids.begin() + r1);
      p.new_token_count = r1 - r0;
      const int32_t q0 = plan.cu_q[s0], kb = plan.cu_k[s0];
      for (uint32_t i = s0; i <= s1; ++i) {
        e.cu_q.push_back(plan.cu_q[i] - q0);
        e.cu_k.push_back(plan.cu_k[i] - kb);
      }
      if (plan.has_prefix)
        e.ctx_slots.assign(plan.ctx_slots.begin() + kb, plan.ctx_slots.begin() + plan.cu_k[s1]);
      for (uint32_t i = s0; i < s1; ++i) {
        e.logits_rows.push_back(plan.logits_idx[i] - q0);
        e.max_q = std::max(e.max_q, uint32_t(plan.cu_q[i + 1] - plan.cu_q[i]));
      }
    } else {
      p.new_token_count = s1 - s0;
      e.block_table_cols = plan.max_blocks;
      e.block_table.assign(plan.block_table.begin() + size_t(s0) * plan.max_blocks,
                           plan.block_table.begin() + size_t(s1) * plan.max_blocks);
      e.context_lens.assign(plan.context_lens.begin() + s0, plan.context_lens.begin() + s1);
    }
    for (uint32_t i = s0; i < s1; ++i) {
      Lane l;
      l.request_id = l.sequence_id = plan.seq_ids[i];
      l.request_generation = base.request_generation;
      l.step_generation = base.step_generation;
      l.request_slot_index = i;
      if (prefill) {
        const int32_t q1 = plan.cu_q[i + 1];
        l.context_token_count = uint32_t(plan.cu_k[i + 1] - plan.cu_k[i]);
        l.input_token_id = uint32_t(plan.token_ids[q1 - 1]);
        l.sequence_position = uint64_t(plan.positions[q1 - 1]);
      } else {
        l.context_token_count = uint32_t(plan.context_lens[i]);
        l.input_token_id = uint32_t(plan.token_ids[i]);
        l.sequence_position = uint64_t(plan.positions[i]);
      }
      p.lanes.push_back(std::move(l));
      e.temperature.push_back(temps ? temps[i] : 0.f);
      e.sample_keys.push_back(keys ? keys[i] : 0);
    }
    p.request_id = p.lanes[0].request_id;
    p.sequence_id = p.lanes[0].sequence_id;
    p.sequence_position = p.lanes[0].sequence_position;
    out.push_back(std::move(p));
  }
  return out;
}

// ----------------------------------------------------------------- KV directory
KvDirectory::KvDirectory(uint32_t cap, uint32_t physical) : physical_(physical) {
  if (cap == 0 || physical == 0) fail(Status::InvalidArgument, "KvDirectory: zero capacity");
  uint32_t sz = 16;
  while (sz < cap * 2) sz <<= 1;  // load factor <= 0.5
  table_.resize(sz);
  used_.assign(sz, 0);
  reset();
}

void KvDirectory::reset() {
  std::fill(used_.begin(), used_.end(), 0);
  free_blocks_.clear();
  for (uint32_t b = physical_; b-- > 0;) free_blocks_.push_back(b);
  block_owner_.assign(physical_, -1);
  block_refs_.assign(physical_, 0);
  live_ = 0;
  hand_ = 0;
  ++generation_;
}

size_t KvDirectory::slot_of(const KvKey& k) const {
  uint64_t h = k.sequence_id * 0x9E3779B97F4A7C15ull ^ (uint64_t(k.logical_block) * 0xC2B2AE3D27D4EB4Full);
  h ^= h >> 29;
  return size_t(h) & (table_.size() - 1);
}

int64_t KvDirectory::lookup(const KvKey& k) const {
  for (size_t s = slot_of(k), n = 0; n < table_.size(); s = (s + 1) & (table_.size() - 1), ++n) {
    if (!used_[s]) return -1;
    if (table_[s].key == k) return int64_t(s);
  }
  return -1;
}

const KvDirectoryEntry* KvDirectory::find(const KvKey& k) const {
  const int64_t s = lookup(k);
  return s < 0 ? nullptr : &table_[size_t(s)];
}

void KvDirectory::erase_slot(size_t s) {
  // backward-shift deletion keeps linear probing chains intact
  const uint32_t b = table_[s].physical_block;
  if (block_refs_[b] && --block_refs_[b] == 0) {
    block_owner_[b] = -1;
    free_blocks_.push_back(b);
  }
  used_[s] = 0;
  --live_;
  size_t hole = s;
  for (size_t j = (s + 1) & (table_.size() - 1); used_[j]; j = (j + 1) & (table_.size() - 1)) {
    const size_t home = slot_of(table_[j].key);
    const bool movable = (j > hole) ? (home <= hole || home > j) : (home <= hole && home > j);
    if (movable) {
      table_[hole] = table_[j];
      used_[hole] = 1;
      used_[j] = 0;
      const uint32_t pb = table_[hole].physical_block;
      if (block_owner_[pb] == int64_t(j)) block_owner_[pb] = int64_t(hole);
      hole = j;
    }
  }
}

uint32_t KvDirectory::sweep_victim() {
  // clock sweep over the table: skip pinned / in-flight, clear reference bits
  for (size_t n = 0; n < 2 * table_.size() + 2; ++n) {
    const size_t s = hand_;
    hand_ = uint32_t((hand_ + 1) & (table_.size() - 1));
    if (!used_[s]) continue;
    KvDirectoryEntry& e = table_[s];
    if (e.pins || e.state == KvEntryState::InFlight) continue;
    if (e.referenced) { e.referenced = 0; continue; }
    const uint32_t b = e.physical_block;
    erase_slot(s);
    ++sweeps_;
    if (!block_refs_[b]) {
      // the block went back to the free list inside erase_slot
      auto it = std::find(free_blocks_.begin(), free_blocks_.end(), b);
      free_blocks_.erase(it);
      return b;
    }
  }
  fail(Status::CapacityExceeded, "KvDirectory: every block is pinned or in flight");
}

uint32_t KvDirectory::acquire(const KvKey& k, uint64_t content, bool* hit) {
  const int64_t s0 = lookup(k);
  if (s0 >= 0) {
    table_[size_t(s0)].referenced = 1;
    if (hit) *hit = table_[size_t(s0)].state == KvEntryState::Resident;
    return table_[size_t(s0)].physical_block;
  }
  if (live_ * 2 >= table_.size()) fail(Status::CapacityExceeded, "KvDirectory: table full");
  uint32_t block = 0xffffffffu;
  bool shared = false;
  if (content) {
    for (size_t s = 0; s < table_.size(); ++s) {
      if (used_[s] && table_[s].content_key == content && table_[s].state == KvEntryState::Resident) {
        block = table_[s].physical_block;
        shared = true;
        break;
      }
    }
  }
  if (!shared) {
    if (free_blocks_.empty()) block = sweep_victim();
    else { block = free_blocks_.back(); free_blocks_.pop_back(); }
  }
  size_t s = slot_of(k);
  while (used_[s]) s = (s + 1) & (table_.size() - 1);
  used_[s] = 1;
  table_[s] = KvDirectoryEntry{k, block, shared ? KvEntryState::Resident : KvEntryState::Missing, KvResidency::Gpu,
                               0, content, 1};
  ++live_;
  ++block_refs_[block];
  if (!shared) block_owner_[block] = int64_t(s);
  else ++shared_;
  if (hit) *hit = shared;
  return block;
}

void KvDirectory::mark_resident(const KvKey& k) {
  const int64_t s = lookup(k);
  if (s < 0) fail(Status::NotFound, "KvDirectory: unknown key");
  table_[size_t(s)].state = KvEntryState::Resident;
}
void KvDirectory::mark_in_flight(const KvKey& k) {
  const int64_t s = lookup(k);
  if (s < 0) fail(Status::NotFound, "KvDirectory: unknown key");
  table_[size_t(s)].state = KvEntryState::InFlight;
}
void KvDirectory::set_residency(const KvKey& k, KvResidency r) {
  const int64_t s = lookup(k);
  if (s < 0) fail(Status::NotFound, "KvDirectory: unknown key");
  table_[size_t(s)].residency = r;
}
void KvDirectory::pin(const KvKey& k) {
  const int64_t s = lookup(k);
  if (s < 0) fail(Status::NotFound, "KvDirectory: unknown key");
  ++table_[size_t(s)].pins;
}
void KvDirectory::unpin(const KvKey& k) {
  const int64_t s = lookup(k);
  if (s < 0 || table_[size_t(s)].pins == 0) fail(Status::InvalidArgument, "KvDirectory: unpin without pin");
  --table_[size_t(s)].pins;
}
void KvDirectory::release_sequence(uint64_t seq) {
  for (bool again = true; again;) {
    again = false;
    for (size_t s = 0; s < table_.size(); ++s) {
      if (used_[s] && table_[s].key.sequence_id == seq) {
        erase_slot(s);
        again = true;  // backward shift may have moved an entry of the same sequence into s
        break;
      }
    }
  }
}

}  // namespace wc
}  // namespace spc
