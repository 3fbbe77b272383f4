#include "rank_daemon.h"

#include <algorithm>
#include <unordered_set>

namespace spc {
namespace rd {

namespace {
struct W {
  std::string b;
  void u32(uint32_t v) {
    for (int i = 0; i < 4; ++i) b.push_back(char(v >> (8 * i)));
  }
  void u64(uint64_t v) {
    for (int i = 0; i < 8; ++i) b.push_back(char(v >> (8 * i)));
  }
  void pad(size_t to) { b.resize(to, '\0'); }
};
struct R {
  const std::string& b;
  size_t o = 0;
  uint32_t u32() {
    const uint32_t v = get_u32(reinterpret_cast<const uint8_t*>(b.data()) + o);
    o += 4;
    return v;
  }
  uint64_t u64() {
    const uint64_t v = get_u64(reinterpret_cast<const uint8_t*>(b.data()) + o);
    o += 8;
    return v;
  }
};
void put_identity(W& w, const wc::Identity& i) {
  w.u64(i.control_generation);
  w.u64(i.transaction_id);
  w.u64(i.dispatch_generation);
  w.u64(i.request_generation);
  w.u64(i.step_generation);
  w.u32(i.step_chunk_index);
  w.u32(i.step_chunk_count);
  w.u32(i.transaction_phase);
  w.u32(0);
}
wc::Identity get_identity(R& r) {
  wc::Identity i;
  i.control_generation = r.u64();
  i.transaction_id = r.u64();
  i.dispatch_generation = r.u64();
  i.request_generation = r.u64();
  i.step_generation = r.u64();
  i.step_chunk_index = r.u32();
  i.step_chunk_count = r.u32();
  i.transaction_phase = r.u32();
  r.u32();
  return i;
}
bool same(const wc::Identity& a, const wc::Identity& b) {
  return a.control_generation == b.control_generation && a.transaction_id == b.transaction_id &&
         a.dispatch_generation == b.dispatch_generation && a.request_generation == b.request_generation &&
         a.step_generation == b.step_generation && a.step_chunk_index == b.step_chunk_index &&
         a.step_chunk_count == b.step_chunk_count && a.transaction_phase == b.transaction_phase;
}
std::vector<uint64_t> sequences_of(const wc::Packet& p) {
  std::vector<uint64_t> s;
  for (const wc::Lane& l : p.lanes) s.push_back(l.sequence_id);
  if (s.empty() && p.sequence_id) s.push_back(p.sequence_id);
  return s;
}
}  // namespace

// ------------------------------------------------------------------ wire records
std::string identity_to_wire(const wc::Identity& id) {
  W w;
  put_identity(w, id);
  return w.b;
}
wc::Identity identity_from_wire(const std::string& b) {
  if (b.size() != kIdentityBytes) fail(Status::AbiMismatch, "rank daemon: identity must be 56 bytes");
  R r{b};
  return get_identity(r);
}
uint64_t identity_fingerprint(const wc::Identity& id) {
  const std::string b = identity_to_wire(id);
  return wc::fingerprint_bytes(reinterpret_cast<const uint8_t*>(b.data()), b.size());
}
uint32_t packet_dedup_hash32(const uint8_t* d, size_t n) { return fnv1a32(d, n); }

std::string ack_to_wire(const Ack& a) {
  W w;
  w.u32(kAckMagic);
  w.u32(kWireAbi);
  w.u32(uint32_t(kAckBytes));
  w.u32(a.status);
  w.u32(a.state);
  w.u32(0);
  put_identity(w, a.identity);
  w.u64(a.packet_fingerprint);
  w.u64(0);
  return w.b;
}
Ack ack_from_wire(const std::string& b) {
  if (b.size() != kAckBytes) fail(Status::AbiMismatch, "rank daemon: acknowledgement must be 96 bytes");
  R r{b};
  if (r.u32() != kAckMagic || r.u32() != kWireAbi || r.u32() != kAckBytes)
    fail(Status::AbiMismatch, "rank daemon: bad acknowledgement header");
  Ack a;
  a.status = r.u32();
  a.state = r.u32();
  if (r.u32() != 0) fail(Status::ValidationFailed, "rank daemon: acknowledgement reserved word set");
  a.identity = get_identity(r);
  a.packet_fingerprint = r.u64();
  return a;
}

std::string final_event_to_wire(const FinalEvent& e) {
  if (e.token_ids.size() > kMaxFinalTokens || e.draft_token_ids.size() > kMaxFinalTokens)
    fail(Status::CapacityExceeded, "rank daemon: at most 8 tokens per final event");
  W w;
  w.u32(kFinalMagic);
  w.u32(uint32_t(kFinalEventBytes));
  w.u32(e.status);
  w.u32(e.program_id);
  w.u32(e.slot);
  w.u32(e.accepted_token_count);
  w.u32(e.completion_flags);
  w.u32(uint32_t(e.token_ids.size()));
  for (uint32_t i = 0; i < kMaxFinalTokens; ++i) w.u32(i < e.token_ids.size() ? e.token_ids[i] : 0);
  w.u32(uint32_t(e.draft_token_ids.size()));
  for (uint32_t i = 0; i < kMaxFinalTokens; ++i) w.u32(i < e.draft_token_ids.size() ? e.draft_token_ids[i] : 0);
  w.u32(0);
  w.u64(e.request_id);
  w.u64(e.sequence_id);
  w.u64(e.sequence_position);
  w.u64(e.service_time_ns);
  put_identity(w, e.identity);
  w.u32(0);  // extension flags
  w.u32(0);
  w.pad(kFinalEventBytes);  // speculative-draft extension region (reserved)
  return w.b;
}
FinalEvent final_event_from_wire(const std::string& b) {
  if (b.size() != kFinalEventBytes) fail(Status::AbiMismatch, "rank daemon: final event must be 272 bytes");
  R r{b};
  if (r.u32() != kFinalMagic || r.u32() != kFinalEventBytes) fail(Status::AbiMismatch, "rank daemon: bad final event");
  FinalEvent e;
  e.status = r.u32();
  e.program_id = r.u32();
  e.slot = r.u32();
  e.accepted_token_count = r.u32();
  e.completion_flags = r.u32();
  const uint32_t n = std::min(r.u32(), kMaxFinalTokens);
  for (uint32_t i = 0; i < kMaxFinalTokens; ++i) {
    const uint32_t v = r.u32();
    if (i < n) e.token_ids.push_back(v);
  }
  const uint32_t nd = std::min(r.u32(), kMaxFinalTokens);
  for (uint32_t i = 0; i < kMaxFinalTokens; ++i) {
    const uint32_t v = r.u32();
    if (i < nd) e.draft_token_ids.push_back(v);
  }
  r.u32();
  e.request_id = r.u64();
  e.sequence_id = r.u64();
  e.sequence_position = r.u64();
  e.service_time_ns = r.u64();
  e.identity = get_identity(r);
  return e;
}

// ------------------------------------------------------------------ ledger
TransactionLedger::TransactionLedger(uint32_t capacity) : table_(capacity) {
  if (!capacity) fail(Status::InvalidArgument, "ledger: zero capacity");
}

uint32_t TransactionLedger::start(const wc::Identity& id) const {
  return uint32_t(identity_fingerprint(id) % table_.size());
}

int64_t TransactionLedger::find_index(const wc::Identity& id) const {
  const uint32_t n = uint32_t(table_.size()), s = start(id);
  for (uint32_t k = 0; k < n; ++k) {
    const uint32_t i = (s + k) % n;
    if (table_[i].state == Empty) return -1;
    if (table_[i].state != Tombstone && same(table_[i].identity, id)) return i;
  }
  return -1;
}

void TransactionLedger::reset(uint64_t generation) {
  std::fill(table_.begin(), table_.end(), LedgerEntry{});
  entry_count_ = active_count_ = terminal_count_ = tombstone_count_ = 0;
  epoch_ = 0;
  generation_ = generation;
}

void TransactionLedger::prepare_generation(uint64_t g) {
  if (generation_ == 0 || g == generation_) {
    if (generation_ == 0) reset(g);
    return;
  }
  if (g < generation_) fail(Status::ValidationFailed, "ledger: stale control generation");
  if (active_count_) fail(Status::Busy, "ledger: active transactions block a generation change");
  reset(g);
}

void TransactionLedger::recycle_oldest_terminal() {
  int64_t best = -1;
  uint64_t oldest = UINT64_MAX;
  for (size_t i = 0; i < table_.size(); ++i)
    if (tx_terminal(table_[i].state) && table_[i].last_observed_epoch < oldest) {
      oldest = table_[i].last_observed_epoch;
      best = int64_t(i);
    }
  if (best < 0) fail(Status::CapacityExceeded, "ledger: full of active transactions");
  table_[best] = LedgerEntry{};
  table_[best].state = Tombstone;
  --entry_count_;
  --terminal_count_;
  ++tombstone_count_;
}

int64_t TransactionLedger::insertion_index(const wc::Identity& id) {
  const uint32_t n = uint32_t(table_.size()), s = start(id);
  int64_t tomb = -1;
  for (uint32_t k = 0; k < n; ++k) {
    const uint32_t i = (s + k) % n;
    if (table_[i].state == Tombstone) {
      if (tomb < 0) tomb = i;
      continue;
    }
    if (table_[i].state == Empty) {
      if (tomb >= 0) {
        --tombstone_count_;
        return tomb;
      }
      return i;
    }
  }
  if (tomb >= 0) {
    --tombstone_count_;
    return tomb;
  }
  return -1;
}

Observation TransactionLedger::observe(const wc::Identity& id, uint64_t fp) {
  if (!fp) fail(Status::InvalidArgument, "ledger: zero payload fingerprint");
  wc::validate_identity(id);
  prepare_generation(id.control_generation);
  if (++epoch_ == 0) epoch_ = 1;
  const int64_t i = find_index(id);
  if (i >= 0) {
    LedgerEntry& e = table_[i];
    e.last_observed_epoch = epoch_;
    if (e.payload_fingerprint != fp) return Observation::Conflict;
    return tx_terminal(e.state) ? Observation::ReplayTerminal : Observation::ReplayActive;
  }
  int64_t slot = insertion_index(id);
  if (slot < 0) {
    recycle_oldest_terminal();
    slot = insertion_index(id);
    if (slot < 0) fail(Status::CapacityExceeded, "ledger: no free entry");
  }
  LedgerEntry& e = table_[slot];
  e = LedgerEntry{};
  e.identity = id;
  e.payload_fingerprint = fp;
  e.last_observed_epoch = epoch_;
  e.state = Prepared;
  ++entry_count_;
  ++active_count_;
  return Observation::New;
}

void TransactionLedger::transition(const wc::Identity& id, uint32_t target, Status terminal_status) {
  wc::validate_identity(id);
  if (target < Prepared || target > Failed) fail(Status::InvalidArgument, "ledger: bad target state");
  const int64_t i = find_index(id);
  if (i < 0) fail(Status::NotFound, "ledger: unknown transaction");
  LedgerEntry& e = table_[i];
  if (tx_terminal(e.state)) {
    if (e.state == target && e.terminal_status == uint32_t(terminal_status))
      fail(Status::Duplicate, "ledger: transition already applied");
    fail(Status::InvalidArgument, "ledger: transaction already terminal");
  }
  const bool legal = e.state == target || (e.state == Prepared && (target == Accepted || target == Cancelled || target == Failed)) ||
                     (e.state == Accepted && (target == Executing || target == Cancelled || target == Failed)) ||
                     (e.state == Executing && (target == Committed || target == Cancelled || target == Failed));
  if (!legal) fail(Status::InvalidArgument, "ledger: illegal transition");
  if (++epoch_ == 0) epoch_ = 1;
  e.last_observed_epoch = epoch_;
  if (tx_terminal(target)) {
    --active_count_;
    ++terminal_count_;
    e.terminal_status = uint32_t(terminal_status);
  } else {
    e.terminal_status = uint32_t(Status::Pending);
  }
  e.state = target;
}

const LedgerEntry* TransactionLedger::find(const wc::Identity& id) const {
  const int64_t i = find_index(id);
  return i < 0 ? nullptr : &table_[i];
}

// ------------------------------------------------------------------ daemon
RankDaemon::RankDaemon(const DaemonConfig& cfg, ForwardFn forward, ExecuteFn execute, FinalFn final_event)
    : cfg_(cfg), forward_(std::move(forward)), execute_(std::move(execute)), final_(std::move(final_event)),
      ledger_(cfg.ledger_capacity) {
  if (cfg_.world == 0 || cfg_.rank >= cfg_.world || cfg_.queue_capacity == 0)
    fail(Status::InvalidArgument, "rank daemon: bad configuration");
  cfg_.work.validate();
}

std::string RankDaemon::submit(const std::string& wire) {
  ++st_.submitted;
  Ack ack;
  ack.state = Prepared;
  const uint32_t h = packet_dedup_hash32(reinterpret_cast<const uint8_t*>(wire.data()), wire.size());
  wc::Packet p;
  try {
    p = wc::deserialize(reinterpret_cast<const uint8_t*>(wire.data()), wire.size());
    wc::validate_packet(p, cfg_.work);
  } catch (const StatusError& e) {
    ++st_.rejected;
    ack.status = uint32_t(e.status);
    ack.state = Failed;
    return ack_to_wire(ack);
  }
  ack.identity = p.identity;
  ack.packet_fingerprint = wc::fingerprint(p);
  if (recent_count_.count(h)) {  // the same bytes again: a retransmission
    ++st_.duplicates;
    const LedgerEntry* e = ledger_.find(p.identity);
    ack.status = uint32_t(Status::Duplicate);
    ack.state = e ? e->state : Prepared;
    return ack_to_wire(ack);
  }
  if (queue_.size() >= cfg_.queue_capacity) {
    ack.status = uint32_t(Status::Busy);
    return ack_to_wire(ack);
  }
  Observation obs;
  try {
    obs = ledger_.observe(p.identity, ack.packet_fingerprint);
  } catch (const StatusError& e) {
    ++st_.rejected;
    ack.status = uint32_t(e.status);
    ack.state = Failed;
    return ack_to_wire(ack);
  }
  if (obs == Observation::Conflict) {
    ++st_.conflicts;
    ack.status = uint32_t(Status::ValidationFailed);
    ack.state = ledger_.find(p.identity)->state;
    return ack_to_wire(ack);
  }
  if (obs != Observation::New) {
    ++st_.duplicates;
    ack.status = uint32_t(Status::Duplicate);
    ack.state = ledger_.find(p.identity)->state;
    return ack_to_wire(ack);
  }
  ledger_.transition(p.identity, Accepted);
  recent_.push_back(h);
  ++recent_count_[h];
  while (recent_.size() > cfg_.dedup_window) {
    const uint32_t old = recent_.front();
    recent_.pop_front();
    if (--recent_count_[old] == 0) recent_count_.erase(old);
  }
  queue_.push_back(Item{std::move(p), wire, ack.packet_fingerprint});
  ++st_.accepted;
  ack.status = uint32_t(Status::Ok);
  ack.state = Accepted;
  return ack_to_wire(ack);
}

uint32_t RankDaemon::pump(uint32_t max_packets) {
  uint32_t n = 0;
  std::unordered_set<uint64_t> held;  // sequences of packets held back in this pass keep their order
  for (auto it = queue_.begin(); it != queue_.end() && n < max_packets;) {
    const std::vector<uint64_t> seqs = sequences_of(it->packet);
    bool ok = true;
    for (uint64_t s : seqs)
      if (busy_seq_.count(s) || held.count(s)) ok = false;
    if (!ok) {
      for (uint64_t s : seqs) held.insert(s);
      ++it;
      continue;
    }
    Item item = std::move(*it);
    it = queue_.erase(it);
    if (cfg_.rank + 1 < cfg_.world && forward_) {
      forward_(item.wire);
      ++st_.forwarded;
    }
    ledger_.transition(item.packet.identity, Executing);
    for (uint64_t s : seqs) ++busy_seq_[s];
    const uint64_t tid = item.packet.identity.transaction_id;
    const std::string wire = item.wire;
    inflight_.emplace(tid, std::move(item));
    ++st_.executed;
    ++n;
    if (execute_) execute_(wire);
  }
  return n;
}

RankDaemon::Item RankDaemon::retire(const wc::Identity& id, Status status) {
  auto it = inflight_.find(id.transaction_id);
  if (it == inflight_.end() || !same(it->second.packet.identity, id))
    fail(Status::NotFound, "rank daemon: completion of an unknown transaction");
  Item item = std::move(it->second);
  inflight_.erase(it);
  for (uint64_t s : sequences_of(item.packet)) {
    auto b = busy_seq_.find(s);
    if (b != busy_seq_.end() && --b->second == 0) busy_seq_.erase(b);
  }
  const LedgerEntry* e = ledger_.find(id);
  if (e && !tx_terminal(e->state)) ledger_.transition(id, status == Status::Ok ? Committed : Failed, status);
  if (status == Status::Ok) ++st_.committed;
  else ++st_.failed;
  return item;
}

void RankDaemon::complete_lanes(const wc::Identity& id, Status status,
                                const std::vector<std::vector<uint32_t>>& lane_tokens, uint64_t service_time_ns) {
  Item item = retire(id, status);
  if (cfg_.rank + 1 != cfg_.world || !final_) return;
  if (lane_tokens.size() != item.packet.lanes.size())
    fail(Status::InvalidArgument, "rank daemon: one token list per lane");
  for (size_t i = 0; i < item.packet.lanes.size(); ++i) {
    const wc::Lane& l = item.packet.lanes[i];
    FinalEvent fe;
    fe.status = uint32_t(status);
    fe.program_id = item.packet.pipeline_slot;
    fe.slot = l.request_slot_index;
    const auto& t = lane_tokens[i];
    fe.token_ids.assign(t.begin(), t.begin() + std::min<size_t>(t.size(), kMaxFinalTokens));
    fe.accepted_token_count = uint32_t(fe.token_ids.size());
    fe.request_id = l.request_id;
    fe.sequence_id = l.sequence_id;
    fe.sequence_position = l.sequence_position;
    fe.service_time_ns = service_time_ns;
    fe.identity = id;
    final_(final_event_to_wire(fe));
    ++st_.final_events;
  }
}

void RankDaemon::complete(const wc::Identity& id, Status status, const std::vector<uint32_t>& tokens,
                          uint64_t service_time_ns) {
  Item item = retire(id, status);
  if (cfg_.rank + 1 == cfg_.world && final_) {
    FinalEvent fe;
    fe.status = uint32_t(status);
    fe.program_id = item.packet.pipeline_slot;
    fe.token_ids.assign(tokens.begin(), tokens.begin() + std::min<size_t>(tokens.size(), kMaxFinalTokens));
    fe.accepted_token_count = uint32_t(fe.token_ids.size());
    fe.request_id = item.packet.request_id;
    fe.sequence_id = item.packet.sequence_id;
    fe.sequence_position = item.packet.sequence_position;
    fe.service_time_ns = service_time_ns;
    fe.identity = id;
    final_(final_event_to_wire(fe));
    ++st_.final_events;
  }
}

void RankDaemon::cancel(const wc::Identity& id) {
  for (auto it = queue_.begin(); it != queue_.end(); ++it)
    if (same(it->packet.identity, id)) {
      queue_.erase(it);
      ledger_.transition(id, Cancelled, Status::Ok);
      ++st_.cancelled;
      return;
    }
  auto f = inflight_.find(id.transaction_id);
  if (f != inflight_.end()) {
    // in flight: the executor's completion still arrives and releases the sequences
    const LedgerEntry* e = ledger_.find(id);
    if (e && !tx_terminal(e->state)) ledger_.transition(id, Cancelled, Status::Ok);
    ++st_.cancelled;
    return;
  }
  fail(Status::NotFound, "rank daemon: nothing to cancel");
}

DaemonStats RankDaemon::stats() const {
  DaemonStats s = st_;
  s.queued = uint32_t(queue_.size());
  s.inflight = uint32_t(inflight_.size());
  return s;
}

}  // namespace rd
}  // namespace spc
