#include "runtime_completion.h"

#include <set>

namespace spc {
namespace rc {

// ---------------------------------------------------------------- credits
CreditLedger::CreditLedger(const std::array<uint32_t, kCreditDomains>& capacities) : cap_(capacities) {
  for (uint32_t c : cap_)
    if (!c) fail(Status::InvalidArgument, "credit ledger: every domain needs a nonzero capacity");
}
void CreditLedger::check(uint32_t d) {
  if (d >= kCreditDomains) fail(Status::InvalidArgument, "credit ledger: unknown domain");
}
bool CreditLedger::acquire(uint32_t d, uint32_t n) {
  check(d);
  if (!n) fail(Status::InvalidArgument, "credit ledger: zero credits");
  if (cap_[d] - used_[d] < n) return false;
  used_[d] += n;
  return true;
}
void CreditLedger::release(uint32_t d, uint32_t n) {
  check(d);
  if (!n || n > used_[d]) fail(Status::InvalidArgument, "credit ledger: release of credits not held");
  used_[d] -= n;
}
uint32_t CreditLedger::available(uint32_t d) const {
  check(d);
  return cap_[d] - used_[d];
}
uint32_t CreditLedger::in_use(uint32_t d) const {
  check(d);
  return used_[d];
}
uint32_t CreditLedger::capacity(uint32_t d) const {
  check(d);
  return cap_[d];
}

// ---------------------------------------------------------------- final events
namespace {
bool same_identity(const wc::Identity& a, const wc::Identity& b) {
  return a.control_generation == b.control_generation && a.transaction_id == b.transaction_id &&
         a.dispatch_generation == b.dispatch_generation && a.request_generation == b.request_generation &&
         a.step_generation == b.step_generation && a.step_chunk_index == b.step_chunk_index &&
         a.step_chunk_count == b.step_chunk_count && a.transaction_phase == b.transaction_phase;
}
}  // namespace

FinalEventQueue::FinalEventQueue(uint32_t capacity) : capacity_(capacity) {
  if (!capacity) fail(Status::InvalidArgument, "final event queue: zero capacity");
}

uint64_t FinalEventQueue::push(FinalEvent e) {
  if (events_.size() >= capacity_) fail(Status::CapacityExceeded, "final event queue: full");
  wc::validate_identity(e.identity);
  if (!e.payload_fingerprint) fail(Status::InvalidArgument, "final event queue: zero payload fingerprint");
  e.generation = next_generation_++;
  e.state = EventPending;
  events_.push_back(e);
  return e.generation;
}

const FinalEvent* FinalEventQueue::peek() const { return events_.empty() ? nullptr : &events_.front(); }

Status FinalEventQueue::acknowledge(const wc::Identity& id, uint64_t generation, uint64_t fp) {
  // pending events are in generation order: binary search would do, but the queue is short
  for (auto it = events_.begin(); it != events_.end(); ++it) {
    if (it->generation != generation) continue;
    if (!same_identity(it->identity, id) || it->payload_fingerprint != fp) return Status::InvalidArgument;
    events_.erase(it);
    return Status::Ok;
  }
  return Status::NotFound;
}

// ---------------------------------------------------------------- transmission window
TransmissionWindow::TransmissionWindow(uint32_t capacity) : slots_(capacity) {
  if (!capacity) fail(Status::InvalidArgument, "transmission window: zero capacity");
  for (uint32_t i = 0; i < capacity; ++i) slots_[i].slot_index = i;
}

const TransmissionSlot& TransmissionWindow::slot(uint32_t i) const {
  if (i >= slots_.size()) fail(Status::InvalidArgument, "transmission window: slot out of range");
  return slots_[i];
}

TransmissionSlot& TransmissionWindow::live(uint32_t i, uint64_t generation) {
  if (i >= slots_.size()) fail(Status::InvalidArgument, "transmission window: slot out of range");
  TransmissionSlot& s = slots_[i];
  if (s.state == SlotFree || s.generation != generation)
    fail(Status::NotFound, "transmission window: stale slot generation");
  return s;
}

std::pair<uint32_t, uint64_t> TransmissionWindow::reserve(const wc::Identity& id, uint64_t fp) {
  wc::validate_identity(id);
  if (!fp) fail(Status::InvalidArgument, "transmission window: zero payload fingerprint");
  int64_t free_slot = -1;
  for (auto& s : slots_) {
    if (s.state == SlotFree) {
      if (free_slot < 0) free_slot = s.slot_index;
      continue;
    }
    if (same_identity(s.identity, id)) {
      if (s.payload_fingerprint != fp) fail(Status::Duplicate, "transmission window: identity held with another payload");
      return {s.slot_index, s.generation};
    }
  }
  if (free_slot < 0) fail(Status::Busy, "transmission window: full");
  TransmissionSlot& s = slots_[free_slot];
  s.state = SlotReserved;
  s.generation = next_generation_++;
  s.identity = id;
  s.payload_fingerprint = fp;
  s.last_send_epoch = 0;
  s.retry_count = 0;
  ++in_use_;
  return {s.slot_index, s.generation};
}

void TransmissionWindow::mark_sent(uint32_t i, uint64_t generation) {
  TransmissionSlot& s = live(i, generation);
  if (s.state == SlotSent) ++s.retry_count;
  s.state = SlotSent;
  s.last_send_epoch = ++send_epoch_;
}

Status TransmissionWindow::acknowledge(uint32_t i, uint64_t generation, const wc::Identity& id, uint64_t fp) {
  if (i >= slots_.size()) fail(Status::InvalidArgument, "transmission window: slot out of range");
  TransmissionSlot& s = slots_[i];
  if (s.state == SlotFree || s.generation != generation) return Status::NotFound;
  if (!same_identity(s.identity, id) || s.payload_fingerprint != fp) return Status::InvalidArgument;
  if (s.state != SlotSent) fail(Status::InvalidArgument, "transmission window: acknowledgement of an unsent slot");
  s.state = SlotFree;  // acknowledged: the slot is reusable at once, under a new generation
  --in_use_;
  return Status::Ok;
}

bool TransmissionWindow::next_replay(uint32_t* slot, uint64_t* generation) const {
  const TransmissionSlot* best = nullptr;
  for (const auto& s : slots_)
    if (s.state == SlotSent && (!best || s.last_send_epoch < best->last_send_epoch)) best = &s;
  if (!best) return false;
  *slot = best->slot_index;
  *generation = best->generation;
  return true;
}

// ---------------------------------------------------------------- controller
Controller::Controller(std::vector<Participant> participants, uint32_t transaction_capacity,
                       uint32_t final_event_capacity, const std::array<uint32_t, kCreditDomains>& credits)
    : parts_(std::move(participants)),
      ledger_(transaction_capacity),
      events_(final_event_capacity),
      credits_(credits) {
  if (parts_.empty() || parts_.size() > kMaxParticipants)
    fail(Status::InvalidArgument, "runtime controller: 1 to 32 participants");
  std::set<std::string> names;
  for (const auto& p : parts_) {
    if (p.name.empty() || !names.insert(p.name).second)
      fail(Status::InvalidArgument, "runtime controller: participant names are nonempty and unique");
    if ((p.flags & ~kRequiredFlags) != 0) fail(Status::InvalidArgument, "runtime controller: unknown participant flag");
    if ((p.flags & kRequiredFlags) != kRequiredFlags)
      fail(Status::Unsupported, "runtime controller: participant " + p.name +
                                    " lacks transactional staging, an infallible commit or an idempotent cancel");
    if (!p.restart_epoch) fail(Status::InvalidArgument, "runtime controller: zero restart epoch");
    if (!p.prepare || !p.execute || !p.commit || !p.cancel)
      fail(Status::InvalidArgument, "runtime controller: participant " + p.name + " lacks an entry point");
  }
}

uint64_t Controller::validate(const Request& r) const {
  wc::validate_identity(r.identity);
  if (!r.request_id) fail(Status::InvalidArgument, "runtime controller: zero request id");
  if (r.payload.empty()) fail(Status::InvalidArgument, "runtime controller: empty payload");
  return wc::fingerprint_bytes(reinterpret_cast<const uint8_t*>(r.payload.data()), r.payload.size());
}

namespace {
template <typename F>
Status guarded(F&& f) {  // an entry point that throws counts as an internal error of that participant
  try {
    return f();
  } catch (...) {
    return Status::InternalError;
  }
}
}  // namespace

uint32_t Controller::cancel_all(const Request& r, size_t upto, Status reason) {
  uint32_t n = 0;
  for (size_t i = upto; i-- > 0;) {
    try {
      parts_[i].cancel(r, reason);
    } catch (...) {
      // cancel is declared idempotent and must not fail; a throw is swallowed so the
      // remaining participants still release their staging
    }
    ++n;
  }
  return n;
}

Result Controller::run(const Request& r) {
  Result res;
  res.payload_fingerprint = validate(r);
  const uint64_t key = rd::identity_fingerprint(r.identity);
  const rd::LedgerEntry* prior = ledger_.find(r.identity);
  if (!prior) {
    // a new transaction needs room for its outcome before anything is recorded
    if (credits_.available(Execution) == 0 || credits_.available(CompletionOwnership) == 0 ||
        events_.pending() >= events_.capacity()) {
      res.status = Status::Busy;
      return res;
    }
  }
  switch (ledger_.observe(r.identity, res.payload_fingerprint)) {
    case rd::Observation::Conflict:
      res.status = Status::Duplicate;  // same identity, another payload
      return res;
    case rd::Observation::ReplayActive:
      res.replayed = true;
      res.status = Status::Busy;
      return res;
    case rd::Observation::ReplayTerminal: {
      const rd::LedgerEntry* e = ledger_.find(r.identity);
      res.replayed = true;
      res.status = Status(e->terminal_status);
      auto g = generation_of_.find(key);
      res.final_event_generation = g == generation_of_.end() ? 0 : g->second;
      return res;
    }
    case rd::Observation::New:
      break;
  }
  credits_.acquire(Execution, 1);
  credits_.acquire(CompletionOwnership, 1);
  Status st = Status::Ok;
  size_t i = 0;
  for (; i < parts_.size() && st == Status::Ok; ++i) st = guarded([&] { return parts_[i].prepare(r); });
  if (st != Status::Ok) {
    res.cancelled = cancel_all(r, i, st);  // the failing participant's staging too (cancel is idempotent)
    ledger_.transition(r.identity, rd::Cancelled, st);
  } else {
    ledger_.transition(r.identity, rd::Accepted);
    ledger_.transition(r.identity, rd::Executing);
    for (i = 0; i < parts_.size() && st == Status::Ok; ++i) st = guarded([&] { return parts_[i].execute(r); });
    if (st != Status::Ok) {
      res.cancelled = cancel_all(r, parts_.size(), st);
      ledger_.transition(r.identity, rd::Failed, st);
    } else {
      for (auto& p : parts_) {
        try {
          p.commit(r);
        } catch (...) {
          // commit is declared infallible: the outcome is already decided
        }
        ++res.committed;
      }
      ledger_.transition(r.identity, rd::Committed, Status::Ok);
    }
  }
  credits_.release(Execution, 1);
  FinalEvent ev;
  ev.identity = r.identity;
  ev.payload_fingerprint = res.payload_fingerprint;
  ev.request_id = r.request_id;
  ev.sequence_id = r.sequence_id;
  ev.sequence_position = r.sequence_position;
  ev.status = st;
  res.final_event_generation = events_.push(ev);
  res.status = st;
  generation_of_[key] = res.final_event_generation;
  generation_order_.push_back(key);
  while (generation_order_.size() > ledger_.capacity()) {
    generation_of_.erase(generation_order_.front());
    generation_order_.pop_front();
  }
  return res;
}

Status Controller::acknowledge_final_event(const wc::Identity& id, uint64_t generation, uint64_t fp) {
  const Status s = events_.acknowledge(id, generation, fp);
  if (s == Status::Ok) credits_.release(CompletionOwnership, 1);
  return s;
}

}  // namespace rc
}  // namespace spc
