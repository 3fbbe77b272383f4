// Runtime completion: how one unit of work is carried to a single, acknowledged
// final outcome across the parts of the runtime that each hold some of its state.
//
//   credit ledger        four bounded credit domains (transport window, resident
//                        reservation, execution, completion ownership); a
//                        transaction holds one execution credit while it runs and
//                        one completion-ownership credit until its final event is
//                        acknowledged, so neither runs past its bound
//   participants         up to 32 parts of the runtime (KV reservation, scheduler
//                        slot, transport, ...) with prepare / execute / commit /
//                        cancel entry points. Each must declare transactional
//                        staging (prepare leaves nothing visible), an infallible
//                        commit and an idempotent cancel; the controller refuses any
//                        that does not
//   controller           runs a transaction: the transaction ledger (rank_daemon.h)
//                        classifies it as new, an in-flight replay, a finished replay
//                        (answered from the record, no participant called again) or a
//                        conflict (same identity, other payload). A new one is
//                        prepared by every participant in order, executed by every
//                        participant in order, then committed by all; a failure in
//                        either phase cancels every participant in reverse order
//                        with the failing status. Its outcome is queued as a final
//                        event
//   final event queue    pending outcomes in generation order; acknowledged by
//                        (identity, generation, payload fingerprint)
//   transmission window  bounded slots of work sent to a peer and not yet
//                        acknowledged: reserve (idempotent for the same identity and
//                        payload), mark sent, acknowledge, and the oldest unacknowledged
//                        send picked for replay after a peer restart or a timeout
//
// Reference behaviour: crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_runtime_completion.h:13-226
// (participant flags, slot and final-event states, controller API) and
// spark_work_transaction.h:38-42 (credit domains), :171-183 (credit ledger API).
// The records and the algorithm here are this runtime's own.
#pragma once

#include <array>
#include <cstdint>
#include <deque>
#include <functional>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.h"
#include "rank_daemon.h"
#include "work_control.h"

namespace spc {
namespace rc {

constexpr uint32_t kMaxParticipants = 32;
enum CreditDomain : uint32_t { TransportWindow = 0, ResidentReservation = 1, Execution = 2, CompletionOwnership = 3 };
constexpr uint32_t kCreditDomains = 4;

constexpr uint32_t kFlagTransactionalStaging = 0x1, kFlagCommitInfallible = 0x2, kFlagCancelIdempotent = 0x4;
constexpr uint32_t kRequiredFlags = kFlagTransactionalStaging | kFlagCommitInfallible | kFlagCancelIdempotent;

// ---------------------------------------------------------------- credits
class CreditLedger {
 public:
  explicit CreditLedger(const std::array<uint32_t, kCreditDomains>& capacities);
  bool acquire(uint32_t domain, uint32_t n);  // false (nothing taken) when fewer than n are free
  void release(uint32_t domain, uint32_t n);  // throws on releasing more than is held
  uint32_t available(uint32_t domain) const;
  uint32_t in_use(uint32_t domain) const;
  uint32_t capacity(uint32_t domain) const;

 private:
  static void check(uint32_t domain);
  std::array<uint32_t, kCreditDomains> cap_{}, used_{};
};

// ---------------------------------------------------------------- final events
enum FinalEventState : uint32_t { EventFree = 0, EventPending = 1, EventAcknowledged = 2 };
struct FinalEvent {
  uint32_t state = EventFree;
  uint64_t generation = 0;
  wc::Identity identity;
  uint64_t payload_fingerprint = 0, request_id = 0, sequence_id = 0, sequence_position = 0;
  Status status = Status::Pending;
};

class FinalEventQueue {
 public:
  explicit FinalEventQueue(uint32_t capacity);
  uint64_t push(FinalEvent e);                // assigns the generation; CapacityExceeded when full
  const FinalEvent* peek() const;             // oldest pending, or null
  // Ok, NotFound (no pending event of that generation) or InvalidArgument (identity
  // or payload fingerprint differ from the event's)
  Status acknowledge(const wc::Identity& id, uint64_t generation, uint64_t payload_fingerprint);
  uint32_t pending() const { return uint32_t(events_.size()); }
  uint32_t capacity() const { return capacity_; }
  uint64_t next_generation() const { return next_generation_; }

 private:
  uint32_t capacity_;
  uint64_t next_generation_ = 1;
  std::deque<FinalEvent> events_;  // pending, generation order
};

// ---------------------------------------------------------------- transmission window
enum SlotState : uint32_t { SlotFree = 0, SlotReserved = 1, SlotSent = 2, SlotAcknowledged = 3 };
struct TransmissionSlot {
  uint32_t state = SlotFree, slot_index = 0;
  uint64_t generation = 0;
  wc::Identity identity;
  uint64_t payload_fingerprint = 0, last_send_epoch = 0;
  uint32_t retry_count = 0;
};

class TransmissionWindow {
 public:
  explicit TransmissionWindow(uint32_t capacity);
  // (slot, generation). The same identity and payload already in the window return
  // its slot; the same identity with another payload is Duplicate; a full window Busy.
  std::pair<uint32_t, uint64_t> reserve(const wc::Identity& id, uint64_t payload_fingerprint);
  void mark_sent(uint32_t slot, uint64_t generation);  // a re-send counts a retry
  // Ok (slot freed), NotFound (stale generation: already acknowledged) or
  // InvalidArgument (identity / payload fingerprint differ)
  Status acknowledge(uint32_t slot, uint64_t generation, const wc::Identity& id, uint64_t payload_fingerprint);
  // The sent, unacknowledged slot sent longest ago; false when there is none.
  bool next_replay(uint32_t* slot, uint64_t* generation) const;
  uint32_t in_use() const { return in_use_; }
  uint32_t capacity() const { return uint32_t(slots_.size()); }
  const TransmissionSlot& slot(uint32_t i) const;

 private:
  TransmissionSlot& live(uint32_t slot, uint64_t generation);
  std::vector<TransmissionSlot> slots_;
  uint32_t in_use_ = 0;
  uint64_t next_generation_ = 1, send_epoch_ = 0;
};

// ---------------------------------------------------------------- controller
struct Request {
  wc::Identity identity;
  uint64_t request_id = 0, sequence_id = 0, sequence_position = 0;
  std::string payload;
};

struct Participant {
  std::string name;
  uint32_t flags = kRequiredFlags;
  uint64_t restart_epoch = 1;
  std::function<Status(const Request&)> prepare, execute;
  std::function<void(const Request&)> commit;
  std::function<void(const Request&, Status)> cancel;
};

struct Result {
  bool replayed = false;
  uint32_t committed = 0, cancelled = 0;
  uint64_t payload_fingerprint = 0, final_event_generation = 0;
  Status status = Status::Pending;
};

class Controller {
 public:
  Controller(std::vector<Participant> participants, uint32_t transaction_capacity, uint32_t final_event_capacity,
             const std::array<uint32_t, kCreditDomains>& credits);
  uint64_t validate(const Request& r) const;  // payload fingerprint; throws on a malformed request
  Result run(const Request& r);
  // Acknowledges a final event and returns its completion-ownership credit.
  Status acknowledge_final_event(const wc::Identity& id, uint64_t generation, uint64_t payload_fingerprint);
  uint32_t participant_count() const { return uint32_t(parts_.size()); }
  const Participant& participant(uint32_t i) const { return parts_.at(i); }
  const rd::TransactionLedger& ledger() const { return ledger_; }
  const FinalEventQueue& final_events() const { return events_; }
  const CreditLedger& credits() const { return credits_; }

 private:
  uint32_t cancel_all(const Request& r, size_t upto, Status reason);
  std::vector<Participant> parts_;
  rd::TransactionLedger ledger_;
  FinalEventQueue events_;
  CreditLedger credits_;
  std::unordered_map<uint64_t, uint64_t> generation_of_;  // identity fingerprint -> final event generation
  std::deque<uint64_t> generation_order_;                  // bounds generation_of_ to the ledger's capacity
};

}  // namespace rc
}  // namespace spc
