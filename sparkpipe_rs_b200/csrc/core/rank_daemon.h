// Per-rank work daemon of a pipeline: idempotent work transactions over the
// work-control packets (work_control.h).
//
//   submit(packet bytes)  dedup (FNV-32 of the wire bytes over a recent window),
//                         parse, ledger handshake (observe: new / replay / conflict),
//                         queue; answers with a 96-byte acknowledgement
//   pump()                takes queued packets in order, holding back any packet
//                         whose sequences still have an earlier step in flight,
//                         forwards each to the next rank first, then hands it to the
//                         local executor (forward-then-submit)
//   complete(...)         executor's completion: ledger commit / failure, the
//                         sequences' next steps released, and on the last rank a
//                         272-byte final event for rank 0
//
// The transaction ledger is an open-addressed table keyed by the transaction
// identity (linear probing from the identity fingerprint, tombstones reused,
// oldest terminal entry recycled when full, reset on a newer control generation;
// states PREPARED -> ACCEPTED -> EXECUTING -> COMMITTED | CANCELLED | FAILED).
//
// Reference behaviour: crates/spark-node/src/rank_daemon/work_ledger.rs (ledger),
// wire.rs (identity 56 B / acknowledgement 96 B / final event 272 B, packet dedup
// hash), daemon.rs (queue, ordering, pump). The wire records keep the reference's
// sizes and field order so acknowledgements and final events interoperate.
#pragma once

#include <deque>
#include <functional>
#include <map>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.h"
#include "work_control.h"

namespace spc {
namespace rd {

constexpr uint32_t kAckMagic = 0x4b434157u;    // "WACK"
constexpr uint32_t kFinalMagic = 0x4e494647u;  // "GFIN"
constexpr uint32_t kWireAbi = 1;
constexpr size_t kIdentityBytes = 56;
constexpr size_t kAckBytes = 96;
constexpr size_t kFinalEventBytes = 272;
constexpr uint32_t kMaxFinalTokens = 8;

enum TxState : uint32_t { Empty = 0, Prepared, Accepted, Executing, Committed, Cancelled, Failed, Tombstone };
inline bool tx_terminal(uint32_t s) { return s == Committed || s == Cancelled || s == Failed; }

std::string identity_to_wire(const wc::Identity& id);
wc::Identity identity_from_wire(const std::string& b);
uint64_t identity_fingerprint(const wc::Identity& id);
uint32_t packet_dedup_hash32(const uint8_t* data, size_t n);

struct Ack {
  uint32_t status = 0, state = 0;
  wc::Identity identity;
  uint64_t packet_fingerprint = 0;
};
std::string ack_to_wire(const Ack& a);
Ack ack_from_wire(const std::string& b);  // AbiMismatch on bad magic / size

struct FinalEvent {
  uint32_t status = 0, program_id = 0, slot = 0, accepted_token_count = 0, completion_flags = 0;
  std::vector<uint32_t> token_ids;        // <= 8
  std::vector<uint32_t> draft_token_ids;  // <= 8
  uint64_t request_id = 0, sequence_id = 0, sequence_position = 0, service_time_ns = 0;
  wc::Identity identity;
};
std::string final_event_to_wire(const FinalEvent& e);
FinalEvent final_event_from_wire(const std::string& b);

// ------------------------------------------------------------------ ledger
enum class Observation : uint32_t { New = 0, ReplayActive, ReplayTerminal, Conflict };

struct LedgerEntry {
  wc::Identity identity;
  uint64_t payload_fingerprint = 0, last_observed_epoch = 0;
  uint32_t state = Empty;
  uint32_t terminal_status = uint32_t(Status::Pending);
};

class TransactionLedger {
 public:
  explicit TransactionLedger(uint32_t capacity);
  Observation observe(const wc::Identity& id, uint64_t payload_fingerprint);  // throws on bad input / full
  void transition(const wc::Identity& id, uint32_t target, Status terminal_status = Status::Ok);
  const LedgerEntry* find(const wc::Identity& id) const;
  uint32_t entries() const { return entry_count_; }
  uint32_t active() const { return active_count_; }
  uint32_t terminal() const { return terminal_count_; }
  uint32_t tombstones() const { return tombstone_count_; }
  uint64_t control_generation() const { return generation_; }
  uint32_t capacity() const { return uint32_t(table_.size()); }

 private:
  int64_t find_index(const wc::Identity& id) const;
  uint32_t start(const wc::Identity& id) const;
  void reset(uint64_t generation);
  void prepare_generation(uint64_t generation);
  void recycle_oldest_terminal();
  int64_t insertion_index(const wc::Identity& id);
  std::vector<LedgerEntry> table_;
  uint32_t entry_count_ = 0, active_count_ = 0, terminal_count_ = 0, tombstone_count_ = 0;
  uint64_t epoch_ = 0, generation_ = 0;
};

// ------------------------------------------------------------------ daemon
struct DaemonConfig {
  uint32_t rank = 0, world = 1;         // pipeline position
  uint32_t queue_capacity = 64;
  uint32_t ledger_capacity = 4096;
  uint32_t dedup_window = 256;          // recent packet hashes remembered
  wc::Config work;                      // packet geometry (validation)
};

struct DaemonStats {
  uint64_t submitted = 0, accepted = 0, duplicates = 0, conflicts = 0, rejected = 0;
  uint64_t forwarded = 0, executed = 0, committed = 0, failed = 0, cancelled = 0, final_events = 0;
  uint32_t queued = 0, inflight = 0;
};

class RankDaemon {
 public:
  using ForwardFn = std::function<void(const std::string& packet_wire)>;
  using ExecuteFn = std::function<void(const std::string& packet_wire)>;
  using FinalFn = std::function<void(const std::string& final_event_wire)>;

  RankDaemon(const DaemonConfig& cfg, ForwardFn forward, ExecuteFn execute, FinalFn final_event);
  // Returns the acknowledgement (96 bytes). Never throws for bad packets: they are
  // acknowledged with a failure status.
  std::string submit(const std::string& packet_wire);
  // Dispatches up to `max_packets` ready packets; returns how many.
  uint32_t pump(uint32_t max_packets = 64);
  // Completion of an executed packet (by its transaction identity).
  void complete(const wc::Identity& id, Status status, const std::vector<uint32_t>& tokens,
                uint64_t service_time_ns);
  // Completion of a batched packet: on the last rank, one final event per lane with
  // that lane's tokens (lane_tokens[i] for packet lane i).
  void complete_lanes(const wc::Identity& id, Status status, const std::vector<std::vector<uint32_t>>& lane_tokens,
                      uint64_t service_time_ns);
  void cancel(const wc::Identity& id);
  const TransactionLedger& ledger() const { return ledger_; }
  DaemonStats stats() const;

 private:
  struct Item {
    wc::Packet packet;
    std::string wire;
    uint64_t fingerprint;
  };
  bool ready(const Item& it) const;
  Item retire(const wc::Identity& id, Status status);  // ledger + bookkeeping of a completion
  DaemonConfig cfg_;
  ForwardFn forward_;
  ExecuteFn execute_;
  FinalFn final_;
  TransactionLedger ledger_;
  std::deque<Item> queue_;
  std::deque<uint32_t> recent_;                    // dedup window (FIFO)
  std::unordered_map<uint32_t, uint32_t> recent_count_;
  std::unordered_map<uint64_t, uint32_t> busy_seq_;  // sequence id -> in-flight packets
  std::map<uint64_t, Item> inflight_;                // transaction id -> packet
  DaemonStats st_;
};

}  // namespace rd
}  // namespace spc
