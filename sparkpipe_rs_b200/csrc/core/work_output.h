// Work-output plane of a pipeline rank: the bounded queue of work packets bound for
// the next rank, the non-blocking socket they travel on, the write / acknowledge
// choreography, and the ring of sequence releases waiting to be sent.
//
//   queue        packets are validated and serialised on enqueue; the head packet
//                is written (resuming at the byte where a short write stopped),
//                then its 96-byte acknowledgement (rank_daemon.h) is read and
//                checked against the packet's identity and fingerprint. Ok or
//                Duplicate pops the packet; CapacityExceeded (the next rank's queue
//                was full) rewinds it for a later resend; any other status is a hard
//                negative: resending byte-identical content would be refused the
//                same way forever, so the packet's owner is told and the packet is
//                dropped. A socket error drops the socket; the head packet is resent
//                whole on the next connection (the receiver deduplicates it)
//   socket       non-blocking: connect to the next rank's host and port, or adopt a
//                connected descriptor. pump() never blocks: it answers Busy when the
//                socket would block and RouteNotFound when the connection broke
//   releases     (request, generation, sequence, token count) records queued by the
//                scheduler when sequences finish, packed into release packets of at
//                most `lanes` records and popped once sent
//
// Reference behaviour: crates/spark-node/src/backend/work_output.rs (queue :44-110,
// socket :286-350, flush and acknowledgement handling :350-465, release ring
// :465-565). The code is this runtime's own.
#pragma once

#include <cstdint>
#include <deque>
#include <functional>
#include <string>
#include <vector>

#include "common.h"
#include "rank_daemon.h"
#include "work_control.h"

namespace spc {
namespace wo {

struct ReleaseRecord {
  uint64_t request_id = 0, request_generation = 0, sequence_id = 0;
  uint32_t token_count = 0;
};

struct WorkOutputStats {
  uint64_t enqueued = 0, sent = 0, acknowledged = 0, duplicates = 0, resent = 0, hard_failures = 0;
  uint64_t socket_drops = 0, releases_queued = 0, releases_sent = 0;
};

class WorkOutput {
 public:
  using FailFn = std::function<void(const wc::Packet&, Status)>;
  WorkOutput(const wc::Config& cfg, bool has_next, std::string next_host, uint32_t next_port,
             uint32_t execution_row_capacity, uint32_t queue_capacity, uint32_t release_capacity);
  ~WorkOutput();
  WorkOutput(const WorkOutput&) = delete;
  WorkOutput& operator=(const WorkOutput&) = delete;

  void enqueue(const wc::Packet& p);      // validates; CapacityExceeded when full
  void adopt_socket(int fd);              // takes ownership of a connected descriptor
  void drop_socket();
  // Ok when the queue drained, Busy when it would block, RouteNotFound on a broken
  // connection (the socket is dropped; the next pump reconnects).
  Status pump(const FailFn& on_hard_failure = nullptr);

  void queue_release(const ReleaseRecord& r);  // CapacityExceeded when full
  // A release packet of the first min(pending, lanes) records (not popped).
  wc::Packet build_release_packet(const wc::Identity& id, uint32_t lanes) const;
  void pop_releases(uint32_t n);

  bool has_next() const { return has_next_; }
  bool has_socket() const { return fd_ >= 0; }
  uint32_t queued() const { return uint32_t(queue_.size()); }
  uint32_t queue_capacity() const { return queue_capacity_; }
  uint32_t releases() const { return uint32_t(releases_.size()); }
  const ReleaseRecord& release(uint32_t i) const { return releases_.at(i); }
  const WorkOutputStats& stats() const { return st_; }

 private:
  struct Item {
    wc::Packet packet;
    std::vector<uint8_t> bytes;
    uint64_t fingerprint;
  };
  Status ensure_socket();
  void reset_ack();
  wc::Config cfg_;
  bool has_next_;
  std::string host_;
  uint32_t port_, rows_, queue_capacity_, release_capacity_;
  std::deque<Item> queue_;
  std::deque<ReleaseRecord> releases_;
  int fd_ = -1;
  bool connecting_ = false, awaiting_ack_ = false, resending_ = false;
  size_t write_off_ = 0, ack_off_ = 0;
  std::string ack_;
  WorkOutputStats st_;
};

}  // namespace wo
}  // namespace spc
