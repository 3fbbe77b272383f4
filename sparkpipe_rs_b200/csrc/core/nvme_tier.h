// Tier 3 of the KV cache: blocks on a drive, fetched just in time.
//
// Device memory (tier 1) and pinned host memory (tier 2, serving/kv_offload.py)
// hold tens of gigabytes; a drive holds a terabyte. This tier answers one
// question: can a block's bytes be upstairs before the step that reads it? It
// reads the schedule instead of fetching on a miss: the planner turns "block h is
// needed by step s" into a deadline-ordered prefetch queue, and `pump` (called
// between steps) issues reads early enough, given the configured drive bandwidth
// and step time, that the transfer hides behind compute.
//
//   - Eviction is a generation bump on a clock sweep (never a write-back): the
//     bytes can be re-fetched from the source tier or recomputed by prefill. A
//     read that lands in a slot evicted meanwhile is discarded by its generation.
//   - `request_demand` never blocks, never allocates a slot and never evicts: it
//     answers READY (bytes in a staging buffer), IN_FLIGHT (joined a running
//     read), STARTED (issued the read) or MISS (not on the drive: recompute).
//     A MISS is the only legitimate stall and is counted; a demand that finds
//     every staging buffer held is a sizing error and is counted separately.
//   - Writes are two-phase: reserve a slot (not readable), write the bytes at the
//     reservation's offset, then commit (now readable) or abort.
//   - The drive is an interface (submit / poll / cancel, nothing blocks). The file
//     device reads a file or block device with O_DIRECT where it is accepted
//     (4096-byte aligned offsets, sizes and buffers) on worker threads; tests use
//     a device that completes a read after a programmed number of polls.
//
// Single owner thread: every mutable call comes from the engine's thread.
//
// Reference behaviour: crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_nvme_tier.h
// (JIT tier design :3-37, sizing defaults :51-76, device contract :109-126, demand
// states, residency assessment and statistics). The reference ships the interface;
// the slot table, queue, staging pool and file device here are this framework's own.
#pragma once

#include <condition_variable>
#include <cstdint>
#include <deque>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "common.h"

namespace spc {
namespace nvt {

constexpr uint32_t kIoAlignment = 4096;
constexpr uint64_t kDefaultBudgetBytes = 1ull << 40;              // 1 TB region
constexpr uint64_t kDefaultBytesPerSecond = 5000000000ull;        // conservative drive read rate
constexpr uint32_t kDefaultStepMicroseconds = 67700;              // one decode step
constexpr uint32_t kMaxStagingBuffers = 16;
constexpr uint32_t kDefaultPendingCapacity = 256;

struct Config {
  uint64_t budget_bytes = kDefaultBudgetBytes;
  uint64_t base_offset = 0;
  uint32_t block_bytes = 0;              // multiple of kIoAlignment
  uint32_t staging_buffers = 4;          // >= 2
  uint32_t demand_reserve = 1;           // staging buffers prefetch may never take
  uint32_t pending_capacity = kDefaultPendingCapacity;
  uint64_t device_bytes_per_second = kDefaultBytesPerSecond;
  uint32_t step_microseconds = kDefaultStepMicroseconds;
};

// The asynchronous block device. submit_read queues a read of `bytes` at `offset`
// into `dst` (owned by the device until poll answers Ok / IoError, or cancel Ok);
// poll answers Ok, Busy or IoError; cancel answers Ok (the device will not touch
// dst again) or Busy (still device-owned: keep polling).
class BlockDevice {
 public:
  virtual ~BlockDevice() = default;
  virtual Status submit_read(uint64_t offset, void* dst, uint32_t bytes, uint64_t* ticket) = 0;
  virtual Status poll(uint64_t ticket) = 0;
  virtual Status cancel(uint64_t ticket) { (void)ticket; return Status::Busy; }
  // Synchronous write used by the write-back path (never on the decode path).
  virtual Status write(uint64_t offset, const void* src, uint32_t bytes) = 0;
};

// A file or block device. O_DIRECT is requested and dropped if the file system
// refuses it; reads run on `threads` worker threads.
class FileDevice : public BlockDevice {
 public:
  FileDevice(const std::string& path, uint64_t size_bytes, uint32_t threads = 2);
  ~FileDevice() override;
  Status submit_read(uint64_t offset, void* dst, uint32_t bytes, uint64_t* ticket) override;
  Status poll(uint64_t ticket) override;
  Status write(uint64_t offset, const void* src, uint32_t bytes) override;
  bool direct() const { return direct_; }

 private:
  struct Req {
    uint64_t ticket;
    uint64_t offset;
    void* dst;
    uint32_t bytes;
  };
  void worker();
  int fd_ = -1;
  bool direct_ = false;
  std::mutex mu_;
  std::condition_variable cv_;
  std::deque<Req> queue_;
  std::unordered_map<uint64_t, Status> done_;
  uint64_t next_ticket_ = 1;
  bool stop_ = false;
  std::vector<std::thread> workers_;
};

// Completes a read after `latency_polls` polls (copying from its own memory), so
// the tier's schedule logic is testable without a drive.
class MockDevice : public BlockDevice {
 public:
  MockDevice(uint64_t size_bytes, uint32_t latency_polls);
  Status submit_read(uint64_t offset, void* dst, uint32_t bytes, uint64_t* ticket) override;
  Status poll(uint64_t ticket) override;
  Status cancel(uint64_t ticket) override;
  Status write(uint64_t offset, const void* src, uint32_t bytes) override;
  void fail_next_read() { fail_next_ = true; }
  uint64_t reads() const { return reads_; }

 private:
  struct Req {
    uint64_t offset;
    void* dst;
    uint32_t bytes;
    uint32_t polls_left;
    bool fail;
  };
  std::vector<uint8_t> mem_;
  uint32_t latency_;
  std::unordered_map<uint64_t, Req> live_;
  uint64_t next_ticket_ = 1;
  uint64_t reads_ = 0;
  bool fail_next_ = false;
};

enum class Demand : uint32_t { Ready = 0, InFlight = 1, Started = 2, Miss = 3 };
enum class Confidence : uint32_t { All = 0, Partial = 1, None = 2 };

struct Need {
  uint64_t hash = 0;
  uint32_t need_by_step = 0;
};

struct Reservation {
  uint64_t hash = 0;
  uint64_t offset = 0;
  uint32_t slot = 0;
  uint32_t generation = 0;
  bool already_present = false;
};

struct PlanReport {
  uint32_t ready = 0, inflight = 0, queued = 0, absent = 0, queue_full = 0, late_risk = 0;
};

struct Residency {
  Confidence confidence = Confidence::All;
  uint32_t ready = 0, inflight_on_time = 0, planned_on_time = 0, late = 0, absent = 0;
};

struct Stats {
  uint64_t write_reservations = 0, publishes = 0, write_aborts = 0, evictions = 0, pinned_skips = 0;
  uint64_t demand_hits = 0, demand_joins = 0, demand_loads = 0, demand_misses = 0, demand_stalls = 0;
  uint64_t prefetch_issues = 0, prefetch_landings = 0, prefetch_late = 0, prefetch_preemptions = 0;
  uint64_t prefetch_dropped = 0, stale_completions = 0, io_errors = 0, read_bytes = 0;
  uint64_t slot_count = 0, slots_in_use = 0;
};

class Tier {
 public:
  Tier(const Config& cfg, std::shared_ptr<BlockDevice> device);
  ~Tier();

  Reservation reserve_write(uint64_t hash);
  void commit_write(const Reservation& r);
  void abort_write(const Reservation& r);
  bool offset_of(uint64_t hash, uint64_t* offset) const;

  PlanReport plan_lookahead(const std::vector<Need>& needs, uint32_t step_now);
  Demand request_demand(uint64_t hash, uint32_t step_now, const uint8_t** staging);
  void pump(uint32_t step_now);
  bool consume(uint64_t hash);
  bool pin(uint64_t hash, bool on);
  Residency will_be_resident_by(const std::vector<uint64_t>& hashes, uint32_t step_now,
                                uint32_t step_deadline) const;

  const Stats& stats() const { return stats_; }
  uint32_t transfer_steps() const { return transfer_steps_; }
  const Config& config() const { return cfg_; }
  // Reads in flight that must land (or be cancelled) before the staging memory can
  // be released; `drain` polls them (bounded by `max_polls`) and reports what is left.
  uint32_t inflight() const;
  uint32_t drain(uint32_t max_polls);

 private:
  enum SlotState : uint8_t { Free = 0, Reserved = 1, Committed = 2 };
  struct Slot {
    uint64_t hash = 0;
    uint32_t generation = 0;
    uint8_t state = Free;
    bool referenced = false;
    int32_t pins = 0;
  };
  enum BufState : uint8_t { Idle = 0, Reading = 1, Ready = 2 };
  struct Buffer {
    uint8_t state = Idle;
    bool demand = false;      // held for a demand (never preempted)
    bool cancelling = false;  // device still owns it after a cancel request
    uint64_t hash = 0;
    uint32_t slot = 0, generation = 0;
    uint64_t ticket = 0;
    uint32_t issued_step = 0, need_by = 0;
  };
  struct Pending {
    uint64_t hash;
    uint32_t need_by;
    bool demand;  // a demand that found no staging buffer, retried first
  };
  int buffer_of(uint64_t hash) const;
  int free_buffer(bool for_demand);
  bool issue(int b, uint32_t slot, bool demand, uint32_t step_now, uint32_t need_by);
  uint32_t evict_one();

  Config cfg_;
  std::shared_ptr<BlockDevice> dev_;
  std::vector<Slot> slots_;
  std::unordered_map<uint64_t, uint32_t> index_;  // committed hash -> slot
  std::vector<uint32_t> free_;
  uint32_t hand_ = 0;
  std::vector<Buffer> bufs_;
  uint8_t* staging_ = nullptr;
  std::vector<Pending> pending_;  // sorted by need_by
  uint32_t transfer_steps_ = 1;
  Stats stats_;
};

}  // namespace nvt
}  // namespace spc
