// KV backing tier: fingerprinted block keys, a batch get/put store interface, the
// stage client that drives it, the pressure-limited restore lookahead, and the
// restore/evict work control of a model whose per-sequence state is paged KV blocks
// plus one recurrent-state record (the Qwen 3.6 hybrid: gated delta-net state).
//
//   format_key          binds model fingerprint, cache-layout fingerprint, rank,
//                       sequence and logical block, so a model or layout change
//                       can never read stale KV
//   Store / MemoryStore batch submit + poll (poll answers Ok on delivery; the batch
//                       outcome travels in the completion's status); MemoryStore
//                       keeps blocks in host memory and completes batches on a
//                       worker thread
//   StageKvClient       explicit enablement ("none" = disabled), batch ids, the
//                       in-flight bound
//   select_lookahead    how many queued packets to restore ahead: the largest n
//                       within the normalised lookahead whose cumulative
//                       non-resident blocks fit both the free physical blocks and
//                       the staging capacity
//   TierMover           one restore (GET) and one evict (PUT) channel over the
//                       client: restore batches take whole lanes (state record
//                       first, then the lane's blocks), chosen by binary search
//                       over the lanes' monotone record prefix sums; each channel
//                       is Free -> InFlight -> Landed -> collected
//
// Reference behaviour: crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_kv_store.h
// (constants, operations, completion contract), spark_stage_kv_client.h (client, key
// binding), and the Qwen 3.6 work control's batch rules
// (V/model-families/qwen36/include/sparkpipe/spark_qwen36_work_control.h: lanes
// whole, state record first, one restore and one evict batch outstanding). The
// reference ships no store or client implementation; these are this framework's own.
#pragma once

#include <condition_variable>
#include <cstdint>
#include <deque>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "common.h"

namespace spc {
namespace kvt {

constexpr uint32_t kMaxKeyBytes = 192;
constexpr uint32_t kMaxBatchBlocks = 128;
constexpr uint32_t kMaxInflightBatches = 8;
constexpr uint32_t kDefaultLookahead = 3;
constexpr uint32_t kMaxLookahead = 8;
constexpr uint32_t kStateBlock = 0xffffffffu;  // logical block id of the recurrent-state record

enum Op : uint32_t { Get = 1, Put = 2 };

struct Block {
  uint32_t op = 0;
  std::string key;
  uint8_t* payload = nullptr;
  uint32_t bytes = 0;
};

struct Completion {
  uint64_t batch_id = 0;
  Status status = Status::Pending;
  uint32_t completed_blocks = 0;
};

std::string format_key(uint64_t model_fp, uint64_t layout_fp, uint32_t rank, uint64_t sequence, uint32_t block);
uint32_t normalize_lookahead(uint32_t lookahead, uint32_t queue_depth);
uint32_t select_lookahead(uint32_t lookahead, uint32_t queue_depth, uint32_t physical_capacity,
                          uint32_t allocated, uint32_t staging_capacity, const std::vector<uint32_t>& cumulative);

class Store {
 public:
  virtual ~Store() = default;
  virtual Status submit(uint64_t batch_id, const std::vector<Block>& blocks, uint32_t priority) = 0;
  // Ok with the completion once the batch is done; Pending while it runs; NotFound
  // for an unknown batch id.
  virtual Status poll(uint64_t batch_id, Completion& out) = 0;
};

// Host-memory store: a worker thread executes batches in submission order.
class MemoryStore : public Store {
 public:
  MemoryStore();
  ~MemoryStore() override;
  Status submit(uint64_t batch_id, const std::vector<Block>& blocks, uint32_t priority) override;
  Status poll(uint64_t batch_id, Completion& out) override;
  size_t stored_blocks() const;
  void set_paused(bool paused);  // tests: hold batches in the queue

 private:
  struct Job {
    uint64_t id;
    std::vector<Block> blocks;
  };
  void run();
  mutable std::mutex mu_;
  std::condition_variable cv_;
  std::deque<Job> queue_;
  std::unordered_map<uint64_t, Completion> done_;
  std::unordered_map<uint64_t, bool> known_;
  std::unordered_map<std::string, std::vector<uint8_t>> data_;
  bool stop_ = false, paused_ = false;
  std::thread worker_;
};

class StageKvClient {
 public:
  // provider "none" disables the tier (submissions are refused with NotFound).
  StageKvClient(const std::string& provider, std::shared_ptr<Store> store, uint32_t rank, uint64_t model_fp,
                uint64_t layout_fp);
  bool enabled() const { return enabled_; }
  uint64_t submit(uint32_t op, const std::vector<Block>& blocks, uint32_t priority);
  Status poll(uint64_t batch_id, Completion& out);
  uint32_t inflight() const { return uint32_t(inflight_.size()); }
  uint32_t rank() const { return rank_; }
  uint64_t model_fp() const { return model_fp_; }
  uint64_t layout_fp() const { return layout_fp_; }

 private:
  bool enabled_;
  std::shared_ptr<Store> store_;
  uint32_t rank_;
  uint64_t model_fp_, layout_fp_, next_id_ = 1;
  std::map<uint64_t, bool> inflight_;
};

// ---------------------------------------------------------------- tier mover
// Moves the KV of a model whose per-sequence state is paged KV blocks plus one
// recurrent-state record between the device's staging area and the backing store.
struct PlanConfig {
  uint64_t model_fp = 0, layout_fp = 0;
  uint32_t rank = 0, block_bytes = 0, state_bytes = 0;
  uint32_t lookahead = kDefaultLookahead, physical_capacity = 0, allocated = 0, staging_capacity = 0;
};

struct PendingLane {
  uint64_t sequence = 0;
  std::vector<uint32_t> blocks;  // non-resident logical blocks
  bool state_nonresident = false;
};

// Host staging records: block records of block_bytes at `blocks`, state records of
// state_bytes at `states`; `batch_blocks` caps the records of one batch.
struct Staging {
  uint8_t* blocks = nullptr;
  uint32_t block_records = 0;
  uint8_t* states = nullptr;
  uint32_t state_records = 0;
  uint32_t batch_blocks = 0;
};

enum class Direction : uint32_t { Restore = 0, Evict = 1 };
enum ChannelStage : uint32_t { Free = 0, InFlight = 1, Landed = 2 };
constexpr uint32_t kPriorityImmediate = 0, kPrioritySpeculative = 1;

struct Channel {
  uint64_t batch_id = 0;
  uint32_t stage = Free, blocks = 0;
  Status outcome = Status::Ok;
};

struct RestoreBatch {
  std::vector<Block> blocks;
  uint32_t lanes_built = 0, block_records = 0, state_records = 0;
};

uint32_t state_block_equivalents(uint32_t state_bytes, uint32_t block_bytes);
// Non-resident block counts summed packet by packet (a packet owns consecutive lanes).
std::vector<uint32_t> cumulative_nonresident(const std::vector<PendingLane>& lanes,
                                             const std::vector<uint32_t>& packet_lane_counts,
                                             uint32_t state_equivalents);

// One restore channel and one evict channel over a stage KV client. A restore takes
// whole lanes in order, each lane's state record ahead of its blocks; the batch ends
// before the first lane whose records would overflow the batch or either staging
// area (CapacityExceeded when even the first lane does not fit).
class TierMover {
 public:
  TierMover(const PlanConfig& c, StageKvClient& client, const Staging& staging);
  // how many queued packets to restore ahead under the current memory pressure
  uint32_t restore_packets(const std::vector<uint32_t>& cumulative) const;
  RestoreBatch plan_restore(const std::vector<PendingLane>& lanes,
                            const std::vector<uint32_t>& packet_lane_counts) const;
  // Evicted bytes are read from the caller's buffers: resident[i] at block_src + i * block_bytes.
  std::vector<Block> plan_evict(uint64_t sequence, const std::vector<uint32_t>& resident, bool include_state,
                                const uint8_t* block_src, const uint8_t* state_src) const;
  void start(Direction d, const std::vector<Block>& blocks, uint32_t priority);
  void poll();                         // advances both channels; never blocks
  const Channel& channel(Direction d) const { return ch_[uint32_t(d)]; }
  Status collect(Direction d);         // outcome of a landed batch; frees the channel
  const PlanConfig& plan() const { return cfg_; }
  void set_pressure(uint32_t physical_capacity, uint32_t allocated, uint32_t staging_capacity);

 private:
  Block record(uint64_t sequence, uint32_t logical, uint32_t op, uint8_t* at, uint32_t bytes) const;
  PlanConfig cfg_;
  StageKvClient& client_;
  Staging st_;
  Channel ch_[2];
};

}  // namespace kvt
}  // namespace spc
