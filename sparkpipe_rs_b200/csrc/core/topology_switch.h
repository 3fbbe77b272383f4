// Live re-shard between parallel layouts (tensor-parallel <-> pipeline-parallel
// recipes) with requests in flight.
//
// STEADY -> QUIESCE (admissions closed; wait until every tracked sequence is at
// a token boundary or finished) -> CHECKPOINT (pin each sequence's KV blocks on
// the tier, write one manifest per sequence) -> SWAP (start + poll the weight
// swap) -> RESUME (a sequence whose blocks all survived is WARM: its blocks are
// planned into the tier lookahead and prefill is skipped; one missing block
// makes it RECOMPUTE) -> STEADY. Every phase retries on the next `advance`
// instead of aborting; there is no cancel (a half-swapped residency is worse
// than either recipe).
//
// Tier keys are strategy-neutral: FNV-1a seeded with the model/geometry
// namespace over the block's content hash, so re-sharding moves residency
// without invalidating content.
//
// Reference behaviour: crates/spark-sched/src/topology_switch.rs (states
// :113-180, seams :182-260, keys :262-280, machine :330-866). The manifest
// record (sequence id, recipe id, position, block count, keys; little-endian)
// and the key derivation are kept so checkpoints stay interchangeable.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "common.h"

namespace spc {
namespace ts {

constexpr uint64_t kManifestDomain = 0x9e3779b97f4a7c15ull;
constexpr size_t kPlanChunk = 16;
constexpr uint64_t kManifestHeaderBytes = 24;

enum class Strategy : uint32_t { TensorParallel = 0, PipelineParallel = 1 };
enum class State : uint32_t { Steady = 0, Quiesce, Checkpoint, Swap, Resume };
enum class ResumeClass : uint32_t { Pending = 0, Warm, Recompute };

struct Recipe {
  uint64_t recipe_id = 0;
  uint64_t weight_pack_bytes = 0;
  Strategy strategy = Strategy::TensorParallel;
};

struct Budget {
  uint64_t quiesce_us = 0, checkpoint_us = 0, swap_fixed_us = 0, swap_stream_us = 0, resume_warm_us = 0, total_us = 0;
};

struct Stats {
  uint64_t switches_completed = 0, sequences_checkpointed = 0, resumed_warm = 0, resumed_recompute = 0;
  uint64_t completed_mid_switch = 0, blocks_pinned = 0, manifest_writes = 0, manifest_bytes = 0;
  uint64_t tier_blocks_found = 0, tier_blocks_absent = 0, swaps_started = 0;
};

struct Config {
  uint64_t kv_namespace = 0;
  uint32_t max_sequences = 0, max_blocks_per_sequence = 0, step_time_us = 0, manifest_block_bytes = 0;
  uint64_t read_bytes_per_s = 0, write_bytes_per_s = 0, swap_fixed_us = 0;
  Recipe initial;
};

struct TierNeed {
  uint64_t key = 0;
  uint32_t need_by_step = 0;
};
struct WriteReservation {
  uint64_t device_offset = 0;
  bool already_present = false;
};

// Seams; implementations return a Status (Ok, NotFound, Busy, ...).
class Tier {
 public:
  virtual ~Tier() = default;
  virtual Status pin(uint64_t key, bool pinned) = 0;
  virtual Status offset_of(uint64_t key, uint64_t* offset) = 0;
  virtual Status reserve_write(uint64_t key, WriteReservation* out) = 0;
  virtual Status commit_write(const WriteReservation& r) = 0;
  virtual void abort_write(const WriteReservation& r) = 0;
  virtual Status plan_lookahead(const std::vector<TierNeed>& needs, uint32_t step_now) = 0;
};
class SwapDevice {
 public:
  virtual ~SwapDevice() = default;
  virtual Status begin_swap(const Recipe& from, const Recipe& to) = 0;
  virtual Status poll_swap() = 0;  // Ok when resident, Busy while streaming
};
class ManifestWriter {
 public:
  virtual ~ManifestWriter() = default;
  virtual Status write_block(uint64_t device_offset, const std::string& payload) = 0;
};

uint64_t kv_key(uint64_t kv_namespace, uint64_t content_hash);
uint64_t manifest_key(uint64_t kv_namespace, uint64_t sequence_id);
Budget estimate_budget(const Config& c, const Recipe& target, uint32_t active_sequences, uint64_t warm_kv_bytes);

class TopologySwitch {
 public:
  // The seams are borrowed and must outlive the switch.
  TopologySwitch(const Config& c, Tier* tier, SwapDevice* swap, ManifestWriter* writer);
  bool admissions_open() const { return state_ == State::Steady; }
  State state() const { return state_; }
  const Recipe& current_recipe() const { return current_; }
  Status last_error() const { return last_error_; }
  const Stats& stats() const { return st_; }
  uint32_t tracked() const { return tracked_; }

  void track_sequence(uint64_t sequence_id, uint64_t recipe_id);
  void set_sequence_kv(uint64_t sequence_id, uint32_t position, const std::vector<uint64_t>& content_hashes);
  void sequence_at_boundary(uint64_t sequence_id);
  void sequence_complete(uint64_t sequence_id);
  void begin(const Recipe& target);
  State advance(uint32_t step_now);
  ResumeClass resume_class_of(uint64_t sequence_id) const;

 private:
  enum class Slot : uint8_t { Free, Active, AtBoundary };
  struct Seq {
    uint64_t id = 0, recipe = 0;
    uint32_t position = 0, blocks = 0;
    Slot slot = Slot::Free;
    ResumeClass resume = ResumeClass::Pending;
    bool pinned = false, checkpointed = false;
  };
  int find(uint64_t id) const;
  bool checkpoint_all();
  Status checkpoint(size_t i);
  void resume(size_t i, uint32_t step_now);
  uint64_t* keys_of(size_t i) { return &keys_[i * cfg_.max_blocks_per_sequence]; }

  Config cfg_;
  Tier* tier_;
  SwapDevice* swap_;
  ManifestWriter* writer_;
  std::vector<Seq> seqs_;
  std::vector<uint64_t> keys_;
  Recipe current_, target_;
  State state_ = State::Steady;
  uint32_t tracked_ = 0;
  size_t cursor_ = 0;
  bool swap_started_ = false;
  Status last_error_ = Status::Ok;
  Stats st_;
};

}  // namespace ts
}  // namespace spc
