// Host-side expert batching queue: one FIFO of token rows per (layer, expert).
//
//   LowLatency   a slot fires once it holds `firing_threshold_rows` rows or its oldest
//                row has waited `firing_deadline_ns`; a firing takes at most
//                kMaxFiringRows rows, oldest first.
//   SealedBatch  rows accumulate until the layer is sealed; then every non-empty slot
//                of the layer fires whole, and the layer unseals once drained.
//
// next_firing() scans layers, then experts, in index order and returns the first slot
// that should fire. Row storage is a fixed pool (kMaxRows) with a free list, so the
// queue never allocates after construction.
//
// On the GPU path the same batching is done on the device (moe_align / ep_recv_align
// build the per-expert row ranges of a step); this queue is for hosts that drive
// experts themselves (CPU offload, batched prefill across requests).
//
// Reference behaviour: V/model-families/glm52/src/spark_glm52_expert_queue.c:31-230
// (validation, enqueue, seal, SlotShouldFire :152-168, NextFiring :170-230).
#pragma once

#include <cstdint>
#include <vector>

#include "common.h"

namespace spc {
namespace eq {

constexpr uint32_t kMaxLayers = 8;
constexpr uint32_t kMaxExperts = 256;
constexpr uint32_t kMaxRows = 1u << 20;
constexpr uint32_t kMaxFiringRows = 1024;

enum class Mode : uint32_t { Invalid = 0, LowLatency = 1, SealedBatch = 2 };

struct Config {
  uint32_t layer_count = 0, expert_count = 0, firing_threshold_rows = 0;
  uint64_t firing_deadline_ns = 0;
  Mode mode = Mode::Invalid;
};

struct Firing {
  uint32_t layer = 0, expert = 0;
  std::vector<uint64_t> row_ids;
};

struct Stats {
  uint64_t firings = 0, fired_rows = 0;
  uint32_t enqueued = 0;
};

class ExpertQueue {
 public:
  explicit ExpertQueue(const Config& c);  // InvalidArgument on a bad configuration
  void enqueue(uint32_t layer, uint32_t expert, uint64_t row_id, uint64_t arrival_ns);
  void seal(uint32_t layer);
  void set_firing_threshold(uint32_t rows);
  // The next slot to fire at `now_ns`; false when none is due.
  bool next_firing(uint64_t now_ns, Firing& out);
  uint32_t slot_rows(uint32_t layer, uint32_t expert) const;
  uint32_t layer_rows(uint32_t layer) const { return layer_rows_.at(layer); }
  bool sealed(uint32_t layer) const { return sealed_.at(layer) != 0; }
  Stats stats() const { return st_; }
  const Config& config() const { return cfg_; }

 private:
  static constexpr uint32_t kNil = 0xffffffffu;
  struct Node {
    uint64_t row_id, arrival_ns;
    uint32_t next;
  };
  struct Slot {
    uint32_t head = kNil, tail = kNil, count = 0;
    uint64_t oldest_ns = 0;
  };
  Slot& slot(uint32_t l, uint32_t e) { return slots_[size_t(l) * cfg_.expert_count + e]; }
  const Slot& slot(uint32_t l, uint32_t e) const { return slots_[size_t(l) * cfg_.expert_count + e]; }
  bool due(uint32_t layer, const Slot& s, uint64_t now_ns) const;
  uint32_t take_node();
  Config cfg_;
  std::vector<Node> pool_;
  uint32_t free_ = kNil, used_high_ = 0;
  std::vector<Slot> slots_;
  std::vector<uint32_t> layer_rows_, sealed_;
  Stats st_;
};

}  // namespace eq
}  // namespace spc
