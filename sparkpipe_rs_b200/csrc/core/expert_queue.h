// Host-side expert batching queue: token rows wait per (layer, expert) slot until the
// slot is due, then leave as one firing.
//
//   LowLatency   a slot is due once it holds `firing_threshold_rows` rows or its oldest
//                row has waited `firing_deadline_ns`; a firing takes at most
//                kMaxFiringRows rows, oldest first.
//   SealedBatch  rows accumulate until their layer is sealed; then every non-empty slot
//                of the layer fires whole, and the layer unseals once drained.
//
// When several slots are due, the one with the lowest (layer, expert) index fires first.
//
// Design. Every slot keeps its rows in its own ring buffer (arrival order is the
// buffer order). Each slot also carries one "due key": 0 when it is due regardless of
// the clock (threshold reached, or its layer is sealed), its oldest arrival plus the
// deadline when only time can make it due, and kNever when it is empty. The keys sit
// in the leaves of a min tournament tree over the slot index, so next_firing(now) is a
// descent to the leftmost leaf whose key is <= now: O(log slots) per firing instead
// of a scan of every slot, and the lowest-index rule falls out of the left-first
// descent. A key changes only when its slot gains its first row, crosses the threshold
// or fires, or when its layer is sealed / unsealed, and each change is one leaf-to-root
// update.
//
// On the GPU path the same batching is done on the device (moe_align / ep_recv_align
// build the per-expert row ranges of a step); this queue is for hosts that drive
// experts themselves (CPU offload, batched prefill across requests).
//
// Reference behaviour (limits, statuses, firing rule): the GLM-5.2 expert queue,
// V/model-families/glm52/include/sparkpipe/spark_glm52_expert_queue.h:7-91.
#pragma once

#include <cstdint>
#include <vector>

#include "common.h"

namespace spc {
namespace eq {

constexpr uint32_t kMaxLayers = 8;
constexpr uint32_t kMaxExperts = 256;
constexpr uint32_t kMaxRows = 1u << 20;       // rows queued at once over all slots
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
  uint32_t enqueued = 0;  // rows waiting now
};

class ExpertQueue {
 public:
  explicit ExpertQueue(const Config& c);  // InvalidArgument on a bad configuration
  void enqueue(uint32_t layer, uint32_t expert, uint64_t row_id, uint64_t arrival_ns);
  void seal(uint32_t layer);
  void set_firing_threshold(uint32_t rows);
  // The slot due at `now_ns` with the lowest (layer, expert) index; false when none is.
  bool next_firing(uint64_t now_ns, Firing& out);
  uint32_t slot_rows(uint32_t layer, uint32_t expert) const;
  uint32_t layer_rows(uint32_t layer) const { return layers_.at(layer).rows; }
  bool sealed(uint32_t layer) const { return layers_.at(layer).sealed; }
  Stats stats() const { return st_; }
  const Config& config() const { return cfg_; }

 private:
  static constexpr uint64_t kNever = ~0ull;
  struct Row {
    uint64_t id, arrival_ns;
  };
  // A growable ring of rows; capacity is a power of two.
  class Ring {
   public:
    uint32_t size() const { return n_; }
    const Row& front() const { return buf_[head_]; }
    void push(const Row& r);
    Row pop();

   private:
    std::vector<Row> buf_;
    uint32_t head_ = 0, n_ = 0;
  };
  struct Layer {
    uint32_t rows = 0;
    bool sealed = false;
  };
  uint32_t index(uint32_t l, uint32_t e) const { return l * cfg_.expert_count + e; }
  uint64_t due_key(uint32_t slot) const;
  void refresh(uint32_t slot);  // recompute the slot's key and its path to the root
  void refresh_layer(uint32_t layer);
  int leftmost_due(uint64_t now_ns) const;

  Config cfg_;
  std::vector<Ring> rings_;
  std::vector<Layer> layers_;
  uint32_t leaves_ = 1;          // tournament tree: leaves_ leaves, node i has children 2i, 2i+1
  std::vector<uint64_t> tree_;   // tree_[leaves_ + slot] = due key of slot
  uint32_t queued_ = 0;
  Stats st_;
};

}  // namespace eq
}  // namespace spc
