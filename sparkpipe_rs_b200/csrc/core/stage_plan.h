// Pipeline stage planner: splits a model's layers into pipeline stages.
//
// Cut rules: the dense prefix (layers before the first routed/MoE layer) stays
// whole inside stage 0, and no stage holds more than
// `max_routed_layers_per_stage` routed layers. Builders: an explicit
// layer-count table, uniform costs, or the exact min-max partition over a
// per-layer cost profile (dynamic program over (stage, layer) with the final,
// token-emitting stage charged an extra cost for the LM head + sampling).
//
// `StagePlanner` keeps cost profiles per decode batch bucket (measured on the
// device by timing each layer, or scaled from the nearest measured bucket) and
// caches the plan per (bucket, stage count), so admission never re-runs the DP.
//
// Reference behaviour: crates/spark-sched/src/stage_plan.rs (constants :27-90,
// validation :300-365, table builder :368-398, DP :404-484, profile scaling
// :583-597, chunk shape :783-806). The descriptor layout (4 u32 header words +
// 13 stages x 16 bytes) and flag values are kept so serialized plans stay
// compatible.
#pragma once

#include <cstdint>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "common.h"

namespace spc {
namespace sp {

constexpr uint32_t kAbiVersion = 1;
constexpr uint32_t kMaxStages = 13;
constexpr uint32_t kDescriptorBytes = 16 + kMaxStages * 16;
constexpr uint32_t kMaxLayers = 128;
constexpr uint32_t kDefaultMaxRoutedPerStage = 8;

constexpr uint32_t kFlagFinalToken = 0x1;
constexpr uint32_t kFlagInputHidden = 0x2;
constexpr uint32_t kFlagOutputHidden = 0x4;
constexpr uint32_t kFlagDensePrefix = 0x8;
constexpr uint32_t kKnownFlags = 0xF;

struct Geometry {
  uint32_t layer_count = 0;
  uint32_t first_routed_layer = 0;
  uint32_t max_routed_layers_per_stage = kDefaultMaxRoutedPerStage;
};

struct Stage {
  uint32_t first_layer = 0, layer_count = 0, flags = 0;
};

struct StagePlan {
  std::vector<Stage> stages;
  uint32_t total_layers() const {
    uint32_t n = 0;
    for (const Stage& s : stages) n += s.layer_count;
    return n;
  }
  std::string serialize() const;                     // C descriptor layout, little-endian
  static StagePlan deserialize(const std::string&);  // AbiMismatch on a bad header
};

uint32_t routed_layers_in(const Geometry& g, uint32_t first, uint32_t count);
bool range_is_valid(const Geometry& g, uint32_t first, uint32_t count);
void validate(const Geometry& g, const StagePlan& p);  // throws StatusError
StagePlan build_from_layer_counts(const Geometry& g, const std::vector<uint32_t>& counts);
StagePlan build_balanced(const Geometry& g, const std::vector<uint64_t>& layer_cost_ns, uint64_t final_extra_ns,
                         uint32_t stage_count);
StagePlan build_uniform(const Geometry& g, uint32_t stage_count);
uint64_t max_stage_cost(const StagePlan& p, const std::vector<uint64_t>& layer_cost_ns, uint64_t final_extra_ns);

struct CostProfile {
  std::vector<uint64_t> layer_cost_ns;
  uint64_t final_extra_ns = 0;
  bool measured = false;
};

class StagePlanner {
 public:
  explicit StagePlanner(const Geometry& g);
  const Geometry& geometry() const { return g_; }
  // Records a measured profile for a batch bucket; drops cached plans.
  void record_profile(uint32_t bucket, const std::vector<uint64_t>& layer_cost_ns, uint64_t final_extra_ns);
  // Measured profile of `bucket`, else the nearest measured bucket scaled
  // linearly by bucket size (ceil), else uniform (1 ns per layer).
  CostProfile profile(uint32_t bucket) const;
  const StagePlan& plan(uint32_t bucket, uint32_t stage_count);
  uint64_t plan_builds() const { return builds_; }
  uint64_t plan_hits() const { return hits_; }

 private:
  Geometry g_;
  std::map<uint32_t, CostProfile> measured_;
  std::map<std::pair<uint32_t, uint32_t>, StagePlan> cache_;
  mutable std::mutex mu_;
  uint64_t builds_ = 0, hits_ = 0;
};

}  // namespace sp
}  // namespace spc
