#include "stage_plan.h"

#include <algorithm>
#include <limits>

namespace spc {
namespace sp {

namespace {
constexpr uint64_t kInf = std::numeric_limits<uint64_t>::max();

void assign_flags(const Geometry& g, StagePlan& p) {
  const size_t n = p.stages.size();
  for (size_t i = 0; i < n; ++i) {
    Stage& s = p.stages[i];
    s.flags = kFlagInputHidden | (i + 1 < n ? kFlagOutputHidden : kFlagFinalToken);
    if (s.first_layer == 0 && s.layer_count >= g.first_routed_layer) s.flags |= kFlagDensePrefix;
  }
}
}  // namespace

uint32_t routed_layers_in(const Geometry& g, uint32_t first, uint32_t count) {
  const uint32_t lo = std::max(first, g.first_routed_layer);
  const uint32_t hi = std::min(first + count, g.layer_count);
  return hi > lo ? hi - lo : 0;
}

bool range_is_valid(const Geometry& g, uint32_t first, uint32_t count) {
  if (count == 0 || first >= g.layer_count || count > g.layer_count - first) return false;
  if (g.first_routed_layer < g.layer_count) {
    // the dense prefix cannot be split: a stage may start inside it only at
    // layer 0, and that stage must reach past it
    if (first != 0 && first < g.first_routed_layer) return false;
    if (first + count < g.first_routed_layer) return false;
  }
  return routed_layers_in(g, first, count) <= g.max_routed_layers_per_stage;
}

void validate(const Geometry& g, const StagePlan& p) {
  if (p.stages.empty() || p.stages.size() > kMaxStages)
    fail(Status::InvalidArgument, "stage plan: stage count outside 1..13");
  uint32_t next = 0, finals = 0;
  for (size_t i = 0; i < p.stages.size(); ++i) {
    const Stage& s = p.stages[i];
    if (s.flags & ~kKnownFlags) fail(Status::InvalidArgument, "stage plan: unknown stage flags");
    if (s.first_layer != next) fail(Status::InvalidArgument, "stage plan: stages are not contiguous");
    if (!range_is_valid(g, s.first_layer, s.layer_count))
      fail(Status::InvalidArgument, "stage plan: stage breaks the cut rules");
    if (s.flags & kFlagFinalToken) {
      ++finals;
      if (i + 1 != p.stages.size()) fail(Status::InvalidArgument, "stage plan: final-token stage is not last");
    } else if (!(s.flags & kFlagOutputHidden)) {
      fail(Status::InvalidArgument, "stage plan: a non-final stage must emit hidden state");
    }
    next = s.first_layer + s.layer_count;
  }
  if (next != g.layer_count) fail(Status::InvalidArgument, "stage plan: layers not fully covered");
  if (finals != 1) fail(Status::InvalidArgument, "stage plan: exactly one final-token stage required");
}

StagePlan build_from_layer_counts(const Geometry& g, const std::vector<uint32_t>& counts) {
  if (counts.empty() || counts.size() > kMaxStages) fail(Status::InvalidArgument, "stage plan: bad table size");
  StagePlan p;
  uint32_t first = 0;
  for (uint32_t c : counts) {
    if (c == 0 || c > g.layer_count - std::min(first, g.layer_count))
      fail(Status::InvalidArgument, "stage plan: bad table layer count");
    p.stages.push_back(Stage{first, c, 0});
    first += c;
  }
  assign_flags(g, p);
  validate(g, p);
  return p;
}

StagePlan build_balanced(const Geometry& g, const std::vector<uint64_t>& cost, uint64_t final_extra,
                         uint32_t stage_count) {
  const uint32_t L = g.layer_count;
  if (L == 0 || L > kMaxLayers || cost.size() < L || stage_count == 0 || stage_count > kMaxStages)
    fail(Status::InvalidArgument, "stage plan: bad balanced-plan input");
  std::vector<uint64_t> prefix(L + 1, 0);
  for (uint32_t i = 0; i < L; ++i) {
    if (cost[i] == 0) fail(Status::InvalidArgument, "stage plan: zero layer cost");
    if (prefix[i] > kInf / 4 - cost[i]) fail(Status::CapacityExceeded, "stage plan: cost overflow");
    prefix[i + 1] = prefix[i] + cost[i];
  }
  // best[e]: minimal bottleneck covering layers [0, e) with `s` stages;
  // from[s][e]: where the last of those stages starts
  std::vector<uint64_t> best(L + 1, kInf), next(L + 1);
  std::vector<std::vector<uint32_t>> from(stage_count + 1, std::vector<uint32_t>(L + 1, UINT32_MAX));
  best[0] = 0;
  for (uint32_t s = 1; s <= stage_count; ++s) {
    std::fill(next.begin(), next.end(), kInf);
    const bool last = s == stage_count;
    for (uint32_t e = 1; e <= L; ++e) {
      if (last && e != L) continue;  // the final stage must end at the last layer
      for (uint32_t b = 0; b < e; ++b) {
        if (best[b] == kInf || !range_is_valid(g, b, e - b)) continue;
        const uint64_t seg = prefix[e] - prefix[b] + (last ? final_extra : 0);
        const uint64_t cand = std::max(best[b], seg);
        if (cand < next[e]) {
          next[e] = cand;
          from[s][e] = b;
        }
      }
    }
    best.swap(next);
  }
  if (best[L] == kInf) fail(Status::CapacityExceeded, "stage plan: stage count cannot satisfy the cut rules");
  StagePlan p;
  p.stages.resize(stage_count);
  uint32_t e = L;
  for (uint32_t s = stage_count; s >= 1; --s) {
    const uint32_t b = from[s][e];
    if (b == UINT32_MAX) fail(Status::InternalError, "stage plan: backtrack failed");
    p.stages[s - 1] = Stage{b, e - b, 0};
    e = b;
  }
  assign_flags(g, p);
  validate(g, p);
  return p;
}

StagePlan build_uniform(const Geometry& g, uint32_t stage_count) {
  return build_balanced(g, std::vector<uint64_t>(g.layer_count, 1), 0, stage_count);
}

uint64_t max_stage_cost(const StagePlan& p, const std::vector<uint64_t>& cost, uint64_t final_extra) {
  uint64_t worst = 0;
  for (const Stage& s : p.stages) {
    uint64_t c = (s.flags & kFlagFinalToken) ? final_extra : 0;
    for (uint32_t i = 0; i < s.layer_count; ++i) c += cost.at(s.first_layer + i);
    worst = std::max(worst, c);
  }
  return worst;
}

std::string StagePlan::serialize() const {
  std::string b(kDescriptorBytes, '\0');
  uint8_t* p = reinterpret_cast<uint8_t*>(&b[0]);
  put_u32(p, kAbiVersion);
  put_u32(p + 4, kDescriptorBytes);
  put_u32(p + 8, uint32_t(stages.size()));
  for (size_t i = 0; i < stages.size() && i < kMaxStages; ++i) {
    uint8_t* q = p + 16 + 16 * i;
    put_u32(q, stages[i].first_layer);
    put_u32(q + 4, stages[i].layer_count);
    put_u32(q + 8, stages[i].flags);
  }
  return b;
}

StagePlan StagePlan::deserialize(const std::string& b) {
  const uint8_t* p = reinterpret_cast<const uint8_t*>(b.data());
  if (b.size() != kDescriptorBytes || get_u32(p) != kAbiVersion || get_u32(p + 4) != kDescriptorBytes)
    fail(Status::AbiMismatch, "stage plan: descriptor ABI mismatch");
  const uint32_t n = get_u32(p + 8);
  if (n == 0 || n > kMaxStages) fail(Status::InvalidArgument, "stage plan: bad stage count");
  StagePlan s;
  for (uint32_t i = 0; i < n; ++i) {
    const uint8_t* q = p + 16 + 16 * i;
    s.stages.push_back(Stage{get_u32(q), get_u32(q + 4), get_u32(q + 8)});
  }
  return s;
}

// ------------------------------------------------------------------ planner
StagePlanner::StagePlanner(const Geometry& g) : g_(g) {
  if (g.layer_count == 0 || g.layer_count > kMaxLayers || g.first_routed_layer > g.layer_count)
    fail(Status::InvalidArgument, "stage planner: bad geometry");
}

void StagePlanner::record_profile(uint32_t bucket, const std::vector<uint64_t>& cost, uint64_t final_extra) {
  if (!bucket || cost.size() != g_.layer_count) fail(Status::InvalidArgument, "stage planner: bad profile");
  for (uint64_t c : cost)
    if (!c) fail(Status::InvalidArgument, "stage planner: zero layer cost");
  std::lock_guard<std::mutex> l(mu_);
  measured_[bucket] = CostProfile{cost, final_extra, true};
  cache_.clear();
}

CostProfile StagePlanner::profile(uint32_t bucket) const {
  std::lock_guard<std::mutex> l(mu_);
  auto it = measured_.find(bucket);
  if (it != measured_.end()) return it->second;
  if (measured_.empty()) return CostProfile{std::vector<uint64_t>(g_.layer_count, 1), 0, false};
  // nearest measured bucket (ties toward the larger one), scaled by bucket ratio
  const CostProfile* src = nullptr;
  uint32_t src_bucket = 0;
  uint64_t best_dist = kInf;
  for (const auto& kv : measured_) {
    const uint64_t d = kv.first > bucket ? kv.first - bucket : bucket - kv.first;
    if (d < best_dist || (d == best_dist && kv.first > src_bucket)) {
      best_dist = d;
      src = &kv.second;
      src_bucket = kv.first;
    }
  }
  CostProfile out;
  for (uint64_t c : src->layer_cost_ns) out.layer_cost_ns.push_back(std::max<uint64_t>(1, (c * bucket + src_bucket - 1) / src_bucket));
  out.final_extra_ns = (src->final_extra_ns * bucket + src_bucket - 1) / src_bucket;
  return out;
}

const StagePlan& StagePlanner::plan(uint32_t bucket, uint32_t stage_count) {
  {
    std::lock_guard<std::mutex> l(mu_);
    auto it = cache_.find({bucket, stage_count});
    if (it != cache_.end()) {
      ++hits_;
      return it->second;
    }
  }
  const CostProfile prof = profile(bucket);
  StagePlan p = build_balanced(g_, prof.layer_cost_ns, prof.final_extra_ns, stage_count);
  std::lock_guard<std::mutex> l(mu_);
  ++builds_;
  return cache_.emplace(std::make_pair(bucket, stage_count), std::move(p)).first->second;
}

}  // namespace sp
}  // namespace spc
