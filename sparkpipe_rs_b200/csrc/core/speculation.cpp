#include "speculation.h"

#include <algorithm>

#include "common.h"

namespace spc {
namespace spec {

void observe_verify(LaneState& s, uint32_t committed, uint32_t full_budget) {
  const int32_t delta = int32_t(committed * 1000u) - int32_t(s.ema_milli);
  s.ema_milli = uint32_t(int32_t(s.ema_milli) + delta / kEmaDivisor);
  if (s.ema_milli < kSuppressMilli) {
    s.budget = 0;
    s.countdown = kReprobeInterval;
  } else {
    s.budget = full_budget;
    s.countdown = 0;
  }
}

void observe_plain(LaneState& s, uint32_t committed, uint32_t full_budget) {
  if (s.budget != 0 || s.countdown == 0) return;
  if (s.countdown > committed) {
    s.countdown -= committed;
  } else {
    s.countdown = 0;
    s.budget = full_budget;
  }
}

uint32_t alpha_milli(uint32_t ema) {
  if (ema <= kMilli) return 0;
  const uint32_t a = uint32_t(uint64_t(ema - kMilli) * kMilli / ema);
  return std::min(a, kAlphaCeiling);
}

uint32_t row_allocator_assign(const std::vector<SlotInput>& lanes, uint32_t cap, uint32_t cost_milli,
                              std::vector<uint32_t>& out) {
  if (cap == 0) return 0;
  const uint32_t n = (uint32_t)lanes.size();
  out.assign(n, 0);
  const uint32_t base = std::min(n, cap);
  uint32_t left = cap - base;
  // probes: a fixed grant in lane order, before any value-ranked grant
  for (uint32_t i = 0; i < n && left; ++i) {
    if (!lanes[i].probe || !lanes[i].maximum_draft_depth) continue;
    out[i] = std::min({kProbeRows, lanes[i].maximum_draft_depth, left});
    left -= out[i];
  }
  // greedy: the next draft row of the lane whose marginal value alpha^(d+1) x 1000 / cost is highest
  const uint32_t cost = cost_milli ? cost_milli : kMilli;
  std::vector<uint32_t> alpha(n);
  for (uint32_t i = 0; i < n; ++i) alpha[i] = alpha_milli(lanes[i].commit_ema_milli);
  while (left) {
    uint32_t best = n, best_v = 0;
    for (uint32_t i = 0; i < n; ++i) {
      if (lanes[i].probe || out[i] >= lanes[i].maximum_draft_depth || alpha[i] == 0) continue;
      uint32_t v = uint32_t(uint64_t(alpha[i]) * kMilli / cost);
      for (uint32_t d = 0; d < out[i]; ++d) v = uint32_t(uint64_t(v) * alpha[i] / kMilli);
      if (v > best_v) { best_v = v; best = i; }
    }
    if (best == n || best_v == 0) break;
    ++out[best];
    --left;
  }
  uint32_t total = base;
  for (uint32_t v : out) total += v;
  return total;
}

uint64_t expected_committed_scaled(const Totals& t) {
  return (t.committed + kPriorRounds * kPriorCommitted) * kUtilityScale / (t.rounds + kPriorRounds);
}

bool outranks_plain(uint64_t e, uint32_t n_plain, uint32_t n_spec, uint64_t plain_ns, uint64_t round_ns) {
  if (!n_plain || !n_spec) return false;
  return e * uint64_t(n_spec) * plain_ns > kUtilityMargin * uint64_t(n_plain) * round_ns;
}

void StepCost::set(uint32_t kind, uint32_t seqs, uint64_t ns) {
  if (kind >= 4 || seqs == 0) fail(Status::InvalidArgument, "StepCost: kind 0..3 and a nonzero batch");
  auto& v = pts_[kind];
  auto it = std::lower_bound(v.begin(), v.end(), std::make_pair(seqs, uint64_t(0)),
                             [](const auto& a, const auto& b) { return a.first < b.first; });
  if (it != v.end() && it->first == seqs) it->second = ns;
  else v.insert(it, {seqs, ns});
}

bool StepCost::measured(uint32_t kind) const { return kind < 4 && !pts_[kind].empty(); }

uint64_t StepCost::estimate(uint32_t kind, uint32_t seqs, uint32_t rows_per_seq) const {
  if (kind >= 4 || pts_[kind].empty()) return 1000000ull + 20000ull * uint64_t(seqs) * rows_per_seq;
  const auto& v = pts_[kind];
  if (seqs <= v.front().first) return v.front().second;
  if (seqs >= v.back().first) return v.back().second;
  auto hi = std::lower_bound(v.begin(), v.end(), std::make_pair(seqs, uint64_t(0)),
                             [](const auto& a, const auto& b) { return a.first < b.first; });
  if (hi->first == seqs) return hi->second;
  auto lo = hi - 1;
  const double f = double(seqs - lo->first) / double(hi->first - lo->first);
  return uint64_t(double(lo->second) + f * (double(hi->second) - double(lo->second)));
}

}  // namespace spec
}  // namespace spc
