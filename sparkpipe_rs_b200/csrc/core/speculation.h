// Speculative-decode policy of the serving scheduler.
//
//   lane state     per request: an EMA of the tokens committed per verify round
//                  (milli fixed point, starts at 2.9 tokens), the draft budget of
//                  its next round, and a reprobe countdown. A lane whose EMA falls
//                  below 1.15 tokens is suppressed (budget 0) and decodes plainly
//                  until it has committed 16 more tokens, then probes again.
//   row allocator  divides a verify wave's row cap between one base row per lane
//                  and draft rows, granted greedily by the marginal expected commit
//                  of the next draft row, alpha^depth with alpha = (ema - 1) / ema
//                  (the chain survival probability that inverts the geometric
//                  expectation), ties to the lower lane index. Milli fixed point
//                  throughout, so the assignment is deterministic.
//   utility        verify instead of plain decode only when the expected tokens of
//                  a round (an average over every resolved round, with a prior of 13
//                  rounds of 2 tokens) per unit of measured round time beat one token
//                  per plain step by a 1.25 margin.
//
// Reference behaviour: the MTP policy of crates/spark-serve/src/request_api/
// speculation.rs:263-335, 501-690 with the constants of request_api/mod.rs:153-176,
// and the row allocator of crates/spark-core/src/row_allocator.rs (cases of
// crates/spark-core/tests/row_allocator.rs). The round-cost term differs on purpose:
// the reference prices its draft chain as two plain decode steps of the full model,
// while here the draft is a separate small model whose cost is inside the measured
// time of a verify round.
#pragma once

#include <cstdint>
#include <vector>

namespace spc {
namespace spec {

constexpr uint32_t kMaxDraftTokens = 8;         // per lane and round
constexpr uint32_t kMaxSpeculativeTokens = 7;   // chain draft length cap
constexpr int32_t kEmaDivisor = 4;
constexpr uint32_t kEmaInitialMilli = 2900;
constexpr uint32_t kSuppressMilli = 1150;
constexpr uint32_t kReprobeInterval = 16;       // committed tokens
constexpr uint64_t kUtilityScale = 1000;
constexpr uint64_t kUtilityMargin = 1250;
constexpr uint64_t kPriorCommitted = 2;         // tokens per prior round (half the tree's maximum)
constexpr uint64_t kPriorRounds = 13;
constexpr uint32_t kMilli = 1000;
constexpr uint32_t kAlphaCeiling = 999;
constexpr uint32_t kProbeRows = 2;

struct LaneState {
  uint32_t ema_milli = kEmaInitialMilli;
  uint32_t budget = 0;      // draft tokens of the next round; 0 = decode plainly
  uint32_t countdown = 0;   // committed tokens until a suppressed lane probes again
  bool disabled = false;    // sampled requests and explicit opt-outs never speculate
};

// After a verify round that committed `committed` tokens (>= 1): EMA update with
// int32 truncation toward zero, then suppression (budget 0, countdown 16) below the
// threshold, else `full_budget`.
void observe_verify(LaneState& s, uint32_t committed, uint32_t full_budget);
// After a plain decode step of a suppressed lane: the countdown runs down by the
// committed tokens; at zero the lane gets `full_budget` again.
void observe_plain(LaneState& s, uint32_t committed, uint32_t full_budget);
// The allocator's cap on a lane's draft depth: 0 while suppressed and counting down.
inline uint32_t max_depth(const LaneState& s, uint32_t full_budget) {
  return (s.budget == 0 && s.countdown != 0) || s.disabled ? 0 : full_budget;
}

struct SlotInput {
  uint32_t commit_ema_milli = 0;
  uint32_t maximum_draft_depth = 0;
  uint32_t probe = 0;  // nonzero: a fixed two-row grant first, no further competition
};
uint32_t alpha_milli(uint32_t commit_ema_milli);
// Fills out[i] with lane i's draft rows; returns base rows + draft rows granted (<= cap).
uint32_t row_allocator_assign(const std::vector<SlotInput>& lanes, uint32_t firing_row_cap,
                              uint32_t spec_row_relative_cost_milli, std::vector<uint32_t>& out);

struct Totals {
  uint64_t rounds = 0;       // verify rounds (one per lane)
  uint64_t proposed = 0;     // draft tokens proposed
  uint64_t accepted = 0;     // draft tokens accepted
  uint64_t committed = 0;    // tokens committed by verify rounds (accepted + one per round)
  uint64_t verify_steps = 0; // verify batches
  uint64_t suppressed = 0;   // lane suppressions
  uint64_t reprobes = 0;     // suppressed lanes re-enabled
};
// Expected committed tokens per round x 1000, with the prior.
uint64_t expected_committed_scaled(const Totals& t);
// E x n_spec x plain_ns > margin x n_plain x round_ns (wrapping u64 products).
bool outranks_plain(uint64_t expected_scaled, uint32_t n_plain, uint32_t n_spec, uint64_t plain_ns,
                    uint64_t round_ns);

// Measured device time of a step by kind (plain decode / verify round) and padded
// batch; an estimate for an unmeasured batch interpolates linearly between measured
// neighbours (a flat extrapolation past the ends), and with none measured falls back
// to a fixed 1 ms + 20 us per row.
class StepCost {
 public:
  void set(uint32_t kind, uint32_t seqs, uint64_t ns);
  uint64_t estimate(uint32_t kind, uint32_t seqs, uint32_t rows_per_seq) const;
  bool measured(uint32_t kind) const;

 private:
  std::vector<std::pair<uint32_t, uint64_t>> pts_[4];  // sorted by seqs
};

}  // namespace spec
}  // namespace spc
