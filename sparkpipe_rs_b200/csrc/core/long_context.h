// Long-context policy: which KV tokens a bounded decode step reads, and how a
// long prompt is cut into prefill chunks.
//
// Bounded selection = a sink prefix + an evenly strided sample of the middle +
// the recent tail, de-duplicated, padded with kInvalidToken to the capacity.
// Contexts that fit the capacity and scan budget are read whole. Prefill plans
// split a prompt into `max_prefill_tokens_per_step` chunks.
//
// Reference behaviour: crates/spark-sched/src/long_context.rs (defaults and
// flags :40-106, normalisation/validation :231-300, prefill plan :303-345,
// decode selection :347-470, bounded selection :520-599). Flag values,
// defaults and the selection rule are kept so plans agree token for token.
#pragma once

#include <cstdint>
#include <vector>

#include "common.h"

namespace spc {
namespace lc {

constexpr uint32_t kInvalidToken = 0xffffffffu;
constexpr uint32_t kMaxSelected = 4096;
constexpr uint32_t kDefaultBlockTokens = 16;
constexpr uint32_t kDefaultRecent = 1536;
constexpr uint32_t kDefaultSink = 128;
constexpr uint32_t kDefaultStride = 384;
constexpr uint32_t kDefaultLongThreshold = 8192;

constexpr uint32_t kRequireBounded = 0x01;
constexpr uint32_t kIncludeSink = 0x02;
constexpr uint32_t kIncludeStrided = 0x04;
constexpr uint32_t kIncludeRecent = 0x08;
constexpr uint32_t kFailOnOverflow = 0x10;
constexpr uint32_t kAllowFullScan = 0x20;
constexpr uint32_t kDefaultFlags = kRequireBounded | kIncludeSink | kIncludeStrided | kIncludeRecent | kFailOnOverflow;
constexpr uint32_t kKnownFlags = kDefaultFlags | kAllowFullScan;

constexpr uint32_t kPlanBounded = 0x01;
constexpr uint32_t kPlanFullScan = 0x02;
constexpr uint32_t kPlanLongContext = 0x04;
constexpr uint32_t kPlanTruncated = 0x08;
constexpr uint32_t kPlanPadded = 0x10;
constexpr uint32_t kPrefillChunked = 0x01;
constexpr uint32_t kPrefillLongContext = 0x02;

enum class Mode : uint32_t { BoundedWindow = 0, FullScan = 1 };

struct DecodePlan {
  uint32_t flags = 0, context_tokens = 0, selected = 0, capacity = 0, padded = 0, selected_blocks = 0;
  uint32_t block_tokens = 0, context_blocks = 0, first_recent = 0, max_scan = 0;
  uint32_t sink = 0, strided = 0, recent = 0;
  uint64_t est_reads = 0, avoided_reads = 0;
};

struct PrefillPlan {
  uint32_t flags = 0, prompt_tokens = 0, tokens_per_step = 0, chunks = 0, final_chunk_tokens = 0;
  uint32_t block_tokens = 0, prompt_blocks = 0;
  uint64_t visits = 0;
};

// Zero fields take their defaults (max_context / selected_capacity from the
// constructor, the rest from the constants above).
struct Policy {
  Mode mode = Mode::BoundedWindow;
  uint32_t flags = kDefaultFlags;
  uint32_t max_context_tokens = 0, selected_capacity = 0, block_tokens = kDefaultBlockTokens;
  uint32_t recent = kDefaultRecent, sink = kDefaultSink, strided = kDefaultStride;
  uint32_t max_scan = 0, prefill_chunk = 0, long_threshold = kDefaultLongThreshold;

  Policy() = default;
  Policy(uint32_t max_context, uint32_t capacity);
  Policy normalized() const;
  void validate() const;  // InvalidArgument
  PrefillPlan prefill_plan(uint32_t prompt_tokens, uint32_t tokens_per_step) const;
  // Fills `out` (its size is the requested capacity, clamped to the policy's).
  DecodePlan decode_selection(uint32_t context_tokens, std::vector<uint32_t>& out) const;
  // One selection per lane into rows of `stride` entries, `capacity` used per row.
  std::vector<DecodePlan> lane_batch(const std::vector<uint32_t>& contexts, std::vector<uint32_t>& out,
                                     size_t stride, size_t capacity) const;
};

}  // namespace lc
}  // namespace spc
