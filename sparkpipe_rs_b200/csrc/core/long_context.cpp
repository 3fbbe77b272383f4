#include "long_context.h"

#include <algorithm>
#include <unordered_set>

namespace spc {
namespace lc {

namespace {
uint32_t ceil_div(uint32_t a, uint32_t b) { return b ? uint32_t((uint64_t(a) + b - 1) / b) : 0; }

void fill_full(const Policy& p, uint32_t ctx, std::vector<uint32_t>& out, uint32_t cap, DecodePlan& d) {
  if (ctx > cap || ctx > p.max_scan) fail(Status::CapacityExceeded, "long context: context exceeds the scan budget");
  for (uint32_t i = 0; i < cap; ++i) out[i] = i < ctx ? i : kInvalidToken;
  d.selected = ctx;
  d.padded = cap - ctx;
  d.selected_blocks = ceil_div(ctx, p.block_tokens);
  d.est_reads = ctx;
  if (ctx < cap) d.flags |= kPlanPadded;
  d.flags |= p.mode == Mode::FullScan ? kPlanFullScan : kPlanBounded;
}

// sink prefix, strided middle, recent tail; de-duplicated in selection order
void fill_bounded(const Policy& p, uint32_t ctx, std::vector<uint32_t>& out, uint32_t cap, DecodePlan& d) {
  std::vector<uint32_t> sel;
  sel.reserve(cap);
  std::unordered_set<uint32_t> seen;
  auto take = [&](uint32_t t) {
    if (sel.size() >= cap || t == kInvalidToken || !seen.insert(t).second) return;
    sel.push_back(t);
  };
  uint32_t sink = 0, recent = 0, strided = 0;
  if (p.flags & kIncludeSink) {
    sink = std::min({p.sink, ctx, cap});
    for (uint32_t t = 0; t < sink; ++t) take(t);
  }
  if ((p.flags & kIncludeRecent) && sel.size() < cap) recent = std::min({p.recent, uint32_t(cap - sel.size()), ctx});
  const uint32_t recent_begin = std::max(ctx > recent ? ctx - recent : 0u, sink);
  const uint32_t mid_begin = sink, mid_end = recent_begin;
  const uint32_t mid = mid_end > mid_begin ? mid_end - mid_begin : 0;
  if ((p.flags & kIncludeStrided) && mid && sel.size() < cap) {
    strided = std::min({p.strided, uint32_t(cap - sel.size()), mid});
    for (uint32_t i = 0; i < strided; ++i) {
      // sample i of `strided` evenly spaced interior points of the middle span
      uint32_t t = mid_begin + uint32_t((uint64_t(i) + 1) * mid / (uint64_t(strided) + 1));
      take(std::min(t, mid_end - 1));
    }
  }
  for (uint32_t t = recent_begin; t < ctx && sel.size() < cap; ++t) take(t);

  std::copy(sel.begin(), sel.end(), out.begin());
  std::fill(out.begin() + sel.size(), out.begin() + cap, kInvalidToken);
  std::unordered_set<uint32_t> blocks;
  for (uint32_t t : sel) blocks.insert(t / p.block_tokens);
  const uint32_t n = uint32_t(sel.size());
  d.flags |= kPlanBounded;
  d.selected = n;
  d.padded = cap - n;
  d.selected_blocks = uint32_t(blocks.size());
  d.first_recent = recent_begin;
  d.sink = sink;
  d.strided = strided;
  d.recent = ctx - recent_begin;
  d.est_reads = n;
  d.avoided_reads = ctx > n ? ctx - n : 0;
  if (n < cap) d.flags |= kPlanPadded;
  if (ctx > n) d.flags |= kPlanTruncated;
}
}  // namespace

Policy::Policy(uint32_t max_context, uint32_t capacity)
    : max_context_tokens(max_context), selected_capacity(capacity), max_scan(capacity), prefill_chunk(capacity) {}

Policy Policy::normalized() const {
  Policy p = *this;
  if (!p.flags) p.flags = kDefaultFlags;
  if (!p.block_tokens) p.block_tokens = kDefaultBlockTokens;
  if (!p.recent) p.recent = kDefaultRecent;
  if (!p.sink) p.sink = kDefaultSink;
  if (!p.strided) p.strided = kDefaultStride;
  if (!p.max_scan) p.max_scan = p.selected_capacity;
  if (!p.prefill_chunk) p.prefill_chunk = p.selected_capacity;
  if (!p.long_threshold) p.long_threshold = kDefaultLongThreshold;
  return p;
}

void Policy::validate() const {
  const Policy p = normalized();
  auto bad = [](const char* w) { fail(Status::InvalidArgument, std::string("long context: ") + w); };
  if (p.flags & ~kKnownFlags) bad("unknown flags");
  if (!p.max_context_tokens || !p.selected_capacity || p.selected_capacity > kMaxSelected) bad("bad capacity");
  if (!p.block_tokens || !p.max_scan || p.max_scan > p.selected_capacity || !p.prefill_chunk) bad("bad budgets");
  if ((p.flags & kRequireBounded) && p.mode == Mode::FullScan && !(p.flags & kAllowFullScan))
    bad("full scan is not allowed under a bounded-decode requirement");
  if (!(p.flags & (kIncludeSink | kIncludeStrided | kIncludeRecent))) bad("selection includes nothing");
}

PrefillPlan Policy::prefill_plan(uint32_t prompt, uint32_t per_step) const {
  if (!prompt) fail(Status::InvalidArgument, "long context: empty prompt");
  validate();
  const Policy p = normalized();
  if (prompt > p.max_context_tokens && (p.flags & kFailOnOverflow))
    fail(Status::CapacityExceeded, "long context: prompt exceeds the context limit");
  if (!per_step) per_step = p.prefill_chunk;
  PrefillPlan r;
  r.prompt_tokens = prompt;
  r.tokens_per_step = per_step;
  r.chunks = ceil_div(prompt, per_step);
  r.final_chunk_tokens = prompt % per_step ? prompt % per_step : per_step;
  r.block_tokens = p.block_tokens;
  r.prompt_blocks = ceil_div(prompt, p.block_tokens);
  r.visits = prompt;
  if (r.chunks > 1) r.flags |= kPrefillChunked;
  if (prompt >= p.long_threshold) r.flags |= kPrefillLongContext;
  return r;
}

DecodePlan Policy::decode_selection(uint32_t ctx, std::vector<uint32_t>& out) const {
  if (!ctx || out.empty()) fail(Status::InvalidArgument, "long context: empty context or selection buffer");
  validate();
  const Policy p = normalized();
  const uint32_t cap = std::min<uint32_t>(uint32_t(out.size()), p.selected_capacity);
  if (ctx > p.max_context_tokens && (p.flags & kFailOnOverflow))
    fail(Status::CapacityExceeded, "long context: context exceeds the context limit");
  DecodePlan d;
  d.context_tokens = ctx;
  d.capacity = cap;
  d.block_tokens = p.block_tokens;
  d.context_blocks = ceil_div(ctx, p.block_tokens);
  d.max_scan = p.max_scan;
  if (ctx >= p.long_threshold) d.flags |= kPlanLongContext;
  if (p.mode == Mode::FullScan) {
    if (!(p.flags & kAllowFullScan)) fail(Status::InvalidArgument, "long context: full scan not allowed");
    fill_full(p, ctx, out, cap, d);
    return d;
  }
  if (ctx <= cap && ctx <= p.max_scan) {
    fill_full(p, ctx, out, cap, d);
    return d;
  }
  fill_bounded(p, ctx, out, cap, d);
  if (d.selected > p.max_scan) fail(Status::CapacityExceeded, "long context: selection exceeds the scan budget");
  return d;
}

std::vector<DecodePlan> Policy::lane_batch(const std::vector<uint32_t>& contexts, std::vector<uint32_t>& out,
                                           size_t stride, size_t capacity) const {
  if (contexts.empty() || !stride || !capacity || stride < capacity ||
      out.size() < (contexts.size() - 1) * stride + capacity)
    fail(Status::InvalidArgument, "long context: bad lane batch buffer");
  std::vector<DecodePlan> plans;
  std::vector<uint32_t> lane(capacity);
  for (size_t i = 0; i < contexts.size(); ++i) {
    plans.push_back(decode_selection(contexts[i], lane));
    std::copy(lane.begin(), lane.end(), out.begin() + i * stride);
  }
  return plans;
}

}  // namespace lc
}  // namespace spc
