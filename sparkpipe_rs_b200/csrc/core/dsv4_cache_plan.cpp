#include "dsv4_cache_plan.h"

#include <limits>

namespace spc {
namespace dsv4 {

namespace {
constexpr uint64_t kMax = std::numeric_limits<uint64_t>::max();

uint64_t add(uint64_t a, uint64_t b) {
  if (a > kMax - b) fail(Status::CapacityExceeded, "dsv4 cache plan: size overflow");
  return a + b;
}
uint64_t mul(uint64_t a, uint64_t b) {
  if (a && b > kMax / a) fail(Status::CapacityExceeded, "dsv4 cache plan: size overflow");
  return a * b;
}
bool pow2(uint64_t v) { return v && !(v & (v - 1)); }
uint64_t align_up(uint64_t v, uint64_t a) { return add(v, a - 1) & ~(a - 1); }
uint64_t packed_bytes(uint64_t elements, uint32_t bits) { return add(mul(elements, bits), 7) / 8; }

// Places a region of `bytes` at the next aligned cursor position; empty regions sit at 0.
struct Cursor {
  uint64_t at = 0;
  uint32_t alignment;
  uint64_t place(uint64_t bytes) {
    if (!bytes) return 0;
    const uint64_t off = align_up(at, alignment);
    at = add(off, bytes);
    return off;
  }
  uint64_t end() const { return align_up(at, alignment); }
};

AttnClass class_of(uint32_t ratio) {
  switch (ratio) {
    case 0: return AttnClass::Sliding;
    case 4: return AttnClass::CompressedSparse;
    case 128: return AttnClass::HeavilyCompressed;
  }
  fail(Status::InvalidArgument, "dsv4 cache plan: unknown compression ratio");
}

LayerPlan layer_plan(const PlanConfig& c, const Geometry& g, uint32_t absolute, bool mtp, uint32_t ratio) {
  LayerPlan L;
  L.absolute_layer = absolute;
  L.mtp_layer = mtp;
  L.ratio = ratio;
  L.attn_class = class_of(ratio);
  const uint64_t content_dim = g.head_dim - g.rope_dim;
  const bool csa = L.attn_class == AttnClass::CompressedSparse;
  // sliding window: one sequence's content then RoPE parts
  L.sliding_entries_per_sequence = g.sliding_window - 1;
  Cursor s{0, c.alignment};
  L.sliding_content_offset = s.place(packed_bytes(mul(L.sliding_entries_per_sequence, content_dim), c.content_bits));
  L.sliding_rope_offset = s.place(packed_bytes(mul(L.sliding_entries_per_sequence, g.rope_dim), c.rope_bits));
  L.sliding_sequence_stride = s.end();
  if (!ratio) return L;
  // compressed history, shared by all sequences: ceil(capacity / r) entries in whole pages
  uint64_t entries = c.aggregate_context_token_capacity / ratio + (c.aggregate_context_token_capacity % ratio ? 1 : 0);
  entries = mul((entries + c.page_entries - 1) / c.page_entries, c.page_entries);
  if (entries > std::numeric_limits<uint32_t>::max()) fail(Status::CapacityExceeded, "dsv4 cache plan: history entries");
  L.compressed_entries = uint32_t(entries);
  Cursor h{0, c.alignment};
  L.compressed_content_offset = h.place(packed_bytes(mul(entries, content_dim), c.content_bits));
  L.compressed_rope_offset = h.place(packed_bytes(mul(entries, g.rope_dim), c.rope_bits));
  if (csa) L.indexer_history_offset = h.place(packed_bytes(mul(entries, g.index_head_dim), c.indexer_bits));
  L.history_arena_bytes = h.end();
  // compressor state of one sequence
  Cursor st{0, c.alignment};
  auto state = [&](uint64_t tokens, uint64_t width) { return st.place(packed_bytes(mul(tokens, width), c.state_bits)); };
  L.compressor_buffer_tokens = ratio - 1;
  const uint64_t cw = csa ? 2ull * g.head_dim : g.head_dim;
  L.compressor_kv_offset = state(L.compressor_buffer_tokens, cw);
  L.compressor_gate_offset = state(L.compressor_buffer_tokens, cw);
  if (csa) {
    L.indexer_buffer_tokens = ratio - 1;
    const uint64_t iw = 2ull * g.index_head_dim;
    L.indexer_kv_offset = state(L.indexer_buffer_tokens, iw);
    L.indexer_gate_offset = state(L.indexer_buffer_tokens, iw);
    L.compressor_overlap_kv_offset = state(ratio, g.head_dim);
    L.compressor_overlap_gate_offset = state(ratio, g.head_dim);
    L.indexer_overlap_kv_offset = state(ratio, g.index_head_dim);
    L.indexer_overlap_gate_offset = state(ratio, g.index_head_dim);
  }
  L.state_sequence_stride = st.end();
  return L;
}
}  // namespace

Geometry geometry(Variant v) {
  switch (v) {
    case Variant::Flash: return Geometry{43, 1, 512, 64, 128, 128, 1u << 20};
    case Variant::Pro: return Geometry{61, 1, 512, 64, 128, 128, 1u << 20};
  }
  fail(Status::InvalidArgument, "dsv4 cache plan: unknown model variant");
}

uint32_t compression_ratio(Variant v, uint32_t layer, bool mtp) {
  const Geometry g = geometry(v);
  if (mtp) return 0;
  if (layer >= g.backbone_layers) fail(Status::InvalidArgument, "dsv4 cache plan: layer out of range");
  if (layer < 2) return v == Variant::Flash ? 0 : 128;
  return layer % 2 == 0 ? 4 : 128;
}

Plan build_plan(const PlanConfig& c) {
  auto bits_ok = [](uint32_t b) { return b == 4 || b == 8 || b == 16 || b == 32; };
  if (!c.backbone_layer_count || !c.active_sequence_capacity || !c.max_context_tokens_per_sequence ||
      !c.aggregate_context_token_capacity || c.aggregate_context_token_capacity < c.active_sequence_capacity ||
      !pow2(c.page_entries) || !pow2(c.alignment) || !bits_ok(c.content_bits) || !bits_ok(c.rope_bits) ||
      !bits_ok(c.indexer_bits) || !bits_ok(c.state_bits))
    fail(Status::InvalidArgument, "dsv4 cache plan: invalid configuration");
  const Geometry g = geometry(c.variant);
  if (c.max_context_tokens_per_sequence > g.max_context_tokens)
    fail(Status::InvalidArgument, "dsv4 cache plan: context above the model's maximum");
  if (uint64_t(c.first_backbone_layer) + c.backbone_layer_count > g.backbone_layers)
    fail(Status::InvalidArgument, "dsv4 cache plan: layer range outside the backbone");
  if (c.include_mtp_layer && g.mtp_layers != 1) fail(Status::InvalidArgument, "dsv4 cache plan: no MTP layer");
  const uint32_t n = c.backbone_layer_count + (c.include_mtp_layer ? 1 : 0);
  if (n > kMaxLayers) fail(Status::InvalidArgument, "dsv4 cache plan: too many layers");

  Plan p;
  p.config = c;
  Cursor sl{0, c.alignment}, hi{0, c.alignment}, st{0, c.alignment};
  for (uint32_t i = 0; i < n; ++i) {
    const bool mtp = i >= c.backbone_layer_count;
    const uint32_t absolute = mtp ? g.backbone_layers : c.first_backbone_layer + i;
    LayerPlan L = layer_plan(c, g, absolute, mtp, compression_ratio(c.variant, absolute, mtp));
    switch (L.attn_class) {
      case AttnClass::Sliding: ++p.sliding_layers; break;
      case AttnClass::CompressedSparse: ++p.compressed_sparse_layers; break;
      case AttnClass::HeavilyCompressed: ++p.heavily_compressed_layers; break;
    }
    // arena offsets are aligned even for empty regions, so a layer's view is always well formed
    L.sliding_arena_bytes = mul(L.sliding_sequence_stride, c.active_sequence_capacity);
    L.sliding_arena_offset = align_up(sl.at, c.alignment);
    sl.at = add(L.sliding_arena_offset, L.sliding_arena_bytes);
    L.history_arena_offset = align_up(hi.at, c.alignment);
    hi.at = add(L.history_arena_offset, L.history_arena_bytes);
    L.state_arena_bytes = mul(L.state_sequence_stride, c.active_sequence_capacity);
    L.state_arena_offset = align_up(st.at, c.alignment);
    st.at = add(L.state_arena_offset, L.state_arena_bytes);
    p.layers.push_back(L);
  }
  p.sliding_arena_bytes = sl.end();
  p.history_arena_bytes = hi.end();
  p.state_arena_bytes = st.end();
  p.total_arena_bytes = add(add(p.sliding_arena_bytes, p.history_arena_bytes), p.state_arena_bytes);
  // worst class per region: ratio 4 has the largest history (and the same sliding
  // window as any class), ratio 128 the largest compressor state
  const LayerPlan csa = layer_plan(c, g, 0, false, 4), hca = layer_plan(c, g, 0, false, 128);
  p.worst_sliding_bytes = mul(mul(csa.sliding_sequence_stride, c.active_sequence_capacity), n);
  p.worst_history_bytes = mul(csa.history_arena_bytes, n);
  p.worst_state_bytes = mul(mul(hca.state_sequence_stride, c.active_sequence_capacity), n);
  p.worst_total_bytes = add(add(p.worst_sliding_bytes, p.worst_history_bytes), p.worst_state_bytes);
  return p;
}

}  // namespace dsv4
}  // namespace spc
