// KV cache plan of the DeepSeek-V4 family (Flash and Pro): how much device memory
// each layer's attention state takes and where it sits in three arenas.
//
// Every layer keeps a sliding window of raw KV (window - 1 entries per sequence,
// content and RoPE parts stored apart). A layer with compression ratio r > 0 also
// keeps a compressed history shared by all sequences: one entry per r tokens of the
// aggregate context capacity, rounded up to whole pages; ratio-4 layers
// ("compressed sparse") add a 128-wide indexer key per entry, ratio-128 layers
// ("heavily compressed") do not. Such a layer also keeps per-sequence compressor
// state: the r - 1 tokens not yet folded into an entry (KV and gate projections;
// twice as wide for ratio 4, which also buffers indexer projections and the r-token
// overlap window of both). Ratio 0 layers are sliding only.
//
//   arenas      sliding (per sequence x layer), compressed history (per layer),
//               compressor state (per sequence x layer); every region and every
//               arena offset aligned to the allocation alignment (256 B default:
//               a TMA box never straddles it)
//   element bits 4, 8, 16 or 32 per tensor family (content, RoPE, indexer,
//               compressor state); sizes are packed bits rounded up to bytes
//   worst class the footprint had every planned layer been of the largest class,
//               for sizing a pool before the layer range is known
//
// Layer classes follow the model's published compress ratios: Flash has 43 layers
// (0 and 1 sliding, then ratio 4 / 128 alternating from layer 2, MTP layer sliding);
// Pro has 61 (0 and 1 ratio 128, then ratio 4 / 128 alternating, MTP layer sliding).
//
// Reference behaviour: crates/spark-abi/vendor/sparkpipe/model-families/dsv4/include/sparkpipe/
// spark_dsv4_cache_plan.h:12-126 (configuration, layer plan and plan records),
// spark_dsv4_flash_model.h / spark_dsv4_pro_model.h (geometry and ratios), src/
// spark_dsv4_cache_plan.c (region order within a layer, page rounding, worst class).
// The region order and rounding are kept so plans agree byte for byte; the code is
// this runtime's own.
#pragma once

#include <cstdint>
#include <vector>

#include "common.h"

namespace spc {
namespace dsv4 {

constexpr uint32_t kMaxLayers = 63;
constexpr uint32_t kDefaultAlignment = 256;
constexpr uint32_t kDefaultPageEntries = 512;

enum class Variant : uint32_t { Flash = 1, Pro = 2 };
enum class AttnClass : uint32_t { Sliding = 1, CompressedSparse = 2, HeavilyCompressed = 3 };

struct Geometry {
  uint32_t backbone_layers, mtp_layers, head_dim, rope_dim, index_head_dim, sliding_window;
  uint32_t max_context_tokens;
};
Geometry geometry(Variant v);
// 0 (sliding only), 4 or 128
uint32_t compression_ratio(Variant v, uint32_t absolute_layer, bool mtp_layer);

struct PlanConfig {
  Variant variant = Variant::Flash;
  uint32_t first_backbone_layer = 0, backbone_layer_count = 0;
  bool include_mtp_layer = false;
  uint32_t active_sequence_capacity = 0, max_context_tokens_per_sequence = 0;
  uint64_t aggregate_context_token_capacity = 0;
  uint32_t page_entries = kDefaultPageEntries;
  uint32_t content_bits = 8, rope_bits = 16, indexer_bits = 8, state_bits = 32;
  uint32_t alignment = kDefaultAlignment;
};

struct LayerPlan {
  uint32_t absolute_layer = 0;
  bool mtp_layer = false;
  AttnClass attn_class = AttnClass::Sliding;
  uint32_t ratio = 0;
  uint32_t sliding_entries_per_sequence = 0, compressed_entries = 0;
  uint32_t compressor_buffer_tokens = 0, indexer_buffer_tokens = 0;
  // sliding: offsets within one sequence's stride; arena offset / bytes of the layer
  uint64_t sliding_content_offset = 0, sliding_rope_offset = 0, sliding_sequence_stride = 0;
  uint64_t sliding_arena_offset = 0, sliding_arena_bytes = 0;
  // compressed history: offsets within the layer's region
  uint64_t compressed_content_offset = 0, compressed_rope_offset = 0, indexer_history_offset = 0;
  uint64_t history_arena_offset = 0, history_arena_bytes = 0;
  // compressor state: offsets within one sequence's stride
  uint64_t compressor_kv_offset = 0, compressor_gate_offset = 0, indexer_kv_offset = 0, indexer_gate_offset = 0;
  uint64_t compressor_overlap_kv_offset = 0, compressor_overlap_gate_offset = 0;
  uint64_t indexer_overlap_kv_offset = 0, indexer_overlap_gate_offset = 0;
  uint64_t state_sequence_stride = 0, state_arena_offset = 0, state_arena_bytes = 0;
};

struct Plan {
  PlanConfig config;
  std::vector<LayerPlan> layers;
  uint32_t sliding_layers = 0, compressed_sparse_layers = 0, heavily_compressed_layers = 0;
  uint64_t sliding_arena_bytes = 0, history_arena_bytes = 0, state_arena_bytes = 0, total_arena_bytes = 0;
  uint64_t worst_sliding_bytes = 0, worst_history_bytes = 0, worst_state_bytes = 0, worst_total_bytes = 0;
};

Plan build_plan(const PlanConfig& cfg);  // throws InvalidArgument / CapacityExceeded

}  // namespace dsv4
}  // namespace spc
