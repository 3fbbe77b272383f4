// Tensor-parallel sharding: how each weight of an MLA-MoE model splits over a TP
// group, and the node configuration a (TP degree, rank, PP stage) shape implies.
//
// Classes (weights stored [out_features, in_features]): REPLICATED (whole on every
// rank: the head-agnostic MLA latent projections and their norms, the router, norms,
// embedding), OUTPUT_DIM_HEADS / INPUT_DIM_HEADS (split on whole-head boundaries:
// q_b / kv_b outputs, o_proj input), OUTPUT_DIM / INPUT_DIM (MLP intermediates:
// gate|up outputs, down input), CONCAT_OUTPUT (a stacked [gate; up] tensor: each half
// splits and the halves re-concatenate per rank, so a rank's slice is two row
// ranges). Unknown names classify UNKNOWN and are refused for any degree above one.
// Output-dimension shards need no collective; input-dimension shards produce partial
// sums closed by the layer's all-reduce / reduce-scatter.
//
// Reference behaviour: the shard classes and view of
// crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_tp_shard.h:10-148 (the
// engine itself is absent there), the name table of
// V/model-families/glm52/src/spark_glm52_tp_shard.c, and the node-config derivation
// crates/spark-node/src/rank_daemon/shape.rs:180-250, whose configuration hash (FNV-1a
// over the little-endian struct images, seed 1469598103934665603) is reproduced bit for
// bit so the same shape hashes the same in both.
#pragma once

#include <string>
#include <vector>

#include "common.h"

namespace spc {
namespace tp {

constexpr uint32_t kShardAbi = 1;
constexpr uint32_t kShapeConfigAbi = 1;

enum class ShardClass : uint32_t {
  Unknown = 0,
  Replicated,
  OutputDimHeads,
  OutputDim,
  InputDimHeads,
  InputDim,
  ConcatOutput,
};

struct Shape {
  uint32_t tp_degree = 1, tp_rank = 0, pp_stage_count = 1, pp_stage_index = 0;
};

// head blocks of the attention projections, in elements: q_b out = nope + rope per
// head, kv_b out = nope + value per head, o_proj in = value per head
struct Geometry {
  uint32_t head_count = 0, q_b_head_block = 0, kv_b_head_block = 0, o_proj_head_block = 0;
};

struct TensorSpec {
  std::string name;
  std::vector<uint64_t> dims;  // [out, in] for matrices (leading expert dim allowed)
  uint32_t element_bytes = 2;
};

struct View {
  ShardClass shard_class = ShardClass::Unknown;
  uint32_t split_dimension = 0;
  // one range per part (one part, or two for CONCAT_OUTPUT), in elements of split_dimension
  std::vector<std::pair<uint64_t, uint64_t>> ranges;  // (offset, extent)
  uint64_t shard_bytes = 0;
};

ShardClass classify(const std::string& tensor_name);
uint64_t head_block(const std::string& tensor_name, const Geometry& g);
// Throws InvalidArgument on unsupported degree, rank out of range, unknown class at
// degree > 1, or indivisible dimensions.
View compute_view(const TensorSpec& spec, const Shape& shape, const Geometry& g);
// Order-sensitive FNV-1a over the shape, the tensor identity and the view: a shard
// built under another degree, rank or geometry hashes differently.
uint64_t geometry_hash(const TensorSpec& spec, const Shape& shape, const View& view);

// ---- node configuration of a shape
struct ModelInputs {
  uint32_t total_layer_count = 0, hidden_dimension = 0, moe_intermediate_dimension = 0;
  uint32_t dense_intermediate_dimension = 0, kv_latent_plus_rope_dimension = 0, kv_bytes_per_element = 2;
};
struct NodeConfig {
  uint32_t first_layer_index = 0, layer_count = 0, heads_per_rank = 0, moe_intermediate_per_rank = 0;
  uint32_t dense_intermediate_per_rank = 0, q_b_output_per_rank = 0, kv_b_output_per_rank = 0;
  uint32_t o_proj_input_per_rank = 0;
  uint64_t kv_bytes_per_token = 0, configuration_hash = 0;
};
NodeConfig derive_node_config(const Shape& shape, const Geometry& g, const ModelInputs& in);

}  // namespace tp
}  // namespace spc
