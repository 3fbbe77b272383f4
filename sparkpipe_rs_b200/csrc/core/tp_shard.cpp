#include "tp_shard.h"

namespace spc {
namespace tp {

namespace {
bool ends_with(const std::string& s, const char* suf) {
  const size_t n = std::char_traits<char>::length(suf);
  return s.size() >= n && s.compare(s.size() - n, n, suf) == 0;
}
bool degree_ok(uint32_t d) { return d == 1 || d == 2 || d == 4 || d == 8 || d == 16; }
void put32(std::string& b, uint32_t v) {
  for (int i = 0; i < 4; ++i) b.push_back(char(v >> (8 * i)));
}
void put64(std::string& b, uint64_t v) {
  for (int i = 0; i < 8; ++i) b.push_back(char(v >> (8 * i)));
}
constexpr uint64_t kShapeHashSeed = 1469598103934665603ull;
}  // namespace

ShardClass classify(const std::string& n) {
  // this engine's weight names (models/weights.py) first, then Hugging Face names
  if (ends_with(n, "w_q_b") || ends_with(n, "w_kv_b") || ends_with(n, "self_attn.q_b_proj.weight") ||
      ends_with(n, "self_attn.kv_b_proj.weight") || ends_with(n, "self_attn.q_proj.weight"))
    return ShardClass::OutputDimHeads;
  if (ends_with(n, "w_o") || ends_with(n, "self_attn.o_proj.weight")) return ShardClass::InputDimHeads;
  if (ends_with(n, "w13") || ends_with(n, "e_w13")) return ShardClass::ConcatOutput;
  if (ends_with(n, "mlp.gate_proj.weight") || ends_with(n, "mlp.up_proj.weight") ||
      ends_with(n, "shared_experts.gate_proj.weight") || ends_with(n, "shared_experts.up_proj.weight") ||
      ends_with(n, "lm_head") || ends_with(n, "lm_head.weight"))
    return ShardClass::OutputDim;
  if (ends_with(n, "w2") || ends_with(n, "e_w2") || ends_with(n, "mlp.down_proj.weight") ||
      ends_with(n, "shared_experts.down_proj.weight"))
    return ShardClass::InputDim;
  if (ends_with(n, "w_qkv_a") || ends_with(n, "q_a_norm") || ends_with(n, "kv_a_norm") || ends_with(n, "in_norm") ||
      ends_with(n, "post_norm") || ends_with(n, "final_norm") || ends_with(n, "gate") || ends_with(n, "gate_bias") ||
      ends_with(n, "embed") || ends_with(n, "self_attn.q_a_proj.weight") ||
      ends_with(n, "self_attn.kv_a_proj_with_mqa.weight") || ends_with(n, "self_attn.q_a_layernorm.weight") ||
      ends_with(n, "self_attn.kv_a_layernorm.weight") || ends_with(n, "mlp.gate.weight") ||
      ends_with(n, "mlp.gate.e_score_correction_bias") || ends_with(n, "input_layernorm.weight") ||
      ends_with(n, "post_attention_layernorm.weight") || ends_with(n, "model.norm.weight") ||
      ends_with(n, "model.embed_tokens.weight"))
    return ShardClass::Replicated;
  return ShardClass::Unknown;
}

uint64_t head_block(const std::string& n, const Geometry& g) {
  if (ends_with(n, "w_q_b") || ends_with(n, "q_b_proj.weight") || ends_with(n, "q_proj.weight")) return g.q_b_head_block;
  if (ends_with(n, "w_kv_b") || ends_with(n, "kv_b_proj.weight")) return g.kv_b_head_block;
  return g.o_proj_head_block;
}

View compute_view(const TensorSpec& spec, const Shape& shape, const Geometry& g) {
  if (!degree_ok(shape.tp_degree)) fail(Status::InvalidArgument, "tp shard: degree must be 1, 2, 4, 8 or 16");
  if (shape.tp_rank >= shape.tp_degree) fail(Status::InvalidArgument, "tp shard: rank out of range");
  if (spec.dims.empty() || spec.element_bytes == 0) fail(Status::InvalidArgument, "tp shard: empty tensor spec");
  uint64_t total = spec.element_bytes;
  for (uint64_t d : spec.dims) total *= d;
  View v;
  v.shard_class = classify(spec.name);
  const size_t rank_dims = spec.dims.size();
  // matrices are [.., out, in]; a leading expert dimension is carried whole
  const uint32_t out_dim = uint32_t(rank_dims >= 2 ? rank_dims - 2 : 0);
  const uint32_t in_dim = uint32_t(rank_dims - 1);
  if (shape.tp_degree == 1 || v.shard_class == ShardClass::Replicated) {
    if (v.shard_class == ShardClass::Unknown && shape.tp_degree > 1)
      fail(Status::InvalidArgument, "tp shard: unknown tensor " + spec.name);
    v.shard_class = shape.tp_degree == 1 && v.shard_class == ShardClass::Unknown ? ShardClass::Replicated : v.shard_class;
    if (shape.tp_degree == 1) v.shard_class = ShardClass::Replicated;
    v.split_dimension = 0;
    v.ranges = {{0, spec.dims[0]}};
    v.shard_bytes = total;
    return v;
  }
  if (v.shard_class == ShardClass::Unknown) fail(Status::InvalidArgument, "tp shard: unknown tensor " + spec.name);
  if (rank_dims < 2) fail(Status::InvalidArgument, "tp shard: a split tensor must be a matrix");
  const uint64_t D = shape.tp_degree, r = shape.tp_rank;
  auto split = [&](uint32_t dim, uint64_t block) {
    const uint64_t n = spec.dims[dim];
    if (block == 0 || n % block) fail(Status::InvalidArgument, "tp shard: dimension not a whole number of blocks");
    const uint64_t units = n / block;
    if (units % D) fail(Status::InvalidArgument, "tp shard: dimension not divisible by the degree");
    const uint64_t per = units / D * block;
    v.split_dimension = dim;
    v.ranges = {{r * per, per}};
  };
  switch (v.shard_class) {
    case ShardClass::OutputDimHeads: split(out_dim, head_block(spec.name, g)); break;
    case ShardClass::InputDimHeads: split(in_dim, head_block(spec.name, g)); break;
    case ShardClass::OutputDim: split(out_dim, 1); break;
    case ShardClass::InputDim: split(in_dim, 1); break;
    case ShardClass::ConcatOutput: {
      const uint64_t n = spec.dims[out_dim];
      if (n % (2 * D)) fail(Status::InvalidArgument, "tp shard: concatenated halves not divisible by the degree");
      const uint64_t half = n / 2, per = half / D;
      v.split_dimension = out_dim;
      v.ranges = {{r * per, per}, {half + r * per, per}};
      break;
    }
    default: fail(Status::InternalError, "tp shard: unhandled class");
  }
  uint64_t extent = 0;
  for (const auto& rg : v.ranges) extent += rg.second;
  v.shard_bytes = total / spec.dims[v.split_dimension] * extent;
  return v;
}

uint64_t geometry_hash(const TensorSpec& spec, const Shape& shape, const View& view) {
  std::string b;
  put32(b, kShardAbi);
  put32(b, shape.tp_degree);
  put32(b, shape.tp_rank);
  put32(b, shape.pp_stage_count);
  put32(b, shape.pp_stage_index);
  b += spec.name;
  b.push_back('\0');
  for (uint64_t d : spec.dims) put64(b, d);
  put32(b, spec.element_bytes);
  put32(b, uint32_t(view.shard_class));
  put32(b, view.split_dimension);
  for (const auto& rg : view.ranges) {
    put64(b, rg.first);
    put64(b, rg.second);
  }
  put64(b, view.shard_bytes);
  return fnv1a64(b.data(), b.size());
}

NodeConfig derive_node_config(const Shape& s, const Geometry& g, const ModelInputs& in) {
  if (!degree_ok(s.tp_degree)) fail(Status::InvalidArgument, "shape: unsupported TP degree");
  if (s.tp_rank >= s.tp_degree || s.pp_stage_count == 0 || s.pp_stage_index >= s.pp_stage_count)
    fail(Status::InvalidArgument, "shape: rank or stage out of range");
  if (in.total_layer_count == 0 || in.total_layer_count % s.pp_stage_count)
    fail(Status::InvalidArgument, "shape: layers do not split evenly over the stages");
  if (g.head_count == 0 || g.head_count % s.tp_degree || in.moe_intermediate_dimension % s.tp_degree ||
      in.dense_intermediate_dimension % s.tp_degree)
    fail(Status::InvalidArgument, "shape: heads or intermediates not divisible by the TP degree");
  NodeConfig c;
  c.layer_count = in.total_layer_count / s.pp_stage_count;
  c.first_layer_index = s.pp_stage_index * c.layer_count;
  c.heads_per_rank = g.head_count / s.tp_degree;
  c.moe_intermediate_per_rank = in.moe_intermediate_dimension / s.tp_degree;
  c.dense_intermediate_per_rank = in.dense_intermediate_dimension / s.tp_degree;
  c.q_b_output_per_rank = c.heads_per_rank * g.q_b_head_block;
  c.kv_b_output_per_rank = c.heads_per_rank * g.kv_b_head_block;
  c.o_proj_input_per_rank = c.heads_per_rank * g.o_proj_head_block;
  // every TP rank of a stage keeps the full head-agnostic latent of its layers
  c.kv_bytes_per_token = uint64_t(c.layer_count) * in.kv_latent_plus_rope_dimension * in.kv_bytes_per_element;
  // configuration hash over the little-endian images of the shape, geometry,
  // inputs and the derived prefix (each prefixed by its ABI word)
  std::string b;
  for (uint32_t v : {kShardAbi, s.tp_degree, s.tp_rank, s.pp_stage_count, s.pp_stage_index}) put32(b, v);
  for (uint32_t v : {kShardAbi, g.head_count, g.q_b_head_block, g.kv_b_head_block, g.o_proj_head_block}) put32(b, v);
  for (uint32_t v : {kShapeConfigAbi, in.total_layer_count, in.hidden_dimension, in.moe_intermediate_dimension,
                     in.dense_intermediate_dimension, in.kv_latent_plus_rope_dimension, in.kv_bytes_per_element})
    put32(b, v);
  for (uint32_t v : {kShapeConfigAbi, c.first_layer_index, c.layer_count, c.heads_per_rank, c.moe_intermediate_per_rank,
                     c.dense_intermediate_per_rank, c.q_b_output_per_rank, c.kv_b_output_per_rank,
                     c.o_proj_input_per_rank, 0u})
    put32(b, v);
  put64(b, c.kv_bytes_per_token);
  c.configuration_hash = fnv1a64(b.data(), b.size(), kShapeHashSeed);
  return c;
}

}  // namespace tp
}  // namespace spc
