#include "ring_runtime.h"

#include <algorithm>

namespace spc {
namespace ring {

void Geometry::validate() const {
  uint64_t sum = 0;
  for (uint32_t c : default_stage_layer_counts) sum += c;
  if (!layer_count || !hidden_dimension || !maximum_context_tokens || !dsa_selected_tokens ||
      !max_speculative_rows_per_lane || !max_batch_bucket || !stage_count || stage_count > sp::kMaxStages ||
      default_stage_layer_counts.size() != stage_count || sum != layer_count || host_prefix.empty() ||
      !gpus_per_node || !max_routed_layers_per_stage || shape_inputs.total_layer_count != layer_count ||
      shape_inputs.hidden_dimension != hidden_dimension)
    fail(Status::InvalidArgument, "ring geometry: invalid");
}

uint32_t dsa_candidate_bucket(const Geometry& g, uint32_t ctx) {
  if (!ctx || ctx > g.maximum_context_tokens) return 0;
  uint64_t n = g.dsa_selected_tokens;
  while (n < ctx && n < g.maximum_context_tokens) n <<= 1;
  return uint32_t(std::min<uint64_t>(n, g.maximum_context_tokens));
}

uint32_t execution_row_capacity(const Geometry& g, uint32_t lanes) {
  if (!lanes || lanes > g.max_batch_bucket) return 0;
  return uint32_t(std::min<uint64_t>(uint64_t(lanes) * g.max_speculative_rows_per_lane, g.max_batch_bucket));
}

uint32_t rank_node(const Geometry& g, uint32_t rank) { return rank / g.gpus_per_node; }

std::string rank_host_name(const Geometry& g, uint32_t rank) {
  const std::string h = g.host_prefix + std::to_string(g.host_index_base + rank_node(g, rank));
  if (h.size() > kHostNameMax) fail(Status::CapacityExceeded, "ring: host name too long");
  return h;
}

namespace {
bool has_all(uint32_t f, uint32_t need) { return (f & need) == need; }

std::string route(const std::string& from, uint32_t from_rank, const std::string& to, uint32_t to_rank) {
  const std::string r = from + "." + std::to_string(from_rank) + "_to_" + to + "." + std::to_string(to_rank) + "_hidden";
  if (r.size() > kRouteNameMax) fail(Status::CapacityExceeded, "ring: route name too long");
  return r;
}

Endpoint make_endpoint(const Geometry& g, uint32_t rows, bool same_node, const std::string& name) {
  Endpoint e;
  e.capability_flags = same_node ? kCapsPeerProduction : kCapsHostStaged;
  e.transport = same_node ? "nvlink.peer_memory" : "fabric.host_staged_tcp";
  e.hidden_dimension = g.hidden_dimension;
  e.bytes_per_sequence = g.hidden_bytes_per_sequence();
  e.max_active_sequences = rows;
  e.max_packet_bytes = g.transport_bytes_per_row() * rows;
  e.route_name = name;
  return e;
}

uint32_t checked_port(uint64_t p) {
  if (!p || p > 65535) fail(Status::InvalidArgument, "ring: port out of range");
  return uint32_t(p);
}

// Fills the fields every builder shares, then links the pipeline neighbours.
void finish(const Geometry& g, RankPlan& p, uint32_t lanes, uint32_t port_base, uint32_t prev, uint32_t next) {
  p.lanes = lanes;
  p.speculative_rows_per_lane = g.max_speculative_rows_per_lane;
  p.execution_row_capacity = execution_row_capacity(g, lanes);
  if (!p.execution_row_capacity) fail(Status::InvalidArgument, "ring: lane capacity outside the batch buckets");
  p.hidden_dimension = g.hidden_dimension;
  p.bytes_per_sequence = g.hidden_bytes_per_sequence();
  p.max_packet_bytes = g.transport_bytes_per_row() * p.execution_row_capacity;
  p.host = rank_host_name(g, p.rank);
  p.listen_port = checked_port(uint64_t(port_base) + p.rank);
  p.final_event_host = rank_host_name(g, 0);
  p.final_event_port = checked_port(uint64_t(port_base) + kFinalEventPortOffset);
  if (p.pp_stage_index > 0) {
    p.flags |= kFlagHasPrevious;
    p.previous_rank = prev;
    p.previous_host = rank_host_name(g, prev);
    p.input_route = route(p.previous_host, prev, p.host, p.rank);
    p.has_input_endpoint = true;
    p.input_endpoint = make_endpoint(g, p.execution_row_capacity, rank_node(g, prev) == rank_node(g, p.rank), p.input_route);
  }
  if (p.pp_stage_index + 1 < p.pp_stage_count) {
    p.flags |= kFlagHasNext;
    p.next_rank = next;
    p.next_port = checked_port(uint64_t(port_base) + next);
    p.next_host = rank_host_name(g, next);
    p.output_route = route(p.host, p.rank, p.next_host, next);
    p.has_output_endpoint = true;
    p.output_endpoint = make_endpoint(g, p.execution_row_capacity, rank_node(g, next) == rank_node(g, p.rank), p.output_route);
  } else {
    p.flags |= kFlagFinalStage;
    p.final_event_route = route(p.host, p.rank, p.final_event_host, 0);
  }
  // the stage that starts at layer 0 and holds every dense (unrouted) layer
  if (p.first_layer == 0 && p.layer_count >= g.first_routed_layer) p.flags |= kFlagDensePrefix;
}
}  // namespace

void validate_endpoint(const Endpoint& e) {
  if (e.abi_version != kAbiVersion) fail(Status::AbiMismatch, "hidden transport: ABI version");
  const uint32_t f = e.capability_flags;
  if (f & kCapSimulationOnly) {
    if (!has_all(f, kCapsSimulation) || has_all(f, kCapsPeerProduction) || has_all(f, kCapsHostStaged))
      fail(Status::InvalidArgument, "hidden transport: simulation endpoint claims a production profile");
  } else if (!has_all(f, kCapsPeerProduction) && !has_all(f, kCapsHostStaged)) {
    fail(Status::InvalidArgument, "hidden transport: capabilities meet no profile");
  }
  if (e.transport.empty() || e.route_name.empty() || !e.hidden_dimension || !e.bytes_per_sequence ||
      !e.max_active_sequences || !e.max_packet_bytes)
    fail(Status::InvalidArgument, "hidden transport: incomplete endpoint");
  if (uint64_t(e.bytes_per_sequence) * e.max_active_sequences > e.max_packet_bytes)
    fail(Status::InvalidArgument, "hidden transport: packet bound below one row per sequence");
}

void validate_rank_plan(const Geometry& g, const RankPlan& p) {
  if (!p.layer_count || uint64_t(p.first_layer) + p.layer_count > g.layer_count || !p.tp_degree ||
      p.tp_rank >= p.tp_degree || p.pp_stage_index >= p.pp_stage_count || p.host.empty() ||
      p.execution_row_capacity != execution_row_capacity(g, p.lanes) ||
      p.max_packet_bytes != g.transport_bytes_per_row() * p.execution_row_capacity)
    fail(Status::InvalidArgument, "rank plan: invalid");
  const bool has_prev = p.flags & kFlagHasPrevious, has_next = p.flags & kFlagHasNext;
  if (has_prev != (p.pp_stage_index > 0) || has_next != (p.pp_stage_index + 1 < p.pp_stage_count) ||
      bool(p.flags & kFlagFinalStage) == has_next || has_prev != p.has_input_endpoint ||
      has_next != p.has_output_endpoint)
    fail(Status::InvalidArgument, "rank plan: neighbour flags disagree");
  if (p.has_input_endpoint) validate_endpoint(p.input_endpoint);
  if (p.has_output_endpoint) validate_endpoint(p.output_endpoint);
  if (p.tp_peer_ranks.size() != p.tp_degree - 1 || p.tp_peer_hosts.size() != p.tp_peer_ranks.size() ||
      p.tp_peer_ports.size() != p.tp_peer_ranks.size())
    fail(Status::InvalidArgument, "rank plan: TP peer table");
}

RankPlan build_rank_plan(const Geometry& g, uint32_t rank, uint32_t lanes, uint32_t port_base, Quantization q) {
  g.validate();
  if (rank >= g.stage_count) fail(Status::InvalidArgument, "ring: rank out of range");
  const sp::Geometry sg{g.layer_count, g.first_routed_layer, g.max_routed_layers_per_stage};
  const sp::StagePlan plan = sp::build_from_layer_counts(sg, g.default_stage_layer_counts);
  const sp::Stage& st = plan.stages[rank];
  RankPlan p;
  p.rank = rank;
  p.first_layer = st.first_layer;
  p.layer_count = st.layer_count;
  p.quantization = q;
  p.pp_stage_count = g.stage_count;
  p.pp_stage_index = rank;
  finish(g, p, lanes, port_base, rank - 1, rank + 1);
  // the stage planner's flags are the authority on the final stage and dense prefix
  if (!(st.flags & sp::kFlagFinalToken) != !(p.flags & kFlagFinalStage) ||
      !(st.flags & sp::kFlagDensePrefix) != !(p.flags & kFlagDensePrefix))
    fail(Status::InternalError, "ring: stage flags disagree with the stage plan");
  validate_rank_plan(g, p);
  return p;
}

RankPlan build_shape_rank_plan(const Geometry& g, const tp::Shape& s, uint32_t lanes, uint32_t port_base,
                               uint32_t tp_port_base, Quantization q) {
  g.validate();
  const tp::NodeConfig nc = tp::derive_node_config(s, g.tp_geometry, g.shape_inputs);
  RankPlan p;
  p.rank = s.pp_stage_index * s.tp_degree + s.tp_rank;
  p.first_layer = nc.first_layer_index;
  p.layer_count = nc.layer_count;
  p.quantization = q;
  p.tp_degree = s.tp_degree;
  p.tp_rank = s.tp_rank;
  p.pp_stage_count = s.pp_stage_count;
  p.pp_stage_index = s.pp_stage_index;
  p.shape_configuration_hash = nc.configuration_hash;
  p.tp_collective_port = checked_port(uint64_t(tp_port_base) + p.rank);
  for (uint32_t t = 0; t < s.tp_degree; ++t) {
    if (t == s.tp_rank) continue;
    const uint32_t peer = s.pp_stage_index * s.tp_degree + t;
    p.tp_peer_ranks.push_back(peer);
    p.tp_peer_hosts.push_back(rank_host_name(g, peer));
    p.tp_peer_ports.push_back(checked_port(uint64_t(tp_port_base) + peer));
  }
  // hidden rows travel between the same TP rank of adjacent stages
  finish(g, p, lanes, port_base, p.rank - s.tp_degree, p.rank + s.tp_degree);
  validate_rank_plan(g, p);
  return p;
}

std::vector<RankPlan> build_ring(const Geometry& g, uint32_t tp_degree, uint32_t lanes, uint32_t port_base,
                                 Quantization q) {
  g.validate();
  std::vector<RankPlan> out;
  const uint32_t stages = g.stage_count;
  for (uint32_t st = 0; st < stages; ++st)
    for (uint32_t t = 0; t < tp_degree; ++t) {
      if (tp_degree == 1) {
        out.push_back(build_rank_plan(g, st, lanes, port_base, q));
      } else {
        tp::Shape s;
        s.tp_degree = tp_degree;
        s.tp_rank = t;
        s.pp_stage_count = stages;
        s.pp_stage_index = st;
        out.push_back(build_shape_rank_plan(g, s, lanes, port_base, port_base + 100, q));
      }
    }
  // agreement: neighbours name each other, and every TP rank's stages tile the layers
  for (const RankPlan& p : out) {
    if (p.flags & kFlagHasNext) {
      const RankPlan& n = out.at(p.next_rank);
      if (n.previous_rank != p.rank || n.first_layer != p.first_layer + p.layer_count || n.input_route != p.output_route)
        fail(Status::InternalError, "ring: neighbours disagree");
    }
  }
  for (uint32_t t = 0; t < tp_degree; ++t) {
    uint32_t covered = 0;
    for (uint32_t st = 0; st < stages; ++st) covered += out[st * tp_degree + t].layer_count;
    if (covered != g.layer_count) fail(Status::InternalError, "ring: stages do not tile the layers");
  }
  return out;
}

}  // namespace ring
}  // namespace spc
