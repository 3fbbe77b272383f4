// Ring runtime rank plans: everything one rank of a pipeline (optionally tensor
// parallel inside each stage) needs to know about its place in the ring, derived
// from one model geometry so every rank computes the same plan for every other.
//
//   geometry         model and deployment numbers as configuration: layers and
//                    the first routed layer, hidden size, context and DSA
//                    selection limits, speculative rows per lane, the largest batch
//                    bucket, stage count and default per-stage layer counts, host
//                    naming, GPUs per node, and the tensor-parallel shape inputs
//   rank plan        layer range and stage flags (final stage, dense prefix),
//                    previous / next ranks with their hosts and ports, lane and
//                    execution-row capacities, the largest hidden packet, TP degree /
//                    rank with the TP peers' hosts and collective ports, the shape's
//                    configuration hash (tp_shard.h), input / output routes with their
//                    hidden-transport endpoints, and the final-event route to rank 0
//   endpoints        a hidden-transport endpoint names its transport and declares
//                    capabilities. Between two ranks of one node it is NVLink peer
//                    memory (device resident); across nodes it is host staged (pinned
//                    host memory and the TCP fabric). Validation requires the full
//                    set of one of the two profiles, or a simulation-only set that
//                    does not also claim a production profile
//
// Reference behaviour: crates/spark-node/src/rank_daemon/ring_runtime.rs (constants
// :20-96, geometry :222-300, endpoint validation :378-414, rank plans and the
// fixed / shape builders :430-700). Capability bits, the NVLink-peer transport
// choice inside a node and the record layout are this runtime's own.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "common.h"
#include "stage_plan.h"
#include "tp_shard.h"

namespace spc {
namespace ring {

constexpr uint32_t kAbiVersion = 1;
constexpr uint32_t kDefaultPortBase = 52100;
constexpr uint32_t kFinalEventPortOffset = 200;
constexpr size_t kHostNameMax = 15, kRouteNameMax = 63;
constexpr uint32_t kNoRank = 0xffffffffu;

constexpr uint32_t kFlagHasPrevious = 0x1, kFlagHasNext = 0x2, kFlagFinalStage = 0x4, kFlagDensePrefix = 0x8;

// hidden-transport capabilities
constexpr uint32_t kCapBf16Rows = 0x01, kCapOrdered = 0x02, kCapBoundedWait = 0x04, kCapDeviceResident = 0x08,
                   kCapPeerMemory = 0x10, kCapHostStaged = 0x20, kCapSimulationOnly = 0x80000000u;
constexpr uint32_t kCapsPeerProduction = kCapBf16Rows | kCapOrdered | kCapBoundedWait | kCapDeviceResident | kCapPeerMemory;
constexpr uint32_t kCapsHostStaged = kCapBf16Rows | kCapOrdered | kCapBoundedWait | kCapHostStaged;
constexpr uint32_t kCapsSimulation = kCapBf16Rows | kCapOrdered | kCapSimulationOnly;

enum class Quantization : uint32_t { Bf16 = 0, Fp8E4m3 = 2 };

struct Geometry {
  uint32_t layer_count = 0, first_routed_layer = 0, hidden_dimension = 0;
  uint32_t maximum_context_tokens = 0, dsa_selected_tokens = 0, dsa_index_bytes_per_sequence = 0;
  uint32_t max_speculative_rows_per_lane = 1, max_batch_bucket = 0;
  uint32_t stage_count = 0;
  std::vector<uint32_t> default_stage_layer_counts;
  uint32_t max_routed_layers_per_stage = sp::kDefaultMaxRoutedPerStage;
  std::string host_prefix = "node";
  uint32_t host_index_base = 0;
  uint32_t gpus_per_node = 8;
  tp::Geometry tp_geometry;
  tp::ModelInputs shape_inputs;
  void validate() const;
  uint32_t hidden_bytes_per_sequence() const { return hidden_dimension * 2; }
  uint64_t transport_bytes_per_row() const { return uint64_t(hidden_bytes_per_sequence()) + dsa_index_bytes_per_sequence; }
};

// smallest power-of-two multiple of the DSA selection that covers the context (capped
// at the maximum context); 0 for an empty or oversized context
uint32_t dsa_candidate_bucket(const Geometry& g, uint32_t context_tokens);
// lanes x speculative rows, capped at the largest batch bucket; 0 for a bad lane count
uint32_t execution_row_capacity(const Geometry& g, uint32_t lanes);
// host of a rank: prefix + (base + node index), where a node holds gpus_per_node ranks
std::string rank_host_name(const Geometry& g, uint32_t rank);
uint32_t rank_node(const Geometry& g, uint32_t rank);

struct Endpoint {
  uint32_t abi_version = kAbiVersion, capability_flags = 0, hidden_dimension = 0, bytes_per_sequence = 0;
  uint32_t max_active_sequences = 0;
  uint64_t max_packet_bytes = 0, validated_latency_ns = 0;
  std::string transport, route_name;
};
void validate_endpoint(const Endpoint& e);  // AbiMismatch / InvalidArgument

struct RankPlan {
  uint32_t rank = 0, flags = 0, first_layer = 0, layer_count = 0;
  uint32_t previous_rank = kNoRank, next_rank = kNoRank;
  uint32_t listen_port = 0, next_port = 0, final_event_port = 0;
  uint32_t lanes = 0, speculative_rows_per_lane = 0, execution_row_capacity = 0;
  uint32_t hidden_dimension = 0, bytes_per_sequence = 0;
  Quantization quantization = Quantization::Bf16;
  uint32_t tp_degree = 1, tp_rank = 0, pp_stage_count = 1, pp_stage_index = 0, tp_collective_port = 0;
  uint64_t shape_configuration_hash = 0, max_packet_bytes = 0;
  std::string host, previous_host, next_host, final_event_host;
  std::vector<uint32_t> tp_peer_ranks, tp_peer_ports;
  std::vector<std::string> tp_peer_hosts;
  std::string input_route, output_route, final_event_route;
  bool has_input_endpoint = false, has_output_endpoint = false;
  Endpoint input_endpoint, output_endpoint;
};

// Pure pipeline: stage r of the geometry's default layer counts on rank r.
RankPlan build_rank_plan(const Geometry& g, uint32_t rank, uint32_t lanes, uint32_t port_base = kDefaultPortBase,
                         Quantization q = Quantization::Bf16);
// TP x PP: rank = pp_stage_index * tp_degree + tp_rank; stages of equal layer share
// from the shape (tp_shard.h derive_node_config); TP peers are the other ranks of the stage.
RankPlan build_shape_rank_plan(const Geometry& g, const tp::Shape& shape, uint32_t lanes,
                               uint32_t port_base = kDefaultPortBase, uint32_t tp_port_base = kDefaultPortBase + 100,
                               Quantization q = Quantization::Bf16);
void validate_rank_plan(const Geometry& g, const RankPlan& p);
// Every rank's plan of a shape, checked for agreement: each rank's next is the
// following stage's previous, and the ranges tile the layers.
std::vector<RankPlan> build_ring(const Geometry& g, uint32_t tp_degree, uint32_t lanes,
                                 uint32_t port_base = kDefaultPortBase, Quantization q = Quantization::Bf16);

}  // namespace ring
}  // namespace spc
