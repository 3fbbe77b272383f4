// Bindings of the ring runtime rank plans (submodule `ring_runtime`).
#include "registry.h"
#include "ring_runtime.h"

#include <pybind11/stl.h>

namespace py = pybind11;
using namespace spc;

static BindRegistrar reg([](py::module_& m) {
  auto r = m.def_submodule("ring_runtime", "rank plans of a pipeline / TP ring and hidden-transport endpoints");
  r.attr("DEFAULT_PORT_BASE") = ring::kDefaultPortBase;
  r.attr("FINAL_EVENT_PORT_OFFSET") = ring::kFinalEventPortOffset;
  r.attr("NO_RANK") = ring::kNoRank;
  r.attr("FLAG_HAS_PREVIOUS") = ring::kFlagHasPrevious;
  r.attr("FLAG_HAS_NEXT") = ring::kFlagHasNext;
  r.attr("FLAG_FINAL_STAGE") = ring::kFlagFinalStage;
  r.attr("FLAG_DENSE_PREFIX") = ring::kFlagDensePrefix;
  r.attr("CAPS_PEER_PRODUCTION") = ring::kCapsPeerProduction;
  r.attr("CAPS_HOST_STAGED") = ring::kCapsHostStaged;
  r.attr("CAPS_SIMULATION") = ring::kCapsSimulation;
  r.attr("CAP_SIMULATION_ONLY") = ring::kCapSimulationOnly;
  py::enum_<ring::Quantization>(r, "Quantization")
      .value("BF16", ring::Quantization::Bf16)
      .value("FP8_E4M3", ring::Quantization::Fp8E4m3);

#define RW(T, f) .def_readwrite(#f, &T::f)
  py::class_<ring::Geometry>(r, "Geometry")
      .def(py::init<>())
      RW(ring::Geometry, layer_count) RW(ring::Geometry, first_routed_layer) RW(ring::Geometry, hidden_dimension)
      RW(ring::Geometry, maximum_context_tokens) RW(ring::Geometry, dsa_selected_tokens)
      RW(ring::Geometry, dsa_index_bytes_per_sequence) RW(ring::Geometry, max_speculative_rows_per_lane)
      RW(ring::Geometry, max_batch_bucket) RW(ring::Geometry, stage_count) RW(ring::Geometry, default_stage_layer_counts)
      RW(ring::Geometry, max_routed_layers_per_stage) RW(ring::Geometry, host_prefix) RW(ring::Geometry, host_index_base)
      RW(ring::Geometry, gpus_per_node) RW(ring::Geometry, tp_geometry) RW(ring::Geometry, shape_inputs)
      .def("validate", &ring::Geometry::validate)
      .def("transport_bytes_per_row", &ring::Geometry::transport_bytes_per_row);
  py::class_<ring::Endpoint>(r, "Endpoint")
      .def(py::init<>())
      RW(ring::Endpoint, abi_version) RW(ring::Endpoint, capability_flags) RW(ring::Endpoint, hidden_dimension)
      RW(ring::Endpoint, bytes_per_sequence) RW(ring::Endpoint, max_active_sequences) RW(ring::Endpoint, max_packet_bytes)
      RW(ring::Endpoint, validated_latency_ns) RW(ring::Endpoint, transport) RW(ring::Endpoint, route_name);
#undef RW
#define RO(f) .def_readonly(#f, &ring::RankPlan::f)
  py::class_<ring::RankPlan>(r, "RankPlan")
      RO(rank) RO(flags) RO(first_layer) RO(layer_count) RO(previous_rank) RO(next_rank) RO(listen_port) RO(next_port)
      RO(final_event_port) RO(lanes) RO(speculative_rows_per_lane) RO(execution_row_capacity) RO(hidden_dimension)
      RO(bytes_per_sequence) RO(quantization) RO(tp_degree) RO(tp_rank) RO(pp_stage_count) RO(pp_stage_index)
      RO(tp_collective_port) RO(shape_configuration_hash) RO(max_packet_bytes) RO(host) RO(previous_host) RO(next_host)
      RO(final_event_host) RO(tp_peer_ranks) RO(tp_peer_ports) RO(tp_peer_hosts) RO(input_route) RO(output_route)
      RO(final_event_route) RO(has_input_endpoint) RO(has_output_endpoint) RO(input_endpoint) RO(output_endpoint);
#undef RO
  r.def("dsa_candidate_bucket", &ring::dsa_candidate_bucket);
  r.def("execution_row_capacity", &ring::execution_row_capacity);
  r.def("rank_host_name", &ring::rank_host_name);
  r.def("validate_endpoint", &ring::validate_endpoint);
  r.def("validate_rank_plan", &ring::validate_rank_plan);
  r.def("build_rank_plan", &ring::build_rank_plan, py::arg("geometry"), py::arg("rank"), py::arg("lanes"),
        py::arg("port_base") = ring::kDefaultPortBase, py::arg("quantization") = ring::Quantization::Bf16);
  r.def("build_shape_rank_plan", &ring::build_shape_rank_plan, py::arg("geometry"), py::arg("shape"), py::arg("lanes"),
        py::arg("port_base") = ring::kDefaultPortBase, py::arg("tp_port_base") = ring::kDefaultPortBase + 100,
        py::arg("quantization") = ring::Quantization::Bf16);
  r.def("build_ring", &ring::build_ring, py::arg("geometry"), py::arg("tp_degree"), py::arg("lanes"),
        py::arg("port_base") = ring::kDefaultPortBase, py::arg("quantization") = ring::Quantization::Bf16);
});
