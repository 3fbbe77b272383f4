// Bindings of tensor-parallel sharding and shape derivation (submodule `tp`).
#include "registry.h"
#include "tp_shard.h"

namespace py = pybind11;
using namespace spc;

static BindRegistrar reg([](py::module_& m) {
  auto t = m.def_submodule("tp", "tensor-parallel shard views and node configs");
  py::enum_<tp::ShardClass>(t, "ShardClass")
      .value("UNKNOWN", tp::ShardClass::Unknown)
      .value("REPLICATED", tp::ShardClass::Replicated)
      .value("OUTPUT_DIM_HEADS", tp::ShardClass::OutputDimHeads)
      .value("OUTPUT_DIM", tp::ShardClass::OutputDim)
      .value("INPUT_DIM_HEADS", tp::ShardClass::InputDimHeads)
      .value("INPUT_DIM", tp::ShardClass::InputDim)
      .value("CONCAT_OUTPUT", tp::ShardClass::ConcatOutput);
  py::class_<tp::Shape>(t, "Shape")
      .def(py::init([](uint32_t d, uint32_t r, uint32_t sc, uint32_t si) { return tp::Shape{d, r, sc, si}; }),
           py::arg("tp_degree") = 1, py::arg("tp_rank") = 0, py::arg("pp_stage_count") = 1,
           py::arg("pp_stage_index") = 0)
      .def_readwrite("tp_degree", &tp::Shape::tp_degree)
      .def_readwrite("tp_rank", &tp::Shape::tp_rank)
      .def_readwrite("pp_stage_count", &tp::Shape::pp_stage_count)
      .def_readwrite("pp_stage_index", &tp::Shape::pp_stage_index);
  py::class_<tp::Geometry>(t, "Geometry")
      .def(py::init([](uint32_t h, uint32_t q, uint32_t kv, uint32_t o) { return tp::Geometry{h, q, kv, o}; }),
           py::arg("head_count"), py::arg("q_b_head_block"), py::arg("kv_b_head_block"), py::arg("o_proj_head_block"));
  py::class_<tp::TensorSpec>(t, "TensorSpec")
      .def(py::init([](std::string n, std::vector<uint64_t> d, uint32_t b) { return tp::TensorSpec{n, d, b}; }),
           py::arg("name"), py::arg("dims"), py::arg("element_bytes") = 2);
  py::class_<tp::View>(t, "View")
      .def_readonly("shard_class", &tp::View::shard_class)
      .def_readonly("split_dimension", &tp::View::split_dimension)
      .def_readonly("ranges", &tp::View::ranges)
      .def_readonly("shard_bytes", &tp::View::shard_bytes);
  t.def("classify", &tp::classify);
  t.def("compute_view", &tp::compute_view);
  t.def("geometry_hash", &tp::geometry_hash);
  py::class_<tp::ModelInputs>(t, "ModelInputs")
      .def(py::init([](uint32_t L, uint32_t H, uint32_t moe, uint32_t dense, uint32_t kv, uint32_t eb) {
             return tp::ModelInputs{L, H, moe, dense, kv, eb};
           }),
           py::arg("total_layer_count"), py::arg("hidden_dimension"), py::arg("moe_intermediate_dimension"),
           py::arg("dense_intermediate_dimension"), py::arg("kv_latent_plus_rope_dimension"),
           py::arg("kv_bytes_per_element") = 2);
  py::class_<tp::NodeConfig>(t, "NodeConfig")
      .def_readonly("first_layer_index", &tp::NodeConfig::first_layer_index)
      .def_readonly("layer_count", &tp::NodeConfig::layer_count)
      .def_readonly("heads_per_rank", &tp::NodeConfig::heads_per_rank)
      .def_readonly("moe_intermediate_per_rank", &tp::NodeConfig::moe_intermediate_per_rank)
      .def_readonly("dense_intermediate_per_rank", &tp::NodeConfig::dense_intermediate_per_rank)
      .def_readonly("q_b_output_per_rank", &tp::NodeConfig::q_b_output_per_rank)
      .def_readonly("kv_b_output_per_rank", &tp::NodeConfig::kv_b_output_per_rank)
      .def_readonly("o_proj_input_per_rank", &tp::NodeConfig::o_proj_input_per_rank)
      .def_readonly("kv_bytes_per_token", &tp::NodeConfig::kv_bytes_per_token)
      .def_readonly("configuration_hash", &tp::NodeConfig::configuration_hash);
  t.def("derive_node_config", &tp::derive_node_config);
});
