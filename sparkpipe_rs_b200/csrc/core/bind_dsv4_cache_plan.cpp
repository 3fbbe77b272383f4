// Bindings of the DeepSeek-V4 cache plan (submodule `dsv4_cache_plan`).
#include "dsv4_cache_plan.h"
#include "registry.h"

#include <pybind11/stl.h>

namespace py = pybind11;
using namespace spc;

static BindRegistrar reg([](py::module_& m) {
  auto d = m.def_submodule("dsv4_cache_plan", "per-layer sliding / compressed / indexer KV cache plan of DeepSeek-V4");
  d.attr("MAX_LAYERS") = dsv4::kMaxLayers;
  d.attr("DEFAULT_ALIGNMENT") = dsv4::kDefaultAlignment;
  d.attr("DEFAULT_PAGE_ENTRIES") = dsv4::kDefaultPageEntries;
  py::enum_<dsv4::Variant>(d, "Variant").value("FLASH", dsv4::Variant::Flash).value("PRO", dsv4::Variant::Pro);
  py::enum_<dsv4::AttnClass>(d, "AttnClass")
      .value("SLIDING", dsv4::AttnClass::Sliding)
      .value("COMPRESSED_SPARSE", dsv4::AttnClass::CompressedSparse)
      .value("HEAVILY_COMPRESSED", dsv4::AttnClass::HeavilyCompressed);
  py::class_<dsv4::Geometry>(d, "Geometry")
      .def_readonly("backbone_layers", &dsv4::Geometry::backbone_layers)
      .def_readonly("mtp_layers", &dsv4::Geometry::mtp_layers)
      .def_readonly("head_dim", &dsv4::Geometry::head_dim)
      .def_readonly("rope_dim", &dsv4::Geometry::rope_dim)
      .def_readonly("index_head_dim", &dsv4::Geometry::index_head_dim)
      .def_readonly("sliding_window", &dsv4::Geometry::sliding_window)
      .def_readonly("max_context_tokens", &dsv4::Geometry::max_context_tokens);
  d.def("geometry", &dsv4::geometry);
  d.def("compression_ratio", &dsv4::compression_ratio, py::arg("variant"), py::arg("layer"), py::arg("mtp_layer") = false);

  py::class_<dsv4::PlanConfig>(d, "PlanConfig")
      .def(py::init<>())
      .def_readwrite("variant", &dsv4::PlanConfig::variant)
      .def_readwrite("first_backbone_layer", &dsv4::PlanConfig::first_backbone_layer)
      .def_readwrite("backbone_layer_count", &dsv4::PlanConfig::backbone_layer_count)
      .def_readwrite("include_mtp_layer", &dsv4::PlanConfig::include_mtp_layer)
      .def_readwrite("active_sequence_capacity", &dsv4::PlanConfig::active_sequence_capacity)
      .def_readwrite("max_context_tokens_per_sequence", &dsv4::PlanConfig::max_context_tokens_per_sequence)
      .def_readwrite("aggregate_context_token_capacity", &dsv4::PlanConfig::aggregate_context_token_capacity)
      .def_readwrite("page_entries", &dsv4::PlanConfig::page_entries)
      .def_readwrite("content_bits", &dsv4::PlanConfig::content_bits)
      .def_readwrite("rope_bits", &dsv4::PlanConfig::rope_bits)
      .def_readwrite("indexer_bits", &dsv4::PlanConfig::indexer_bits)
      .def_readwrite("state_bits", &dsv4::PlanConfig::state_bits)
      .def_readwrite("alignment", &dsv4::PlanConfig::alignment);

#define RO(f) .def_readonly(#f, &dsv4::LayerPlan::f)
  py::class_<dsv4::LayerPlan>(d, "LayerPlan")
      RO(absolute_layer) RO(mtp_layer) RO(attn_class) RO(ratio) RO(sliding_entries_per_sequence)
      RO(compressed_entries) RO(compressor_buffer_tokens) RO(indexer_buffer_tokens) RO(sliding_content_offset)
      RO(sliding_rope_offset) RO(sliding_sequence_stride) RO(sliding_arena_offset) RO(sliding_arena_bytes)
      RO(compressed_content_offset) RO(compressed_rope_offset) RO(indexer_history_offset) RO(history_arena_offset)
      RO(history_arena_bytes) RO(compressor_kv_offset) RO(compressor_gate_offset) RO(indexer_kv_offset)
      RO(indexer_gate_offset) RO(compressor_overlap_kv_offset) RO(compressor_overlap_gate_offset)
      RO(indexer_overlap_kv_offset) RO(indexer_overlap_gate_offset) RO(state_sequence_stride)
      RO(state_arena_offset) RO(state_arena_bytes);
#undef RO
#define RO(f) .def_readonly(#f, &dsv4::Plan::f)
  py::class_<dsv4::Plan>(d, "Plan")
      RO(config) RO(layers) RO(sliding_layers) RO(compressed_sparse_layers) RO(heavily_compressed_layers)
      RO(sliding_arena_bytes) RO(history_arena_bytes) RO(state_arena_bytes) RO(total_arena_bytes)
      RO(worst_sliding_bytes) RO(worst_history_bytes) RO(worst_state_bytes) RO(worst_total_bytes);
#undef RO
  d.def("build_plan", &dsv4::build_plan);
});
