// Bindings of the scheduling-plane planners: pipeline stage planner,
// long-context policy and the live topology switch (submodules `stage_plan`,
// `long_context`, `topology_switch`).
#include "long_context.h"
#include "registry.h"
#include "stage_plan.h"
#include "topology_switch.h"

namespace py = pybind11;
using namespace spc;

namespace {
// Python-implemented seams for the topology switch (tests drive mocks).
struct PyTier : ts::Tier {
  Status pin(uint64_t key, bool pinned) override { PYBIND11_OVERRIDE_PURE(Status, ts::Tier, pin, key, pinned); }
  Status offset_of(uint64_t key, uint64_t* off) override {
    py::gil_scoped_acquire g;
    py::function f = py::get_override(static_cast<const ts::Tier*>(this), "offset_of");
    py::object r = f(key);  // int offset, or None when absent
    if (r.is_none()) return Status::NotFound;
    *off = r.cast<uint64_t>();
    return Status::Ok;
  }
  Status reserve_write(uint64_t key, ts::WriteReservation* out) override {
    py::gil_scoped_acquire g;
    py::function f = py::get_override(static_cast<const ts::Tier*>(this), "reserve_write");
    py::object r = f(key);  // (status, offset, already_present)
    auto t = r.cast<std::tuple<Status, uint64_t, bool>>();
    out->device_offset = std::get<1>(t);
    out->already_present = std::get<2>(t);
    return std::get<0>(t);
  }
  Status commit_write(const ts::WriteReservation& r) override {
    PYBIND11_OVERRIDE_PURE(Status, ts::Tier, commit_write, r);
  }
  void abort_write(const ts::WriteReservation& r) override { PYBIND11_OVERRIDE_PURE(void, ts::Tier, abort_write, r); }
  Status plan_lookahead(const std::vector<ts::TierNeed>& needs, uint32_t step) override {
    PYBIND11_OVERRIDE_PURE(Status, ts::Tier, plan_lookahead, needs, step);
  }
};
struct PySwap : ts::SwapDevice {
  Status begin_swap(const ts::Recipe& a, const ts::Recipe& b) override {
    PYBIND11_OVERRIDE_PURE(Status, ts::SwapDevice, begin_swap, a, b);
  }
  Status poll_swap() override { PYBIND11_OVERRIDE_PURE(Status, ts::SwapDevice, poll_swap, ); }
};
struct PyWriter : ts::ManifestWriter {
  Status write_block(uint64_t off, const std::string& payload) override {
    py::gil_scoped_acquire g;
    py::function f = py::get_override(static_cast<const ts::ManifestWriter*>(this), "write_block");
    return f(off, py::bytes(payload)).cast<Status>();
  }
};
}  // namespace

static BindRegistrar reg([](py::module_& m) {
  // ---------------------------------------------------------------- stage plan
  auto s = m.def_submodule("stage_plan", "pipeline stage planner");
  s.attr("ABI_VERSION") = sp::kAbiVersion;
  s.attr("MAX_STAGES") = sp::kMaxStages;
  s.attr("DESCRIPTOR_BYTES") = sp::kDescriptorBytes;
  s.attr("FLAG_FINAL_TOKEN") = sp::kFlagFinalToken;
  s.attr("FLAG_INPUT_HIDDEN") = sp::kFlagInputHidden;
  s.attr("FLAG_OUTPUT_HIDDEN") = sp::kFlagOutputHidden;
  s.attr("FLAG_DENSE_PREFIX") = sp::kFlagDensePrefix;
  py::class_<sp::Geometry>(s, "Geometry")
      .def(py::init([](uint32_t layers, uint32_t first_routed, uint32_t max_routed) {
             return sp::Geometry{layers, first_routed, max_routed};
           }),
           py::arg("layer_count"), py::arg("first_routed_layer"),
           py::arg("max_routed_layers_per_stage") = sp::kDefaultMaxRoutedPerStage)
      .def_readwrite("layer_count", &sp::Geometry::layer_count)
      .def_readwrite("first_routed_layer", &sp::Geometry::first_routed_layer)
      .def_readwrite("max_routed_layers_per_stage", &sp::Geometry::max_routed_layers_per_stage);
  py::class_<sp::Stage>(s, "Stage")
      .def(py::init([](uint32_t f, uint32_t n, uint32_t fl) { return sp::Stage{f, n, fl}; }),
           py::arg("first_layer"), py::arg("layer_count"), py::arg("flags") = 0)
      .def_readwrite("first_layer", &sp::Stage::first_layer)
      .def_readwrite("layer_count", &sp::Stage::layer_count)
      .def_readwrite("flags", &sp::Stage::flags)
      .def("__repr__", [](const sp::Stage& x) {
        return "Stage(" + std::to_string(x.first_layer) + ", " + std::to_string(x.layer_count) + ", flags=" +
               std::to_string(x.flags) + ")";
      });
  py::class_<sp::StagePlan>(s, "StagePlan")
      .def(py::init<>())
      .def_readwrite("stages", &sp::StagePlan::stages)
      .def_property_readonly("stage_count", [](const sp::StagePlan& p) { return p.stages.size(); })
      .def("total_layers", &sp::StagePlan::total_layers)
      .def("serialize", [](const sp::StagePlan& p) { return py::bytes(p.serialize()); })
      .def_static("deserialize", [](py::bytes b) { return sp::StagePlan::deserialize(std::string(b)); })
      .def("layer_counts", [](const sp::StagePlan& p) {
        std::vector<uint32_t> v;
        for (const auto& x : p.stages) v.push_back(x.layer_count);
        return v;
      });
  s.def("routed_layers_in", &sp::routed_layers_in);
  s.def("range_is_valid", &sp::range_is_valid);
  s.def("validate", &sp::validate);
  s.def("build_from_layer_counts", &sp::build_from_layer_counts);
  s.def("build_balanced", &sp::build_balanced, py::arg("geometry"), py::arg("layer_cost_ns"),
        py::arg("final_extra_ns") = 0, py::arg("stage_count") = 1);
  s.def("build_uniform", &sp::build_uniform);
  s.def("max_stage_cost", &sp::max_stage_cost);
  py::class_<sp::CostProfile>(s, "CostProfile")
      .def_readonly("layer_cost_ns", &sp::CostProfile::layer_cost_ns)
      .def_readonly("final_extra_ns", &sp::CostProfile::final_extra_ns)
      .def_readonly("measured", &sp::CostProfile::measured);
  py::class_<sp::StagePlanner>(s, "StagePlanner")
      .def(py::init<const sp::Geometry&>())
      .def("record_profile", &sp::StagePlanner::record_profile)
      .def("profile", &sp::StagePlanner::profile)
      .def("plan", &sp::StagePlanner::plan, py::return_value_policy::copy)
      .def_property_readonly("plan_builds", &sp::StagePlanner::plan_builds)
      .def_property_readonly("plan_hits", &sp::StagePlanner::plan_hits);

  // ---------------------------------------------------------------- long context
  auto l = m.def_submodule("long_context", "bounded decode selection and chunked-prefill plans");
  l.attr("INVALID_TOKEN") = lc::kInvalidToken;
  l.attr("MAX_SELECTED") = lc::kMaxSelected;
  l.attr("REQUIRE_BOUNDED") = lc::kRequireBounded;
  l.attr("INCLUDE_SINK") = lc::kIncludeSink;
  l.attr("INCLUDE_STRIDED") = lc::kIncludeStrided;
  l.attr("INCLUDE_RECENT") = lc::kIncludeRecent;
  l.attr("FAIL_ON_OVERFLOW") = lc::kFailOnOverflow;
  l.attr("ALLOW_FULL_SCAN") = lc::kAllowFullScan;
  l.attr("DEFAULT_FLAGS") = lc::kDefaultFlags;
  l.attr("PLAN_BOUNDED") = lc::kPlanBounded;
  l.attr("PLAN_FULL_SCAN") = lc::kPlanFullScan;
  l.attr("PLAN_LONG_CONTEXT") = lc::kPlanLongContext;
  l.attr("PLAN_TRUNCATED") = lc::kPlanTruncated;
  l.attr("PLAN_PADDED") = lc::kPlanPadded;
  l.attr("PREFILL_CHUNKED") = lc::kPrefillChunked;
  l.attr("PREFILL_LONG_CONTEXT") = lc::kPrefillLongContext;
  py::enum_<lc::Mode>(l, "Mode").value("BOUNDED_WINDOW", lc::Mode::BoundedWindow).value("FULL_SCAN", lc::Mode::FullScan);
  py::class_<lc::DecodePlan>(l, "DecodePlan")
      .def_readonly("flags", &lc::DecodePlan::flags)
      .def_readonly("context_tokens", &lc::DecodePlan::context_tokens)
      .def_readonly("selected", &lc::DecodePlan::selected)
      .def_readonly("capacity", &lc::DecodePlan::capacity)
      .def_readonly("padded", &lc::DecodePlan::padded)
      .def_readonly("selected_blocks", &lc::DecodePlan::selected_blocks)
      .def_readonly("block_tokens", &lc::DecodePlan::block_tokens)
      .def_readonly("context_blocks", &lc::DecodePlan::context_blocks)
      .def_readonly("first_recent", &lc::DecodePlan::first_recent)
      .def_readonly("max_scan", &lc::DecodePlan::max_scan)
      .def_readonly("sink", &lc::DecodePlan::sink)
      .def_readonly("strided", &lc::DecodePlan::strided)
      .def_readonly("recent", &lc::DecodePlan::recent)
      .def_readonly("est_reads", &lc::DecodePlan::est_reads)
      .def_readonly("avoided_reads", &lc::DecodePlan::avoided_reads);
  py::class_<lc::PrefillPlan>(l, "PrefillPlan")
      .def_readonly("flags", &lc::PrefillPlan::flags)
      .def_readonly("prompt_tokens", &lc::PrefillPlan::prompt_tokens)
      .def_readonly("tokens_per_step", &lc::PrefillPlan::tokens_per_step)
      .def_readonly("chunks", &lc::PrefillPlan::chunks)
      .def_readonly("final_chunk_tokens", &lc::PrefillPlan::final_chunk_tokens)
      .def_readonly("block_tokens", &lc::PrefillPlan::block_tokens)
      .def_readonly("prompt_blocks", &lc::PrefillPlan::prompt_blocks)
      .def_readonly("visits", &lc::PrefillPlan::visits);
  py::class_<lc::Policy>(l, "Policy")
      .def(py::init<uint32_t, uint32_t>(), py::arg("max_context_tokens"), py::arg("selected_capacity"))
      .def_readwrite("mode", &lc::Policy::mode)
      .def_readwrite("flags", &lc::Policy::flags)
      .def_readwrite("max_context_tokens", &lc::Policy::max_context_tokens)
      .def_readwrite("selected_capacity", &lc::Policy::selected_capacity)
      .def_readwrite("block_tokens", &lc::Policy::block_tokens)
      .def_readwrite("recent", &lc::Policy::recent)
      .def_readwrite("sink", &lc::Policy::sink)
      .def_readwrite("strided", &lc::Policy::strided)
      .def_readwrite("max_scan", &lc::Policy::max_scan)
      .def_readwrite("prefill_chunk", &lc::Policy::prefill_chunk)
      .def_readwrite("long_threshold", &lc::Policy::long_threshold)
      .def("validate", &lc::Policy::validate)
      .def("prefill_plan", &lc::Policy::prefill_plan, py::arg("prompt_tokens"), py::arg("tokens_per_step") = 0)
      .def("decode_selection", [](const lc::Policy& p, uint32_t ctx, uint32_t capacity) {
        std::vector<uint32_t> out(capacity);
        lc::DecodePlan d = p.decode_selection(ctx, out);
        return py::make_tuple(d, out);
      })
      .def("lane_batch", [](const lc::Policy& p, const std::vector<uint32_t>& ctx, size_t stride, size_t capacity) {
        std::vector<uint32_t> out(ctx.empty() ? 0 : (ctx.size() - 1) * stride + capacity, lc::kInvalidToken);
        auto plans = p.lane_batch(ctx, out, stride, capacity);
        return py::make_tuple(plans, out);
      });

  // ---------------------------------------------------------------- topology switch
  auto t = m.def_submodule("topology_switch", "TP <-> PP live re-shard state machine");
  t.attr("MANIFEST_DOMAIN") = ts::kManifestDomain;
  py::enum_<ts::Strategy>(t, "Strategy")
      .value("TENSOR_PARALLEL", ts::Strategy::TensorParallel)
      .value("PIPELINE_PARALLEL", ts::Strategy::PipelineParallel);
  py::enum_<ts::State>(t, "State")
      .value("STEADY", ts::State::Steady)
      .value("QUIESCE", ts::State::Quiesce)
      .value("CHECKPOINT", ts::State::Checkpoint)
      .value("SWAP", ts::State::Swap)
      .value("RESUME", ts::State::Resume);
  py::enum_<ts::ResumeClass>(t, "ResumeClass")
      .value("PENDING", ts::ResumeClass::Pending)
      .value("WARM", ts::ResumeClass::Warm)
      .value("RECOMPUTE", ts::ResumeClass::Recompute);
  py::class_<ts::Recipe>(t, "Recipe")
      .def(py::init([](uint64_t id, uint64_t bytes, ts::Strategy st) { return ts::Recipe{id, bytes, st}; }),
           py::arg("recipe_id"), py::arg("weight_pack_bytes") = 0, py::arg("strategy") = ts::Strategy::TensorParallel)
      .def_readwrite("recipe_id", &ts::Recipe::recipe_id)
      .def_readwrite("weight_pack_bytes", &ts::Recipe::weight_pack_bytes)
      .def_readwrite("strategy", &ts::Recipe::strategy);
  py::class_<ts::Budget>(t, "Budget")
      .def_readonly("quiesce_us", &ts::Budget::quiesce_us)
      .def_readonly("checkpoint_us", &ts::Budget::checkpoint_us)
      .def_readonly("swap_fixed_us", &ts::Budget::swap_fixed_us)
      .def_readonly("swap_stream_us", &ts::Budget::swap_stream_us)
      .def_readonly("resume_warm_us", &ts::Budget::resume_warm_us)
      .def_readonly("total_us", &ts::Budget::total_us);
  py::class_<ts::Stats>(t, "Stats")
      .def_readonly("switches_completed", &ts::Stats::switches_completed)
      .def_readonly("sequences_checkpointed", &ts::Stats::sequences_checkpointed)
      .def_readonly("resumed_warm", &ts::Stats::resumed_warm)
      .def_readonly("resumed_recompute", &ts::Stats::resumed_recompute)
      .def_readonly("completed_mid_switch", &ts::Stats::completed_mid_switch)
      .def_readonly("blocks_pinned", &ts::Stats::blocks_pinned)
      .def_readonly("manifest_writes", &ts::Stats::manifest_writes)
      .def_readonly("manifest_bytes", &ts::Stats::manifest_bytes)
      .def_readonly("tier_blocks_found", &ts::Stats::tier_blocks_found)
      .def_readonly("tier_blocks_absent", &ts::Stats::tier_blocks_absent)
      .def_readonly("swaps_started", &ts::Stats::swaps_started);
  py::class_<ts::Config>(t, "Config")
      .def(py::init<>())
      .def_readwrite("kv_namespace", &ts::Config::kv_namespace)
      .def_readwrite("max_sequences", &ts::Config::max_sequences)
      .def_readwrite("max_blocks_per_sequence", &ts::Config::max_blocks_per_sequence)
      .def_readwrite("step_time_us", &ts::Config::step_time_us)
      .def_readwrite("manifest_block_bytes", &ts::Config::manifest_block_bytes)
      .def_readwrite("read_bytes_per_s", &ts::Config::read_bytes_per_s)
      .def_readwrite("write_bytes_per_s", &ts::Config::write_bytes_per_s)
      .def_readwrite("swap_fixed_us", &ts::Config::swap_fixed_us)
      .def_readwrite("initial", &ts::Config::initial);
  py::class_<ts::TierNeed>(t, "TierNeed")
      .def_readonly("key", &ts::TierNeed::key)
      .def_readonly("need_by_step", &ts::TierNeed::need_by_step);
  py::class_<ts::WriteReservation>(t, "WriteReservation")
      .def_readonly("device_offset", &ts::WriteReservation::device_offset)
      .def_readonly("already_present", &ts::WriteReservation::already_present);
  py::class_<ts::Tier, PyTier>(t, "Tier").def(py::init<>());
  py::class_<ts::SwapDevice, PySwap>(t, "SwapDevice").def(py::init<>());
  py::class_<ts::ManifestWriter, PyWriter>(t, "ManifestWriter").def(py::init<>());
  t.def("kv_key", &ts::kv_key);
  t.def("manifest_key", &ts::manifest_key);
  t.def("estimate_budget", &ts::estimate_budget);
  py::class_<ts::TopologySwitch>(t, "TopologySwitch")
      .def(py::init<const ts::Config&, ts::Tier*, ts::SwapDevice*, ts::ManifestWriter*>(), py::keep_alive<1, 3>(),
           py::keep_alive<1, 4>(), py::keep_alive<1, 5>())
      .def_property_readonly("admissions_open", &ts::TopologySwitch::admissions_open)
      .def_property_readonly("state", &ts::TopologySwitch::state)
      .def_property_readonly("current_recipe", &ts::TopologySwitch::current_recipe)
      .def_property_readonly("last_error", [](const ts::TopologySwitch& x) { return uint32_t(x.last_error()); })
      .def_property_readonly("stats", &ts::TopologySwitch::stats)
      .def_property_readonly("tracked", &ts::TopologySwitch::tracked)
      .def("track_sequence", &ts::TopologySwitch::track_sequence)
      .def("set_sequence_kv", &ts::TopologySwitch::set_sequence_kv)
      .def("sequence_at_boundary", &ts::TopologySwitch::sequence_at_boundary)
      .def("sequence_complete", &ts::TopologySwitch::sequence_complete)
      .def("begin", &ts::TopologySwitch::begin)
      .def("advance", &ts::TopologySwitch::advance)
      .def("resume_class_of", &ts::TopologySwitch::resume_class_of);
});
