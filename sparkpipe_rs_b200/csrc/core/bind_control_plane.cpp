// Bindings of the driver control plane (submodule `control_plane`): model
// descriptions, the module library, the driver compiler and the orchestrator.
#include "control_plane.h"
#include "registry.h"

#include <pybind11/stl.h>

namespace py = pybind11;
using namespace spc;

static BindRegistrar reg([](py::module_& m) {
  auto c = m.def_submodule("control_plane", "model descriptions, module library, driver compiler, orchestrator");
  c.def("sha256_hex", [](py::bytes b) { return ctl::sha256_hex(std::string(b)); });
  c.def("file_sha256_hex", &ctl::file_sha256_hex);
  c.def("op_kind_name", [](uint32_t k) { return ctl::op_kind_name(ctl::OpKind(k)); });
  py::class_<ctl::Operation>(c, "Operation")
      .def_readonly("name", &ctl::Operation::name)
      .def_readonly("module_id", &ctl::Operation::module_id)
      .def_readonly("configuration_json", &ctl::Operation::configuration_json)
      .def_property_readonly("kind", [](const ctl::Operation& o) { return std::string(ctl::op_kind_name(o.kind)); });
  py::class_<ctl::Scheduling>(c, "Scheduling")
      .def_readonly("max_active_slots", &ctl::Scheduling::max_active_slots)
      .def_readonly("max_new_tokens", &ctl::Scheduling::max_new_tokens)
      .def_readonly("target_latency_ns", &ctl::Scheduling::target_latency_ns);
  py::class_<ctl::Program>(c, "Program")
      .def_readonly("name", &ctl::Program::name)
      .def_readonly("program_id", &ctl::Program::program_id)
      .def_readonly("max_inflight", &ctl::Program::max_inflight)
      .def_readonly("external_completion", &ctl::Program::external_completion)
      .def_readonly("scheduling", &ctl::Program::scheduling)
      .def_readonly("operations", &ctl::Program::operations);
  py::class_<ctl::Stage>(c, "Stage")
      .def_readonly("name", &ctl::Stage::name)
      .def_readonly("target", &ctl::Stage::target)
      .def_readonly("programs", &ctl::Stage::programs);
  py::class_<ctl::ModelDescription>(c, "ModelDescription")
      .def_readonly("schema_version", &ctl::ModelDescription::schema_version)
      .def_readonly("model_id", &ctl::ModelDescription::model_id)
      .def_readonly("model_revision", &ctl::ModelDescription::model_revision)
      .def_readonly("metadata_json", &ctl::ModelDescription::metadata_json)
      .def_readonly("source_sha256", &ctl::ModelDescription::source_sha256)
      .def_readonly("stages", &ctl::ModelDescription::stages);
  c.def("parse_model_description", &ctl::parse_model_description);
  c.def("load_model_description", &ctl::load_model_description);
  py::class_<ctl::ModuleArtifact>(c, "ModuleArtifact")
      .def_readonly("module_id", &ctl::ModuleArtifact::module_id)
      .def_readonly("target", &ctl::ModuleArtifact::target)
      .def_readonly("artifact_sha256", &ctl::ModuleArtifact::artifact_sha256)
      .def_readonly("link_unit_path", &ctl::ModuleArtifact::link_unit_path)
      .def_readonly("validator_sha256", &ctl::ModuleArtifact::validator_sha256)
      .def_readonly("execute_symbol", &ctl::ModuleArtifact::execute_symbol)
      .def_readonly("validated", &ctl::ModuleArtifact::validated);
  py::class_<ctl::PublishReport>(c, "PublishReport")
      .def_readonly("validation_reused", &ctl::PublishReport::validation_reused)
      .def_readonly("artifact_sha256", &ctl::PublishReport::artifact_sha256)
      .def_readonly("validator_sha256", &ctl::PublishReport::validator_sha256)
      .def_readonly("record_path", &ctl::PublishReport::record_path)
      .def_readonly("active_record_path", &ctl::PublishReport::active_record_path)
      .def_readonly("stored_link_unit_path", &ctl::PublishReport::stored_link_unit_path);
  c.def(
      "publish_module",
      [](const std::string& root, const std::string& module_id, const std::string& target,
         const std::string& link_unit, const std::string& recipe, const std::string& init_symbol,
         const std::string& execute_symbol, const std::string& destroy_symbol, const std::string& validator,
         const std::vector<std::string>& validator_args) {
        ctl::PublishRequest r;
        r.library_root = root;
        r.module_id = module_id;
        r.target = target;
        r.link_unit_path = link_unit;
        r.validation_recipe = recipe;
        r.init_symbol = init_symbol;
        r.execute_symbol = execute_symbol;
        r.destroy_symbol = destroy_symbol;
        r.validator_path = validator;
        r.validator_args = validator_args;
        return ctl::publish_module(r);
      },
      py::arg("library_root"), py::arg("module_id"), py::arg("target"), py::arg("link_unit"), py::arg("recipe"),
      py::arg("init_symbol"), py::arg("execute_symbol"), py::arg("destroy_symbol"), py::arg("validator"),
      py::arg("validator_args") = std::vector<std::string>{});
  c.def("resolve_module", &ctl::resolve_module);
  c.def("load_module_record", &ctl::load_module_record);
  py::class_<ctl::CompileReport>(c, "CompileReport")
      .def_readonly("program_count", &ctl::CompileReport::program_count)
      .def_readonly("operation_count", &ctl::CompileReport::operation_count)
      .def_readonly("link_unit_count", &ctl::CompileReport::link_unit_count)
      .def_readonly("model_description_sha256", &ctl::CompileReport::model_description_sha256)
      .def_readonly("compiled_program_sha256", &ctl::CompileReport::compiled_program_sha256)
      .def_readonly("driver_sha256", &ctl::CompileReport::driver_sha256)
      .def_readonly("generated_source_path", &ctl::CompileReport::generated_source_path)
      .def_readonly("driver_path", &ctl::CompileReport::driver_path)
      .def_readonly("manifest_path", &ctl::CompileReport::manifest_path);
  c.def(
      "compile_driver",
      [](const std::string& description, const std::string& stage, const std::string& root, const std::string& out,
         const std::string& compiler, const std::string& include_dir) {
        ctl::CompileRequest r;
        r.model_description_path = description;
        r.stage_name = stage;
        r.library_root = root;
        r.output_directory = out;
        r.compiler = compiler;
        r.include_directory = include_dir;
        return ctl::compile_driver(r);
      },
      py::arg("model_description"), py::arg("stage"), py::arg("library_root"), py::arg("output_directory"),
      py::arg("compiler") = "cc", py::arg("include_directory") = "");
  py::class_<ctl::Orchestrator>(c, "Orchestrator")
      .def(py::init<>())
      .def("add_node", &ctl::Orchestrator::add_node)
      .def("attach_driver", &ctl::Orchestrator::attach_driver, py::arg("node"), py::arg("driver_path"),
           py::arg("config_json") = "{}")
      .def("resolve_route", &ctl::Orchestrator::resolve_route)
      .def("submit",
           [](ctl::Orchestrator& o, uint32_t route, py::bytes input, size_t cap) {
             return py::bytes(o.submit(route, std::string(input), cap));
           })
      .def("outstanding", &ctl::Orchestrator::outstanding)
      .def("snapshot",
           [](ctl::Orchestrator& o, uint32_t d) {
             const spb_snapshot s = o.snapshot(d);
             return py::make_tuple(s.submits, s.completions, s.inflight);
           })
      .def_property_readonly("node_count", &ctl::Orchestrator::node_count)
      .def_property_readonly("driver_count", &ctl::Orchestrator::driver_count);
});
