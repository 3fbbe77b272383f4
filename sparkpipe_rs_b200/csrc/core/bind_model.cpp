// Bindings of the model seam: contract documents and the model-driver loader
// (submodules `contract`, `driver`).
#include "contract.h"
#include "driver_loader.h"
#include "registry.h"

namespace py = pybind11;
using namespace spc;

static BindRegistrar reg([](py::module_& m) {
  auto c = m.def_submodule("contract", "model contract documents");
  py::class_<ModelGeometry>(c, "ModelGeometry")
      .def_readonly("total_parameters", &ModelGeometry::total_parameters)
      .def_readonly("active_parameters", &ModelGeometry::active_parameters)
      .def_readonly("hidden_dimension", &ModelGeometry::hidden_dimension)
      .def_readonly("layer_count", &ModelGeometry::layer_count)
      .def_readonly("vocabulary_size", &ModelGeometry::vocabulary_size)
      .def_readonly("maximum_context_tokens", &ModelGeometry::maximum_context_tokens)
      .def_readonly("first_routed_layer", &ModelGeometry::first_routed_layer);
  py::class_<ContractDocument>(c, "ContractDocument")
      .def_static("parse", &ContractDocument::parse, py::arg("text"), py::arg("path") = "<memory>")
      .def_property_readonly("schema_version", &ContractDocument::schema_version)
      .def_property_readonly("model_id", &ContractDocument::model_id)
      .def_property_readonly("architecture", &ContractDocument::architecture)
      .def("geometry", &ContractDocument::geometry)
      .def("section_json", [](const ContractDocument& d, const std::string& name) -> py::object {
        const Json* s = d.section(name);
        if (!s) return py::none();
        return py::str(s->dump());
      })
      .def("raw_json", [](const ContractDocument& d) { return d.raw().dump(); })
      .def("as_k27_json", [](const ContractDocument& d) { return d.as_k27().dump(); })
      .def("family", &ContractDocument::family);

  auto d = m.def_submodule("driver", "model-driver loader");
  d.attr("ABI_VERSION") = SPB_MODEL_DRIVER_ABI_VERSION;
  d.attr("SYMBOL") = SPB_MODEL_DRIVER_SYMBOL;
  d.attr("PROGRAM_EXTERNAL_COMPLETION") = SPB_PROGRAM_EXTERNAL_COMPLETION;
  d.attr("PROGRAM_STREAM_ORDERED") = SPB_PROGRAM_STREAM_ORDERED;
  d.attr("PROGRAM_CAPTURED_CUDA_GRAPH") = SPB_PROGRAM_CAPTURED_CUDA_GRAPH;
  d.attr("PROGRAM_NO_HOST_STAGING") = SPB_PROGRAM_NO_HOST_STAGING;
  d.attr("PROGRAM_NO_DEVICE_MEMCPY") = SPB_PROGRAM_NO_DEVICE_MEMCPY;
  d.attr("PROGRAM_VALIDATED_LATENCY") = SPB_PROGRAM_VALIDATED_LATENCY;
  d.attr("PROGRAM_PRIVATE_QUEUES") = SPB_PROGRAM_PRIVATE_QUEUES;
  d.attr("PROGRAM_KNOWN_FLAGS") = SPB_PROGRAM_KNOWN_FLAGS;
  py::class_<DriverProgramInfo>(d, "ProgramInfo")
      .def_readonly("program_id", &DriverProgramInfo::program_id)
      .def_readonly("flags", &DriverProgramInfo::flags)
      .def_readonly("max_inflight", &DriverProgramInfo::max_inflight)
      .def_readonly("name", &DriverProgramInfo::name);
  py::class_<spb_snapshot>(d, "Snapshot")
      .def_readonly("submits", &spb_snapshot::submits)
      .def_readonly("completions", &spb_snapshot::completions)
      .def_readonly("inflight", &spb_snapshot::inflight);
  py::class_<ModelDriver>(d, "ModelDriver")
      .def_static("load", &ModelDriver::load, py::arg("path"), py::arg("expected_target") = "",
                  py::return_value_policy::take_ownership)
      .def_property_readonly("model_id", &ModelDriver::model_id)
      .def_property_readonly("model_revision", &ModelDriver::model_revision)
      .def_property_readonly("stage_name", &ModelDriver::stage_name)
      .def_property_readonly("target", &ModelDriver::target)
      .def_property_readonly("model_description_sha256", &ModelDriver::model_description_sha256)
      .def_property_readonly("compiled_program_sha256", &ModelDriver::compiled_program_sha256)
      .def_property_readonly("module_instance_count", &ModelDriver::module_instance_count)
      .def("programs", &ModelDriver::programs)
      .def("find_program", [](const ModelDriver& m, const std::string& n) -> py::object {
        DriverProgramInfo p;
        if (!m.find_program(n, &p)) return py::none();
        return py::cast(p);
      })
      .def("create", &ModelDriver::create, py::arg("config_json") = "{}")
      .def("destroy", &ModelDriver::destroy)
      .def_property_readonly("has_instance", &ModelDriver::has_instance)
      .def("admit", &ModelDriver::admit)
      .def("snapshot", &ModelDriver::snapshot)
      .def("submit", [](ModelDriver& m, uint32_t pid, py::bytes input, size_t cap) {
        return py::bytes(m.submit(pid, std::string(input), cap));
      }, py::arg("program_id"), py::arg("input"), py::arg("output_capacity") = 4096);
  d.def("sha256_hex_is_valid", [](const std::string& s) { return sha256_hex_is_valid(s.c_str()); });
  d.def("abi_layout", [] {
    py::dict out;
    for (const auto& kv : driver_abi_layout()) out[py::str(kv.first)] = kv.second;
    return out;
  });
});
