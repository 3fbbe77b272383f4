// Bindings of the ring node context (submodule `node_context`).
#include "node_context.h"
#include "registry.h"

#include <pybind11/functional.h>
#include <pybind11/stl.h>

namespace py = pybind11;
using namespace spc;

static BindRegistrar reg([](py::module_& m) {
  auto n = m.def_submodule("node_context", "prefill / decode / submit_work seam of one ring rank over its model driver");
  py::class_<nc::NodeContextConfig>(n, "NodeContextConfig")
      .def(py::init<>())
      .def_readwrite("plan", &nc::NodeContextConfig::plan)
      .def_readwrite("driver_path", &nc::NodeContextConfig::driver_path)
      .def_readwrite("target", &nc::NodeContextConfig::target)
      .def_readwrite("driver_config_json", &nc::NodeContextConfig::driver_config_json)
      .def_readwrite("prefill_program", &nc::NodeContextConfig::prefill_program)
      .def_readwrite("decode_program", &nc::NodeContextConfig::decode_program)
      .def_readwrite("work", &nc::NodeContextConfig::work)
      .def_readwrite("queue_capacity", &nc::NodeContextConfig::queue_capacity)
      .def_readwrite("release_capacity", &nc::NodeContextConfig::release_capacity)
      .def_readwrite("output_capacity", &nc::NodeContextConfig::output_capacity);
  py::class_<nc::WorkResult>(n, "WorkResult")
      .def_readonly("status", &nc::WorkResult::status)
      .def_readonly("forwarded", &nc::WorkResult::forwarded)
      .def_readonly("final_stage", &nc::WorkResult::final_stage)
      .def_property_readonly("output", [](const nc::WorkResult& r) { return py::bytes(r.output); })
      .def_readonly("final_event", &nc::WorkResult::final_event);
  py::class_<nc::NodeContext>(n, "NodeContext")
      .def_static("build", [](const nc::NodeContextConfig& c) { return nc::NodeContext::build(c).release(); },
                  py::return_value_policy::take_ownership)
      .def("submit_work", &nc::NodeContext::submit_work)
      .def("prefill", &nc::NodeContext::prefill)
      .def("decode", &nc::NodeContext::decode)
      .def("pump_output", &nc::NodeContext::pump_output, py::arg("on_hard_failure") = nullptr)
      .def("adopt_output_socket", [](nc::NodeContext& c, int fd) {
        if (!c.work_output()) throw std::invalid_argument("node context: final stage has no output plane");
        c.work_output()->adopt_socket(fd);
      })
      .def_property_readonly("queued_output", [](nc::NodeContext& c) { return c.work_output() ? c.work_output()->queued() : 0u; })
      .def_property_readonly("submitted", &nc::NodeContext::submitted)
      .def_property_readonly("plan", &nc::NodeContext::plan);
});
