// Bindings of the work-output plane (submodule `work_output`).
#include "registry.h"
#include "work_output.h"

#include <pybind11/functional.h>
#include <pybind11/stl.h>

namespace py = pybind11;
using namespace spc;

static BindRegistrar reg([](py::module_& m) {
  auto w = m.def_submodule("work_output", "bounded work queue and non-blocking next-rank socket with acknowledgements");
  py::class_<wo::ReleaseRecord>(w, "ReleaseRecord")
      .def(py::init([](uint64_t req, uint64_t gen, uint64_t seq, uint32_t tokens) {
             return wo::ReleaseRecord{req, gen, seq, tokens};
           }),
           py::arg("request_id"), py::arg("request_generation"), py::arg("sequence_id"), py::arg("token_count"))
      .def_readonly("request_id", &wo::ReleaseRecord::request_id)
      .def_readonly("request_generation", &wo::ReleaseRecord::request_generation)
      .def_readonly("sequence_id", &wo::ReleaseRecord::sequence_id)
      .def_readonly("token_count", &wo::ReleaseRecord::token_count);
  py::class_<wo::WorkOutputStats>(w, "WorkOutputStats")
      .def_readonly("enqueued", &wo::WorkOutputStats::enqueued)
      .def_readonly("sent", &wo::WorkOutputStats::sent)
      .def_readonly("acknowledged", &wo::WorkOutputStats::acknowledged)
      .def_readonly("duplicates", &wo::WorkOutputStats::duplicates)
      .def_readonly("resent", &wo::WorkOutputStats::resent)
      .def_readonly("hard_failures", &wo::WorkOutputStats::hard_failures)
      .def_readonly("socket_drops", &wo::WorkOutputStats::socket_drops)
      .def_readonly("releases_queued", &wo::WorkOutputStats::releases_queued)
      .def_readonly("releases_sent", &wo::WorkOutputStats::releases_sent);
  py::class_<wo::WorkOutput>(w, "WorkOutput")
      .def(py::init<const wc::Config&, bool, std::string, uint32_t, uint32_t, uint32_t, uint32_t>(), py::arg("config"),
           py::arg("has_next"), py::arg("next_host"), py::arg("next_port"), py::arg("execution_row_capacity"),
           py::arg("queue_capacity"), py::arg("release_capacity"))
      .def("enqueue", &wo::WorkOutput::enqueue)
      .def("adopt_socket", &wo::WorkOutput::adopt_socket)
      .def("drop_socket", &wo::WorkOutput::drop_socket)
      .def("pump", &wo::WorkOutput::pump, py::arg("on_hard_failure") = nullptr)
      .def("queue_release", &wo::WorkOutput::queue_release)
      .def("build_release_packet", &wo::WorkOutput::build_release_packet)
      .def("pop_releases", &wo::WorkOutput::pop_releases)
      .def_property_readonly("has_next", &wo::WorkOutput::has_next)
      .def_property_readonly("has_socket", &wo::WorkOutput::has_socket)
      .def_property_readonly("queued", &wo::WorkOutput::queued)
      .def_property_readonly("releases", &wo::WorkOutput::releases)
      .def("release", &wo::WorkOutput::release, py::return_value_policy::copy)
      .def_property_readonly("stats", [](const wo::WorkOutput& o) { return o.stats(); });
});
