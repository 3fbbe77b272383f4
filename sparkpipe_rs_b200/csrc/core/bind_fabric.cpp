// Bindings of the multi-node host fabric (submodule `fabric`): memlink planning and
// transfer over buffer-protocol objects (bytes / bytearray / numpy), and the fabric
// topology model. Transfers release the GIL.
#include "fabric.h"
#include "registry.h"

#include <pybind11/stl.h>

namespace py = pybind11;
using namespace spc;

static BindRegistrar reg([](py::module_& m) {
  auto f = m.def_submodule("fabric", "memlink neighbour transfers and the fabric topology model");
  f.attr("DEFAULT_BASE_PORT") = fabric::kDefaultBasePort;
  f.attr("DEFAULT_LANES") = fabric::kDefaultLanes;
  f.attr("MAX_LANES") = fabric::kMaxLanes;
  f.attr("DEFAULT_STORE_BYTES") = fabric::kDefaultStoreBytes;
  f.attr("CHUNK_BYTES") = fabric::kChunkBytes;
  f.attr("NO_NODE") = fabric::kNoNode;
  f.attr("FLAG_DEBUG_ONLY") = fabric::kFlagDebugOnly;
  f.attr("FLAG_SWITCHED") = fabric::kFlagSwitched;
  f.attr("FLAG_FUTURE_ONLY") = fabric::kFlagFutureOnly;
  py::enum_<fabric::Direction>(f, "Direction")
      .value("PREVIOUS", fabric::Direction::Previous)
      .value("NEXT", fabric::Direction::Next);
  py::enum_<fabric::Mode>(f, "Mode")
      .value("INVALID", fabric::Mode::Invalid)
      .value("RING_DEBUG_SINGLE_RAIL", fabric::Mode::RingDebugSingleRail)
      .value("SINGLE_SWITCH_SINGLE_RAIL", fabric::Mode::SingleSwitchSingleRail)
      .value("DUAL_SWITCH_DUAL_RAIL", fabric::Mode::DualSwitchDualRail);
  py::class_<fabric::Partition>(f, "Partition")
      .def_readonly("lane", &fabric::Partition::lane)
      .def_readonly("lanes", &fabric::Partition::lanes)
      .def_readonly("offset", &fabric::Partition::offset)
      .def_readonly("bytes", &fabric::Partition::bytes);
  py::class_<fabric::Endpoint>(f, "Endpoint")
      .def_readonly("host", &fabric::Endpoint::host)
      .def_readonly("base_port", &fabric::Endpoint::base_port)
      .def_readonly("lanes", &fabric::Endpoint::lanes);
  f.def("validate_lanes", &fabric::validate_lanes);
  f.def("partition", &fabric::partition, py::arg("total"), py::arg("lanes"), py::arg("lane"),
        py::arg("chunk") = fabric::kChunkBytes);
  f.def("neighbor_rank", &fabric::neighbor_rank);
  f.def("host_from_template", &fabric::host_from_template);
  f.def("neighbor_endpoint", &fabric::neighbor_endpoint, py::arg("rank"), py::arg("ranks"), py::arg("direction"),
        py::arg("host_template"), py::arg("base_port") = fabric::kDefaultBasePort,
        py::arg("lanes") = fabric::kDefaultLanes);
  f.def("send",
        [](const std::string& host, uint16_t port, uint32_t lanes, py::buffer src, uint32_t timeout_ms) {
          py::buffer_info b = src.request();
          const uint64_t n = uint64_t(b.size) * b.itemsize;
          py::gil_scoped_release nogil;
          return fabric::Memlink::send(host, port, lanes, static_cast<const uint8_t*>(b.ptr), n, timeout_ms);
        },
        py::arg("host"), py::arg("base_port"), py::arg("lanes"), py::arg("src"), py::arg("timeout_ms") = 30000);
  f.def("receive",
        [](uint16_t port, uint32_t lanes, py::buffer dst, uint32_t timeout_ms) {
          py::buffer_info b = dst.request(true);
          const uint64_t n = uint64_t(b.size) * b.itemsize;
          py::gil_scoped_release nogil;
          return fabric::Memlink::receive(port, lanes, static_cast<uint8_t*>(b.ptr), n, timeout_ms);
        },
        py::arg("base_port"), py::arg("lanes"), py::arg("dst"), py::arg("timeout_ms") = 30000);
  py::class_<fabric::TopologyConfig>(f, "TopologyConfig")
      .def(py::init<>())
      .def_readwrite("mode", &fabric::TopologyConfig::mode)
      .def_readwrite("flags", &fabric::TopologyConfig::flags)
      .def_readwrite("nodes", &fabric::TopologyConfig::nodes)
      .def_readwrite("local", &fabric::TopologyConfig::local)
      .def_readwrite("rails", &fabric::TopologyConfig::rails)
      .def_readwrite("switches", &fabric::TopologyConfig::switches)
      .def_readwrite("ports", &fabric::TopologyConfig::ports)
      .def_readwrite("link_gbps", &fabric::TopologyConfig::link_gbps)
      .def_readwrite("mtu", &fabric::TopologyConfig::mtu);
  py::class_<fabric::Route>(f, "Route")
      .def_readonly("mode", &fabric::Route::mode)
      .def_readonly("rail", &fabric::Route::rail)
      .def_readonly("src", &fabric::Route::src)
      .def_readonly("dst", &fabric::Route::dst)
      .def_readonly("port", &fabric::Route::port)
      .def_readonly("first_hop", &fabric::Route::first_hop)
      .def_readonly("hops", &fabric::Route::hops)
      .def_readonly("switched", &fabric::Route::switched);
  f.def("default_topology", &fabric::default_topology, py::arg("mode"), py::arg("nodes"), py::arg("local"),
        py::arg("mtu") = 9000);
  f.def("validate", &fabric::validate);
  f.def("resolve_route", &fabric::resolve_route);
  f.def("mode_name", &fabric::mode_name);
});
