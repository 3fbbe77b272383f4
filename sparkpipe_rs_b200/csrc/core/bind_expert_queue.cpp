// Bindings of the host-side expert batching queue (submodule `expert_queue`).
#include "expert_queue.h"
#include "registry.h"

namespace py = pybind11;
using namespace spc;

static BindRegistrar reg([](py::module_& m) {
  auto q = m.def_submodule("expert_queue", "host-side per-(layer, expert) row batching");
  q.attr("MAX_LAYERS") = eq::kMaxLayers;
  q.attr("MAX_EXPERTS") = eq::kMaxExperts;
  q.attr("MAX_ROWS") = eq::kMaxRows;
  q.attr("MAX_FIRING_ROWS") = eq::kMaxFiringRows;
  py::enum_<eq::Mode>(q, "Mode")
      .value("INVALID", eq::Mode::Invalid)
      .value("LOW_LATENCY", eq::Mode::LowLatency)
      .value("SEALED_BATCH", eq::Mode::SealedBatch);
  py::class_<eq::Config>(q, "Config")
      .def(py::init([](uint32_t layers, uint32_t experts, uint32_t threshold, uint64_t deadline_ns, eq::Mode mode) {
             eq::Config c;
             c.layer_count = layers;
             c.expert_count = experts;
             c.firing_threshold_rows = threshold;
             c.firing_deadline_ns = deadline_ns;
             c.mode = mode;
             return c;
           }),
           py::arg("layer_count"), py::arg("expert_count"), py::arg("firing_threshold_rows"),
           py::arg("firing_deadline_ns"), py::arg("mode"))
      .def_readwrite("layer_count", &eq::Config::layer_count)
      .def_readwrite("expert_count", &eq::Config::expert_count)
      .def_readwrite("firing_threshold_rows", &eq::Config::firing_threshold_rows)
      .def_readwrite("firing_deadline_ns", &eq::Config::firing_deadline_ns)
      .def_readwrite("mode", &eq::Config::mode);
  py::class_<eq::Stats>(q, "Stats")
      .def_readonly("firings", &eq::Stats::firings)
      .def_readonly("fired_rows", &eq::Stats::fired_rows)
      .def_readonly("enqueued", &eq::Stats::enqueued);
  py::class_<eq::ExpertQueue>(q, "ExpertQueue")
      .def(py::init<const eq::Config&>())
      .def("enqueue", &eq::ExpertQueue::enqueue, py::arg("layer"), py::arg("expert"), py::arg("row_id"),
           py::arg("arrival_ns"))
      .def("seal", &eq::ExpertQueue::seal)
      .def("set_firing_threshold", &eq::ExpertQueue::set_firing_threshold)
      .def("next_firing",
           [](eq::ExpertQueue& self, uint64_t now_ns) -> py::object {
             eq::Firing f;
             if (!self.next_firing(now_ns, f)) return py::none();
             return py::make_tuple(f.layer, f.expert, f.row_ids);
           },
           "(layer, expert, row_ids) of the next slot due at now_ns, or None")
      .def("slot_rows", &eq::ExpertQueue::slot_rows)
      .def("layer_rows", &eq::ExpertQueue::layer_rows)
      .def("sealed", &eq::ExpertQueue::sealed)
      .def("stats", &eq::ExpertQueue::stats);
});
