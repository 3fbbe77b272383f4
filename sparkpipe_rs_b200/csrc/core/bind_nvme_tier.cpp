// Bindings of the drive-backed KV tier (submodule `nvme_tier`). Staging data is
// handed back as bytes (a copy) plus its host address for zero-copy consumers.
#include "nvme_tier.h"
#include "registry.h"

#include <pybind11/stl.h>

#include <cstdlib>
#include <cstring>

namespace py = pybind11;
using namespace spc;

static Status device_write(nvt::BlockDevice& d, uint64_t offset, const py::bytes& data) {
  const std::string buf = data;  // O_DIRECT wants an aligned source: copy into one
  const size_t n = (buf.size() + nvt::kIoAlignment - 1) / nvt::kIoAlignment * nvt::kIoAlignment;
  void* a = std::aligned_alloc(nvt::kIoAlignment, n ? n : nvt::kIoAlignment);
  if (!a) return Status::CapacityExceeded;
  std::memset(a, 0, n);
  std::memcpy(a, buf.data(), buf.size());
  const Status s = d.write(offset, a, (uint32_t)n);
  std::free(a);
  return s;
}

static BindRegistrar reg([](py::module_& m) {
  auto t = m.def_submodule("nvme_tier", "just-in-time drive-backed KV tier");
  t.attr("IO_ALIGNMENT") = nvt::kIoAlignment;
  t.attr("DEFAULT_BUDGET_BYTES") = nvt::kDefaultBudgetBytes;
  t.attr("DEFAULT_BYTES_PER_SECOND") = nvt::kDefaultBytesPerSecond;
  t.attr("DEFAULT_STEP_MICROSECONDS") = nvt::kDefaultStepMicroseconds;
  py::enum_<nvt::Demand>(t, "Demand")
      .value("READY", nvt::Demand::Ready)
      .value("IN_FLIGHT", nvt::Demand::InFlight)
      .value("STARTED", nvt::Demand::Started)
      .value("MISS", nvt::Demand::Miss);
  py::enum_<nvt::Confidence>(t, "Confidence")
      .value("ALL", nvt::Confidence::All)
      .value("PARTIAL", nvt::Confidence::Partial)
      .value("NONE", nvt::Confidence::None);
  py::class_<nvt::Config>(t, "Config")
      .def(py::init<>())
      .def_readwrite("budget_bytes", &nvt::Config::budget_bytes)
      .def_readwrite("base_offset", &nvt::Config::base_offset)
      .def_readwrite("block_bytes", &nvt::Config::block_bytes)
      .def_readwrite("staging_buffers", &nvt::Config::staging_buffers)
      .def_readwrite("demand_reserve", &nvt::Config::demand_reserve)
      .def_readwrite("pending_capacity", &nvt::Config::pending_capacity)
      .def_readwrite("device_bytes_per_second", &nvt::Config::device_bytes_per_second)
      .def_readwrite("step_microseconds", &nvt::Config::step_microseconds);
  py::class_<nvt::BlockDevice, std::shared_ptr<nvt::BlockDevice>>(t, "BlockDevice")
      .def("write", [](nvt::BlockDevice& d, uint64_t off, const py::bytes& b) { return device_write(d, off, b); });
  py::class_<nvt::FileDevice, nvt::BlockDevice, std::shared_ptr<nvt::FileDevice>>(t, "FileDevice")
      .def(py::init<const std::string&, uint64_t, uint32_t>(), py::arg("path"), py::arg("size_bytes"),
           py::arg("threads") = 2)
      .def_property_readonly("direct", &nvt::FileDevice::direct);
  py::class_<nvt::MockDevice, nvt::BlockDevice, std::shared_ptr<nvt::MockDevice>>(t, "MockDevice")
      .def(py::init<uint64_t, uint32_t>(), py::arg("size_bytes"), py::arg("latency_polls"))
      .def("fail_next_read", &nvt::MockDevice::fail_next_read)
      .def_property_readonly("reads", &nvt::MockDevice::reads);
  py::class_<nvt::Need>(t, "Need")
      .def(py::init([](uint64_t h, uint32_t s) { return nvt::Need{h, s}; }), py::arg("hash"), py::arg("need_by_step"))
      .def_readwrite("hash", &nvt::Need::hash)
      .def_readwrite("need_by_step", &nvt::Need::need_by_step);
  py::class_<nvt::Reservation>(t, "Reservation")
      .def_readonly("hash", &nvt::Reservation::hash)
      .def_readonly("offset", &nvt::Reservation::offset)
      .def_readonly("slot", &nvt::Reservation::slot)
      .def_readonly("generation", &nvt::Reservation::generation)
      .def_readonly("already_present", &nvt::Reservation::already_present);
  py::class_<nvt::PlanReport>(t, "PlanReport")
      .def_readonly("ready", &nvt::PlanReport::ready)
      .def_readonly("inflight", &nvt::PlanReport::inflight)
      .def_readonly("queued", &nvt::PlanReport::queued)
      .def_readonly("absent", &nvt::PlanReport::absent)
      .def_readonly("queue_full", &nvt::PlanReport::queue_full)
      .def_readonly("late_risk", &nvt::PlanReport::late_risk);
  py::class_<nvt::Residency>(t, "Residency")
      .def_readonly("confidence", &nvt::Residency::confidence)
      .def_readonly("ready", &nvt::Residency::ready)
      .def_readonly("inflight_on_time", &nvt::Residency::inflight_on_time)
      .def_readonly("planned_on_time", &nvt::Residency::planned_on_time)
      .def_readonly("late", &nvt::Residency::late)
      .def_readonly("absent", &nvt::Residency::absent);
  py::class_<nvt::Stats>(t, "Stats")
#define STAT(n) .def_readonly(#n, &nvt::Stats::n)
      STAT(write_reservations) STAT(publishes) STAT(write_aborts) STAT(evictions) STAT(pinned_skips)
      STAT(demand_hits) STAT(demand_joins) STAT(demand_loads) STAT(demand_misses) STAT(demand_stalls)
      STAT(prefetch_issues) STAT(prefetch_landings) STAT(prefetch_late) STAT(prefetch_preemptions)
      STAT(prefetch_dropped) STAT(stale_completions) STAT(io_errors) STAT(read_bytes) STAT(slot_count)
      STAT(slots_in_use);
#undef STAT
  py::class_<nvt::Tier>(t, "Tier")
      .def(py::init<const nvt::Config&, std::shared_ptr<nvt::BlockDevice>>(), py::keep_alive<1, 3>())
      .def("reserve_write", &nvt::Tier::reserve_write)
      .def("commit_write", &nvt::Tier::commit_write)
      .def("abort_write", &nvt::Tier::abort_write)
      .def("offset_of",
           [](const nvt::Tier& t, uint64_t h) -> py::object {
             uint64_t off;
             if (!t.offset_of(h, &off)) return py::none();
             return py::int_(off);
           })
      .def("plan_lookahead", &nvt::Tier::plan_lookahead)
      .def("request_demand",
           [](nvt::Tier& t, uint64_t h, uint32_t step) {
             const uint8_t* p = nullptr;
             const nvt::Demand d = t.request_demand(h, step, &p);
             py::object data = p ? py::object(py::bytes(reinterpret_cast<const char*>(p), t.config().block_bytes))
                                 : py::object(py::none());
             return py::make_tuple(d, data, reinterpret_cast<uintptr_t>(p));
           })
      .def("pump", &nvt::Tier::pump)
      .def("consume", &nvt::Tier::consume)
      .def("pin", &nvt::Tier::pin)
      .def("will_be_resident_by", &nvt::Tier::will_be_resident_by)
      .def("inflight", &nvt::Tier::inflight)
      .def("drain", &nvt::Tier::drain)
      .def_property_readonly("transfer_steps", &nvt::Tier::transfer_steps)
      .def_property_readonly("stats", &nvt::Tier::stats);
});
