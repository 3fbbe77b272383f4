// Bindings of the stage-module services (submodule `stage_module`). Device
// pointers cross as integers; the CUDA allocator is implemented in Python on the
// kernels extension's raw allocation calls (core/stage_module.py).
#include "registry.h"
#include "stage_module.h"

#include <pybind11/stl.h>

namespace py = pybind11;
using namespace spc;

namespace {
struct PyAllocator : stm::Allocator {
  Status allocate(uint64_t bytes, void** ptr) override {
    py::gil_scoped_acquire g;
    py::function f = py::get_override(static_cast<const stm::Allocator*>(this), "allocate");
    if (!f) return Status::Unsupported;
    const uint64_t p = f(bytes).cast<uint64_t>();
    *ptr = reinterpret_cast<void*>(uintptr_t(p));
    return p ? Status::Ok : Status::CapacityExceeded;
  }
  void release(void* ptr) override {
    py::gil_scoped_acquire g;
    py::function f = py::get_override(static_cast<const stm::Allocator*>(this), "release");
    if (f) f(uint64_t(reinterpret_cast<uintptr_t>(ptr)));
  }
  Status zero(void* ptr, uint64_t bytes) override {
    py::gil_scoped_acquire g;
    py::function f = py::get_override(static_cast<const stm::Allocator*>(this), "zero");
    if (!f) return Status::Unsupported;
    return f(uint64_t(reinterpret_cast<uintptr_t>(ptr)), bytes).cast<Status>();
  }
  Status copy_from_host(void* dst, const void* src, uint64_t bytes) override {
    py::gil_scoped_acquire g;
    py::function f = py::get_override(static_cast<const stm::Allocator*>(this), "copy_from_host");
    if (!f) return Status::Unsupported;
    return f(uint64_t(reinterpret_cast<uintptr_t>(dst)), uint64_t(reinterpret_cast<uintptr_t>(src)), bytes)
        .cast<Status>();
  }
};

std::FILE* open_pack(const std::string& path) {
  std::FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) fail(Status::IoError, "stage module: cannot open pack " + path);
  return f;
}
}  // namespace

static BindRegistrar reg([](py::module_& m) {
  auto s = m.def_submodule("stage_module", "stage-module services: device ledger, pack regions, slot claims");
  s.attr("MAX_DEVICE_ALLOCATIONS") = stm::kMaxDeviceAllocations;
  s.attr("STAGING_CHUNK_BYTES") = stm::kStagingChunkBytes;
  s.attr("QUIESCE_TIMEOUT_NS") = stm::kQuiesceTimeoutNs;
  py::class_<stm::Allocator, PyAllocator, std::shared_ptr<stm::Allocator>>(s, "Allocator").def(py::init<>());
  py::class_<stm::HostAllocator, stm::Allocator, std::shared_ptr<stm::HostAllocator>>(s, "HostAllocator")
      .def(py::init<>());
  py::class_<stm::DeviceLedger>(s, "DeviceLedger")
      .def(py::init<std::string, std::shared_ptr<stm::Allocator>>(), py::keep_alive<1, 3>())
      .def("allocate",
           [](stm::DeviceLedger& l, uint64_t bytes, bool zeroed) {
             return uint64_t(reinterpret_cast<uintptr_t>(l.allocate(bytes, zeroed)));
           },
           py::arg("bytes"), py::arg("zeroed") = false)
      .def("rollback", &stm::DeviceLedger::rollback)
      .def("release_all", &stm::DeviceLedger::release_all)
      .def_property_readonly("count", &stm::DeviceLedger::count)
      .def_property_readonly("bytes_resident", &stm::DeviceLedger::bytes_resident)
      .def_property_readonly("tag", &stm::DeviceLedger::tag);
  s.def("pack_read", [](const std::string& path, uint64_t offset, uint64_t bytes) {
    std::FILE* f = open_pack(path);
    std::string buf(bytes, '\0');
    try {
      stm::pack_read(path, f, offset, buf.data(), bytes);
    } catch (...) {
      std::fclose(f);
      throw;
    }
    std::fclose(f);
    return py::bytes(buf);
  });
  s.def("load_device_region", [](stm::DeviceLedger& l, const std::string& path, uint64_t offset, uint64_t bytes) {
    std::FILE* f = open_pack(path);
    void* p = nullptr;
    try {
      p = stm::load_device_region(l, f, offset, bytes);
    } catch (...) {
      std::fclose(f);
      throw;
    }
    std::fclose(f);
    return uint64_t(reinterpret_cast<uintptr_t>(p));
  });
  py::class_<stm::SlotTable>(s, "SlotTable")
      .def(py::init<uint32_t>())
      .def("claim",
           [](stm::SlotTable& t) -> py::object {
             uint32_t i;
             if (!t.claim(&i)) return py::none();
             return py::int_(i);
           })
      .def("release", &stm::SlotTable::release)
      .def("claim_set", &stm::SlotTable::claim_set)
      .def("release_set", &stm::SlotTable::release_set)
      .def("claimed", &stm::SlotTable::claimed)
      .def_property_readonly("free_count", &stm::SlotTable::free_count)
      .def_property_readonly("size", &stm::SlotTable::size)
      .def("wait_all_free", &stm::SlotTable::wait_all_free, py::arg("timeout_ns") = stm::kQuiesceTimeoutNs,
           py::call_guard<py::gil_scoped_release>())
      .def("admit", [](const stm::SlotTable& t, uint32_t sequences) {
        // the driver ABI's admission record: how many of the requested sequences the free slots take
        return std::min(sequences, t.free_count());
      });
  s.def("env_text", &stm::env_text);
  s.def("env_unsigned", &stm::env_unsigned);
});
