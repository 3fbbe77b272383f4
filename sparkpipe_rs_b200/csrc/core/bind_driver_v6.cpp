// Bindings of the ABI-v6 stage-driver loader (submodule `driver_v6`).
#include "driver_v6.h"
#include "registry.h"

namespace py = pybind11;
using namespace spc;

namespace {

py::dict completion_dict(const v6::Completion& c) {
  py::dict d;
  d["request_id"] = c.request_id;
  d["sequence_id"] = c.sequence_id;
  d["sequence_position"] = c.sequence_position;
  d["program_id"] = c.program_id;
  d["driver_dispatch_slot"] = c.driver_dispatch_slot;
  d["accepted_token_count"] = c.accepted_token_count;
  d["completion_flags"] = c.completion_flags;
  d["token_ids"] = c.token_ids;
  d["draft_token_ids"] = c.draft_token_ids;
  d["status"] = c.status;
  d["queue_delay_ns"] = c.queue_delay_ns;
  d["service_time_ns"] = c.service_time_ns;
  d["device_memcpy_bytes"] = c.device_memcpy_bytes;
  d["host_staging_bytes"] = c.host_staging_bytes;
  return d;
}

std::string text(const char* s) { return s ? std::string(s) : std::string(); }

}  // namespace

static BindRegistrar reg([](py::module_& m) {
  auto v = m.def_submodule("driver_v6", "loader for stage drivers of the reference's model-driver ABI v6");
  v.attr("ABI_VERSION") = SP6_ABI_VERSION;
  v.attr("INTERFACE_SYMBOL") = SP6_INTERFACE_SYMBOL;
  v.attr("BUFFER_READ") = SP6_BUFFER_READ;
  v.attr("BUFFER_WRITE") = SP6_BUFFER_WRITE;
  v.attr("FRAME_PREFILL") = SP6_FRAME_PREFILL;
  v.attr("PROGRAM_EXTERNAL_COMPLETION") = SP6_PROGRAM_EXTERNAL_COMPLETION;
  v.attr("PROGRAM_NO_HOST_STAGING") = SP6_PROGRAM_NO_HOST_STAGING;
  v.attr("PROGRAM_VALIDATED_LATENCY") = SP6_PROGRAM_VALIDATED_LATENCY;
  v.def("abi_layout", &v6::abi_layout, "sizeof / offsetof of the v6 structs as laid out by this build");
  py::class_<v6::Driver>(v, "Driver")
      .def_static("load", &v6::Driver::load, py::arg("path"), py::arg("expected_target") = "")
      .def_property_readonly("model_id", [](const v6::Driver& d) { return text(d.descriptor().model_id); })
      .def_property_readonly("model_revision", [](const v6::Driver& d) { return text(d.descriptor().model_revision); })
      .def_property_readonly("stage_name", [](const v6::Driver& d) { return text(d.descriptor().stage_name); })
      .def_property_readonly("target", [](const v6::Driver& d) { return text(d.descriptor().target); })
      .def_property_readonly("model_description_sha256",
                             [](const v6::Driver& d) { return text(d.descriptor().model_description_sha256); })
      .def_property_readonly("compiled_program_sha256",
                             [](const v6::Driver& d) { return text(d.descriptor().compiled_program_sha256); })
      .def_property_readonly("module_instance_count",
                             [](const v6::Driver& d) { return d.descriptor().module_instance_count; })
      .def("programs",
           [](const v6::Driver& d) {
             py::list out;
             for (const auto& p : d.programs()) {
               py::dict x;
               x["program_id"] = p.program_id;
               x["flags"] = p.flags;
               x["max_inflight"] = p.max_inflight;
               x["name"] = p.name;
               x["max_active_slots"] = p.profile.max_active_slots;
               x["max_new_tokens"] = p.profile.max_new_tokens;
               x["validated_latency_ns"] = p.profile.validated_latency_ns;
               out.append(x);
             }
             return out;
           })
      .def("create", &v6::Driver::create, py::arg("node_id"), py::arg("node_target"), py::arg("node_context") = 0)
      .def("destroy", &v6::Driver::destroy)
      .def_property_readonly("has_instance", &v6::Driver::has_instance)
      .def(
          "admit",
          [](v6::Driver& d, uint32_t program_id, uint64_t request_id, uint64_t sequence_id, uint64_t position,
             uint64_t deadline_ns, uint32_t active_slots, uint32_t new_tokens, uint32_t priority, uint32_t frame_flags) {
            sp6_admission_request r{};
            r.program_id = program_id;
            r.request_id = request_id;
            r.sequence_id = sequence_id;
            r.sequence_position = position;
            r.deadline_time_ns = deadline_ns;
            r.active_slot_count = active_slots;
            r.new_token_count = new_tokens;
            r.priority = priority;
            r.frame_flags = frame_flags;
            const sp6_admission_decision x = d.admit(r);
            py::dict out;
            out["accepted"] = bool(x.accepted);
            out["rejection_reason"] = x.rejection_reason;
            out["driver_dispatch_slot"] = x.driver_dispatch_slot;
            out["estimated_queue_delay_ns"] = x.estimated_queue_delay_ns;
            out["estimated_service_time_ns"] = x.estimated_service_time_ns;
            out["available_dispatch_slot_count"] = x.available_dispatch_slot_count;
            out["driver_dispatch_generation"] = x.driver_dispatch_generation;
            out["driver_dispatch_cookie0"] = x.driver_dispatch_cookie0;
            out["driver_dispatch_cookie1"] = x.driver_dispatch_cookie1;
            return out;
          },
          py::arg("program_id"), py::arg("request_id") = 0, py::arg("sequence_id") = 0, py::arg("position") = 0,
          py::arg("deadline_ns") = 0, py::arg("active_slots") = 1, py::arg("new_tokens") = 1, py::arg("priority") = 0,
          py::arg("frame_flags") = 0)
      .def(
          "submit",
          [](v6::Driver& d, uint32_t program_id, uint64_t request_id, uint64_t sequence_id, uint64_t position,
             uint32_t new_tokens, const std::vector<uint64_t>& scalars,
             const std::vector<std::tuple<uint32_t, uint32_t, uint64_t, uint64_t>>& buffers, uint32_t flags,
             uint32_t active_slots, uint32_t priority, uint64_t deadline_ns, uint64_t stream,
             const py::object& dispatch) {
            if (scalars.size() > SP6_SCALARS) fail(Status::InvalidArgument, "v6 driver: at most 8 scalars");
            v6::FrameArgs a;
            a.request_id = request_id;
            a.sequence_id = sequence_id;
            a.sequence_position = position;
            a.new_token_count = new_tokens;
            a.active_slot_count = active_slots;
            a.priority = priority;
            a.deadline_time_ns = deadline_ns;
            a.flags = flags;
            a.execution_stream = stream;
            for (size_t i = 0; i < scalars.size(); ++i) a.scalar[i] = scalars[i];
            for (const auto& b : buffers)
              a.buffers.push_back(sp6_buffer{std::get<0>(b), std::get<1>(b),
                                             reinterpret_cast<void*>(uintptr_t(std::get<2>(b))), std::get<3>(b)});
            if (!dispatch.is_none()) {  // an admission decision: its slot, generation and cookies
              const py::dict x = dispatch.cast<py::dict>();
              a.driver_dispatch_slot = x["driver_dispatch_slot"].cast<uint32_t>();
              a.driver_dispatch_generation = x["driver_dispatch_generation"].cast<uint64_t>();
              a.driver_dispatch_cookie0 = x["driver_dispatch_cookie0"].cast<uint64_t>();
              a.driver_dispatch_cookie1 = x["driver_dispatch_cookie1"].cast<uint64_t>();
              a.flags |= 0x00000001u;  // the dispatch slot is valid
            }
            py::gil_scoped_release nogil;
            return uint32_t(d.submit(program_id, a));
          },
          py::arg("program_id"), py::arg("request_id"), py::arg("sequence_id") = 0, py::arg("position") = 0,
          py::arg("new_tokens") = 1, py::arg("scalars") = std::vector<uint64_t>{},
          py::arg("buffers") = std::vector<std::tuple<uint32_t, uint32_t, uint64_t, uint64_t>>{},
          py::arg("flags") = 0, py::arg("active_slots") = 1, py::arg("priority") = 0, py::arg("deadline_ns") = 0,
          py::arg("stream") = 0, py::arg("dispatch") = py::none())
      .def(
          "poll",
          [](v6::Driver& d, size_t max, int timeout_ms) {
            std::vector<v6::Completion> cs;
            {
              py::gil_scoped_release nogil;
              cs = d.poll(max, timeout_ms);
            }
            py::list out;
            for (const auto& c : cs) out.append(completion_dict(c));
            return out;
          },
          py::arg("max") = 64, py::arg("timeout_ms") = 0)
      .def("snapshot",
           [](v6::Driver& d, uint32_t program_id) {
             const sp6_runtime_snapshot s = d.snapshot(program_id);
             py::dict out;
             out["submitted_count"] = s.submitted_count;
             out["completed_count"] = s.completed_count;
             out["rejected_count"] = s.rejected_count;
             out["active_submission_count"] = s.active_submission_count;
             out["available_dispatch_slot_count"] = s.available_dispatch_slot_count;
             out["resident_sequence_count"] = s.resident_sequence_count;
             out["resident_token_count"] = s.resident_token_count;
             out["kv_token_capacity"] = s.kv_token_capacity;
             out["host_callback_completion_count"] = s.host_callback_completion_count;
             out["stale_admission_count"] = s.stale_admission_count;
             return out;
           })
      .def_property_readonly("wakes", &v6::Driver::wakes)
      .def_property_readonly("frames_in_flight", &v6::Driver::frames_in_flight);
});
