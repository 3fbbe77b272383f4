// Bindings of the per-rank work daemon (submodule `rank_daemon`).
#include "rank_daemon.h"
#include "registry.h"

namespace py = pybind11;
using namespace spc;

static BindRegistrar reg([](py::module_& m) {
  auto r = m.def_submodule("rank_daemon", "idempotent pipeline work transactions");
  r.attr("IDENTITY_BYTES") = rd::kIdentityBytes;
  r.attr("ACK_BYTES") = rd::kAckBytes;
  r.attr("FINAL_EVENT_BYTES") = rd::kFinalEventBytes;
  r.attr("STATE_PREPARED") = uint32_t(rd::Prepared);
  r.attr("STATE_ACCEPTED") = uint32_t(rd::Accepted);
  r.attr("STATE_EXECUTING") = uint32_t(rd::Executing);
  r.attr("STATE_COMMITTED") = uint32_t(rd::Committed);
  r.attr("STATE_CANCELLED") = uint32_t(rd::Cancelled);
  r.attr("STATE_FAILED") = uint32_t(rd::Failed);
  r.def("identity_to_wire", [](const wc::Identity& i) { return py::bytes(rd::identity_to_wire(i)); });
  r.def("identity_from_wire", [](py::bytes b) { return rd::identity_from_wire(std::string(b)); });
  r.def("identity_fingerprint", &rd::identity_fingerprint);
  r.def("packet_dedup_hash32", [](py::bytes b) {
    std::string s(b);
    return rd::packet_dedup_hash32(reinterpret_cast<const uint8_t*>(s.data()), s.size());
  });
  py::class_<rd::Ack>(r, "Ack")
      .def(py::init<>())
      .def_readwrite("status", &rd::Ack::status)
      .def_readwrite("state", &rd::Ack::state)
      .def_readwrite("identity", &rd::Ack::identity)
      .def_readwrite("packet_fingerprint", &rd::Ack::packet_fingerprint);
  r.def("ack_to_wire", [](const rd::Ack& a) { return py::bytes(rd::ack_to_wire(a)); });
  r.def("ack_from_wire", [](py::bytes b) { return rd::ack_from_wire(std::string(b)); });
  py::class_<rd::FinalEvent>(r, "FinalEvent")
      .def(py::init<>())
      .def_readwrite("status", &rd::FinalEvent::status)
      .def_readwrite("program_id", &rd::FinalEvent::program_id)
      .def_readwrite("accepted_token_count", &rd::FinalEvent::accepted_token_count)
      .def_readwrite("token_ids", &rd::FinalEvent::token_ids)
      .def_readwrite("draft_token_ids", &rd::FinalEvent::draft_token_ids)
      .def_readwrite("request_id", &rd::FinalEvent::request_id)
      .def_readwrite("sequence_id", &rd::FinalEvent::sequence_id)
      .def_readwrite("sequence_position", &rd::FinalEvent::sequence_position)
      .def_readwrite("service_time_ns", &rd::FinalEvent::service_time_ns)
      .def_readwrite("identity", &rd::FinalEvent::identity);
  r.def("final_event_to_wire", [](const rd::FinalEvent& e) { return py::bytes(rd::final_event_to_wire(e)); });
  r.def("final_event_from_wire", [](py::bytes b) { return rd::final_event_from_wire(std::string(b)); });
  py::enum_<rd::Observation>(r, "Observation")
      .value("NEW", rd::Observation::New)
      .value("REPLAY_ACTIVE", rd::Observation::ReplayActive)
      .value("REPLAY_TERMINAL", rd::Observation::ReplayTerminal)
      .value("CONFLICT", rd::Observation::Conflict);
  py::class_<rd::LedgerEntry>(r, "LedgerEntry")
      .def_readonly("identity", &rd::LedgerEntry::identity)
      .def_readonly("payload_fingerprint", &rd::LedgerEntry::payload_fingerprint)
      .def_readonly("state", &rd::LedgerEntry::state)
      .def_readonly("terminal_status", &rd::LedgerEntry::terminal_status);
  py::class_<rd::TransactionLedger>(r, "TransactionLedger")
      .def(py::init<uint32_t>())
      .def("observe", &rd::TransactionLedger::observe)
      .def("transition", &rd::TransactionLedger::transition, py::arg("identity"), py::arg("target"),
           py::arg("terminal_status") = Status::Ok)
      .def("find", [](const rd::TransactionLedger& l, const wc::Identity& i) -> py::object {
        const rd::LedgerEntry* e = l.find(i);
        if (!e) return py::none();
        return py::cast(*e);
      })
      .def_property_readonly("entries", &rd::TransactionLedger::entries)
      .def_property_readonly("active", &rd::TransactionLedger::active)
      .def_property_readonly("terminal", &rd::TransactionLedger::terminal)
      .def_property_readonly("tombstones", &rd::TransactionLedger::tombstones)
      .def_property_readonly("control_generation", &rd::TransactionLedger::control_generation)
      .def_property_readonly("capacity", &rd::TransactionLedger::capacity);
  py::class_<rd::DaemonConfig>(r, "DaemonConfig")
      .def(py::init<>())
      .def_readwrite("rank", &rd::DaemonConfig::rank)
      .def_readwrite("world", &rd::DaemonConfig::world)
      .def_readwrite("queue_capacity", &rd::DaemonConfig::queue_capacity)
      .def_readwrite("ledger_capacity", &rd::DaemonConfig::ledger_capacity)
      .def_readwrite("dedup_window", &rd::DaemonConfig::dedup_window)
      .def_readwrite("work", &rd::DaemonConfig::work);
  py::class_<rd::DaemonStats>(r, "DaemonStats")
      .def_readonly("submitted", &rd::DaemonStats::submitted)
      .def_readonly("accepted", &rd::DaemonStats::accepted)
      .def_readonly("duplicates", &rd::DaemonStats::duplicates)
      .def_readonly("conflicts", &rd::DaemonStats::conflicts)
      .def_readonly("rejected", &rd::DaemonStats::rejected)
      .def_readonly("forwarded", &rd::DaemonStats::forwarded)
      .def_readonly("executed", &rd::DaemonStats::executed)
      .def_readonly("committed", &rd::DaemonStats::committed)
      .def_readonly("failed", &rd::DaemonStats::failed)
      .def_readonly("cancelled", &rd::DaemonStats::cancelled)
      .def_readonly("final_events", &rd::DaemonStats::final_events)
      .def_readonly("queued", &rd::DaemonStats::queued)
      .def_readonly("inflight", &rd::DaemonStats::inflight);
  py::class_<rd::RankDaemon>(r, "RankDaemon")
      .def(py::init([](const rd::DaemonConfig& c, py::object fwd, py::object exe, py::object fin) {
             auto wrap = [](py::object f) -> std::function<void(const std::string&)> {
               if (f.is_none()) return nullptr;
               return [f](const std::string& b) {
                 py::gil_scoped_acquire g;
                 f(py::bytes(b));
               };
             };
             return new rd::RankDaemon(c, wrap(fwd), wrap(exe), wrap(fin));
           }),
           py::arg("config"), py::arg("forward") = py::none(), py::arg("execute") = py::none(),
           py::arg("final_event") = py::none())
      .def("submit", [](rd::RankDaemon& d, py::bytes b) { return py::bytes(d.submit(std::string(b))); })
      .def("pump", &rd::RankDaemon::pump, py::arg("max_packets") = 64)
      .def("complete", &rd::RankDaemon::complete, py::arg("identity"), py::arg("status") = Status::Ok,
           py::arg("tokens") = std::vector<uint32_t>{}, py::arg("service_time_ns") = 0)
      .def("complete_lanes", &rd::RankDaemon::complete_lanes, py::arg("identity"), py::arg("status"),
           py::arg("lane_tokens"), py::arg("service_time_ns") = 0)
      .def("cancel", &rd::RankDaemon::cancel)
      .def_property_readonly("ledger", &rd::RankDaemon::ledger, py::return_value_policy::reference_internal)
      .def("stats", &rd::RankDaemon::stats);
});
