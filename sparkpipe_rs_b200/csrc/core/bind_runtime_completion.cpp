// Bindings of runtime completion (submodule `runtime_completion`): credit ledger,
// final event queue, transmission window and the transaction controller whose
// participants are Python callables.
#include "registry.h"
#include "runtime_completion.h"

#include <pybind11/stl.h>

namespace py = pybind11;
using namespace spc;

namespace {
rc::Participant participant_from(py::handle o) {
  rc::Participant p;
  p.name = py::cast<std::string>(o.attr("name"));
  if (py::hasattr(o, "flags")) p.flags = py::cast<uint32_t>(o.attr("flags"));
  if (py::hasattr(o, "restart_epoch")) p.restart_epoch = py::cast<uint64_t>(o.attr("restart_epoch"));
  py::object prep = o.attr("prepare"), exec = o.attr("execute"), commit = o.attr("commit"), cancel = o.attr("cancel");
  // called with the GIL held: the controller runs from Python
  p.prepare = [prep](const rc::Request& r) { return Status(py::cast<uint32_t>(prep(r))); };
  p.execute = [exec](const rc::Request& r) { return Status(py::cast<uint32_t>(exec(r))); };
  p.commit = [commit](const rc::Request& r) { commit(r); };
  p.cancel = [cancel](const rc::Request& r, Status s) { cancel(r, uint32_t(s)); };
  return p;
}
std::array<uint32_t, rc::kCreditDomains> credits_from(const std::vector<uint32_t>& v) {
  if (v.size() != rc::kCreditDomains) throw std::invalid_argument("four credit capacities");
  return {v[0], v[1], v[2], v[3]};
}
}  // namespace

static BindRegistrar reg([](py::module_& m) {
  auto c = m.def_submodule("runtime_completion", "transaction controller, final events, transmission window, credits");
  c.attr("MAX_PARTICIPANTS") = rc::kMaxParticipants;
  c.attr("DOMAIN_TRANSPORT_WINDOW") = uint32_t(rc::TransportWindow);
  c.attr("DOMAIN_RESIDENT_RESERVATION") = uint32_t(rc::ResidentReservation);
  c.attr("DOMAIN_EXECUTION") = uint32_t(rc::Execution);
  c.attr("DOMAIN_COMPLETION_OWNERSHIP") = uint32_t(rc::CompletionOwnership);
  c.attr("FLAG_TRANSACTIONAL_STAGING") = rc::kFlagTransactionalStaging;
  c.attr("FLAG_COMMIT_INFALLIBLE") = rc::kFlagCommitInfallible;
  c.attr("FLAG_CANCEL_IDEMPOTENT") = rc::kFlagCancelIdempotent;
  c.attr("REQUIRED_FLAGS") = rc::kRequiredFlags;
  c.attr("SLOT_FREE") = uint32_t(rc::SlotFree);
  c.attr("SLOT_RESERVED") = uint32_t(rc::SlotReserved);
  c.attr("SLOT_SENT") = uint32_t(rc::SlotSent);

  py::class_<rc::CreditLedger>(c, "CreditLedger")
      .def(py::init([](const std::vector<uint32_t>& caps) { return rc::CreditLedger(credits_from(caps)); }))
      .def("acquire", &rc::CreditLedger::acquire)
      .def("release", &rc::CreditLedger::release)
      .def("available", &rc::CreditLedger::available)
      .def("in_use", &rc::CreditLedger::in_use)
      .def("capacity", &rc::CreditLedger::capacity);

  py::class_<rc::FinalEvent>(c, "FinalEvent")
      .def(py::init<>())
      .def_readwrite("state", &rc::FinalEvent::state)
      .def_readwrite("generation", &rc::FinalEvent::generation)
      .def_readwrite("identity", &rc::FinalEvent::identity)
      .def_readwrite("payload_fingerprint", &rc::FinalEvent::payload_fingerprint)
      .def_readwrite("request_id", &rc::FinalEvent::request_id)
      .def_readwrite("sequence_id", &rc::FinalEvent::sequence_id)
      .def_readwrite("sequence_position", &rc::FinalEvent::sequence_position)
      .def_readwrite("status", &rc::FinalEvent::status);
  py::class_<rc::FinalEventQueue>(c, "FinalEventQueue")
      .def(py::init<uint32_t>())
      .def("push", &rc::FinalEventQueue::push)
      .def("peek", [](const rc::FinalEventQueue& q) -> py::object {
        const rc::FinalEvent* e = q.peek();
        return e ? py::cast(*e) : py::none();
      })
      .def("acknowledge", &rc::FinalEventQueue::acknowledge)
      .def_property_readonly("pending", &rc::FinalEventQueue::pending)
      .def_property_readonly("capacity", &rc::FinalEventQueue::capacity);

  py::class_<rc::TransmissionSlot>(c, "TransmissionSlot")
      .def_readonly("state", &rc::TransmissionSlot::state)
      .def_readonly("slot_index", &rc::TransmissionSlot::slot_index)
      .def_readonly("generation", &rc::TransmissionSlot::generation)
      .def_readonly("identity", &rc::TransmissionSlot::identity)
      .def_readonly("payload_fingerprint", &rc::TransmissionSlot::payload_fingerprint)
      .def_readonly("last_send_epoch", &rc::TransmissionSlot::last_send_epoch)
      .def_readonly("retry_count", &rc::TransmissionSlot::retry_count);
  py::class_<rc::TransmissionWindow>(c, "TransmissionWindow")
      .def(py::init<uint32_t>())
      .def("reserve", &rc::TransmissionWindow::reserve)
      .def("mark_sent", &rc::TransmissionWindow::mark_sent)
      .def("acknowledge", &rc::TransmissionWindow::acknowledge)
      .def("next_replay", [](const rc::TransmissionWindow& w) -> py::object {
        uint32_t s;
        uint64_t g;
        if (!w.next_replay(&s, &g)) return py::none();
        return py::make_tuple(s, g);
      })
      .def("slot", &rc::TransmissionWindow::slot, py::return_value_policy::copy)
      .def_property_readonly("in_use", &rc::TransmissionWindow::in_use)
      .def_property_readonly("capacity", &rc::TransmissionWindow::capacity);

  py::class_<rc::Request>(c, "Request")
      .def(py::init<>())
      .def_readwrite("identity", &rc::Request::identity)
      .def_readwrite("request_id", &rc::Request::request_id)
      .def_readwrite("sequence_id", &rc::Request::sequence_id)
      .def_readwrite("sequence_position", &rc::Request::sequence_position)
      .def_property(
          "payload", [](const rc::Request& r) { return py::bytes(r.payload); },
          [](rc::Request& r, py::bytes b) { r.payload = std::string(b); });
  py::class_<rc::Result>(c, "Result")
      .def_readonly("replayed", &rc::Result::replayed)
      .def_readonly("committed", &rc::Result::committed)
      .def_readonly("cancelled", &rc::Result::cancelled)
      .def_readonly("payload_fingerprint", &rc::Result::payload_fingerprint)
      .def_readonly("final_event_generation", &rc::Result::final_event_generation)
      .def_readonly("status", &rc::Result::status);
  py::class_<rc::Controller>(c, "Controller")
      .def(py::init([](py::list participants, uint32_t transaction_capacity, uint32_t final_event_capacity,
                       const std::vector<uint32_t>& credits) {
             std::vector<rc::Participant> ps;
             for (auto o : participants) ps.push_back(participant_from(o));
             return new rc::Controller(std::move(ps), transaction_capacity, final_event_capacity, credits_from(credits));
           }),
           py::arg("participants"), py::arg("transaction_capacity") = 1024, py::arg("final_event_capacity") = 64,
           py::arg("credits") = std::vector<uint32_t>{64, 64, 8, 64})
      .def("validate", &rc::Controller::validate)
      .def("run", &rc::Controller::run)
      .def("acknowledge_final_event", &rc::Controller::acknowledge_final_event)
      .def("peek_final_event", [](const rc::Controller& ctl) -> py::object {
        const rc::FinalEvent* e = ctl.final_events().peek();
        return e ? py::cast(*e) : py::none();
      })
      .def_property_readonly("pending_final_events", [](const rc::Controller& ctl) { return ctl.final_events().pending(); })
      .def("credits_available", [](const rc::Controller& ctl, uint32_t d) { return ctl.credits().available(d); })
      .def("ledger_state", [](const rc::Controller& ctl, const wc::Identity& id) -> py::object {
        const rd::LedgerEntry* e = ctl.ledger().find(id);
        return e ? py::cast(e->state) : py::none();
      })
      .def_property_readonly("participant_count", &rc::Controller::participant_count);
});
