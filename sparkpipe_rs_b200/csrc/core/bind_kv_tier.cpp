// Bindings of the KV backing tier and its restore/evict work control (submodule `kv_tier`).
// Payload and staging buffers are passed as integer host addresses (e.g. a numpy
// array's .ctypes.data); the caller keeps them alive while a batch is in flight.
#include "kv_tier.h"
#include "registry.h"

#include <pybind11/stl.h>

namespace py = pybind11;
using namespace spc;

static uint8_t* addr(uint64_t a) { return reinterpret_cast<uint8_t*>(uintptr_t(a)); }

static BindRegistrar reg([](py::module_& m) {
  auto k = m.def_submodule("kv_tier", "fingerprinted KV backing tier and restore/evict work control");
  k.attr("MAX_KEY_BYTES") = kvt::kMaxKeyBytes;
  k.attr("MAX_BATCH_BLOCKS") = kvt::kMaxBatchBlocks;
  k.attr("MAX_INFLIGHT_BATCHES") = kvt::kMaxInflightBatches;
  k.attr("DEFAULT_LOOKAHEAD") = kvt::kDefaultLookahead;
  k.attr("MAX_LOOKAHEAD") = kvt::kMaxLookahead;
  k.attr("STATE_BLOCK") = kvt::kStateBlock;
  k.attr("GET") = uint32_t(kvt::Get);
  k.attr("PUT") = uint32_t(kvt::Put);
  k.attr("FREE") = uint32_t(kvt::Free);
  k.attr("IN_FLIGHT") = uint32_t(kvt::InFlight);
  k.attr("LANDED") = uint32_t(kvt::Landed);
  k.def("format_key", &kvt::format_key);
  k.def("normalize_lookahead", &kvt::normalize_lookahead);
  k.def("select_lookahead", &kvt::select_lookahead);
  py::class_<kvt::Block>(k, "Block")
      .def(py::init([](uint32_t op, std::string key, uint64_t payload, uint32_t bytes) {
             kvt::Block b;
             b.op = op;
             b.key = std::move(key);
             b.payload = addr(payload);
             b.bytes = bytes;
             return b;
           }),
           py::arg("op"), py::arg("key"), py::arg("payload"), py::arg("bytes"))
      .def_readonly("op", &kvt::Block::op)
      .def_readonly("key", &kvt::Block::key)
      .def_readonly("bytes", &kvt::Block::bytes)
      .def_property_readonly("payload", [](const kvt::Block& b) { return uint64_t(uintptr_t(b.payload)); });
  py::class_<kvt::Completion>(k, "Completion")
      .def_readonly("batch_id", &kvt::Completion::batch_id)
      .def_property_readonly("status", [](const kvt::Completion& c) { return uint32_t(c.status); })
      .def_readonly("completed_blocks", &kvt::Completion::completed_blocks);
  py::class_<kvt::Store, std::shared_ptr<kvt::Store>>(k, "Store");
  py::class_<kvt::MemoryStore, kvt::Store, std::shared_ptr<kvt::MemoryStore>>(k, "MemoryStore")
      .def(py::init<>())
      .def("stored_blocks", &kvt::MemoryStore::stored_blocks)
      .def("set_paused", &kvt::MemoryStore::set_paused);
  py::class_<kvt::StageKvClient>(k, "StageKvClient")
      .def(py::init<const std::string&, std::shared_ptr<kvt::Store>, uint32_t, uint64_t, uint64_t>(),
           py::arg("provider"), py::arg("store"), py::arg("rank"), py::arg("model_fp"), py::arg("layout_fp"))
      .def_property_readonly("enabled", &kvt::StageKvClient::enabled)
      .def_property_readonly("inflight", &kvt::StageKvClient::inflight)
      .def("submit", &kvt::StageKvClient::submit, py::call_guard<py::gil_scoped_release>())
      .def("poll", [](kvt::StageKvClient& c, uint64_t id) -> py::object {
        kvt::Completion out;
        const Status s = c.poll(id, out);
        if (s == Status::Ok) return py::cast(out);
        return py::cast(uint32_t(s));
      });
  py::class_<kvt::PlanConfig>(k, "PlanConfig")
      .def(py::init<>())
      .def_readwrite("model_fp", &kvt::PlanConfig::model_fp)
      .def_readwrite("layout_fp", &kvt::PlanConfig::layout_fp)
      .def_readwrite("rank", &kvt::PlanConfig::rank)
      .def_readwrite("block_bytes", &kvt::PlanConfig::block_bytes)
      .def_readwrite("state_bytes", &kvt::PlanConfig::state_bytes)
      .def_readwrite("lookahead", &kvt::PlanConfig::lookahead)
      .def_readwrite("physical_capacity", &kvt::PlanConfig::physical_capacity)
      .def_readwrite("allocated", &kvt::PlanConfig::allocated)
      .def_readwrite("staging_capacity", &kvt::PlanConfig::staging_capacity);
  py::class_<kvt::PendingLane>(k, "PendingLane")
      .def(py::init([](uint64_t seq, std::vector<uint32_t> blocks, bool state) {
             kvt::PendingLane l;
             l.sequence = seq;
             l.blocks = std::move(blocks);
             l.state_nonresident = state;
             return l;
           }),
           py::arg("sequence"), py::arg("blocks"), py::arg("state_nonresident") = false);
  py::enum_<kvt::Direction>(k, "Direction")
      .value("RESTORE", kvt::Direction::Restore)
      .value("EVICT", kvt::Direction::Evict);
  py::class_<kvt::Channel>(k, "Channel")
      .def_readonly("batch_id", &kvt::Channel::batch_id)
      .def_readonly("stage", &kvt::Channel::stage)
      .def_readonly("blocks", &kvt::Channel::blocks)
      .def_property_readonly("outcome", [](const kvt::Channel& ch) { return uint32_t(ch.outcome); });
  py::class_<kvt::RestoreBatch>(k, "RestoreBatch")
      .def_readonly("blocks", &kvt::RestoreBatch::blocks)
      .def_readonly("lanes_built", &kvt::RestoreBatch::lanes_built)
      .def_readonly("block_records", &kvt::RestoreBatch::block_records)
      .def_readonly("state_records", &kvt::RestoreBatch::state_records);
  k.def("state_block_equivalents", &kvt::state_block_equivalents);
  k.def("cumulative_nonresident", &kvt::cumulative_nonresident);
  py::class_<kvt::TierMover>(k, "TierMover")
      .def(py::init([](const kvt::PlanConfig& c, kvt::StageKvClient& client, uint64_t block_staging,
                       uint32_t block_records, uint64_t state_staging, uint32_t state_records,
                       uint32_t batch_blocks) {
             kvt::Staging s;
             s.blocks = addr(block_staging);
             s.block_records = block_records;
             s.states = addr(state_staging);
             s.state_records = state_records;
             s.batch_blocks = batch_blocks;
             return new kvt::TierMover(c, client, s);
           }),
           py::arg("plan"), py::arg("client"), py::arg("block_staging"), py::arg("block_records"),
           py::arg("state_staging"), py::arg("state_records"), py::arg("batch_blocks"),
           py::keep_alive<1, 3>())
      .def("restore_packets", &kvt::TierMover::restore_packets)
      .def("plan_restore", &kvt::TierMover::plan_restore)
      .def("plan_evict",
           [](const kvt::TierMover& m, uint64_t seq, const std::vector<uint32_t>& resident, bool state,
              uint64_t block_src, uint64_t state_src) {
             return m.plan_evict(seq, resident, state, addr(block_src), addr(state_src));
           })
      .def("start", &kvt::TierMover::start)
      .def("poll", &kvt::TierMover::poll)
      .def("channel", &kvt::TierMover::channel, py::return_value_policy::copy)
      .def("collect", [](kvt::TierMover& m, kvt::Direction d) { return uint32_t(m.collect(d)); })
      .def("set_pressure", &kvt::TierMover::set_pressure);
});
