// Bindings of the work-control plane (packets, identity, MTP tree, KV directory).
#include <pybind11/numpy.h>

#include <cstring>
#include <stdexcept>

#include "registry.h"
#include "work_control.h"

namespace py = pybind11;
using namespace spc;

namespace {
template <typename T>
py::array_t<T> np_copy(const std::vector<T>& v) {
  py::array_t<T> a((py::ssize_t)v.size());
  if (!v.empty()) std::memcpy(a.mutable_data(), v.data(), v.size() * sizeof(T));
  return a;
}
}  // namespace

static BindRegistrar reg([](py::module_& m) {
  auto w = m.def_submodule("work_control", "work packets, transaction identity, MTP tree, KV directory");
  w.attr("ABI_VERSION") = wc::kAbiVersion;
  w.attr("PACKET_MAGIC") = wc::kPacketMagic;
  w.attr("PHASE_PREFILL") = wc::kPhasePrefill;
  w.attr("PHASE_DECODE") = wc::kPhaseDecode;
  w.attr("PHASE_VERIFY") = wc::kPhaseVerify;
  w.attr("PHASE_RELEASE") = wc::kPhaseRelease;
  w.attr("PHASE_CANCEL") = wc::kPhaseCancel;
  w.attr("FLAG_PREFILL") = wc::kFlagPrefill;
  w.attr("FLAG_MTP_TREE_VERIFY") = wc::kFlagMtpTreeVerify;
  w.def("fingerprint_bytes", [](py::bytes b) {
    std::string s = b;
    return wc::fingerprint_bytes(reinterpret_cast<const uint8_t*>(s.data()), s.size());
  });
  w.def("queue_depth", [](uint32_t c) { return wc::queue_depth(c); });
  w.def("select_batch_bucket", &wc::select_batch_bucket);
  w.def("execution_chunk_shape", &wc::execution_chunk_shape);
  py::class_<wc::Identity>(w, "Identity")
      .def(py::init<>())
      .def_readwrite("control_generation", &wc::Identity::control_generation)
      .def_readwrite("transaction_id", &wc::Identity::transaction_id)
      .def_readwrite("dispatch_generation", &wc::Identity::dispatch_generation)
      .def_readwrite("request_generation", &wc::Identity::request_generation)
      .def_readwrite("step_generation", &wc::Identity::step_generation)
      .def_readwrite("step_chunk_index", &wc::Identity::step_chunk_index)
      .def_readwrite("step_chunk_count", &wc::Identity::step_chunk_count)
      .def_readwrite("transaction_phase", &wc::Identity::transaction_phase);
  w.def("validate_identity", &wc::validate_identity);
  py::class_<wc::Config>(w, "Config")
      .def(py::init<>())
      .def_readwrite("mtp_draft_token_count", &wc::Config::mtp_draft_token_count)
      .def_readwrite("max_speculative_token_count", &wc::Config::max_speculative_token_count)
      .def_readwrite("maximum_context_tokens", &wc::Config::maximum_context_tokens)
      .def_readwrite("kv_block_tokens", &wc::Config::kv_block_tokens)
      .def_readwrite("max_prefill_tokens_per_packet", &wc::Config::max_prefill_tokens_per_packet)
      .def_readwrite("output_vocab_count", &wc::Config::output_vocab_count)
      .def_readwrite("max_lane_count", &wc::Config::max_lane_count)
      .def_readwrite("cohort_capacity", &wc::Config::cohort_capacity)
      .def("validate", &wc::Config::validate);
  py::class_<wc::Lane>(w, "Lane")
      .def(py::init<>())
      .def_readwrite("request_id", &wc::Lane::request_id)
      .def_readwrite("sequence_id", &wc::Lane::sequence_id)
      .def_readwrite("sequence_position", &wc::Lane::sequence_position)
      .def_readwrite("context_token_count", &wc::Lane::context_token_count)
      .def_readwrite("input_token_id", &wc::Lane::input_token_id)
      .def_readwrite("speculative_token_count", &wc::Lane::speculative_token_count)
      .def_readwrite("speculative_draft_token_ids", &wc::Lane::speculative_draft_token_ids)
      .def_readwrite("mtp_proposed", &wc::Lane::mtp_proposed)
      .def_readwrite("mtp_accepted", &wc::Lane::mtp_accepted)
      .def_readwrite("mtp_path_id", &wc::Lane::mtp_path_id);
  w.attr("FLAG_EXECUTION_PAYLOAD") = wc::kFlagExecutionPayload;
  w.attr("FLAG_PREFILL") = wc::kFlagPrefill;
  py::class_<wc::ExecPayload>(w, "ExecPayload")
      .def_property_readonly("positions", [](const wc::ExecPayload& e) { return np_copy(e.positions); })
      .def_property_readonly("slots", [](const wc::ExecPayload& e) { return np_copy(e.slots); })
      .def_property_readonly("block_table", [](const wc::ExecPayload& e) { return np_copy(e.block_table); })
      .def_property_readonly("context_lens", [](const wc::ExecPayload& e) { return np_copy(e.context_lens); })
      .def_readonly("block_table_cols", &wc::ExecPayload::block_table_cols)
      .def_property_readonly("cu_q", [](const wc::ExecPayload& e) { return np_copy(e.cu_q); })
      .def_property_readonly("cu_k", [](const wc::ExecPayload& e) { return np_copy(e.cu_k); })
      .def_property_readonly("ctx_slots", [](const wc::ExecPayload& e) { return np_copy(e.ctx_slots); })
      .def_property_readonly("logits_rows", [](const wc::ExecPayload& e) { return np_copy(e.logits_rows); })
      .def_readonly("max_q", &wc::ExecPayload::max_q)
      .def_property_readonly("temperature", [](const wc::ExecPayload& e) { return np_copy(e.temperature); })
      .def_property_readonly("sample_keys", [](const wc::ExecPayload& e) {
        py::array_t<int64_t> a((py::ssize_t)e.sample_keys.size());
        if (!e.sample_keys.empty()) std::memcpy(a.mutable_data(), e.sample_keys.data(), e.sample_keys.size() * 8);
        return a;
      });
  py::class_<wc::Packet>(w, "Packet")
      .def(py::init<>())
      .def_readonly("exec", &wc::Packet::exec)
      .def_property_readonly("input_token_ids", [](const wc::Packet& p) {
        std::vector<int32_t> v;
        for (const auto& l : p.lanes) v.push_back(int32_t(l.input_token_id));
        return np_copy(v);
      })
      .def_property_readonly("prefill_tokens", [](const wc::Packet& p) {
        std::vector<int32_t> v(p.prefill_token_ids.begin(), p.prefill_token_ids.end());
        return np_copy(v);
      })
      .def_property_readonly("sequence_ids", [](const wc::Packet& p) {
        std::vector<int64_t> v;
        for (const auto& l : p.lanes) v.push_back(int64_t(l.sequence_id));
        return np_copy(v);
      })
      .def_readwrite("flags", &wc::Packet::flags)
      .def_readwrite("identity", &wc::Packet::identity)
      .def_readwrite("active_sequence_count", &wc::Packet::active_sequence_count)
      .def_readwrite("new_token_count", &wc::Packet::new_token_count)
      .def_readwrite("block_token_count", &wc::Packet::block_token_count)
      .def_readwrite("execution_row_count", &wc::Packet::execution_row_count)
      .def_readwrite("execution_batch_bucket", &wc::Packet::execution_batch_bucket)
      .def_readwrite("prefill_token_ids", &wc::Packet::prefill_token_ids)
      .def_readwrite("lanes", &wc::Packet::lanes)
      .def("serialize", [](const wc::Packet& p) {
        auto b = wc::serialize(p);
        return py::bytes(reinterpret_cast<const char*>(b.data()), b.size());
      })
      .def("fingerprint", &wc::fingerprint);
  w.def("deserialize", [](py::bytes b) {
    std::string s = b;
    return wc::deserialize(reinterpret_cast<const uint8_t*>(s.data()), s.size());
  });
  w.def("validate_packet", &wc::validate_packet);
  w.def("build_step_packet", &wc::build_step_packet);
  // serialized micro-batch packets of one step (what the rank daemons consume)
  w.def("build_stage_packets",
        [](const StepPlan& plan, const wc::Identity& base, const wc::Config& cfg, uint32_t chunks, py::object temps,
           py::object keys) {
          py::array_t<float, py::array::c_style | py::array::forcecast> ta;
          py::array_t<int64_t, py::array::c_style | py::array::forcecast> ka;
          const float* tp = nullptr;
          const uint64_t* kp = nullptr;
          if (!temps.is_none()) {
            ta = temps.cast<decltype(ta)>();
            if (ta.size() < plan.num_seqs) throw std::invalid_argument("temperatures shorter than the lanes");
            tp = ta.data();
          }
          if (!keys.is_none()) {
            ka = keys.cast<decltype(ka)>();
            if (ka.size() < plan.num_seqs) throw std::invalid_argument("keys shorter than the lanes");
            kp = reinterpret_cast<const uint64_t*>(ka.data());
          }
          py::list out;
          for (const auto& p : wc::build_stage_packets(plan, base, cfg, chunks, tp, kp)) {
            auto b = wc::serialize(p);
            out.append(py::bytes(reinterpret_cast<const char*>(b.data()), b.size()));
          }
          return out;
        },
        py::arg("plan"), py::arg("base"), py::arg("config"), py::arg("chunks"), py::arg("temps") = py::none(),
        py::arg("keys") = py::none());
  auto mt = w.def_submodule("mtp_tree");
  mt.attr("CANDIDATE_COUNT") = wc::mtp::kCandidates;
  mt.attr("VERIFIER_ROW_COUNT") = wc::mtp::kVerifierRows;
  mt.def("accepted_token_count", &wc::mtp::accepted_token_count);
  mt.def("fallback_row_index", &wc::mtp::fallback_row_index);
  mt.def("tail_candidate_index", &wc::mtp::tail_candidate_index);
  mt.def("tail_parent_row_index", &wc::mtp::tail_parent_row_index);
  mt.def("tail_base_position_offset", &wc::mtp::tail_base_position_offset);
  mt.def("resolution_is_valid", &wc::mtp::resolution_is_valid);
  mt.def("topology_is_valid", &wc::mtp::topology_is_valid);
  mt.def("resolve", [](const std::vector<uint32_t>& cand, const std::vector<uint32_t>& ver, uint32_t vocab) {
    if (cand.size() != wc::mtp::kCandidates || ver.size() != wc::mtp::kVerifierRows)
      fail(Status::InvalidArgument, "mtp resolve: 5 candidates and 6 verifier tokens");
    auto r = wc::mtp::resolve(cand.data(), ver.data(), vocab);
    return py::make_tuple(r.path_id, r.accepted_token_count, r.committed_token_count, r.fallback_row_index);
  });
  py::enum_<wc::KvEntryState>(w, "KvEntryState")
      .value("MISSING", wc::KvEntryState::Missing)
      .value("IN_FLIGHT", wc::KvEntryState::InFlight)
      .value("RESIDENT", wc::KvEntryState::Resident)
      .value("TRANSIENT", wc::KvEntryState::Transient);
  py::class_<wc::KvDirectory>(w, "KvDirectory")
      .def(py::init<uint32_t, uint32_t>())
      .def("acquire", [](wc::KvDirectory& d, uint64_t seq, uint32_t blk, uint64_t content) {
        bool hit = false;
        const uint32_t b = d.acquire(wc::KvKey{seq, blk}, content, &hit);
        return py::make_tuple(b, hit);
      }, py::arg("sequence_id"), py::arg("logical_block"), py::arg("content_key") = 0)
      .def("find", [](const wc::KvDirectory& d, uint64_t seq, uint32_t blk) -> py::object {
        const auto* e = d.find(wc::KvKey{seq, blk});
        if (!e) return py::none();
        return py::make_tuple(e->physical_block, e->state, e->pins);
      })
      .def("mark_resident", [](wc::KvDirectory& d, uint64_t s, uint32_t b) { d.mark_resident({s, b}); })
      .def("mark_in_flight", [](wc::KvDirectory& d, uint64_t s, uint32_t b) { d.mark_in_flight({s, b}); })
      .def("pin", [](wc::KvDirectory& d, uint64_t s, uint32_t b) { d.pin({s, b}); })
      .def("unpin", [](wc::KvDirectory& d, uint64_t s, uint32_t b) { d.unpin({s, b}); })
      .def("release_sequence", &wc::KvDirectory::release_sequence)
      .def("reset", &wc::KvDirectory::reset)
      .def_property_readonly("generation", &wc::KvDirectory::generation)
      .def_property_readonly("live_entries", &wc::KvDirectory::live_entries)
      .def_property_readonly("free_blocks", &wc::KvDirectory::free_blocks)
      .def_property_readonly("sweeps", &wc::KvDirectory::sweeps)
      .def_property_readonly("shared_hits", &wc::KvDirectory::shared_hits);
});
