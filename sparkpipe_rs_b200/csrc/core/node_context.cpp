#include "node_context.h"

#include <cstring>

namespace spc {
namespace nc {

std::unique_ptr<NodeContext> NodeContext::build(const NodeContextConfig& cfg) {
  cfg.work.validate();
  if (!cfg.output_capacity) fail(Status::InvalidArgument, "node context: zero output capacity");
  const ring::RankPlan& p = cfg.plan;
  if (!p.layer_count || !p.execution_row_capacity || p.host.empty())
    fail(Status::InvalidArgument, "node context: the rank plan is not built");
  const bool has_next = p.flags & ring::kFlagHasNext;
  if (has_next != p.has_output_endpoint) fail(Status::InvalidArgument, "node context: next-rank flags disagree");
  if (p.has_output_endpoint) ring::validate_endpoint(p.output_endpoint);
  std::unique_ptr<NodeContext> ctx(new NodeContext(cfg));
  ctx->driver_.reset(ModelDriver::load(cfg.driver_path, cfg.target));
  DriverProgramInfo pi;
  if (!ctx->driver_->find_program(cfg.prefill_program, &pi))
    fail(Status::RouteNotFound, "node context: driver has no program " + cfg.prefill_program);
  ctx->prefill_id_ = pi.program_id;
  if (!ctx->driver_->find_program(cfg.decode_program, &pi))
    fail(Status::RouteNotFound, "node context: driver has no program " + cfg.decode_program);
  ctx->decode_id_ = pi.program_id;
  ctx->driver_->create(cfg.driver_config_json);
  if (has_next)
    ctx->out_.reset(new wo::WorkOutput(cfg.work, true, p.next_host, p.next_port, p.execution_row_capacity,
                                       cfg.queue_capacity, cfg.release_capacity));
  return ctx;
}

WorkResult NodeContext::submit_work(const wc::Packet& pk) {
  wc::validate_packet(pk, cfg_.work);
  if (pk.execution_row_count > cfg_.plan.execution_row_capacity)
    fail(Status::InvalidArgument, "node context: packet exceeds the rank's execution rows");
  const uint32_t phase = pk.identity.transaction_phase;
  if (phase != wc::kPhasePrefill && phase != wc::kPhaseDecode && phase != wc::kPhaseVerify)
    fail(Status::InvalidArgument, "node context: not a prefill, decode or verify packet");
  WorkResult r;
  if (out_) {  // forward first: the next stage starts on this packet while this one computes
    out_->enqueue(pk);
    r.forwarded = true;
  }
  const std::vector<uint8_t> wire = wc::serialize(pk);
  const uint32_t program = phase == wc::kPhasePrefill ? prefill_id_ : decode_id_;
  r.output = driver_->submit(program, std::string(reinterpret_cast<const char*>(wire.data()), wire.size()),
                             cfg_.output_capacity);
  ++submitted_;
  if (cfg_.plan.flags & ring::kFlagFinalStage) {
    r.final_stage = true;
    if (r.output.size() % 4) fail(Status::InvalidArgument, "node context: final-stage output is not u32 token ids");
    rd::FinalEvent& e = r.final_event;
    const size_t n = r.output.size() / 4;
    if (n > rd::kMaxFinalTokens) fail(Status::CapacityExceeded, "node context: more tokens than a final event holds");
    for (size_t i = 0; i < n; ++i) {
      uint32_t t;
      std::memcpy(&t, r.output.data() + 4 * i, 4);
      e.token_ids.push_back(t);
    }
    e.status = uint32_t(Status::Ok);
    e.accepted_token_count = uint32_t(n);
    // a packet without its own request fields belongs to its first lane's request
    const bool own = pk.request_id != 0 || pk.lanes.empty();
    e.request_id = own ? pk.request_id : pk.lanes[0].request_id;
    e.sequence_id = own ? pk.sequence_id : pk.lanes[0].sequence_id;
    e.sequence_position = own ? pk.sequence_position : pk.lanes[0].sequence_position;
    e.slot = pk.pipeline_slot;
    e.identity = pk.identity;
  }
  return r;
}

WorkResult NodeContext::prefill(const wc::Packet& p) {
  if (p.identity.transaction_phase != wc::kPhasePrefill) fail(Status::InvalidArgument, "node context: not a prefill packet");
  return submit_work(p);
}

WorkResult NodeContext::decode(const wc::Packet& p) {
  if (p.identity.transaction_phase != wc::kPhaseDecode) fail(Status::InvalidArgument, "node context: not a decode packet");
  return submit_work(p);
}

Status NodeContext::pump_output(const wo::WorkOutput::FailFn& f) { return out_ ? out_->pump(f) : Status::Ok; }

}  // namespace nc
}  // namespace spc
