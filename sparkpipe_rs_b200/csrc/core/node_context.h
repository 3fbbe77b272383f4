// Node context of one ring rank: the seam a serving backend calls (prefill, decode,
// submit_work), built from the rank's plan and its compiled model driver.
//
//   build        loads the stage's model driver against the node's compile target
//                (driver_loader.h: fail-closed ABI / target checks), resolves its
//                prefill and decode programs by name, creates the driver instance,
//                checks the rank plan, and, for a rank with a next stage, opens the
//                work-output plane toward it (work_output.h)
//   submit_work  validates a work packet against the rank's limits (execution rows,
//                phase), hands it on to the next rank first when there is one
//                (forward-then-run, so the next stage's weights start streaming
//                while this one computes), then runs the packet's program on the
//                driver. On the final stage the program's output is read as token ids
//                (little-endian u32) and returned as the packet's final event for
//                rank 0
//   prefill /    submit_work restricted to the prefill or the decode phase
//   decode
//
// Reference behaviour: crates/spark-abi/vendor/sparkpipe/include/sparkpipe/
// spark_ring_node_context_builder.h:87-284 (node contexts built from packs exposing
// prefill / decode / submit_work) and crates/spark-node/src/backend/state.rs:206-290
// (the Rank0NodeContext seam). The composition here is this runtime's own.
#pragma once

#include <cstdint>
#include <memory>
#include <string>

#include "common.h"
#include "driver_loader.h"
#include "rank_daemon.h"
#include "ring_runtime.h"
#include "work_control.h"
#include "work_output.h"

namespace spc {
namespace nc {

struct NodeContextConfig {
  ring::RankPlan plan;
  std::string driver_path, target, driver_config_json = "{}";
  std::string prefill_program = "prefill", decode_program = "decode";
  wc::Config work;
  uint32_t queue_capacity = 64, release_capacity = 256;
  uint32_t output_capacity = 1u << 20;
};

struct WorkResult {
  Status status = Status::Ok;
  bool forwarded = false, final_stage = false;
  std::string output;          // the program's output bytes
  rd::FinalEvent final_event;  // on the final stage
};

class NodeContext {
 public:
  static std::unique_ptr<NodeContext> build(const NodeContextConfig& cfg);
  WorkResult submit_work(const wc::Packet& p);
  WorkResult prefill(const wc::Packet& p);
  WorkResult decode(const wc::Packet& p);
  // drives the work-output plane toward the next rank (Ok when nothing is left)
  Status pump_output(const wo::WorkOutput::FailFn& on_hard_failure = nullptr);
  wo::WorkOutput* work_output() { return out_.get(); }
  const ring::RankPlan& plan() const { return cfg_.plan; }
  ModelDriver& driver() { return *driver_; }
  uint64_t submitted() const { return submitted_; }

 private:
  explicit NodeContext(const NodeContextConfig& cfg) : cfg_(cfg) {}
  NodeContextConfig cfg_;
  std::unique_ptr<ModelDriver> driver_;
  std::unique_ptr<wo::WorkOutput> out_;
  uint32_t prefill_id_ = 0, decode_id_ = 0;
  uint64_t submitted_ = 0;
};

}  // namespace nc
}  // namespace spc
