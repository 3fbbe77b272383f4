// Loader for stage drivers built against the reference's model-driver ABI v6
// (binary layout in include/sparkpipe_b200/spark_driver_abi_v6.h).
//
//   load       dlopen, resolve `SparkModelDriverGetInterface`, validate the whole
//              interface fail-closed before any entry point runs: ABI version and
//              struct sizes, identity strings, 64-hex-digit SHA-256 fields, a
//              non-empty table of programs with unique ids and names, known flag
//              bits, profiles that agree with their programs, flag claims backed
//              by profile numbers, and the node's compile target
//   create     one driver instance per node; completions and wake-ups the driver
//              reports (from any thread) land in a locked queue
//   admit      the driver's admission decision for a prospective frame
//   submit     builds the frame (the loader owns it, and its buffer table, until
//              the frame's completion arrives: a driver may complete after submit
//              returns) and calls the program's submit entry point
//   poll       completions in arrival order, waiting up to a timeout
//   snapshot   per-program runtime counters
//
// Reference behaviour: crates/spark-sys/src/driver.rs (ModelDriver::load,
// validate_program, validate_interface). The implementation is this framework's own.
#pragma once

#include <sparkpipe_b200/spark_driver_abi_v6.h>

#include <condition_variable>
#include <cstdint>
#include <deque>
#include <list>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "common.h"

namespace spc {
namespace v6 {

struct ProgramInfo {
  uint32_t program_id = 0, flags = 0, max_inflight = 0;
  std::string name;
  sp6_program_profile profile{};
};

struct Completion {
  uint64_t request_id = 0, sequence_id = 0, sequence_position = 0;
  uint32_t program_id = 0, driver_dispatch_slot = 0, accepted_token_count = 0, completion_flags = 0;
  std::vector<uint32_t> token_ids, draft_token_ids;
  int32_t status = 0;
  sp6_residency residency{};
  uint64_t queue_delay_ns = 0, service_time_ns = 0, device_memcpy_bytes = 0, host_staging_bytes = 0;
};

// Frame fields a caller sets (the rest — program, completion route — the loader fills).
struct FrameArgs {
  uint64_t request_id = 0, sequence_id = 0, sequence_position = 0, deadline_time_ns = 0;
  uint32_t active_slot_count = 0, new_token_count = 0, priority = 0, flags = 0;
  uint32_t driver_dispatch_slot = SP6_INVALID_DISPATCH_SLOT;
  uint64_t driver_dispatch_generation = 0, driver_dispatch_cookie0 = 0, driver_dispatch_cookie1 = 0;
  uint64_t execution_stream = 0;  // a cudaStream_t as an integer (0 = none)
  std::vector<sp6_buffer> buffers;
  uint64_t scalar[SP6_SCALARS] = {};
  sp6_residency residency{};
};

void validate_interface(const sp6_interface* iface, const std::string& expected_target);

class Driver {
 public:
  // Throws StatusError: DriverLoadError (open / symbol), AbiMismatch, ValidationFailed,
  // Duplicate, TargetMismatch.
  static std::unique_ptr<Driver> load(const std::string& path, const std::string& expected_target);
  ~Driver();
  Driver(const Driver&) = delete;
  Driver& operator=(const Driver&) = delete;

  const sp6_driver_descriptor& descriptor() const { return *iface_->descriptor; }
  std::vector<ProgramInfo> programs() const;

  // node_context is handed to the driver as is (a pointer the caller keeps alive).
  void create(const std::string& node_id, const std::string& node_target, uint64_t node_context);
  void destroy();
  bool has_instance() const { return instance_ != nullptr; }
  sp6_admission_decision admit(const sp6_admission_request& request);
  Status submit(uint32_t program_id, const FrameArgs& args);
  std::vector<Completion> poll(size_t max, int timeout_ms);
  sp6_runtime_snapshot snapshot(uint32_t program_id);
  uint64_t wakes() const;
  size_t frames_in_flight() const;

 private:
  Driver(void* handle, const sp6_interface* iface) : handle_(handle), iface_(iface) {}
  static void on_completion(void* ctx, const sp6_completion* c);
  static void on_wake(void* ctx);
  const sp6_program_descriptor* program(uint32_t id) const;
  struct OwnedFrame {
    sp6_frame frame{};
    std::vector<sp6_buffer> buffers;
  };
  void* handle_;
  const sp6_interface* iface_;
  void* instance_ = nullptr;
  std::string node_id_, node_target_;
  mutable std::mutex mu_;
  std::condition_variable cv_;
  std::deque<Completion> done_;
  std::list<OwnedFrame> inflight_;
  uint64_t wakes_ = 0;
};

// sizeof / offsetof of the v6 structs as this compiler lays them out (compared by the
// layout gate with a C probe and with the natural C layout of the declarations).
std::vector<std::pair<std::string, uint64_t>> abi_layout();

}  // namespace v6
}  // namespace spc
