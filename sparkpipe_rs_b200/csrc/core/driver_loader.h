// Model-driver loader: dlopen a driver library, resolve its interface symbol and
// validate the whole interface fail-closed before anything is called (rules listed
// in include/sparkpipe_b200/model_driver.h). Reference behaviour:
// crates/spark-sys/src/driver.rs (ModelDriver::load :62-110, program checks
// :173-228, interface checks :230-316).
#pragma once

#include <sparkpipe_b200/model_driver.h>

#include <string>
#include <vector>

#include "common.h"

namespace spc {

struct DriverProgramInfo {
  uint32_t program_id, flags, max_inflight;
  std::string name;
};

class ModelDriver {
 public:
  // Throws StatusError: DriverLoadError (open / symbol), AbiMismatch (interface,
  // descriptor, program or profile ABI), ValidationFailed (a flag claim without
  // its profile number), Duplicate (program id or name), TargetMismatch.
  static ModelDriver* load(const std::string& path, const std::string& expected_target);
  ~ModelDriver();
  ModelDriver(const ModelDriver&) = delete;
  ModelDriver& operator=(const ModelDriver&) = delete;

  std::string model_id() const;
  std::string model_revision() const;
  std::string stage_name() const;
  std::string target() const;
  std::string model_description_sha256() const;
  std::string compiled_program_sha256() const;
  uint32_t module_instance_count() const;
  std::vector<DriverProgramInfo> programs() const;
  bool find_program(const std::string& name, DriverProgramInfo* out) const;

  // Instance lifecycle through the driver's entry points.
  void create(const std::string& config_json);
  void destroy();
  bool has_instance() const { return instance_ != nullptr; }
  uint32_t admit(uint32_t program_id, uint32_t sequences, uint32_t tokens);
  spb_snapshot snapshot();
  std::string submit(uint32_t program_id, const std::string& input, size_t output_capacity);

 private:
  ModelDriver(void* handle, const spb_model_driver_interface* iface) : handle_(handle), iface_(iface) {}
  const spb_program_descriptor* program(uint32_t id) const;
  void* handle_;
  const spb_model_driver_interface* iface_;
  void* instance_ = nullptr;
};

// Validation on its own (used by load and by tests on in-memory interfaces).
void validate_driver_interface(const spb_model_driver_interface* iface, const std::string& expected_target);
bool sha256_hex_is_valid(const char* s);

// sizeof / offsetof of the ABI structs as this compiler lays them out (the layout gate
// compares them with a C probe compiled by the system C compiler).
std::vector<std::pair<std::string, uint64_t>> driver_abi_layout();

}  // namespace spc
