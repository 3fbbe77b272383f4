// Control plane of model drivers: what a model is made of, where its validated
// modules live, how a driver is built from them, and how submits are routed to
// loaded drivers.
//
//   model description  a JSON file: model id / revision, stages (name, compile
//                      target), programs (id, in-flight bound, completion mode,
//                      scheduling limits) and their ordered operations (name, kind
//                      from the operation taxonomy, module id, configuration). Loaded
//                      and validated fail-closed; its SHA-256 is its identity.
//   module library     content-addressed store of validated link units (.o / .a):
//                      publishing hashes the unit and the validator, runs the
//                      validator unless an identical validation is on record, stores
//                      the unit and an immutable record under the hash, then swaps
//                      the module's active record atomically. Resolving re-hashes
//                      the stored unit against its record.
//   driver compiler    generates the C source of one stage's model driver (the
//                      driver ABI of include/sparkpipe_b200/model_driver.h) whose
//                      programs run their operations' module entry points in order,
//                      compiles it with the stage's link units into a shared object
//                      and writes a manifest with every hash involved.
//   orchestrator       nodes (id, compile target) with attached drivers (loaded and
//                      validated against the node's target), routes (model id,
//                      revision, stage, program) -> (driver, program), submits,
//                      per-driver outstanding counts and program snapshots.
//
// Module entry points (C, all return 0 on success):
//   int32_t init(const char* configuration_json, void** state);
//   int32_t execute(void* state, const spb_buffer* input, spb_buffer* output);
//   void    destroy(void* state);
//
// Reference behaviour: crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_model_description.h:15-84,
// spark_module_library.h:14-79, spark_driver_compiler.h:13-63, spark_orchestrator.h:14-46
// (the concepts and their records). Formats, paths and the generated driver are
// this framework's own.
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "common.h"
#include "driver_loader.h"

namespace spc {
namespace ctl {

std::string sha256_hex(const std::string& bytes);
std::string file_sha256_hex(const std::string& path);

// ---------------------------------------------------------------- model description
enum class OpKind : uint32_t {
  GlobalAttention, LinearAttention, SlidingAttention, CompressedSparseAttention, HierarchicalCompressedAttention,
  RoutedMoe, GroupedMoe, SharedMoe, HashRoutedMoe, Router, DenseMlp, PositionEncoding, SparseIndex, GateProjection,
  AttentionOutputGate, RecurrentUpdate, RecurrentReplay, DepthStateDelta, HyperConnection, MultiTokenPrediction, Draft,
  OutputHead, Custom
};
const char* op_kind_name(OpKind k);
OpKind op_kind_from_name(const std::string& s);  // throws SchemaError

struct Operation {
  std::string name, module_id, configuration_json;
  OpKind kind = OpKind::Custom;
};
struct Scheduling {
  uint32_t max_active_slots = 0, max_new_tokens = 0, max_resident_sequences = 0;
  uint64_t max_sequence_tokens = 0, target_latency_ns = 0, resident_weight_bytes = 0, resident_kv_bytes = 0;
};
struct Program {
  std::string name;
  uint32_t program_id = 0, max_inflight = 1;
  bool external_completion = false;
  Scheduling scheduling;
  std::vector<Operation> operations;
};
struct Stage {
  std::string name, target;
  std::vector<Program> programs;
};
struct ModelDescription {
  uint32_t schema_version = 1;
  std::string model_id, model_revision, metadata_json, source_sha256;
  std::vector<Stage> stages;
  const Stage* stage(const std::string& name) const;
};
ModelDescription parse_model_description(const std::string& json_text);
ModelDescription load_model_description(const std::string& path);

// ---------------------------------------------------------------- module library
enum class LinkUnit : uint32_t { RelocatableObject = 1, StaticArchive = 2 };
struct ModuleArtifact {
  std::string module_id, target, artifact_sha256, link_unit_path, validation_recipe, validator_sha256;
  std::string init_symbol, execute_symbol, destroy_symbol;
  uint32_t module_abi = 1;
  LinkUnit kind = LinkUnit::RelocatableObject;
  bool validated = false;
};
struct PublishRequest {
  std::string library_root, module_id, target, link_unit_path, validation_recipe;
  std::string init_symbol, execute_symbol, destroy_symbol;
  uint32_t module_abi = 1;
  std::string validator_path;                  // run as: validator [args...] <link unit>; exit 0 = valid
  std::vector<std::string> validator_args;
};
struct PublishReport {
  bool validation_reused = false;
  std::string artifact_sha256, validator_sha256, record_path, active_record_path, stored_link_unit_path;
};
PublishReport publish_module(const PublishRequest& req);
ModuleArtifact resolve_module(const std::string& library_root, const std::string& module_id,
                              const std::string& target);
ModuleArtifact load_module_record(const std::string& record_path);

// ---------------------------------------------------------------- driver compiler
struct CompileRequest {
  std::string model_description_path, stage_name, library_root, output_directory;
  std::string compiler = "cc";
  std::string include_directory;               // where sparkpipe_b200/model_driver.h lives
  std::vector<std::string> extra_args;
};
struct CompileReport {
  uint32_t program_count = 0, operation_count = 0, link_unit_count = 0;
  std::string model_description_sha256, compiled_program_sha256, driver_sha256;
  std::string generated_source_path, driver_path, manifest_path;
};
CompileReport compile_driver(const CompileRequest& req);

// ---------------------------------------------------------------- orchestrator
class Orchestrator {
 public:
  uint32_t add_node(const std::string& node_id, const std::string& target);
  uint32_t attach_driver(uint32_t node, const std::string& driver_path, const std::string& config_json);
  uint32_t resolve_route(const std::string& model_id, const std::string& revision, const std::string& stage,
                         const std::string& program) const;
  std::string submit(uint32_t route, const std::string& input, size_t output_capacity);
  uint64_t outstanding(uint32_t driver) const;
  spb_snapshot snapshot(uint32_t driver);
  uint32_t node_count() const { return (uint32_t)nodes_.size(); }
  uint32_t driver_count() const { return (uint32_t)drivers_.size(); }

 private:
  struct Node {
    std::string id, target;
  };
  struct Attached {
    uint32_t node;
    std::unique_ptr<ModelDriver> driver;
    uint64_t outstanding = 0;
  };
  struct Route {
    uint32_t driver, program_id;
  };
  std::vector<Node> nodes_;
  std::vector<Attached> drivers_;
  mutable std::vector<Route> routes_;
};

}  // namespace ctl
}  // namespace spc
