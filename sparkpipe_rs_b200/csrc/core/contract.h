// Model contract documents: envelope validation, normalized geometry from either
// dialect (a `model` section, or flat top-level keys), section access, the typed
// Kimi-K2-family view (`as_k27`, every required section and field type-checked
// against a declarative schema) and family dispatch by `architecture`.
//
// Reference behaviour: crates/spark-model/src/contract.rs (envelope :84-132,
// geometry :144-170, as_k27 :172-225), k27.rs (sections and field types),
// family.rs (dispatch). The JSON format is the reference's, so the same contract
// files load in both.
#pragma once

#include <string>
#include <vector>

#include "common.h"
#include "json.h"

namespace spc {

struct ModelGeometry {
  // -1 = absent (dialects differ; absence is meaningful to family validators)
  int64_t total_parameters = -1, active_parameters = -1, hidden_dimension = -1, layer_count = -1;
  int64_t vocabulary_size = -1, maximum_context_tokens = -1, first_routed_layer = -1;
};

class ContractDocument {
 public:
  // Throws StatusError: ParseError (bad JSON), SchemaError (bad envelope / no geometry).
  static ContractDocument parse(const std::string& text, const std::string& path = "<memory>");
  int64_t schema_version() const { return schema_version_; }  // -1 if absent
  const std::string& model_id() const { return model_id_; }    // "" if absent
  const std::string& architecture() const { return architecture_; }
  bool has_geometry() const;
  ModelGeometry geometry() const;
  const Json& raw() const { return raw_; }
  const Json* section(const std::string& name) const { return raw_.get(name); }
  // Typed K2-family view: the validated sections (with defaults filled) as one
  // JSON object; SchemaError names the missing or malformed section / field.
  Json as_k27() const;
  // Family of this contract ("k27"); SchemaError without an architecture,
  // Unsupported for an unknown one.
  std::string family() const;

 private:
  Json raw_;
  std::string path_, model_id_, architecture_;
  int64_t schema_version_ = -1;
};

}  // namespace spc
