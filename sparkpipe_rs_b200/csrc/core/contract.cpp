#include "contract.h"

#include <cmath>

namespace spc {

namespace {
enum class FT { U64, F64, Bool, Str, StrList };
struct Field {
  const char* name;
  FT type;
  bool required;  // optional fields get a default
};
struct Section {
  const char* name;
  bool required;
  std::vector<Field> fields;
};

// The K2-family contract schema (field names and types of the reference format).
const std::vector<Section>& k27_schema() {
  static const std::vector<Section> s = {
      {"sources", false,
       {{"checkpoint_config", FT::Str, false}, {"parameter_counts", FT::Str, false}, {"license", FT::Str, false}}},
      {"multimodal_wrapper", true,
       {{"note", FT::Str, false},
        {"text_architecture", FT::Str, false},
        {"text_model_type", FT::Str, false},
        {"media_placeholder_token_id", FT::U64, false}}},
      {"model", true,
       {{"total_parameters", FT::U64, true},
        {"active_parameters", FT::U64, true},
        {"hidden_dimension", FT::U64, true},
        {"layer_count", FT::U64, true},
        {"vocabulary_size", FT::U64, true},
        {"maximum_context_tokens", FT::U64, true},
        {"rms_norm_epsilon", FT::F64, true},
        {"first_routed_layer", FT::U64, true},
        {"tie_word_embeddings", FT::Bool, true}}},
      {"mla", true,
       {{"query_head_count", FT::U64, true},
        {"query_lora_rank", FT::U64, true},
        {"kv_lora_rank", FT::U64, true},
        {"qk_nope_dimension", FT::U64, true},
        {"qk_unrotated_dimension", FT::U64, true},
        {"value_head_dimension", FT::U64, true},
        {"output_gate", FT::Bool, true},
        {"uses_nope", FT::Bool, true},
        {"attention_bias", FT::Bool, true}}},
      {"rope", true,
       {{"type", FT::Str, true},
        {"theta", FT::F64, true},
        {"factor", FT::F64, true},
        {"original_max_position_embeddings", FT::U64, true},
        {"beta_fast", FT::F64, true},
        {"beta_slow", FT::F64, true},
        {"mscale", FT::F64, true},
        {"mscale_all_dim", FT::F64, true},
        {"note", FT::Str, false}}},
      {"moe", true,
       {{"routed_expert_count", FT::U64, true},
        {"experts_per_token", FT::U64, true},
        {"shared_expert_count", FT::U64, true},
        {"expert_intermediate_dimension", FT::U64, true},
        {"dense_intermediate_dimension", FT::U64, true},
        {"routed_scaling_factor", FT::F64, true},
        {"router_activation", FT::Str, true},
        {"top_k_method", FT::Str, true},
        {"router_group_count", FT::U64, true},
        {"renormalize_selected_probabilities", FT::Bool, true},
        {"activation", FT::Str, true},
        {"moe_layer_frequency", FT::U64, true}}},
      {"quantization", true,
       {{"routed_expert_weight_format", FT::Str, true},
        {"routed_expert_group_size", FT::U64, true},
        {"routed_expert_symmetric", FT::Bool, true},
        {"routed_expert_quant_method", FT::Str, true},
        {"non_expert_weight_format", FT::Str, true},
        {"non_expert_activation_format", FT::Str, true},
        {"accumulator_format", FT::Str, true},
        {"kv_cache_format", FT::Str, true},
        {"quantized_components", FT::StrList, true},
        {"unquantized_patterns", FT::StrList, true},
        {"note", FT::Str, false}}},
      {"speculation", true, {{"base_checkpoint_mtp_layer_count", FT::U64, true}, {"note", FT::Str, false}}},
      {"cache", true,
       {{"kv_element_bits", FT::U64, true}, {"kv_page_slots", FT::U64, true}, {"note", FT::Str, false}}},
      {"tokens", true,
       {{"begin_of_sentence", FT::U64, true}, {"end_of_text", FT::U64, true}, {"pad", FT::U64, true}}},
      {"qualification", true,
       {{"cuda_target", FT::Str, true}, {"status", FT::Str, true}, {"production_ready", FT::Bool, true}}},
  };
  return s;
}

bool is_u64(const Json& v) { return v.is_integer() && v.int64() >= 0; }

Json typed_default(FT t) {
  switch (t) {
    case FT::U64: return Json::make_int(0);
    case FT::F64: return Json::make_number(0.0);
    case FT::Bool: return Json::make_bool(false);
    case FT::Str: return Json::make_string("");
    case FT::StrList: return Json::make_array();
  }
  return Json();
}

bool type_ok(const Json& v, FT t) {
  switch (t) {
    case FT::U64: return is_u64(v);
    case FT::F64: return v.is_number();
    case FT::Bool: return v.is_bool();
    case FT::Str: return v.is_string();
    case FT::StrList:
      if (!v.is_array()) return false;
      for (const Json& e : v.arr())
        if (!e.is_string()) return false;
      return true;
  }
  return false;
}

int64_t opt_u64(const Json* obj, const char* key) {
  if (!obj) return -1;
  const Json* v = obj->get(key);
  return (v && is_u64(*v)) ? v->int64() : -1;
}
}  // namespace

ContractDocument ContractDocument::parse(const std::string& text, const std::string& path) {
  ContractDocument d;
  d.path_ = path;
  try {
    d.raw_ = Json::parse(text);
  } catch (const StatusError& e) {
    fail(Status::ParseError, "contract " + path + ": " + e.what());
  }
  if (const Json* v = d.raw_.get("schema_version")) {
    if (!is_u64(*v) || v->int64() == 0)
      fail(Status::SchemaError, "contract " + path + ": schema_version must be a positive integer, found " + v->dump());
    d.schema_version_ = v->int64();
  }
  if (const Json* v = d.raw_.get("model_id")) {
    if (!v->is_string() || v->str().empty())
      fail(Status::SchemaError, "contract " + path + ": model_id must be a non-empty string");
    d.model_id_ = v->str();
  }
  if (const Json* v = d.raw_.get("architecture"))
    if (v->is_string()) d.architecture_ = v->str();
  if (!d.has_geometry())
    fail(Status::SchemaError,
         "contract " + path + ": no model geometry found (neither a 'model' section nor flat geometry keys)");
  return d;
}

bool ContractDocument::has_geometry() const {
  if (raw_.get("model")) return raw_.get("model")->is_object();
  const ModelGeometry g = geometry();
  return g.layer_count >= 0 || g.hidden_dimension >= 0;
}

ModelGeometry ContractDocument::geometry() const {
  const Json* src = raw_.get("model");
  if (src && !src->is_object()) return ModelGeometry{};
  if (!src) src = &raw_;  // flat dialect: geometry keys at the top level
  ModelGeometry g;
  g.total_parameters = opt_u64(src, "total_parameters");
  g.active_parameters = opt_u64(src, "active_parameters");
  g.hidden_dimension = opt_u64(src, "hidden_dimension");
  g.layer_count = opt_u64(src, "layer_count");
  g.vocabulary_size = opt_u64(src, "vocabulary_size");
  if (g.vocabulary_size < 0 && src == &raw_) g.vocabulary_size = opt_u64(src, "vocab_size");
  g.maximum_context_tokens = opt_u64(src, "maximum_context_tokens");
  g.first_routed_layer = opt_u64(src, "first_routed_layer");
  return g;
}

Json ContractDocument::as_k27() const {
  const std::string who = model_id_.empty() ? std::string("unknown") : model_id_;
  Json out = Json::make_object();
  if (schema_version_ >= 0) out.set("schema_version", Json::make_int(schema_version_));
  if (!model_id_.empty()) out.set("model_id", Json::make_string(model_id_));
  if (!architecture_.empty()) out.set("architecture", Json::make_string(architecture_));
  for (const Section& sec : k27_schema()) {
    const Json* src = raw_.get(sec.name);
    if (!src) {
      if (sec.required) fail(Status::SchemaError, "contract " + who + ": missing required section '" + sec.name + "'");
      src = nullptr;
    } else if (!src->is_object()) {
      fail(Status::SchemaError, "contract " + who + ": section '" + sec.name + "' must be an object");
    }
    Json o = Json::make_object();
    for (const Field& f : sec.fields) {
      const Json* v = src ? src->get(f.name) : nullptr;
      if (!v) {
        if (f.required)
          fail(Status::SchemaError,
               "contract " + who + ": section '" + sec.name + "' is missing field '" + f.name + "'");
        o.set(f.name, typed_default(f.type));
        continue;
      }
      if (!type_ok(*v, f.type))
        fail(Status::SchemaError,
             "contract " + who + ": section '" + sec.name + "' field '" + f.name + "' has the wrong type");
      o.set(f.name, *v);
    }
    out.set(sec.name, std::move(o));
  }
  return out;
}

std::string ContractDocument::family() const {
  if (architecture_.empty()) fail(Status::SchemaError, "contract " + model_id_ + ": missing architecture field");
  if (architecture_ == "KimiK25ForConditionalGeneration") return "k27";
  fail(Status::Unsupported, "contract " + model_id_ + ": unsupported architecture '" + architecture_ + "'");
}

}  // namespace spc
