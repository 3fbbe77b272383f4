#include "control_plane.h"

#include <sys/stat.h>
#include <sys/wait.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <set>
#include <sstream>
#include <type_traits>

#include "json.h"

namespace spc {
namespace ctl {

// ---------------------------------------------------------------- SHA-256 (FIPS 180-4)
namespace {
using u128 = unsigned __int128;

// floor(x) with x^n <= v (n = 2 or 3), by bisection on integers
uint64_t iroot(u128 v, int n) {
  uint64_t lo = 0, hi = 1ull << 40;
  while (lo < hi) {
    const uint64_t mid = lo + (hi - lo + 1) / 2;
    u128 p = mid;
    for (int i = 1; i < n; ++i) p *= mid;
    if (p <= v) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

struct Sha256Consts {
  uint32_t k[64], h0[8];
  Sha256Consts() {
    // the first 32 fraction bits of the cube roots (k) and square roots (h0) of the first primes
    int primes[64], n = 0;
    for (int c = 2; n < 64; ++c) {
      bool prime = true;
      for (int d = 2; d * d <= c; ++d)
        if (c % d == 0) { prime = false; break; }
      if (prime) primes[n++] = c;
    }
    for (int i = 0; i < 64; ++i) k[i] = uint32_t(iroot(u128(primes[i]) << 96, 3));
    for (int i = 0; i < 8; ++i) h0[i] = uint32_t(iroot(u128(primes[i]) << 64, 2));
  }
};
const Sha256Consts& consts() {
  static const Sha256Consts c;
  return c;
}
inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }
}  // namespace

std::string sha256_hex(const std::string& bytes) {
  const Sha256Consts& C = consts();
  uint32_t h[8];
  std::memcpy(h, C.h0, sizeof(h));
  std::string msg = bytes;
  const uint64_t bits = uint64_t(bytes.size()) * 8;
  msg.push_back(char(0x80));
  while (msg.size() % 64 != 56) msg.push_back('\0');
  for (int i = 7; i >= 0; --i) msg.push_back(char((bits >> (8 * i)) & 0xff));
  for (size_t off = 0; off < msg.size(); off += 64) {
    uint32_t w[64];
    for (int i = 0; i < 16; ++i) {
      const unsigned char* p = reinterpret_cast<const unsigned char*>(msg.data() + off + 4 * i);
      w[i] = (uint32_t(p[0]) << 24) | (uint32_t(p[1]) << 16) | (uint32_t(p[2]) << 8) | uint32_t(p[3]);
    }
    for (int i = 16; i < 64; ++i) {
      const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
      const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
      w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int i = 0; i < 64; ++i) {
      const uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
      const uint32_t ch = (e & f) ^ (~e & g);
      const uint32_t t1 = hh + S1 + ch + C.k[i] + w[i];
      const uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
      const uint32_t maj = (a & b) ^ (a & c) ^ (b & c);
      const uint32_t t2 = S0 + maj;
      hh = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
    }
    h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
  }
  static const char* hex = "0123456789abcdef";
  std::string out;
  for (uint32_t v : h)
    for (int i = 7; i >= 0; --i) out.push_back(hex[(v >> (4 * i)) & 0xf]);
  return out;
}

namespace {
std::string read_file(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) fail(Status::IoError, "cannot read " + path);
  std::ostringstream ss;
  ss << f.rdbuf();
  return ss.str();
}
void write_file_atomic(const std::string& path, const std::string& data) {
  const std::string tmp = path + ".tmp." + std::to_string(::getpid());
  {
    std::ofstream f(tmp, std::ios::binary | std::ios::trunc);
    if (!f) fail(Status::IoError, "cannot write " + tmp);
    f.write(data.data(), (std::streamsize)data.size());
    if (!f) fail(Status::IoError, "short write " + tmp);
  }
  if (std::rename(tmp.c_str(), path.c_str()) != 0) fail(Status::IoError, "cannot replace " + path);
}
void mkdirs(const std::string& path) {
  std::string cur;
  for (size_t i = 0; i <= path.size(); ++i) {
    if (i == path.size() || path[i] == '/') {
      if (!cur.empty() && ::mkdir(cur.c_str(), 0755) != 0 && errno != EEXIST)
        fail(Status::IoError, "cannot create directory " + cur);
    }
    if (i < path.size()) cur.push_back(path[i]);
  }
}
bool exists(const std::string& p) {
  struct stat st;
  return ::stat(p.c_str(), &st) == 0;
}
// Runs argv[0] with arguments, no shell; returns the exit status (-1: not run).
int run(const std::vector<std::string>& argv) {
  const pid_t pid = ::fork();
  if (pid < 0) return -1;
  if (pid == 0) {
    std::vector<char*> a;
    for (const auto& s : argv) a.push_back(const_cast<char*>(s.c_str()));
    a.push_back(nullptr);
    ::execvp(a[0], a.data());
    ::_exit(127);
  }
  int st = 0;
  while (::waitpid(pid, &st, 0) < 0)
    if (errno != EINTR) return -1;
  return WIFEXITED(st) ? WEXITSTATUS(st) : -1;
}
bool ident_ok(const std::string& s) {
  if (s.empty() || s.size() > 128) return false;
  for (char c : s)
    if (!(std::isalnum((unsigned char)c) || c == '_' || c == '-' || c == '.')) return false;
  return s != "." && s != "..";
}
bool symbol_ok(const std::string& s) {
  if (s.empty() || !(std::isalpha((unsigned char)s[0]) || s[0] == '_')) return false;
  for (char c : s)
    if (!(std::isalnum((unsigned char)c) || c == '_')) return false;
  return true;
}
}  // namespace

std::string file_sha256_hex(const std::string& path) { return sha256_hex(read_file(path)); }

// ---------------------------------------------------------------- model description
namespace {
const std::pair<OpKind, const char*> kKinds[] = {
    {OpKind::GlobalAttention, "global_attention"},
    {OpKind::LinearAttention, "linear_attention"},
    {OpKind::SlidingAttention, "sliding_attention"},
    {OpKind::CompressedSparseAttention, "compressed_sparse_attention"},
    {OpKind::HierarchicalCompressedAttention, "hierarchical_compressed_attention"},
    {OpKind::RoutedMoe, "routed_moe"},
    {OpKind::GroupedMoe, "grouped_moe"},
    {OpKind::SharedMoe, "shared_moe"},
    {OpKind::HashRoutedMoe, "hash_routed_moe"},
    {OpKind::Router, "router"},
    {OpKind::DenseMlp, "dense_mlp"},
    {OpKind::PositionEncoding, "position_encoding"},
    {OpKind::SparseIndex, "sparse_index"},
    {OpKind::GateProjection, "gate_projection"},
    {OpKind::AttentionOutputGate, "attention_output_gate"},
    {OpKind::RecurrentUpdate, "recurrent_update"},
    {OpKind::RecurrentReplay, "recurrent_replay"},
    {OpKind::DepthStateDelta, "depth_state_delta"},
    {OpKind::HyperConnection, "hyper_connection"},
    {OpKind::MultiTokenPrediction, "multi_token_prediction"},
    {OpKind::Draft, "draft"},
    {OpKind::OutputHead, "output_head"},
    {OpKind::Custom, "custom"},
};
uint64_t u64_field(const Json& o, const char* k, uint64_t dflt) {
  const Json* v = o.get(k);
  if (!v) return dflt;
  if (!v->is_integer() || v->int64() < 0) fail(Status::SchemaError, std::string("model description: ") + k);
  return uint64_t(v->int64());
}
std::string str_field(const Json& o, const char* k) {
  const Json* v = o.get(k);
  if (!v || !v->is_string() || v->str().empty())
    fail(Status::SchemaError, std::string("model description: missing string ") + k);
  return v->str();
}
}  // namespace

const char* op_kind_name(OpKind k) {
  for (const auto& p : kKinds)
    if (p.first == k) return p.second;
  return "custom";
}
OpKind op_kind_from_name(const std::string& s) {
  for (const auto& p : kKinds)
    if (s == p.second) return p.first;
  fail(Status::SchemaError, "model description: unknown operation kind " + s);
}

const Stage* ModelDescription::stage(const std::string& name) const {
  for (const auto& s : stages)
    if (s.name == name) return &s;
  return nullptr;
}

ModelDescription parse_model_description(const std::string& text) {
  const Json j = Json::parse(text);
  if (!j.is_object()) fail(Status::SchemaError, "model description: not an object");
  ModelDescription d;
  d.schema_version = (uint32_t)u64_field(j, "schema_version", 0);
  if (d.schema_version != 1) fail(Status::SchemaError, "model description: schema_version must be 1");
  d.model_id = str_field(j, "model_id");
  d.model_revision = str_field(j, "model_revision");
  if (const Json* m = j.get("metadata")) d.metadata_json = m->dump();
  const Json* stages = j.get("stages");
  if (!stages || !stages->is_array() || stages->size() == 0) fail(Status::SchemaError, "model description: no stages");
  std::set<std::string> stage_names;
  for (const Json& sj : stages->arr()) {
    Stage s;
    s.name = str_field(sj, "name");
    s.target = str_field(sj, "target");
    if (!stage_names.insert(s.name).second) fail(Status::Duplicate, "model description: duplicate stage " + s.name);
    const Json* progs = sj.get("programs");
    if (!progs || !progs->is_array() || progs->size() == 0)
      fail(Status::SchemaError, "model description: stage " + s.name + " has no programs");
    std::set<std::string> pnames;
    std::set<uint32_t> pids;
    for (const Json& pj : progs->arr()) {
      Program p;
      p.name = str_field(pj, "name");
      p.program_id = (uint32_t)u64_field(pj, "program_id", 0);
      p.max_inflight = (uint32_t)u64_field(pj, "max_inflight", 1);
      if (p.program_id == 0 || p.max_inflight == 0)
        fail(Status::SchemaError, "model description: program ids and in-flight bounds are nonzero");
      if (!pnames.insert(p.name).second || !pids.insert(p.program_id).second)
        fail(Status::Duplicate, "model description: duplicate program in stage " + s.name);
      if (const Json* c = pj.get("completion")) {
        if (!c->is_string() || (c->str() != "submit_return" && c->str() != "external"))
          fail(Status::SchemaError, "model description: completion is submit_return or external");
        p.external_completion = c->str() == "external";
      }
      if (const Json* sc = pj.get("scheduling")) {
        p.scheduling.max_active_slots = (uint32_t)u64_field(*sc, "max_active_slots", 0);
        p.scheduling.max_new_tokens = (uint32_t)u64_field(*sc, "max_new_tokens", 0);
        p.scheduling.max_resident_sequences = (uint32_t)u64_field(*sc, "max_resident_sequences", 0);
        p.scheduling.max_sequence_tokens = u64_field(*sc, "max_sequence_tokens", 0);
        p.scheduling.target_latency_ns = u64_field(*sc, "target_latency_ns", 0);
        p.scheduling.resident_weight_bytes = u64_field(*sc, "resident_weight_bytes", 0);
        p.scheduling.resident_kv_bytes = u64_field(*sc, "resident_kv_bytes", 0);
      }
      const Json* ops = pj.get("operations");
      if (!ops || !ops->is_array() || ops->size() == 0)
        fail(Status::SchemaError, "model description: program " + p.name + " has no operations");
      for (const Json& oj : ops->arr()) {
        Operation o;
        o.name = str_field(oj, "name");
        o.module_id = str_field(oj, "module_id");
        if (!ident_ok(o.module_id)) fail(Status::SchemaError, "model description: bad module id " + o.module_id);
        o.kind = op_kind_from_name(str_field(oj, "kind"));
        if (const Json* c = oj.get("configuration")) o.configuration_json = c->dump();
        else o.configuration_json = "{}";
        p.operations.push_back(std::move(o));
      }
      s.programs.push_back(std::move(p));
    }
    d.stages.push_back(std::move(s));
  }
  d.source_sha256 = sha256_hex(text);
  return d;
}

ModelDescription load_model_description(const std::string& path) { return parse_model_description(read_file(path)); }

// ---------------------------------------------------------------- module library
namespace {
std::string module_dir(const std::string& root, const std::string& id, const std::string& target) {
  return root + "/" + id + "/" + target;
}
Json artifact_json(const ModuleArtifact& a) {
  Json j = Json::make_object();
  j.set("schema_version", Json::make_int(1));
  j.set("module_abi", Json::make_int(a.module_abi));
  j.set("link_unit_kind", Json::make_string(a.kind == LinkUnit::StaticArchive ? "static_archive" : "relocatable_object"));
  j.set("module_id", Json::make_string(a.module_id));
  j.set("target", Json::make_string(a.target));
  j.set("artifact_sha256", Json::make_string(a.artifact_sha256));
  j.set("link_unit_path", Json::make_string(a.link_unit_path));
  j.set("validation_recipe", Json::make_string(a.validation_recipe));
  j.set("validator_sha256", Json::make_string(a.validator_sha256));
  j.set("init_symbol", Json::make_string(a.init_symbol));
  j.set("execute_symbol", Json::make_string(a.execute_symbol));
  j.set("destroy_symbol", Json::make_string(a.destroy_symbol));
  j.set("validated", Json::make_bool(a.validated));
  return j;
}
}  // namespace

ModuleArtifact load_module_record(const std::string& record_path) {
  const Json j = Json::parse(read_file(record_path));
  ModuleArtifact a;
  a.module_abi = (uint32_t)u64_field(j, "module_abi", 0);
  const std::string kind = str_field(j, "link_unit_kind");
  if (kind != "relocatable_object" && kind != "static_archive")
    fail(Status::SchemaError, "module record: unknown link unit kind");
  a.kind = kind == "static_archive" ? LinkUnit::StaticArchive : LinkUnit::RelocatableObject;
  a.module_id = str_field(j, "module_id");
  a.target = str_field(j, "target");
  a.artifact_sha256 = str_field(j, "artifact_sha256");
  a.link_unit_path = str_field(j, "link_unit_path");
  a.validation_recipe = str_field(j, "validation_recipe");
  a.validator_sha256 = str_field(j, "validator_sha256");
  a.init_symbol = str_field(j, "init_symbol");
  a.execute_symbol = str_field(j, "execute_symbol");
  a.destroy_symbol = str_field(j, "destroy_symbol");
  const Json* v = j.get("validated");
  a.validated = v && v->is_bool() && v->boolean();
  if (!sha256_hex_is_valid(a.artifact_sha256.c_str()) || !sha256_hex_is_valid(a.validator_sha256.c_str()))
    fail(Status::SchemaError, "module record: bad hashes");
  return a;
}

PublishReport publish_module(const PublishRequest& r) {
  if (!ident_ok(r.module_id) || !ident_ok(r.target) || r.library_root.empty())
    fail(Status::InvalidArgument, "module library: bad module id, target or root");
  for (const auto* s : {&r.init_symbol, &r.execute_symbol, &r.destroy_symbol})
    if (!symbol_ok(*s)) fail(Status::InvalidArgument, "module library: bad entry-point symbol " + *s);
  if (r.validation_recipe.empty() || r.validator_path.empty())
    fail(Status::InvalidArgument, "module library: a validation recipe and a validator are required");
  LinkUnit kind;
  const std::string& src = r.link_unit_path;
  if (src.size() > 2 && src.compare(src.size() - 2, 2, ".o") == 0) kind = LinkUnit::RelocatableObject;
  else if (src.size() > 2 && src.compare(src.size() - 2, 2, ".a") == 0) kind = LinkUnit::StaticArchive;
  else fail(Status::InvalidArgument, "module library: link units are .o or .a files");
  PublishReport rep;
  rep.artifact_sha256 = file_sha256_hex(src);
  rep.validator_sha256 = file_sha256_hex(r.validator_path);
  const std::string dir = module_dir(r.library_root, r.module_id, r.target);
  mkdirs(dir);
  rep.record_path = dir + "/" + rep.artifact_sha256 + ".json";
  rep.stored_link_unit_path = dir + "/" + rep.artifact_sha256 + (kind == LinkUnit::StaticArchive ? ".a" : ".o");
  rep.active_record_path = dir + "/active.json";
  bool reuse = false;
  if (exists(rep.record_path)) {
    const ModuleArtifact old = load_module_record(rep.record_path);
    reuse = old.validated && old.validator_sha256 == rep.validator_sha256 &&
            old.validation_recipe == r.validation_recipe && old.execute_symbol == r.execute_symbol &&
            old.init_symbol == r.init_symbol && old.destroy_symbol == r.destroy_symbol;
  }
  if (!reuse) {
    std::vector<std::string> argv{r.validator_path};
    argv.insert(argv.end(), r.validator_args.begin(), r.validator_args.end());
    argv.push_back(src);
    const int code = run(argv);
    if (code != 0)
      fail(Status::ValidationFailed, "module library: validator exited with " + std::to_string(code));
    write_file_atomic(rep.stored_link_unit_path, read_file(src));
    ModuleArtifact a;
    a.module_id = r.module_id;
    a.target = r.target;
    a.artifact_sha256 = rep.artifact_sha256;
    a.link_unit_path = rep.stored_link_unit_path;
    a.validation_recipe = r.validation_recipe;
    a.validator_sha256 = rep.validator_sha256;
    a.init_symbol = r.init_symbol;
    a.execute_symbol = r.execute_symbol;
    a.destroy_symbol = r.destroy_symbol;
    a.module_abi = r.module_abi;
    a.kind = kind;
    a.validated = true;
    write_file_atomic(rep.record_path, artifact_json(a).dump());
  }
  rep.validation_reused = reuse;
  write_file_atomic(rep.active_record_path, read_file(rep.record_path));
  return rep;
}

ModuleArtifact resolve_module(const std::string& root, const std::string& id, const std::string& target) {
  if (!ident_ok(id) || !ident_ok(target)) fail(Status::InvalidArgument, "module library: bad module id or target");
  const std::string active = module_dir(root, id, target) + "/active.json";
  if (!exists(active)) fail(Status::NotFound, "module library: no active " + id + " for " + target);
  ModuleArtifact a = load_module_record(active);
  if (!a.validated) fail(Status::ModuleNotValidated, "module library: " + id + " is not validated");
  if (a.module_id != id || a.target != target) fail(Status::HashMismatch, "module library: record names another module");
  if (file_sha256_hex(a.link_unit_path) != a.artifact_sha256)
    fail(Status::HashMismatch, "module library: stored link unit of " + id + " does not match its record");
  return a;
}

// ---------------------------------------------------------------- driver compiler
namespace {
std::string c_string(const std::string& s) {
  std::string o = "\"";
  for (unsigned char c : s) {
    if (c == '"' || c == '\\') { o.push_back('\\'); o.push_back((char)c); }
    else if (c >= 32 && c < 127) o.push_back((char)c);
    else {
      char buf[8];
      std::snprintf(buf, sizeof(buf), "\\%03o", c);
      o += buf;
    }
  }
  return o + "\"";
}

// Text builder for the generated source. Integers go through std::to_string, not
// the iostream number formatting, whose locale facets have crashed inside the
// Python process this library is loaded into (another C++ runtime's facets).
struct Src {
  std::string s;
  Src& operator<<(const char* v) { s += v; return *this; }
  Src& operator<<(const std::string& v) { s += v; return *this; }
  template <typename T, typename = std::enable_if_t<std::is_integral<T>::value>>
  Src& operator<<(T v) { s += std::to_string(v); return *this; }
  const std::string& str() const { return s; }
};
}  // namespace

CompileReport compile_driver(const CompileRequest& req) {
  const std::string text = read_file(req.model_description_path);
  const ModelDescription d = parse_model_description(text);
  const Stage* st = d.stage(req.stage_name);
  if (!st) fail(Status::NotFound, "driver compiler: no stage " + req.stage_name);
  // resolve every module once
  std::map<std::string, ModuleArtifact> mods;
  std::vector<const Operation*> ops;  // all operations, program by program
  for (const auto& p : st->programs)
    for (const auto& o : p.operations) {
      ops.push_back(&o);
      if (!mods.count(o.module_id)) mods[o.module_id] = resolve_module(req.library_root, o.module_id, st->target);
    }
  Src c;
  c << "/* Model driver of " << d.model_id << " " << d.model_revision << ", stage " << st->name
    << "; generated from a model description. */\n"
    << "#include <sparkpipe_b200/model_driver.h>\n#include <stdlib.h>\n#include <string.h>\n\n";
  std::set<std::string> declared;
  for (const auto& kv : mods) {
    const ModuleArtifact& m = kv.second;
    if (declared.insert(m.init_symbol).second)
      c << "extern int32_t " << m.init_symbol << "(const char*, void**);\n";
    if (declared.insert(m.execute_symbol).second)
      c << "extern int32_t " << m.execute_symbol << "(void*, const spb_buffer*, spb_buffer*);\n";
    if (declared.insert(m.destroy_symbol).second) c << "extern void " << m.destroy_symbol << "(void*);\n";
  }
  const size_t nops = ops.size();
  c << "\n#define NOPS " << nops << "\n"
    << "typedef struct { void* state[NOPS]; uint64_t submits, completions, inflight; } drv_instance;\n"
    << "static const char* const op_config[NOPS] = {";
  for (size_t i = 0; i < nops; ++i) c << (i ? ", " : "") << c_string(ops[i]->configuration_json);
  c << "};\n\n"
    << "static void drv_destroy(void* p) {\n  drv_instance* x = (drv_instance*)p;\n  if (!x) return;\n";
  for (size_t i = nops; i-- > 0;)
    c << "  if (x->state[" << i << "]) " << mods[ops[i]->module_id].destroy_symbol << "(x->state[" << i << "]);\n";
  c << "  free(x);\n}\n\n"
    << "static int32_t drv_create(const char* cfg, void** out) {\n  (void)cfg;\n"
    << "  drv_instance* x = (drv_instance*)calloc(1, sizeof(drv_instance));\n  if (!x) return 2;\n  int32_t r;\n";
  for (size_t i = 0; i < nops; ++i)
    c << "  if ((r = " << mods[ops[i]->module_id].init_symbol << "(op_config[" << i << "], &x->state[" << i
      << "])) != 0) { drv_destroy(x); return r; }\n";
  c << "  *out = x;\n  return 0;\n}\n\n"
    << "static int32_t drv_admit(void* p, spb_admission* a) { (void)p; a->accepted = a->sequences; return 0; }\n"
    << "static int32_t drv_snapshot(void* p, spb_snapshot* s) {\n  drv_instance* x = (drv_instance*)p;\n"
    << "  s->submits = x->submits; s->completions = x->completions; s->inflight = x->inflight; s->reserved = 0;\n"
    << "  return 0;\n}\n\n"
    // operations run in order; each reads the previous one's output (ping-pong buffers of the caller's capacity)
    << "static int32_t run_chain(drv_instance* x, const int* idx, int n, const spb_buffer* in, spb_buffer* out) {\n"
    << "  x->submits++; x->inflight++;\n"
    << "  char* tmp[2] = {0, 0};\n  spb_buffer cur = *in;\n  int32_t r = 0;\n"
    << "  for (int j = 0; j < n && r == 0; ++j) {\n"
    << "    spb_buffer dst;\n"
    << "    if (j == n - 1) dst = *out;\n"
    << "    else {\n      if (!tmp[j & 1]) tmp[j & 1] = (char*)malloc(out->bytes ? out->bytes : 1);\n"
    << "      if (!tmp[j & 1]) { r = 2; break; }\n      dst.data = tmp[j & 1]; dst.bytes = out->bytes;\n    }\n"
    << "    r = op_exec(x, idx[j], &cur, &dst);\n    cur = dst;\n  }\n"
    << "  if (r == 0) out->bytes = cur.bytes;\n  free(tmp[0]); free(tmp[1]);\n"
    << "  x->inflight--; if (r == 0) x->completions++;\n  return r;\n}\n\n";
  // op_exec dispatch must precede run_chain: emit it through a forward declaration
  Src disp;
  disp << "static int32_t op_exec(drv_instance* x, int i, const spb_buffer* in, spb_buffer* out) {\n  switch (i) {\n";
  for (size_t i = 0; i < nops; ++i)
    disp << "    case " << i << ": return " << mods[ops[i]->module_id].execute_symbol << "(x->state[" << i
         << "], in, out);\n";
  disp << "  }\n  return 1;\n}\n\n";
  std::string body = c.str();
  const std::string marker = "static int32_t run_chain(";
  body.insert(body.find(marker), disp.str());
  Src t;
  t << body;
  size_t op0 = 0;
  std::vector<std::string> pnames;
  for (size_t pi = 0; pi < st->programs.size(); ++pi) {
    const Program& p = st->programs[pi];
    t << "static const int prog" << pi << "_ops[] = {";
    for (size_t j = 0; j < p.operations.size(); ++j) t << (j ? ", " : "") << op0 + j;
    t << "};\nstatic int32_t prog" << pi << "_submit(void* p, const spb_buffer* in, spb_buffer* out) {\n"
      << "  return run_chain((drv_instance*)p, prog" << pi << "_ops, " << p.operations.size() << ", in, out);\n}\n";
    const uint32_t flags = p.external_completion ? SPB_PROGRAM_EXTERNAL_COMPLETION : 0u;
    t << "static const spb_program_profile prog" << pi << "_profile = {sizeof(spb_program_profile), "
      << (flags & ~SPB_PROGRAM_EXTERNAL_COMPLETION) << "u, " << p.max_inflight << "u, 0u, 0, 0, "
      << p.scheduling.target_latency_ns << "ull, 0};\n";
    op0 += p.operations.size();
  }
  t << "\nstatic const spb_program_descriptor programs[] = {\n";
  for (size_t pi = 0; pi < st->programs.size(); ++pi) {
    const Program& p = st->programs[pi];
    const uint32_t flags = p.external_completion ? SPB_PROGRAM_EXTERNAL_COMPLETION : 0u;
    t << "  {" << p.program_id << "u, " << flags << "u, " << p.max_inflight << "u, 0u, " << c_string(p.name)
      << ", &prog" << pi << "_profile, prog" << pi << "_submit},\n";
  }
  t << "};\n";
  // the compiled-program hash covers the generated source without its own line
  const std::string source_wo_hash = t.str();
  const std::string program_sha = sha256_hex(source_wo_hash);
  t << "static const spb_model_driver_descriptor descriptor = {SPB_MODEL_DRIVER_ABI_VERSION, "
    << "sizeof(spb_model_driver_descriptor), " << c_string(d.model_id) << ", " << c_string(d.model_revision) << ", "
    << c_string(st->name) << ", " << c_string(st->target) << ", " << c_string(d.source_sha256) << ", "
    << c_string(program_sha) << ", " << st->programs.size() << "u, NOPS, programs};\n"
    << "static const spb_model_driver_interface iface = {SPB_MODEL_DRIVER_ABI_VERSION, "
    << "sizeof(spb_model_driver_interface), &descriptor, drv_create, drv_destroy, drv_admit, drv_snapshot};\n"
    << "const spb_model_driver_interface* spb_model_driver_get_interface(void) { return &iface; }\n";
  mkdirs(req.output_directory);
  CompileReport rep;
  rep.program_count = (uint32_t)st->programs.size();
  rep.operation_count = (uint32_t)nops;
  rep.link_unit_count = (uint32_t)mods.size();
  rep.model_description_sha256 = d.source_sha256;
  rep.compiled_program_sha256 = program_sha;
  const std::string base = req.output_directory + "/" + d.model_id + "." + st->name;
  rep.generated_source_path = base + ".driver.c";
  rep.driver_path = base + ".driver.so";
  rep.manifest_path = base + ".manifest.json";
  write_file_atomic(rep.generated_source_path, t.str());
  std::vector<std::string> argv{req.compiler, "-shared", "-fPIC", "-O2", "-o", rep.driver_path,
                                rep.generated_source_path};
  if (!req.include_directory.empty()) argv.push_back("-I" + req.include_directory);
  for (const auto& kv : mods) argv.push_back(kv.second.link_unit_path);
  argv.insert(argv.end(), req.extra_args.begin(), req.extra_args.end());
  const int code = run(argv);
  if (code != 0) fail(Status::CompilerError, "driver compiler: compiler exited with " + std::to_string(code));
  rep.driver_sha256 = file_sha256_hex(rep.driver_path);
  Json m = Json::make_object();
  m.set("model_id", Json::make_string(d.model_id));
  m.set("model_revision", Json::make_string(d.model_revision));
  m.set("stage", Json::make_string(st->name));
  m.set("target", Json::make_string(st->target));
  m.set("model_description_sha256", Json::make_string(d.source_sha256));
  m.set("compiled_program_sha256", Json::make_string(program_sha));
  m.set("driver_sha256", Json::make_string(rep.driver_sha256));
  Json units = Json::make_array();
  for (const auto& kv : mods) {
    Json u = Json::make_object();
    u.set("module_id", Json::make_string(kv.first));
    u.set("artifact_sha256", Json::make_string(kv.second.artifact_sha256));
    units.push(std::move(u));
  }
  m.set("link_units", std::move(units));
  write_file_atomic(rep.manifest_path, m.dump());
  return rep;
}

// ---------------------------------------------------------------- orchestrator
uint32_t Orchestrator::add_node(const std::string& id, const std::string& target) {
  if (id.empty() || target.empty()) fail(Status::InvalidArgument, "orchestrator: node id and target required");
  for (const auto& n : nodes_)
    if (n.id == id) fail(Status::Duplicate, "orchestrator: duplicate node " + id);
  nodes_.push_back(Node{id, target});
  return (uint32_t)nodes_.size() - 1;
}

uint32_t Orchestrator::attach_driver(uint32_t node, const std::string& path, const std::string& config_json) {
  if (node >= nodes_.size()) fail(Status::NotFound, "orchestrator: no such node");
  std::unique_ptr<ModelDriver> drv(ModelDriver::load(path, nodes_[node].target));
  drv->create(config_json);
  drivers_.push_back(Attached{node, std::move(drv), 0});
  return (uint32_t)drivers_.size() - 1;
}

uint32_t Orchestrator::resolve_route(const std::string& model_id, const std::string& revision, const std::string& stage,
                                     const std::string& program) const {
  for (uint32_t i = 0; i < drivers_.size(); ++i) {
    const ModelDriver& d = *drivers_[i].driver;
    DriverProgramInfo info;
    if (d.model_id() == model_id && d.model_revision() == revision && d.stage_name() == stage &&
        d.find_program(program, &info)) {
      for (uint32_t r = 0; r < routes_.size(); ++r)
        if (routes_[r].driver == i && routes_[r].program_id == info.program_id) return r;
      routes_.push_back(Route{i, info.program_id});
      return (uint32_t)routes_.size() - 1;
    }
  }
  fail(Status::RouteNotFound, "orchestrator: no driver serves " + model_id + "@" + revision + " " + stage + "/" + program);
}

std::string Orchestrator::submit(uint32_t route, const std::string& input, size_t output_capacity) {
  if (route >= routes_.size()) fail(Status::NotFound, "orchestrator: no such route");
  Attached& a = drivers_[routes_[route].driver];
  ++a.outstanding;
  try {
    std::string out = a.driver->submit(routes_[route].program_id, input, output_capacity);
    --a.outstanding;
    return out;
  } catch (...) {
    --a.outstanding;
    throw;
  }
}

uint64_t Orchestrator::outstanding(uint32_t driver) const {
  if (driver >= drivers_.size()) fail(Status::NotFound, "orchestrator: no such driver");
  return drivers_[driver].outstanding;
}

spb_snapshot Orchestrator::snapshot(uint32_t driver) {
  if (driver >= drivers_.size()) fail(Status::NotFound, "orchestrator: no such driver");
  return drivers_[driver].driver->snapshot();
}

}  // namespace ctl
}  // namespace spc
