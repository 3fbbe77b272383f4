#include "driver_loader.h"

#include <dlfcn.h>

#include <cctype>
#include <cstring>

namespace spc {

namespace {
bool text_ok(const char* s) { return s && s[0] != '\0'; }

void validate_program(const spb_program_descriptor& p, uint32_t index) {
  const std::string where = "driver: program " + std::to_string(index);
  if (p.program_id == 0 || !text_ok(p.name) || !p.submit || p.max_inflight == 0 || p.reserved != 0 || !p.profile ||
      (p.flags & ~SPB_PROGRAM_KNOWN_FLAGS))
    fail(Status::AbiMismatch, where + ": bad program descriptor");
  const spb_program_profile& f = *p.profile;
  if (f.descriptor_bytes < sizeof(spb_program_profile) || f.reserved != 0 || f.max_inflight != p.max_inflight ||
      f.profile_flags != (p.flags & ~SPB_PROGRAM_EXTERNAL_COMPLETION) || (f.profile_flags & ~SPB_PROGRAM_KNOWN_FLAGS))
    fail(Status::AbiMismatch, where + ": profile disagrees with its program");
  const std::string name = p.name;
  if ((p.flags & SPB_PROGRAM_NO_HOST_STAGING) && f.host_staging_bytes_ceiling != 0)
    fail(Status::ValidationFailed, "driver: program " + name + " claims no host staging but stages bytes");
  if ((p.flags & SPB_PROGRAM_NO_DEVICE_MEMCPY) && f.device_memcpy_bytes_ceiling != 0)
    fail(Status::ValidationFailed, "driver: program " + name + " claims no device memcpy but copies bytes");
  if ((p.flags & SPB_PROGRAM_VALIDATED_LATENCY) && f.validated_latency_ns == 0)
    fail(Status::ValidationFailed, "driver: program " + name + " claims a validated latency without one");
  if ((p.flags & SPB_PROGRAM_PRIVATE_QUEUES) && f.private_queue_count == 0)
    fail(Status::ValidationFailed, "driver: program " + name + " claims private queues without any");
}
}  // namespace

bool sha256_hex_is_valid(const char* s) {
  if (!s) return false;
  size_t n = 0;
  for (; s[n]; ++n)
    if (!std::isxdigit(static_cast<unsigned char>(s[n]))) return false;
  return n == 64;
}

void validate_driver_interface(const spb_model_driver_interface* iface, const std::string& expected_target) {
  if (!iface || iface->abi_version != SPB_MODEL_DRIVER_ABI_VERSION ||
      iface->interface_bytes < sizeof(spb_model_driver_interface) || !iface->descriptor || !iface->create ||
      !iface->destroy || !iface->admit || !iface->snapshot)
    fail(Status::AbiMismatch, "driver: bad interface");
  const spb_model_driver_descriptor& d = *iface->descriptor;
  if (d.abi_version != SPB_MODEL_DRIVER_ABI_VERSION || d.descriptor_bytes < sizeof(spb_model_driver_descriptor) ||
      !text_ok(d.model_id) || !text_ok(d.model_revision) || !text_ok(d.stage_name) || !text_ok(d.target) ||
      !sha256_hex_is_valid(d.model_description_sha256) || !sha256_hex_is_valid(d.compiled_program_sha256) ||
      d.program_count == 0 || d.module_instance_count == 0 || !d.programs)
    fail(Status::AbiMismatch, "driver: bad descriptor");
  if (!expected_target.empty() && expected_target != d.target)
    fail(Status::TargetMismatch, std::string("driver: compiled for ") + d.target + ", node is " + expected_target);
  for (uint32_t i = 0; i < d.program_count; ++i) {
    validate_program(d.programs[i], i);
    for (uint32_t j = 0; j < i; ++j)
      if (d.programs[j].program_id == d.programs[i].program_id || !std::strcmp(d.programs[j].name, d.programs[i].name))
        fail(Status::Duplicate, "driver: duplicate program id or name");
  }
}

ModelDriver* ModelDriver::load(const std::string& path, const std::string& expected_target) {
  if (path.empty()) fail(Status::InvalidArgument, "driver: empty path");
  void* h = dlopen(path.c_str(), RTLD_NOW | RTLD_LOCAL);
  if (!h) {
    const char* e = dlerror();
    fail(Status::DriverLoadError, "driver: cannot load " + path + ": " + (e ? e : "unknown error"));
  }
  auto get = reinterpret_cast<spb_get_interface_fn>(dlsym(h, SPB_MODEL_DRIVER_SYMBOL));
  if (!get) {
    dlclose(h);
    fail(Status::DriverLoadError, "driver: " + path + " exports no " SPB_MODEL_DRIVER_SYMBOL);
  }
  const spb_model_driver_interface* iface = get();
  try {
    validate_driver_interface(iface, expected_target);
  } catch (...) {
    dlclose(h);
    throw;
  }
  return new ModelDriver(h, iface);
}

ModelDriver::~ModelDriver() {
  if (instance_) iface_->destroy(instance_);
  if (handle_) dlclose(handle_);
}

std::string ModelDriver::model_id() const { return iface_->descriptor->model_id; }
std::string ModelDriver::model_revision() const { return iface_->descriptor->model_revision; }
std::string ModelDriver::stage_name() const { return iface_->descriptor->stage_name; }
std::string ModelDriver::target() const { return iface_->descriptor->target; }
std::string ModelDriver::model_description_sha256() const { return iface_->descriptor->model_description_sha256; }
std::string ModelDriver::compiled_program_sha256() const { return iface_->descriptor->compiled_program_sha256; }
uint32_t ModelDriver::module_instance_count() const { return iface_->descriptor->module_instance_count; }

std::vector<DriverProgramInfo> ModelDriver::programs() const {
  std::vector<DriverProgramInfo> v;
  const spb_model_driver_descriptor& d = *iface_->descriptor;
  for (uint32_t i = 0; i < d.program_count; ++i) {
    const spb_program_descriptor& p = d.programs[i];
    v.push_back(DriverProgramInfo{p.program_id, p.flags, p.max_inflight, p.name});
  }
  return v;
}

bool ModelDriver::find_program(const std::string& name, DriverProgramInfo* out) const {
  for (const DriverProgramInfo& p : programs())
    if (p.name == name) {
      if (out) *out = p;
      return true;
    }
  return false;
}

const spb_program_descriptor* ModelDriver::program(uint32_t id) const {
  const spb_model_driver_descriptor& d = *iface_->descriptor;
  for (uint32_t i = 0; i < d.program_count; ++i)
    if (d.programs[i].program_id == id) return &d.programs[i];
  fail(Status::NotFound, "driver: no program " + std::to_string(id));
}

void ModelDriver::create(const std::string& config_json) {
  if (instance_) fail(Status::Busy, "driver: instance already created");
  void* inst = nullptr;
  const int32_t r = iface_->create(config_json.c_str(), &inst);
  if (r != 0 || !inst) fail(Status(r ? uint32_t(r) : uint32_t(Status::InternalError)), "driver: create failed");
  instance_ = inst;
}

void ModelDriver::destroy() {
  if (!instance_) return;
  iface_->destroy(instance_);
  instance_ = nullptr;
}

uint32_t ModelDriver::admit(uint32_t program_id, uint32_t sequences, uint32_t tokens) {
  if (!instance_) fail(Status::InvalidArgument, "driver: no instance");
  program(program_id);
  spb_admission a{program_id, sequences, tokens, 0};
  const int32_t r = iface_->admit(instance_, &a);
  if (r != 0) fail(Status(uint32_t(r)), "driver: admission refused");
  return a.accepted;
}

spb_snapshot ModelDriver::snapshot() {
  if (!instance_) fail(Status::InvalidArgument, "driver: no instance");
  spb_snapshot s{};
  const int32_t r = iface_->snapshot(instance_, &s);
  if (r != 0) fail(Status(uint32_t(r)), "driver: snapshot failed");
  return s;
}

std::string ModelDriver::submit(uint32_t program_id, const std::string& input, size_t output_capacity) {
  if (!instance_) fail(Status::InvalidArgument, "driver: no instance");
  const spb_program_descriptor* p = program(program_id);
  std::string out(output_capacity, '\0');
  spb_buffer in{const_cast<char*>(input.data()), input.size()};
  spb_buffer o{&out[0], out.size()};
  const int32_t r = p->submit(instance_, &in, &o);
  if (r != 0) fail(Status(uint32_t(r)), "driver: submit failed");
  if (o.bytes > out.size()) fail(Status::CapacityExceeded, "driver: output larger than its buffer");
  out.resize(o.bytes);
  return out;
}

std::vector<std::pair<std::string, uint64_t>> driver_abi_layout() {
#define L(expr) {#expr, uint64_t(expr)}
  return {
      L(sizeof(spb_buffer)),
      L(sizeof(spb_program_profile)),
      L(offsetof(spb_program_profile, host_staging_bytes_ceiling)),
      L(offsetof(spb_program_profile, validated_latency_ns)),
      L(sizeof(spb_program_descriptor)),
      L(offsetof(spb_program_descriptor, name)),
      L(offsetof(spb_program_descriptor, profile)),
      L(offsetof(spb_program_descriptor, submit)),
      L(sizeof(spb_model_driver_descriptor)),
      L(offsetof(spb_model_driver_descriptor, model_id)),
      L(offsetof(spb_model_driver_descriptor, target)),
      L(offsetof(spb_model_driver_descriptor, program_count)),
      L(offsetof(spb_model_driver_descriptor, programs)),
      L(sizeof(spb_admission)),
      L(sizeof(spb_snapshot)),
      L(sizeof(spb_model_driver_interface)),
      L(offsetof(spb_model_driver_interface, descriptor)),
      L(offsetof(spb_model_driver_interface, snapshot)),
      L(alignof(spb_model_driver_descriptor)),
      L(alignof(spb_program_profile)),
  };
#undef L
}

}  // namespace spc
