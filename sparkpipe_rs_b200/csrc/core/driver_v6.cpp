#include "driver_v6.h"

#include <dlfcn.h>

#include <algorithm>
#include <chrono>
#include <cstring>

#include "driver_loader.h"  // sha256_hex_is_valid

namespace spc {
namespace v6 {

namespace {

bool has_text(const char* s) { return s != nullptr && *s != '\0'; }

void check_program(const sp6_program_descriptor& p, uint32_t index) {
  const std::string at = "v6 driver: program " + std::to_string(index);
  if (p.program_id == 0 || !has_text(p.name) || p.submit == nullptr || p.max_inflight == 0 || p.reserved != 0 ||
      p.profile == nullptr || (p.flags & ~SP6_PROGRAM_KNOWN_FLAGS) != 0)
    fail(Status::AbiMismatch, at + ": malformed descriptor");
  const sp6_program_profile& f = *p.profile;
  const uint32_t expect_flags = p.flags & ~SP6_PROGRAM_EXTERNAL_COMPLETION;
  if (f.descriptor_bytes < sizeof(sp6_program_profile) || f.reserved != 0 || f.max_inflight != p.max_inflight ||
      f.profile_flags != expect_flags)
    fail(Status::AbiMismatch, at + ": profile does not match its program");
  // a claim in the flags must be backed by the profile's numbers
  struct Claim {
    uint32_t flag;
    bool broken;
    const char* what;
  };
  const Claim claims[] = {
      {SP6_PROGRAM_NO_HOST_STAGING, f.host_staging_bytes_per_submit_ceiling != 0, "no host staging"},
      {SP6_PROGRAM_NO_DEVICE_MEMCPY, f.device_memcpy_bytes_per_submit_ceiling != 0, "no device memcpy"},
      {SP6_PROGRAM_VALIDATED_LATENCY, f.validated_latency_ns == 0, "a validated latency"},
      {SP6_PROGRAM_PRIVATE_QUEUE_PRESSURE, f.private_queue_count == 0, "private queue pressure"},
  };
  for (const Claim& c : claims)
    if ((p.flags & c.flag) && c.broken)
      fail(Status::ValidationFailed, std::string("v6 driver: program ") + p.name + " claims " + c.what +
                                         " that its profile contradicts");
}

}  // namespace

void validate_interface(const sp6_interface* iface, const std::string& expected_target) {
  if (iface == nullptr || iface->abi_version != SP6_ABI_VERSION || iface->interface_bytes < sizeof(sp6_interface) ||
      iface->descriptor == nullptr || !iface->create || !iface->destroy || !iface->admit || !iface->snapshot)
    fail(Status::AbiMismatch, "v6 driver: interface");
  const sp6_driver_descriptor& d = *iface->descriptor;
  const bool identity_ok = has_text(d.model_id) && has_text(d.model_revision) && has_text(d.stage_name) &&
                           has_text(d.target) && sha256_hex_is_valid(d.model_description_sha256) &&
                           sha256_hex_is_valid(d.compiled_program_sha256);
  if (d.abi_version != SP6_ABI_VERSION || d.descriptor_bytes < sizeof(sp6_driver_descriptor) || !identity_ok ||
      d.program_count == 0 || d.module_instance_count == 0 || d.programs == nullptr)
    fail(Status::AbiMismatch, "v6 driver: descriptor");
  if (!expected_target.empty() && expected_target != d.target)
    fail(Status::TargetMismatch, std::string("v6 driver: built for ") + d.target + ", node is " + expected_target);
  std::vector<std::pair<uint32_t, std::string>> seen;
  for (uint32_t i = 0; i < d.program_count; ++i) {
    check_program(d.programs[i], i);
    const std::string name = d.programs[i].name;
    for (const auto& s : seen)
      if (s.first == d.programs[i].program_id || s.second == name)
        fail(Status::Duplicate, "v6 driver: program id or name used twice");
    seen.emplace_back(d.programs[i].program_id, name);
  }
}

std::unique_ptr<Driver> Driver::load(const std::string& path, const std::string& expected_target) {
  if (path.empty()) fail(Status::InvalidArgument, "v6 driver: empty path");
  void* h = dlopen(path.c_str(), RTLD_NOW | RTLD_LOCAL);
  if (!h) fail(Status::DriverLoadError, std::string("v6 driver: cannot open ") + path + ": " + dlerror());
  auto get = reinterpret_cast<sp6_get_interface_fn>(dlsym(h, SP6_INTERFACE_SYMBOL));
  if (!get) {
    dlclose(h);
    fail(Status::DriverLoadError, "v6 driver: " + path + " exports no " SP6_INTERFACE_SYMBOL);
  }
  const sp6_interface* iface = get();
  try {
    validate_interface(iface, expected_target);
  } catch (...) {
    dlclose(h);
    throw;
  }
  return std::unique_ptr<Driver>(new Driver(h, iface));
}

Driver::~Driver() {
  destroy();
  if (handle_) dlclose(handle_);
}

std::vector<ProgramInfo> Driver::programs() const {
  std::vector<ProgramInfo> out;
  const sp6_driver_descriptor& d = descriptor();
  for (uint32_t i = 0; i < d.program_count; ++i) {
    ProgramInfo p;
    p.program_id = d.programs[i].program_id;
    p.flags = d.programs[i].flags;
    p.max_inflight = d.programs[i].max_inflight;
    p.name = d.programs[i].name;
    p.profile = *d.programs[i].profile;
    out.push_back(std::move(p));
  }
  return out;
}

const sp6_program_descriptor* Driver::program(uint32_t id) const {
  const sp6_driver_descriptor& d = descriptor();
  for (uint32_t i = 0; i < d.program_count; ++i)
    if (d.programs[i].program_id == id) return &d.programs[i];
  return nullptr;
}

void Driver::on_completion(void* ctx, const sp6_completion* c) {
  auto* self = static_cast<Driver*>(ctx);
  if (!self || !c) return;
  Completion r;
  r.request_id = c->request_id;
  r.sequence_id = c->sequence_id;
  r.sequence_position = c->sequence_position;
  r.program_id = c->program_id;
  r.driver_dispatch_slot = c->driver_dispatch_slot;
  r.accepted_token_count = c->accepted_token_count;
  r.completion_flags = c->completion_flags;
  if (c->completion_flags & SP6_COMPLETION_FLAG_TOKEN_IDS)
    r.token_ids.assign(c->token_ids, c->token_ids + std::min(c->token_count, SP6_COMPLETION_TOKENS));
  if (c->completion_flags & SP6_COMPLETION_FLAG_DRAFT_TOKEN_IDS)
    r.draft_token_ids.assign(c->draft_token_ids,
                             c->draft_token_ids + std::min(c->draft_token_count, SP6_COMPLETION_DRAFT_TOKENS));
  r.status = c->status;
  r.residency = c->residency;
  r.queue_delay_ns = c->queue_delay_ns;
  r.service_time_ns = c->service_time_ns;
  r.device_memcpy_bytes = c->device_memcpy_bytes;
  r.host_staging_bytes = c->host_staging_bytes;
  {
    std::lock_guard<std::mutex> lk(self->mu_);
    // the frame of this request is no longer referenced by the driver
    for (auto it = self->inflight_.begin(); it != self->inflight_.end(); ++it)
      if (it->frame.request_id == r.request_id && it->frame.program_id == r.program_id) {
        self->inflight_.erase(it);
        break;
      }
    self->done_.push_back(std::move(r));
  }
  self->cv_.notify_all();
}

void Driver::on_wake(void* ctx) {
  auto* self = static_cast<Driver*>(ctx);
  if (!self) return;
  {
    std::lock_guard<std::mutex> lk(self->mu_);
    ++self->wakes_;
  }
  self->cv_.notify_all();
}

void Driver::create(const std::string& node_id, const std::string& node_target, uint64_t node_context) {
  if (instance_) fail(Status::Busy, "v6 driver: an instance exists");
  node_id_ = node_id;
  node_target_ = node_target;
  sp6_create_request req{};
  req.node_id = node_id_.c_str();
  req.node_target = node_target_.c_str();
  req.node_context = reinterpret_cast<void*>(uintptr_t(node_context));
  req.completion_function = &Driver::on_completion;
  req.completion_context = this;
  req.wake_function = &Driver::on_wake;
  req.wake_context = this;
  void* inst = nullptr;
  const sp6_status s = iface_->create(&req, &inst);
  if (s != 0 || inst == nullptr) fail(s ? Status(s) : Status::DriverLoadError, "v6 driver: create failed");
  instance_ = inst;
}

void Driver::destroy() {
  if (!instance_) return;
  iface_->destroy(instance_);
  instance_ = nullptr;
  std::lock_guard<std::mutex> lk(mu_);
  inflight_.clear();
}

sp6_admission_decision Driver::admit(const sp6_admission_request& request) {
  if (!instance_) fail(Status::InvalidArgument, "v6 driver: no instance");
  if (!program(request.program_id)) fail(Status::NotFound, "v6 driver: unknown program");
  sp6_admission_request r = request;
  r.descriptor_bytes = sizeof(sp6_admission_request);
  sp6_admission_decision d{};
  d.descriptor_bytes = sizeof(sp6_admission_decision);
  const sp6_status s = iface_->admit(instance_, &r, &d);
  if (s != 0) fail(Status(s), "v6 driver: admit failed");
  return d;
}

Status Driver::submit(uint32_t program_id, const FrameArgs& a) {
  if (!instance_) fail(Status::InvalidArgument, "v6 driver: no instance");
  const sp6_program_descriptor* p = program(program_id);
  if (!p) fail(Status::NotFound, "v6 driver: unknown program");
  OwnedFrame* of;
  {
    std::lock_guard<std::mutex> lk(mu_);
    inflight_.emplace_back();
    of = &inflight_.back();
  }
  of->buffers = a.buffers;
  sp6_frame& f = of->frame;
  f.request_id = a.request_id;
  f.sequence_id = a.sequence_id;
  f.sequence_position = a.sequence_position;
  f.deadline_time_ns = a.deadline_time_ns;
  f.active_slot_count = a.active_slot_count;
  f.new_token_count = a.new_token_count;
  f.priority = a.priority;
  f.flags = a.flags;
  f.driver_dispatch_slot = a.driver_dispatch_slot;
  f.program_id = program_id;
  f.driver_dispatch_generation = a.driver_dispatch_generation;
  f.driver_dispatch_cookie0 = a.driver_dispatch_cookie0;
  f.driver_dispatch_cookie1 = a.driver_dispatch_cookie1;
  f.execution_stream = reinterpret_cast<void*>(uintptr_t(a.execution_stream));
  f.buffers = of->buffers.empty() ? nullptr : of->buffers.data();
  f.buffer_count = uint32_t(of->buffers.size());
  std::copy(a.scalar, a.scalar + SP6_SCALARS, f.scalar);
  f.residency = a.residency;
  f.user_context = nullptr;
  f.completion_function = &Driver::on_completion;
  f.completion_context = this;
  const sp6_status s = p->submit(instance_, &f);
  if (s != 0) {
    // refused: the driver keeps no reference to the frame
    std::lock_guard<std::mutex> lk(mu_);
    for (auto it = inflight_.begin(); it != inflight_.end(); ++it)
      if (&*it == of) {
        inflight_.erase(it);
        break;
      }
  }
  return Status(s);
}

std::vector<Completion> Driver::poll(size_t max, int timeout_ms) {
  std::unique_lock<std::mutex> lk(mu_);
  if (done_.empty() && timeout_ms > 0)
    cv_.wait_for(lk, std::chrono::milliseconds(timeout_ms), [&] { return !done_.empty(); });
  std::vector<Completion> out;
  while (!done_.empty() && out.size() < max) {
    out.push_back(std::move(done_.front()));
    done_.pop_front();
  }
  return out;
}

sp6_runtime_snapshot Driver::snapshot(uint32_t program_id) {
  if (!instance_) fail(Status::InvalidArgument, "v6 driver: no instance");
  sp6_runtime_snapshot s{};
  s.descriptor_bytes = sizeof(sp6_runtime_snapshot);
  const sp6_status st = iface_->snapshot(instance_, program_id, &s);
  if (st != 0) fail(Status(st), "v6 driver: snapshot failed");
  return s;
}

uint64_t Driver::wakes() const {
  std::lock_guard<std::mutex> lk(mu_);
  return wakes_;
}

size_t Driver::frames_in_flight() const {
  std::lock_guard<std::mutex> lk(mu_);
  return inflight_.size();
}

std::vector<std::pair<std::string, uint64_t>> abi_layout() {
#define SP6_SIZE(T) {"sizeof(" #T ")", sizeof(T)}
#define SP6_OFF(T, F) {"offsetof(" #T "," #F ")", offsetof(T, F)}
  return {SP6_SIZE(sp6_buffer),
          SP6_SIZE(sp6_residency),
          SP6_SIZE(sp6_completion),
          SP6_OFF(sp6_completion, token_ids),
          SP6_OFF(sp6_completion, status),
          SP6_OFF(sp6_completion, residency),
          SP6_SIZE(sp6_frame),
          SP6_OFF(sp6_frame, execution_stream),
          SP6_OFF(sp6_frame, scalar),
          SP6_OFF(sp6_frame, completion_function),
          SP6_SIZE(sp6_program_profile),
          SP6_OFF(sp6_program_profile, private_queue_count),
          SP6_SIZE(sp6_admission_request),
          SP6_OFF(sp6_admission_request, residency),
          SP6_SIZE(sp6_admission_decision),
          SP6_OFF(sp6_admission_decision, private_queue_pressure),
          SP6_SIZE(sp6_runtime_snapshot),
          SP6_SIZE(sp6_create_request),
          SP6_SIZE(sp6_program_descriptor),
          SP6_OFF(sp6_program_descriptor, submit),
          SP6_SIZE(sp6_driver_descriptor),
          SP6_OFF(sp6_driver_descriptor, programs),
          SP6_SIZE(sp6_interface),
          SP6_OFF(sp6_interface, snapshot)};
#undef SP6_SIZE
#undef SP6_OFF
}

}  // namespace v6
}  // namespace spc
