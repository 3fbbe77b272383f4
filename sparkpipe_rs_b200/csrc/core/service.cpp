#include "service.h"

#include <algorithm>

#include "json.h"
#include "text.h"

namespace spc {
namespace svc {

namespace {
const uint8_t* u8(const std::string& s) { return reinterpret_cast<const uint8_t*>(s.data()); }

std::string body_prefix(size_t bytes) {
  std::string b(bytes, '\0');
  put_u32(reinterpret_cast<uint8_t*>(&b[0]), kAbiVersion);
  put_u32(reinterpret_cast<uint8_t*>(&b[4]), uint32_t(bytes));
  return b;
}

void check_body_prefix(const std::string& body, size_t bytes) {
  if (body.size() < bytes || get_u32(u8(body)) != kAbiVersion || get_u32(u8(body) + 4) != bytes)
    fail(Status::InvalidArgument, "frame: bad body prefix");
}

std::string frame(uint32_t kind, uint32_t flags, uint64_t client_id, uint64_t creq, const std::string& body) {
  FrameHeader h;
  h.kind = kind;
  h.flags = flags;
  h.body_bytes = uint32_t(body.size());
  h.client_id = client_id;
  h.client_request_id = creq;
  return serialize_header(h) + body;
}
}  // namespace

// ------------------------------------------------------------------ frame codec
std::string serialize_header(const FrameHeader& h) {
  std::string b(kHeaderBytes, '\0');
  uint8_t* p = reinterpret_cast<uint8_t*>(&b[0]);
  put_u32(p, kFrameMagic);
  put_u32(p + 4, kAbiVersion);
  put_u32(p + 8, uint32_t(kHeaderBytes));
  put_u32(p + 12, h.kind);
  put_u32(p + 16, h.flags);
  put_u32(p + 20, h.body_bytes);
  put_u64(p + 24, h.client_id);
  put_u64(p + 32, h.client_request_id);
  return b;
}

FrameHeader parse_header(const std::string& bytes) {
  if (bytes.size() < kHeaderBytes) fail(Status::InvalidArgument, "frame: short header");
  const uint8_t* p = u8(bytes);
  if (get_u32(p) != kFrameMagic || get_u32(p + 4) != kAbiVersion || get_u32(p + 8) != kHeaderBytes)
    fail(Status::InvalidArgument, "frame: bad magic, abi version or header size");
  FrameHeader h;
  h.kind = get_u32(p + 12);
  h.flags = get_u32(p + 16);
  h.body_bytes = get_u32(p + 20);
  h.client_id = get_u64(p + 24);
  h.client_request_id = get_u64(p + 32);
  return h;
}

void validate_header(const FrameHeader& h, uint32_t max_body_bytes) {
  const uint32_t limit = max_body_bytes ? max_body_bytes : kMaxFrameBodyBytes;
  if (h.body_bytes > limit) fail(Status::CapacityExceeded, "frame: body too large");
  switch (h.kind) {
    case kFrameSubmitText: case kFrameSubmitTokenIds: case kFrameCancel: case kFramePing:
    case kFrameEvent: case kFrameSubmitAck: case kFrameError: case kFramePong:
      return;
    default:
      fail(Status::InvalidArgument, "frame: unknown kind");
  }
}

std::string build_event_frame(const ServiceEvent& e) {
  std::string b = body_prefix(kEventBodyBytes);
  uint8_t* p = reinterpret_cast<uint8_t*>(&b[0]);
  put_u32(p + 8, e.kind);
  put_u32(p + 12, e.flags);
  put_u32(p + 16, e.status);
  put_u32(p + 20, e.token_id);
  put_u32(p + 24, e.token_index);
  put_u32(p + 28, e.token_count);
  put_u32(p + 32, e.prompt_token_offset);
  put_u32(p + 36, e.prompt_token_count);
  put_u32(p + 40, e.dispatch_kind);
  put_u32(p + 44, e.dispatch_flags);
  put_u64(p + 48, e.client_id);
  put_u64(p + 56, e.client_request_id);
  put_u64(p + 64, e.serving_request_id);
  put_u64(p + 72, e.sequence_id);
  put_u64(p + 80, e.serving_request_handle);
  return frame(kFrameEvent, 0, e.client_id, e.client_request_id, b);
}

ServiceEvent parse_event_body(const std::string& body) {
  check_body_prefix(body, kEventBodyBytes);
  const uint8_t* p = u8(body);
  ServiceEvent e;
  e.kind = get_u32(p + 8);
  e.flags = get_u32(p + 12);
  e.status = get_u32(p + 16);
  e.token_id = get_u32(p + 20);
  e.token_index = get_u32(p + 24);
  e.token_count = get_u32(p + 28);
  e.prompt_token_offset = get_u32(p + 32);
  e.prompt_token_count = get_u32(p + 36);
  e.dispatch_kind = get_u32(p + 40);
  e.dispatch_flags = get_u32(p + 44);
  e.client_id = get_u64(p + 48);
  e.client_request_id = get_u64(p + 56);
  e.serving_request_id = get_u64(p + 64);
  e.sequence_id = get_u64(p + 72);
  e.serving_request_handle = get_u64(p + 80);
  return e;
}

SubmitRequest parse_submit_text_frame(const FrameHeader& h, const std::string& body) {
  validate_header(h);
  if (h.kind != kFrameSubmitText) fail(Status::InvalidArgument, "frame: not a submit-text frame");
  check_body_prefix(body, kSubmitTextBodyBytes);
  const uint8_t* p = u8(body);
  const uint32_t n = get_u32(p + 28);
  if (n == 0 || n > kMaxTextBytes) fail(Status::InvalidArgument, "frame: bad text length");
  if (body.size() != kSubmitTextBodyBytes + n || h.body_bytes != body.size())
    fail(Status::InvalidArgument, "frame: body size mismatch");
  SubmitRequest r;
  r.flags = h.flags;
  r.priority = get_u32(p + 8);
  r.thinking_budget = get_u32(p + 12);
  r.output_budget = get_u32(p + 16);
  r.max_prefill_tokens_per_step = get_u32(p + 20);
  r.tokenizer_flags = get_u32(p + 24);
  r.client_id = h.client_id;
  r.client_request_id = h.client_request_id;
  r.sequence_id = get_u64(p + 32);
  r.text = body.substr(kSubmitTextBodyBytes);
  return r;
}

SubmitRequest parse_submit_tokens_frame(const FrameHeader& h, const std::string& body) {
  validate_header(h);
  if (h.kind != kFrameSubmitTokenIds) fail(Status::InvalidArgument, "frame: not a submit-token-ids frame");
  check_body_prefix(body, kSubmitTokensBodyBytes);
  const uint8_t* p = u8(body);
  const uint32_t n = get_u32(p + 24);
  if (n == 0 || n > kMaxTokenFrameCount) fail(Status::InvalidArgument, "frame: bad token count");
  if (body.size() != kSubmitTokensBodyBytes + size_t(n) * 4 || h.body_bytes != body.size())
    fail(Status::InvalidArgument, "frame: body size mismatch");
  SubmitRequest r;
  r.flags = h.flags;
  r.priority = get_u32(p + 8);
  r.thinking_budget = get_u32(p + 12);
  r.output_budget = get_u32(p + 16);
  r.max_prefill_tokens_per_step = get_u32(p + 20);
  r.client_id = h.client_id;
  r.client_request_id = h.client_request_id;
  r.sequence_id = get_u64(p + 32);
  r.token_ids.resize(n);
  for (uint32_t i = 0; i < n; ++i) r.token_ids[i] = get_u32(p + kSubmitTokensBodyBytes + 4 * i);
  return r;
}

uint64_t parse_cancel_frame(const FrameHeader& h, const std::string& body) {
  validate_header(h);
  if (h.kind != kFrameCancel || body.size() != kCancelBodyBytes || h.body_bytes != body.size())
    fail(Status::InvalidArgument, "frame: bad cancel frame");
  check_body_prefix(body, kCancelBodyBytes);
  const uint64_t in_body = get_u64(u8(body) + 16);
  const uint64_t creq = in_body ? in_body : h.client_request_id;
  if (!creq) fail(Status::InvalidArgument, "frame: cancel without a request id");
  return creq;
}

std::string build_submit_text_frame(const SubmitRequest& r) {
  std::string b = body_prefix(kSubmitTextBodyBytes);
  uint8_t* p = reinterpret_cast<uint8_t*>(&b[0]);
  put_u32(p + 8, r.priority);
  put_u32(p + 12, r.thinking_budget);
  put_u32(p + 16, r.output_budget);
  put_u32(p + 20, r.max_prefill_tokens_per_step);
  put_u32(p + 24, r.tokenizer_flags);
  put_u32(p + 28, uint32_t(r.text.size()));
  put_u64(p + 32, r.sequence_id);
  return frame(kFrameSubmitText, r.flags, r.client_id, r.client_request_id, b + r.text);
}

std::string build_submit_tokens_frame(const SubmitRequest& r) {
  std::string b = body_prefix(kSubmitTokensBodyBytes);
  b.resize(kSubmitTokensBodyBytes + 4 * r.token_ids.size());
  uint8_t* p = reinterpret_cast<uint8_t*>(&b[0]);
  put_u32(p + 8, r.priority);
  put_u32(p + 12, r.thinking_budget);
  put_u32(p + 16, r.output_budget);
  put_u32(p + 20, r.max_prefill_tokens_per_step);
  put_u32(p + 24, uint32_t(r.token_ids.size()));
  put_u64(p + 32, r.sequence_id);
  for (size_t i = 0; i < r.token_ids.size(); ++i) put_u32(p + kSubmitTokensBodyBytes + 4 * i, r.token_ids[i]);
  return frame(kFrameSubmitTokenIds, r.flags, r.client_id, r.client_request_id, b);
}

std::string build_cancel_frame(uint64_t client_id, uint64_t creq) {
  std::string b = body_prefix(kCancelBodyBytes);
  put_u64(reinterpret_cast<uint8_t*>(&b[16]), creq);
  return frame(kFrameCancel, 0, client_id, creq, b);
}

std::string build_ping_frame(uint64_t client_id, uint64_t cookie) {
  return frame(kFramePing, 0, client_id, cookie, "");
}
std::string build_pong_frame(uint64_t client_id, uint64_t cookie) {
  return frame(kFramePong, 0, client_id, cookie, "");
}

std::string build_ack_frame(const SubmitResult& r) {
  std::string b = body_prefix(kAckBodyBytes);
  uint8_t* p = reinterpret_cast<uint8_t*>(&b[0]);
  put_u32(p + 8, r.prompt_token_count);
  put_u32(p + 12, r.required_token_capacity);
  put_u32(p + 16, r.thinking_budget);
  put_u32(p + 20, r.output_budget);
  put_u64(p + 24, r.client_id);
  put_u64(p + 32, r.client_request_id);
  put_u64(p + 40, r.serving_request_id);
  put_u64(p + 48, r.sequence_id);
  put_u64(p + 56, r.serving_request_handle);
  return frame(kFrameSubmitAck, 0, r.client_id, r.client_request_id, b);
}

SubmitResult parse_ack_body(const std::string& body) {
  check_body_prefix(body, kAckBodyBytes);
  const uint8_t* p = u8(body);
  SubmitResult r;
  r.prompt_token_count = get_u32(p + 8);
  r.required_token_capacity = get_u32(p + 12);
  r.thinking_budget = get_u32(p + 16);
  r.output_budget = get_u32(p + 20);
  r.client_id = get_u64(p + 24);
  r.client_request_id = get_u64(p + 32);
  r.serving_request_id = get_u64(p + 40);
  r.sequence_id = get_u64(p + 48);
  r.serving_request_handle = get_u64(p + 56);
  return r;
}

std::string build_error_frame(uint64_t client_id, uint64_t creq, Status s) {
  std::string b = body_prefix(kErrorBodyBytes);
  put_u32(reinterpret_cast<uint8_t*>(&b[8]), uint32_t(s));
  return frame(kFrameError, 0, client_id, creq, b);
}

// ------------------------------------------------------------------ runtime
ServiceRuntime::ServiceRuntime(const ServiceConfig& cfg) : cfg_(cfg) {
  if (!cfg_.flags) cfg_.flags = kCfgDefaultFlags;
  if (!cfg_.request_id_base) cfg_.request_id_base = kDefaultRequestIdBase;
  if (!cfg_.client_capacity || !cfg_.request_capacity || !cfg_.event_capacity)
    fail(Status::InvalidArgument, "service: capacities must be non-zero");
  next_request_ = cfg_.request_id_base;
  st_.event_capacity = cfg_.event_capacity;
}

uint64_t ServiceRuntime::register_client(uint64_t cookie) {
  std::lock_guard<std::mutex> g(mu_);
  if (clients_.size() >= cfg_.client_capacity) fail(Status::CapacityExceeded, "service: client table full");
  const uint64_t id = next_client_++;
  if (!next_client_) next_client_ = 1;
  clients_[id].cookie = cookie;
  ServiceEvent e;
  e.kind = kEvClientConnected;
  e.client_id = id;
  push_locked(e);
  return id;
}

bool ServiceRuntime::has_client(uint64_t client_id) const {
  std::lock_guard<std::mutex> g(mu_);
  return clients_.count(client_id) != 0;
}

std::vector<uint64_t> ServiceRuntime::disconnect_client(uint64_t client_id) {
  std::lock_guard<std::mutex> g(mu_);
  if (!clients_.erase(client_id)) fail(Status::NotFound, "service: unknown client");
  std::vector<uint64_t> handles;
  for (auto it = by_handle_.begin(); it != by_handle_.end();) {
    if (it->second.client_id == client_id) {
      if (it->second.state == MapState::Live) {
        handles.push_back(it->first);
        ++st_.cancelled;
      }
      auto range = by_client_req_.equal_range(key(client_id, it->second.client_request_id));
      for (auto r = range.first; r != range.second; ++r)
        if (r->second == it->first) { by_client_req_.erase(r); break; }
      it = by_handle_.erase(it);
    } else {
      ++it;
    }
  }
  ServiceEvent e;
  e.kind = kEvClientDisconnected;
  e.client_id = client_id;
  push_locked(e);
  return handles;
}

SubmitResult ServiceRuntime::submit(const SubmitRequest& r, uint32_t prompt_tokens) {
  std::lock_guard<std::mutex> g(mu_);
  ++st_.submitted;
  if (r.flags & ~kSubmitKnownFlags) fail(Status::InvalidArgument, "service: unknown submit flags");
  if (r.text.size() > kMaxTextBytes) fail(Status::InvalidArgument, "service: text too large");
  if (prompt_tokens == 0) fail(Status::InvalidArgument, "service: empty prompt");
  if (!clients_.count(r.client_id)) fail(Status::NotFound, "service: unknown client");
  if (r.client_request_id == 0) fail(Status::InvalidArgument, "service: client request id must be non-zero");
  {
    auto range = by_client_req_.equal_range(key(r.client_id, r.client_request_id));
    for (auto it = range.first; it != range.second; ++it) {
      const Mapping& m = by_handle_.at(it->second);
      if (m.client_id == r.client_id && m.client_request_id == r.client_request_id)
        fail(Status::Duplicate, "service: client request id already live");
    }
  }
  if (by_handle_.size() >= cfg_.request_capacity) fail(Status::CapacityExceeded, "service: request map full");
  const BudgetPolicy& b = cfg_.budgets;
  if (prompt_tokens >= b.max_context_tokens) fail(Status::CapacityExceeded, "service: prompt exceeds the context limit");
  uint32_t out = r.output_budget ? r.output_budget : b.default_output_budget;
  out = std::min(out, b.max_output_budget);
  out = std::min(out, b.max_context_tokens - prompt_tokens);
  SubmitResult res;
  res.prompt_token_count = prompt_tokens;
  res.output_budget = out;
  res.thinking_budget = std::min(r.thinking_budget, out);
  res.required_token_capacity = prompt_tokens + out;
  res.client_id = r.client_id;
  res.client_request_id = r.client_request_id;
  res.serving_request_id = next_request_++;
  res.serving_request_handle = res.serving_request_id;
  res.sequence_id = r.sequence_id ? r.sequence_id : next_sequence_++;
  by_handle_[res.serving_request_handle] =
      Mapping{MapState::Live, r.client_id, r.client_request_id, res.serving_request_id, res.sequence_id};
  by_client_req_.emplace(key(r.client_id, r.client_request_id), res.serving_request_handle);
  ++clients_[r.client_id].accepted;
  ++st_.accepted;
  return res;
}

uint64_t ServiceRuntime::cancel(uint64_t client_id, uint64_t creq) {
  std::lock_guard<std::mutex> g(mu_);
  auto range = by_client_req_.equal_range(key(client_id, creq));
  for (auto it = range.first; it != range.second; ++it) {
    Mapping& m = by_handle_.at(it->second);
    if (m.client_id == client_id && m.client_request_id == creq && m.state == MapState::Live) {
      // the mapping stays until the engine reports the cancellation, so the
      // terminal event still reaches the client
      m.state = MapState::Cancelled;
      ++st_.cancelled;
      return it->second;
    }
  }
  fail(Status::NotFound, "service: no live request with that id");
}

bool ServiceRuntime::lookup(uint64_t client_id, uint64_t creq, uint64_t* handle) const {
  std::lock_guard<std::mutex> g(mu_);
  auto range = by_client_req_.equal_range(key(client_id, creq));
  for (auto it = range.first; it != range.second; ++it) {
    const Mapping& m = by_handle_.at(it->second);
    if (m.client_id == client_id && m.client_request_id == creq) {
      if (handle) *handle = it->second;
      return true;
    }
  }
  return false;
}

void ServiceRuntime::push_locked(const ServiceEvent& e) {
  // token / progress events are dropped on a full ring; terminal and client
  // events always queue so no stream is left without its end
  const bool must = event_is_terminal(e.kind) || e.kind == kEvClientConnected || e.kind == kEvClientDisconnected;
  if (ring_.size() >= cfg_.event_capacity && !must) {
    ++st_.dropped_events;
    return;
  }
  ring_.push_back(e);
}

void ServiceRuntime::release_finished_locked() {
  if (!(cfg_.flags & kCfgAutoReleaseCompleted)) return;
  for (uint64_t h : finished_) {
    auto it = by_handle_.find(h);
    if (it == by_handle_.end()) continue;
    auto range = by_client_req_.equal_range(key(it->second.client_id, it->second.client_request_id));
    for (auto r = range.first; r != range.second; ++r)
      if (r->second == h) { by_client_req_.erase(r); break; }
    by_handle_.erase(it);
  }
  finished_.clear();
}

uint32_t ServiceRuntime::forward(const std::vector<EngineEvent>& events) {
  std::lock_guard<std::mutex> g(mu_);
  uint32_t queued = 0;
  for (const EngineEvent& ev : events) {
    auto it = by_handle_.find(ev.handle);
    if (it == by_handle_.end()) continue;
    Mapping& m = it->second;
    ServiceEvent e;
    e.kind = ev.kind;
    e.status = ev.status;
    e.token_id = ev.token_id;
    e.token_index = ev.token_index;
    e.token_count = ev.token_count;
    e.prompt_token_offset = ev.prompt_token_offset;
    e.prompt_token_count = ev.prompt_token_count;
    e.dispatch_kind = ev.dispatch_kind;
    e.dispatch_flags = ev.dispatch_flags;
    e.client_id = m.client_id;
    e.client_request_id = m.client_request_id;
    e.serving_request_id = m.serving_request_id;
    e.sequence_id = m.sequence_id;
    e.serving_request_handle = ev.handle;
    if (event_is_terminal(ev.kind)) {
      if (ev.kind == kEvCompleted) {
        m.state = MapState::Completed;
        auto c = clients_.find(m.client_id);
        if (c != clients_.end()) ++c->second.completed;
      } else {
        m.state = MapState::Cancelled;
      }
      finished_.push_back(ev.handle);
    }
    const size_t before = ring_.size();
    push_locked(e);
    queued += uint32_t(ring_.size() - before);
    ++st_.forwarded_events;
  }
  release_finished_locked();
  return queued;
}

bool ServiceRuntime::pop(ServiceEvent* out) {
  std::lock_guard<std::mutex> g(mu_);
  if (ring_.empty()) return false;
  *out = ring_.front();
  ring_.pop_front();
  return true;
}

std::vector<ServiceEvent> ServiceRuntime::pop_all(size_t max_events) {
  std::lock_guard<std::mutex> g(mu_);
  std::vector<ServiceEvent> v;
  while (!ring_.empty() && v.size() < max_events) {
    v.push_back(ring_.front());
    ring_.pop_front();
  }
  return v;
}

ServiceStats ServiceRuntime::stats() const {
  std::lock_guard<std::mutex> g(mu_);
  ServiceStats s = st_;
  s.connected_clients = uint32_t(clients_.size());
  s.live_requests = 0;
  s.completed_mappings = 0;
  for (const auto& kv : by_handle_) {
    if (kv.second.state == MapState::Live) ++s.live_requests;
    else if (kv.second.state == MapState::Completed) ++s.completed_mappings;
  }
  s.event_count = uint32_t(ring_.size());
  return s;
}

// ------------------------------------------------------------------ compat
namespace {
struct CompatBuilder {
  CompatRequest req;
  ChatWriter w;
  CompatBuilder(size_t cap, const std::string& style) : w(style, cap) {}

  [[noreturn]] static void bad(const char* what) { fail(Status::InvalidArgument, std::string("compat: ") + what); }

  static bool read_u32(const Json& root, const char* name, uint32_t* out) {
    const Json* v = root.get(name);
    if (!v) return false;
    if (!v->is_integer() || v->int64() < 0 || v->num() > 4294967295.0) bad("budget / priority must be a u32");
    *out = uint32_t(v->int64());
    return true;
  }
  bool append_str_member(const Json& obj, const char* name) {
    const Json* v = obj.get(name);
    if (!v) return false;
    if (!v->is_string()) bad("expected a string member");
    w.append(v->str());
    return true;
  }
  bool append_file_content(const Json& obj) {
    for (const char* f : {"content", "file_content", "file_text", "text", "data"})
      if (append_str_member(obj, f)) return true;
    return false;
  }
  void append_file(const Json& obj) {
    w.append("\n[uploaded file: ");
    if (!append_str_member(obj, "filename") && !append_str_member(obj, "file_name")) append_str_member(obj, "name");
    w.append("]\n");
    if (!append_file_content(obj)) bad("file without content");
    w.append("\n[/uploaded file]\n");
  }
  void append_content_object(const Json& el) {
    if (const Json* t = el.get("text")) {
      if (!t->is_string()) bad("text part must be a string");
      w.append(t->str());
      return;
    }
    for (const char* f : {"content", "file_content", "file_text", "data", "filename", "file_name", "name"})
      if (el.get(f)) { append_file(el); return; }
    if (const Json* src = el.get("source"))
      if (src->is_object()) append_file_content(*src);
  }
  void append_content(const Json& c) {
    if (c.is_string()) { w.append(c.str()); return; }
    if (!c.is_array()) bad("content must be a string or an array");
    for (const Json& el : c.arr()) {
      if (el.is_string()) { w.append(el.str()); continue; }
      if (!el.is_object()) bad("content part must be a string or an object");
      append_content_object(el);
    }
  }
  static std::string role_of(const Json& m) {
    const Json* r = m.get("role");
    if (!r || !r->is_string()) return "user";
    const std::string& s = r->str();
    if (s == "user" || s == "system" || s == "assistant" || s == "tool") return s;
    bad("unknown role");
  }
  void append_messages(const Json& msgs) {
    if (!msgs.is_array() || msgs.size() == 0) bad("messages must be a non-empty array");
    for (const Json& m : msgs.arr()) {
      if (!m.is_object()) bad("message must be an object");
      const Json* c = m.get("content");
      if (!c) bad("message without content");
      const std::string role = role_of(m);
      w.begin_message(role);
      append_content(*c);
      w.end_message(role);
    }
  }
  void append_files(const Json& root) {
    for (const char* key : {"files", "attachments"}) {
      const Json* f = root.get(key);
      if (!f) continue;
      if (!f->is_array()) bad("files must be an array");
      for (const Json& file : f->arr()) {
        if (!file.is_object()) bad("file must be an object");
        append_file(file);
      }
    }
  }
  void common(const Json& root) {
    if (!root.is_object()) bad("request body must be a JSON object");
    read_u32(root, "priority", &req.priority);
    read_u32(root, "max_tokens", &req.output_budget);
    read_u32(root, "max_completion_tokens", &req.output_budget);
    uint32_t a = 0, b = 0;
    const bool ha = read_u32(root, "thinking_budget_tokens", &a);
    const bool hb = read_u32(root, "thinking_token_budget", &b);
    if (ha && hb && a != b) bad("conflicting thinking budgets");
    if (!ha && !hb) return;
    req.thinking_budget = ha ? a : b;
    req.chat_flags = kChatAddGenerationPrompt | (req.thinking_budget ? kChatEnableThinking : 0u);
  }
};

Json parse_body(const std::string& text) {
  try {
    return Json::parse(text);
  } catch (const StatusError& e) {
    fail(Status::ParseError, e.what());
  }
}
}  // namespace

CompatRequest prepare_openai_json(const std::string& json, size_t capacity, const std::string& style) {
  if (!capacity) fail(Status::InvalidArgument, "compat: zero capacity");
  const Json root = parse_body(json);
  CompatBuilder b(capacity, style);
  b.common(root);
  const Json* msgs = root.get("messages");
  if (msgs) {
    b.w.begin("Max", b.req.chat_flags);
    b.append_messages(*msgs);
  } else if (const Json* prompt = root.get("prompt")) {
    if (!prompt->is_string()) CompatBuilder::bad("prompt must be a string");
    b.w.append(prompt->str());
  } else {
    CompatBuilder::bad("neither messages nor prompt");
  }
  b.append_files(root);
  if (msgs) b.w.finish(b.req.chat_flags);
  b.req.text = b.w.text();
  return b.req;
}

CompatRequest prepare_anthropic_json(const std::string& json, size_t capacity, const std::string& style) {
  if (!capacity) fail(Status::InvalidArgument, "compat: zero capacity");
  const Json root = parse_body(json);
  CompatBuilder b(capacity, style);
  b.common(root);
  b.w.begin("Max", b.req.chat_flags);
  if (const Json* sys = root.get("system")) {
    b.w.begin_message("system");
    b.append_content(*sys);
    b.w.end_message("system");
  }
  const Json* msgs = root.get("messages");
  if (!msgs) CompatBuilder::bad("messages missing");
  b.append_messages(*msgs);
  b.append_files(root);
  b.w.finish(b.req.chat_flags);
  b.req.text = b.w.text();
  return b.req;
}

}  // namespace svc
}  // namespace spc
