#include "gateway.h"

#include <arpa/inet.h>
#include <fcntl.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <sys/epoll.h>
#include <sys/eventfd.h>
#include <sys/socket.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <chrono>
#include <cstdio>
#include <cstring>

namespace spc {
namespace gw {

const char* const kBodyUnauthorized =
    "{\"error\":{\"type\":\"unauthorized\",\"message\":\"missing or invalid bearer token\"}}\n";
const char* const kBodyNotFound = "{\"error\":{\"type\":\"not_found\",\"message\":\"unknown endpoint\"}}\n";
const char* const kBodyBadRequest =
    "{\"error\":{\"type\":\"bad_request\",\"message\":\"invalid or oversized request\"}}\n";
const char* const kBodyUnavailableJson =
    "{\"error\":{\"type\":\"backend_unavailable\",\"message\":\"GLM52 RING backend is not attached\"}}\n";
const char* const kBodyUnavailableSse =
    "event: error\ndata: {\"error\":{\"type\":\"backend_unavailable\",\"message\":\"GLM52 RING backend is not "
    "attached\"}}\n\n";
const char* const kBodyTimeoutJson =
    "{\"error\":{\"type\":\"request_timeout\",\"message\":\"GLM52 RING request produced no terminal event before "
    "the stream poll budget\"}}\n";
const char* const kBodyTimeoutSse =
    "event: error\ndata: {\"error\":{\"type\":\"request_timeout\",\"message\":\"GLM52 RING request produced no "
    "terminal event before the stream poll budget\"}}\n\n";

// ------------------------------------------------------------------ wire helpers
Route route_request(const std::string& method, const std::string& path) {
  if (method == "OPTIONS") return Route::CorsPreflight;
  if (method == "GET") {
    if (path == "/") return Route::DemoUi;
    if (path == "/health") return Route::Health;
    if (path == "/metrics") return Route::Metrics;
    return Route::None;
  }
  if (method == "POST") {
    if (path == "/v1/chat/completions") return Route::OpenAiChat;
    if (path == "/v1/completions") return Route::OpenAiCompletions;
    if (path == "/v1/messages") return Route::AnthropicMessages;
  }
  return Route::None;
}

bool body_requests_stream(const std::string& body) {
  static const char kMember[] = "\"stream\"";
  const size_t mlen = sizeof(kMember) - 1;
  auto is_ws = [](char ch) { return ch == ' ' || ch == '\t' || ch == '\r' || ch == '\n'; };
  size_t pos = body.find(kMember);
  while (pos != std::string::npos) {
    size_t k = pos + mlen;
    while (k < body.size() && is_ws(body[k])) ++k;
    if (k < body.size() && body[k] == ':') {
      ++k;
      while (k < body.size() && is_ws(body[k])) ++k;
      if (body.compare(k, 4, "true") == 0) return true;
    }
    pos = body.find(kMember, pos + 1);
  }
  return false;
}

bool authorization_matches(const std::string* authorization, const std::string& api_key) {
  if (api_key.empty()) return true;
  const std::string expected = "Bearer " + api_key;
  if (expected.size() >= 512) return false;  // keys past the header buffer never match
  return authorization && *authorization == expected;
}

std::string escape_json_bytes(const std::string& bytes) {
  std::string o;
  o.reserve(bytes.size() + 8);
  for (unsigned char b : bytes) {
    switch (b) {
      case '"': o += "\\\""; break;
      case '\\': o += "\\\\"; break;
      case '\n': o += "\\n"; break;
      case '\r': o += "\\r"; break;
      case '\t': o += "\\t"; break;
      default:
        if (b < 0x20) {
          char buf[8];
          std::snprintf(buf, sizeof buf, "\\u%04x", b);
          o += buf;
        } else {
          o += char(b);
        }
    }
  }
  return o;
}

const char* sse_event_name(uint32_t kind) {
  if (svc::event_is_terminal(kind)) return "done";
  return kind == svc::kEvToken ? "token" : "event";
}

namespace {
struct Out {
  std::string s;
  Out& k(const char* name) {  // "name":
    s += '"';
    s += name;
    s += "\":";
    return *this;
  }
  Out& str(const char* name, const std::string& v) {
    k(name);
    s += '"';
    s += v;
    s += "\",";
    return *this;
  }
  Out& num(const char* name, uint64_t v) {
    k(name);
    s += std::to_string(v);
    s += ',';
    return *this;
  }
};
}  // namespace

std::string build_health_body(bool runtime_initialized, bool local_control_ready) {
  return std::string("{\"schema\":\"sparkpipe.runtime_observation.v1\",\"runtime_initialized\":") +
         (runtime_initialized ? "1" : "0") + ",\"local_control_ready\":" + (local_control_ready ? "1" : "0") +
         ",\"end_to_end_observation_status\":\"NOT_MEASURED\",\"accuracy_status\":\"NOT_MEASURED\","
         "\"performance_status\":\"NOT_MEASURED\"}\n";
}

std::string build_service_health_body(const HealthStats& stats_in, const BackendView& view_in) {
  // an unattached backend reports a zeroed view and zeroed counters
  const HealthStats stats = view_in.attached ? stats_in : HealthStats{};
  const BackendView view = view_in.attached ? view_in : BackendView{};
  const ServingCounters& sv = stats.serving;
  const char* identity = (!view.release_id.empty() && !view.release_git_commit.empty() && view.release_generation)
                             ? "OBSERVED" : "NOT_MEASURED";
  const char* e2e = (sv.completed_streams && sv.decoded_tokens) ? "OBSERVED" : "NOT_MEASURED";
  const char* batching = view.max_active_sequences <= 1 ? "NOT_WORKING"
                         : (sv.max_decode_lanes > 1 || sv.max_prefill_lanes > 1) ? "OBSERVED" : "NOT_MEASURED";
  const char* jit = !(view.request_api_flags & kRequestApiFlagJitKvPrefetch) ? "NOT_WORKING"
                    : sv.jit_prefetch_dispatches ? "OBSERVED" : "NOT_MEASURED";
  const char* mtp = !(view.speculation_flags & kBackendFlagMtp) ? "NOT_WORKING"
                    : sv.mtp_verify_dispatches ? "OBSERVED" : "NOT_MEASURED";
  const char* dspark = !(view.speculation_flags & kBackendFlagDspark) ? "NOT_WORKING" : "NOT_MEASURED";
  const char* transport = view.transport_capability_flags ? "OBSERVED" : "NOT_MEASURED";
  Out o;
  o.s = "{";
  o.str("schema", "sparkpipe.runtime_observation.v1")
      .str("release_identity_status", identity)
      .str("release_id", escape_json_bytes(view.release_id))
      .str("release_git_commit", escape_json_bytes(view.release_git_commit))
      .num("release_generation", view.release_generation)
      .num("runtime_initialized", view.runtime_initialized)
      .num("local_control_ready", view.local_control_ready)
      .num("configured_kv_context_limit_tokens", view.kv_context_limit_tokens)
      .num("configured_max_active_sequences", view.max_active_sequences)
      .num("adaptive_decode_batch_width", view.adaptive_decode_batch_width)
      .num("decode_batch_capacity", view.decode_batch_capacity)
      .num("prefill_wave_token_count", view.prefill_wave_token_count)
      .str("transport_shared_object", escape_json_bytes(view.transport_shared_object_path))
      .num("bound_transport_interface_flags", view.transport_capability_flags)
      .str("transport_binding_status", transport)
      .str("end_to_end_observation_status", e2e)
      .str("accuracy_status", "NOT_MEASURED")
      .str("performance_status", "NOT_MEASURED")
      .str("multi_sequence_batching_status", batching)
      .str("long_context_status", "NOT_MEASURED")
      .str("jit_kv_status", jit)
      .str("dspark_status", dspark)
      .str("mtp_status", mtp)
      .num("connected_clients", stats.connected_clients)
      .num("live_requests", stats.live_requests)
      .num("queued_requests", sv.queued_requests)
      .num("completed_streams", sv.completed_streams)
      .num("prefill_dispatches", sv.prefill_dispatches)
      .num("prefill_batch_dispatches", sv.prefill_batch_dispatches)
      .num("prefill_tokens", sv.prefill_tokens)
      .num("decode_dispatches", sv.decode_dispatches)
      .num("decoded_tokens", sv.decoded_tokens)
      .num("maximum_prefill_active_sequences", sv.max_prefill_active)
      .num("maximum_prefill_lanes", sv.max_prefill_lanes)
      .num("maximum_decode_active_sequences", sv.max_decode_active)
      .num("maximum_decode_lanes", sv.max_decode_lanes)
      .num("event_backlog", stats.event_backlog)
      .num("dropped_events", stats.dropped_events)
      .num("jit_prefetch_dispatches", sv.jit_prefetch_dispatches)
      .num("jit_prefetch_blocks", sv.jit_prefetch_blocks)
      .num("async_jit_prefetch_starts", sv.async_jit_starts)
      .num("async_jit_prefetch_completions", sv.async_jit_completions)
      .num("mtp_draft_tokens", sv.mtp_draft_tokens)
      .num("mtp_verify_dispatches", sv.mtp_verify_dispatches)
      .num("mtp_draft_ready", sv.mtp_draft_ready)
      .num("mtp_accepted_draft_tokens", sv.mtp_accepted_draft_tokens)
      .num("mtp_committed_tokens", sv.mtp_committed_tokens)
      .num("mtp_rejected_tokens", sv.mtp_rejected_tokens);
  o.k("first_blocker");
  o.s += '"' + escape_json_bytes(view.first_blocker) + "\"}\n";
  return o.s;
}

std::string build_metrics_body(const HealthStats& st, const BackendView& v) {
  std::string o;
  auto metric = [&](const char* name, const char* type, uint64_t value) {
    o += "# TYPE sparkpipe_";
    o += name;
    o += ' ';
    o += type;
    o += "\nsparkpipe_";
    o += name;
    o += ' ';
    o += std::to_string(value);
    o += '\n';
  };
  const ServingCounters& s = st.serving;
  metric("backend_attached", "gauge", v.attached);
  metric("runtime_initialized", "gauge", v.runtime_initialized);
  metric("connected_clients", "gauge", st.connected_clients);
  metric("live_requests", "gauge", st.live_requests);
  metric("queued_requests", "gauge", s.queued_requests);
  metric("event_backlog", "gauge", st.event_backlog);
  metric("dropped_events_total", "counter", st.dropped_events);
  metric("completed_streams_total", "counter", s.completed_streams);
  metric("prefill_dispatches_total", "counter", s.prefill_dispatches);
  metric("prefill_tokens_total", "counter", s.prefill_tokens);
  metric("decode_dispatches_total", "counter", s.decode_dispatches);
  metric("decoded_tokens_total", "counter", s.decoded_tokens);
  metric("max_decode_active_sequences", "gauge", s.max_decode_active);
  metric("max_prefill_active_sequences", "gauge", s.max_prefill_active);
  metric("mtp_draft_tokens_total", "counter", s.mtp_draft_tokens);
  metric("mtp_accepted_draft_tokens_total", "counter", s.mtp_accepted_draft_tokens);
  metric("mtp_verify_dispatches_total", "counter", s.mtp_verify_dispatches);
  return o;
}

std::string build_submit_accepted_json(const svc::SubmitResult& r) {
  return "{\"id\":\"spreq-" + std::to_string(r.serving_request_id) +
         "\",\"object\":\"sparkpipe.request\",\"client_request_id\":" + std::to_string(r.client_request_id) +
         ",\"serving_request_id\":" + std::to_string(r.serving_request_id) +
         ",\"sequence_id\":" + std::to_string(r.sequence_id) +
         ",\"prompt_tokens\":" + std::to_string(r.prompt_token_count) +
         ",\"output_token_budget\":" + std::to_string(r.output_budget) + ",\"status\":\"queued\"}\n";
}

std::string build_submit_accepted_sse(const svc::SubmitResult& r) {
  return "event: accepted\ndata: {\"client_request_id\":" + std::to_string(r.client_request_id) +
         ",\"serving_request_id\":" + std::to_string(r.serving_request_id) +
         ",\"sequence_id\":" + std::to_string(r.sequence_id) +
         ",\"prompt_tokens\":" + std::to_string(r.prompt_token_count) +
         ",\"output_token_budget\":" + std::to_string(r.output_budget) + "}\n\n";
}

std::string build_service_event_frame(const svc::ServiceEvent& e, const std::string& token_text) {
  std::string f = "event: ";
  f += sse_event_name(e.kind);
  f += "\ndata: {";
  Out o;
  o.num("kind", e.kind)
      .num("status", e.status)
      .num("client_id", e.client_id)
      .num("client_request_id", e.client_request_id)
      .num("serving_request_id", e.serving_request_id)
      .num("sequence_id", e.sequence_id)
      .num("token_id", e.token_id)
      .num("token_index", e.token_index)
      .k("text");
  f += o.s;
  f += '"';
  f += escape_json_bytes(token_text);
  f += "\"}\n\n";
  return f;
}

const std::string& demo_ui_html() {
  static const std::string page =
      "<!doctype html><html><head><meta charset=\"utf-8\"><title>sparkpipe-rs B200 demo</title>"
      "<style>body{font:15px system-ui,sans-serif;max-width:900px;margin:2em auto;padding:0 1em}"
      "textarea{width:100%;min-height:12em}#out{white-space:pre-wrap;border:1px solid #ccc;padding:.8em;"
      "min-height:8em}label{display:block;margin:.6em 0}</style></head><body>"
      "<h2>sparkpipe-rs B200 demo</h2>"
      "<label>API key <input id=\"key\" type=\"password\" size=\"40\"></label>"
      "<label>Prompt<textarea id=\"msg\">Explain multi-head latent attention in two sentences.</textarea></label>"
      "<label>Attach text files <input id=\"att\" type=\"file\" multiple></label>"
      "<label>Max tokens <input id=\"max\" type=\"number\" value=\"512\"></label>"
      "<button id=\"go\">Generate</button><div id=\"out\"></div>"
      "<script>"
      "async function readFiles(){const fs=document.getElementById('att').files;const r=[];"
      "for(const f of fs){r.push({filename:f.name,content:await f.text()});}return r;}"
      "document.getElementById('go').onclick=async()=>{const out=document.getElementById('out');out.textContent='';"
      "const key=document.getElementById('key').value;const h={'content-type':'application/json'};"
      "if(key)h.authorization='Bearer '+key;"
      "const req={stream:true,max_tokens:+document.getElementById('max').value,"
      "messages:[{role:'user',content:document.getElementById('msg').value}],files:await readFiles()};"
      "const resp=await fetch('/v1/chat/completions',{method:'POST',headers:h,body:JSON.stringify(req)});"
      "const rd=resp.body.getReader();const td=new TextDecoder();let buf='';"
      "for(;;){const c=await rd.read();if(c.done)break;buf+=td.decode(c.value,{stream:true});let i;"
      "while((i=buf.indexOf('\\n\\n'))>=0){const ev=buf.slice(0,i);buf=buf.slice(i+2);"
      "const d=ev.split('\\n').find(l=>l.startsWith('data: '));if(!d)continue;"
      "try{const j=JSON.parse(d.slice(6));if(j.text)out.textContent+=j.text;}catch(e){}}}};"
      "</script></body></html>";
  return page;
}

// ------------------------------------------------------------------ server
struct Gateway::Conn {
  int fd = -1;
  bool frames = false;
  std::string in, out;
  size_t out_off = 0;
  bool close_after_flush = false;
  bool keep_alive = true;
  bool streaming = false;
  bool read_closed = false;
  uint32_t mask = 0;  // epoll interest currently registered
  uint64_t stream_handle = 0;
  uint64_t client_id = 0;
};

namespace {
void set_nonblock(int fd) { fcntl(fd, F_SETFL, fcntl(fd, F_GETFL, 0) | O_NONBLOCK); }

int listen_on(const std::string& host, int port, int* bound) {
  const int fd = socket(AF_INET, SOCK_STREAM | SOCK_CLOEXEC, 0);
  if (fd < 0) fail(Status::IoError, "gateway: socket() failed");
  int one = 1;
  setsockopt(fd, SOL_SOCKET, SO_REUSEADDR, &one, sizeof one);
  sockaddr_in a{};
  a.sin_family = AF_INET;
  a.sin_port = htons(uint16_t(port));
  if (inet_pton(AF_INET, host.c_str(), &a.sin_addr) != 1) {
    close(fd);
    fail(Status::InvalidArgument, "gateway: bad IPv4 host " + host);
  }
  if (bind(fd, reinterpret_cast<sockaddr*>(&a), sizeof a) != 0 || listen(fd, 512) != 0) {
    const std::string err = std::strerror(errno);
    close(fd);
    fail(Status::IoError, "gateway: bind/listen on " + host + ":" + std::to_string(port) + ": " + err);
  }
  socklen_t len = sizeof a;
  getsockname(fd, reinterpret_cast<sockaddr*>(&a), &len);
  *bound = ntohs(a.sin_port);
  set_nonblock(fd);
  return fd;
}

const char* reason(int code) {
  switch (code) {
    case 200: return "OK";
    case 202: return "Accepted";
    case 400: return "Bad Request";
    case 401: return "Unauthorized";
    case 404: return "Not Found";
    case 503: return "Service Unavailable";
    case 504: return "Gateway Timeout";
  }
  return "Status";
}

std::string head(int code, const char* ctype) {
  std::string h = "HTTP/1.1 " + std::to_string(code) + " " + reason(code) + "\r\ncontent-type: " + ctype +
                  "\r\naccess-control-allow-origin: *\r\naccess-control-allow-headers: authorization, "
                  "content-type\r\naccess-control-allow-methods: GET, POST, OPTIONS\r\ncache-control: no-cache\r\n";
  return h;
}

std::string lower(std::string s) {
  for (char& ch : s) ch = char(std::tolower(static_cast<unsigned char>(ch)));
  return s;
}

std::string trim(const std::string& s) {
  size_t a = 0, b = s.size();
  while (a < b && (s[a] == ' ' || s[a] == '\t')) ++a;
  while (b > a && (s[b - 1] == ' ' || s[b - 1] == '\t')) --b;
  return s.substr(a, b - a);
}

// Decodes a chunked body starting at `pos`; 1 = complete (body, end set),
// 0 = needs more bytes, -1 = malformed or over `cap`.
int decode_chunked(const std::string& in, size_t pos, size_t cap, std::string* body, size_t* end) {
  body->clear();
  while (true) {
    const size_t eol = in.find("\r\n", pos);
    if (eol == std::string::npos) return in.size() - pos > 64 ? -1 : 0;
    const std::string line = in.substr(pos, eol - pos);
    char* e = nullptr;
    const unsigned long long n = std::strtoull(line.c_str(), &e, 16);
    if (e == line.c_str()) return -1;
    pos = eol + 2;
    if (n == 0) {
      // trailers until an empty line
      while (true) {
        const size_t t = in.find("\r\n", pos);
        if (t == std::string::npos) return 0;
        if (t == pos) { *end = pos + 2; return 1; }
        pos = t + 2;
      }
    }
    if (body->size() + n > cap) return -1;
    if (in.size() < pos + n + 2) return 0;
    body->append(in, pos, size_t(n));
    pos += size_t(n);
    if (in.compare(pos, 2, "\r\n") != 0) return -1;
    pos += 2;
  }
}
}  // namespace

Gateway::Gateway(const GatewayConfig& cfg, std::shared_ptr<Tokenizer> tok, std::shared_ptr<svc::ServiceRuntime> service)
    : cfg_(cfg), tok_(std::move(tok)), svc_(std::move(service)) {
  if (!svc_) fail(Status::InvalidArgument, "gateway: a service runtime is required");
}

Gateway::~Gateway() { stop(); }

void Gateway::start() {
  if (running_.load()) return;
  stop_ = false;
  lfd_ = listen_on(cfg_.host, cfg_.port, &port_);
  if (cfg_.frame_port >= 0) ffd_ = listen_on(cfg_.host, cfg_.frame_port, &frame_port_);
  epfd_ = epoll_create1(EPOLL_CLOEXEC);
  evfd_ = eventfd(0, EFD_NONBLOCK | EFD_CLOEXEC);
  if (epfd_ < 0 || evfd_ < 0) fail(Status::IoError, "gateway: epoll/eventfd setup failed");
  auto add = [&](int fd) {
    epoll_event ev{};
    ev.events = EPOLLIN;
    ev.data.fd = fd;
    epoll_ctl(epfd_, EPOLL_CTL_ADD, fd, &ev);
  };
  add(lfd_);
  if (ffd_ >= 0) add(ffd_);
  add(evfd_);
  nonstream_client_ = svc_->register_client(0);
  running_ = true;
  th_ = std::thread([this] { loop(); });
}

void Gateway::stop() {
  if (!running_.load()) return;
  stop_ = true;
  wake();
  if (th_.joinable()) th_.join();
  for (auto& kv : conns_) close(kv.first);
  conns_.clear();
  stream_conn_.clear();
  frame_conn_.clear();
  for (int* fd : {&lfd_, &ffd_, &evfd_, &epfd_})
    if (*fd >= 0) { close(*fd); *fd = -1; }
  running_ = false;
  work_cv_.notify_all();
}

void Gateway::wake() {
  if (evfd_ < 0) return;
  const uint64_t one = 1;
  ssize_t r = write(evfd_, &one, sizeof one);
  (void)r;
}

void Gateway::set_backend_view(const BackendView& v) {
  std::lock_guard<std::mutex> g(view_mu_);
  view_ = v;
}

void Gateway::set_serving_counters(const ServingCounters& c) {
  std::lock_guard<std::mutex> g(view_mu_);
  counters_ = c;
}

HealthStats Gateway::health_stats() {
  const svc::ServiceStats s = svc_->stats();
  HealthStats h;
  h.connected_clients = s.connected_clients;
  h.live_requests = s.live_requests;
  h.event_backlog = s.event_count;
  h.dropped_events = s.dropped_events;
  std::lock_guard<std::mutex> g(view_mu_);
  h.serving = counters_;
  return h;
}

std::vector<EngineWork> Gateway::poll_work(int timeout_ms, size_t max_items) {
  std::unique_lock<std::mutex> lk(work_mu_);
  if (work_.empty() && timeout_ms > 0)
    work_cv_.wait_for(lk, std::chrono::milliseconds(timeout_ms), [&] { return !work_.empty() || stop_.load(); });
  std::vector<EngineWork> v;
  while (!work_.empty() && v.size() < max_items) {
    v.push_back(std::move(work_.front()));
    work_.pop_front();
  }
  return v;
}

void Gateway::push_work(EngineWork&& w) {
  {
    std::lock_guard<std::mutex> g(work_mu_);
    work_.push_back(std::move(w));
  }
  work_cv_.notify_one();
}

uint32_t Gateway::publish(const std::vector<svc::EngineEvent>& events) {
  const uint32_t n = svc_->forward(events);
  if (n) wake();
  return n;
}

std::string Gateway::token_text(uint32_t id) const {
  if (!tok_ || id >= tok_->vocab_size() || tok_->is_special(id)) return std::string();
  return tok_->token_bytes(id);
}

void Gateway::loop() {
  std::vector<epoll_event> evs(256);
  while (!stop_.load()) {
    const int n = epoll_wait(epfd_, evs.data(), int(evs.size()), 100);
    for (int i = 0; i < n && !stop_.load(); ++i) {
      const int fd = evs[i].data.fd;
      const uint32_t e = evs[i].events;
      if (fd == lfd_) { accept_on(lfd_, false); continue; }
      if (fd == ffd_) { accept_on(ffd_, true); continue; }
      if (fd == evfd_) {
        uint64_t v;
        while (read(evfd_, &v, sizeof v) > 0) {}
        continue;
      }
      auto it = conns_.find(fd);
      if (it == conns_.end()) continue;
      Conn& c = *it->second;
      if (e & (EPOLLERR | EPOLLHUP)) { close_conn(fd); continue; }
      if (e & EPOLLIN) {
        on_readable(c);
        if (!conns_.count(fd)) continue;
      }
      if (e & EPOLLOUT) on_writable(c);
    }
    deliver_events();
  }
}

void Gateway::accept_on(int lfd, bool frames) {
  while (true) {
    const int fd = accept4(lfd, nullptr, nullptr, SOCK_NONBLOCK | SOCK_CLOEXEC);
    if (fd < 0) return;
    if (conns_.size() >= cfg_.max_connections) { close(fd); continue; }
    int one = 1;
    setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof one);
    auto c = std::make_unique<Conn>();
    c->fd = fd;
    c->frames = frames;
    epoll_event ev{};
    ev.events = EPOLLIN | EPOLLRDHUP;
    ev.data.fd = fd;
    epoll_ctl(epfd_, EPOLL_CTL_ADD, fd, &ev);
    c->mask = ev.events;
    if (frames) {
      try {
        c->client_id = svc_->register_client(uint64_t(fd));
        frame_conn_[c->client_id] = fd;  // its CLIENT_CONNECTED event tells the client its id
      } catch (const StatusError&) {
        close(fd);
        continue;
      }
    }
    conns_[fd] = std::move(c);
    ++accepted_;
  }
}

void Gateway::on_readable(Conn& c) {
  const int fd = c.fd;
  char buf[65536];
  bool peer_closed = false;
  while (true) {
    const ssize_t r = recv(fd, buf, sizeof buf, 0);
    if (r > 0) {
      c.in.append(buf, size_t(r));
      if (c.in.size() > cfg_.max_request_bytes + 65536 && !c.frames) break;
      continue;
    }
    if (r == 0) peer_closed = true;
    else if (errno == EINTR) continue;
    else if (errno != EAGAIN && errno != EWOULDBLOCK) peer_closed = true;
    break;
  }
  if (peer_closed) {
    // a half-closed client still gets the answer to a request it completed,
    // but a client that leaves mid-stream is gone: cancel
    if (c.streaming || c.frames) { close_conn(fd); return; }
    c.close_after_flush = true;
    c.read_closed = true;  // stop polling for input: level-triggered EOF would spin
  }
  const bool ok = c.frames ? process_frames(c) : process_http(c);
  if (!conns_.count(fd)) return;
  if (!ok) c.close_after_flush = true;
  flush(c);
}

void Gateway::on_writable(Conn& c) { flush(c); }

void Gateway::flush(Conn& c) {
  const int fd = c.fd;
  while (c.out_off < c.out.size()) {
    const ssize_t w = send(fd, c.out.data() + c.out_off, c.out.size() - c.out_off, MSG_NOSIGNAL);
    if (w > 0) { c.out_off += size_t(w); continue; }
    if (w < 0 && errno == EINTR) continue;
    if (w < 0 && (errno == EAGAIN || errno == EWOULDBLOCK)) break;
    close_conn(fd);
    return;
  }
  if (c.out_off == c.out.size()) {
    c.out.clear();
    c.out_off = 0;
  } else if (c.out_off > (1u << 20)) {
    c.out.erase(0, c.out_off);
    c.out_off = 0;
  }
  const bool pending = !c.out.empty();
  const uint32_t want = (c.read_closed ? 0u : uint32_t(EPOLLIN | EPOLLRDHUP)) | (pending ? uint32_t(EPOLLOUT) : 0u);
  if (want != c.mask) {
    epoll_event ev{};
    ev.events = want;
    ev.data.fd = fd;
    epoll_ctl(epfd_, EPOLL_CTL_MOD, fd, &ev);
    c.mask = want;
  }
  if (!pending && c.close_after_flush && !c.streaming) close_conn(fd);
}

void Gateway::close_conn(int fd) {
  auto it = conns_.find(fd);
  if (it == conns_.end()) return;
  Conn& c = *it->second;
  if (c.client_id && c.client_id != nonstream_client_) {
    try {
      for (uint64_t h : svc_->disconnect_client(c.client_id)) {
        EngineWork w;
        w.kind = EngineWork::Cancel;
        w.handle = h;
        w.client_id = c.client_id;
        push_work(std::move(w));
        ++disconnect_cancels_;
      }
    } catch (const StatusError&) {
    }
    frame_conn_.erase(c.client_id);
  }
  if (c.streaming) stream_conn_.erase(c.stream_handle);
  epoll_ctl(epfd_, EPOLL_CTL_DEL, fd, nullptr);
  close(fd);
  conns_.erase(it);
}

void Gateway::respond(Conn& c, int code, const char* ctype, const std::string& body) {
  c.out += head(code, ctype);
  c.out += "content-length: " + std::to_string(body.size()) + "\r\n";
  if (!c.keep_alive) c.out += "connection: close\r\n";
  c.out += "\r\n";
  c.out += body;
  if (!c.keep_alive) c.close_after_flush = true;
}

void Gateway::begin_sse(Conn& c) {
  c.out += head(202, "text/event-stream");
  c.out += "transfer-encoding: chunked\r\n";
  if (!c.keep_alive) c.out += "connection: close\r\n";
  c.out += "\r\n";
}

void Gateway::send_chunk(Conn& c, const std::string& data) {
  char hex[20];
  std::snprintf(hex, sizeof hex, "%zx\r\n", data.size());
  c.out += hex;
  c.out += data;
  c.out += "\r\n";
}

bool Gateway::process_http(Conn& c) {
  while (!c.streaming && !c.in.empty()) {
    const size_t he = c.in.find("\r\n\r\n");
    if (he == std::string::npos) {
      if (c.in.size() > 65536) {
        c.keep_alive = false;
        respond(c, 400, "application/json", kBodyBadRequest);
        c.in.clear();
        return false;
      }
      return true;
    }
    // request line
    const size_t le = c.in.find("\r\n");
    const std::string line = c.in.substr(0, le);
    const size_t s1 = line.find(' '), s2 = line.rfind(' ');
    if (s1 == std::string::npos || s2 == s1) {
      c.keep_alive = false;
      respond(c, 400, "application/json", kBodyBadRequest);
      c.in.clear();
      return false;
    }
    const std::string method = line.substr(0, s1);
    std::string target = line.substr(s1 + 1, s2 - s1 - 1);
    const std::string version = line.substr(s2 + 1);
    const size_t q = target.find('?');
    const std::string path = q == std::string::npos ? target : target.substr(0, q);
    // headers
    long long content_length = -1;
    bool chunked = false, have_auth = false;
    std::string auth, connection;
    size_t p = le + 2;
    while (p < he) {
      const size_t e = c.in.find("\r\n", p);
      const std::string h = c.in.substr(p, e - p);
      p = e + 2;
      const size_t colon = h.find(':');
      if (colon == std::string::npos) continue;
      const std::string name = lower(trim(h.substr(0, colon)));
      const std::string value = trim(h.substr(colon + 1));
      if (name == "content-length") {
        char* end = nullptr;
        content_length = std::strtoll(value.c_str(), &end, 10);
        if (end == value.c_str() || *end || content_length < 0) content_length = -2;
      } else if (name == "transfer-encoding") {
        chunked = lower(value).find("chunked") != std::string::npos;
      } else if (name == "authorization") {
        auth = value;
        have_auth = true;
      } else if (name == "connection") {
        connection = lower(value);
      }
    }
    c.keep_alive = version == "HTTP/1.1" ? connection.find("close") == std::string::npos
                                         : connection.find("keep-alive") != std::string::npos;
    if (content_length == -2) {
      c.keep_alive = false;
      respond(c, 400, "application/json", kBodyBadRequest);
      c.in.clear();
      return false;
    }
    std::string body;
    size_t consumed;
    const size_t body_at = he + 4;
    if (chunked) {
      const int r = decode_chunked(c.in, body_at, cfg_.max_request_bytes, &body, &consumed);
      if (r == 0) return true;
      if (r < 0) {
        c.keep_alive = false;
        respond(c, 400, "application/json", kBodyBadRequest);
        c.in.clear();
        return false;
      }
    } else {
      const size_t cl = content_length < 0 ? 0 : size_t(content_length);
      if (cl > cfg_.max_request_bytes) {
        c.keep_alive = false;
        respond(c, 400, "application/json", kBodyBadRequest);
        c.in.clear();
        return false;
      }
      if (c.in.size() < body_at + cl) return true;
      body = c.in.substr(body_at, cl);
      consumed = body_at + cl;
    }
    c.in.erase(0, consumed);
    handle_http(c, method, path, have_auth ? &auth : nullptr, body);
    if (!c.keep_alive) { c.in.clear(); break; }
  }
  return true;
}

void Gateway::handle_http(Conn& c, const std::string& method, const std::string& path, const std::string* auth,
                          const std::string& body) {
  const Route r = route_request(method, path);
  switch (r) {
    case Route::CorsPreflight: respond(c, 200, "text/plain", ""); return;
    case Route::DemoUi: respond(c, 200, "text/html; charset=utf-8", demo_ui_html()); return;
    case Route::Health: {
      BackendView v;
      {
        std::lock_guard<std::mutex> g(view_mu_);
        v = view_;
      }
      respond(c, 200, "application/json", build_service_health_body(health_stats(), v));
      return;
    }
    case Route::Metrics: {
      BackendView v;
      {
        std::lock_guard<std::mutex> g(view_mu_);
        v = view_;
      }
      respond(c, 200, "text/plain; version=0.0.4", build_metrics_body(health_stats(), v));
      return;
    }
    case Route::None: respond(c, 404, "application/json", kBodyNotFound); return;
    default: handle_submission(c, r, auth, body); return;
  }
}

void Gateway::handle_submission(Conn& c, Route r, const std::string* auth, const std::string& body) {
  if (!authorization_matches(auth, cfg_.api_key)) {
    respond(c, 401, "application/json", kBodyUnauthorized);
    return;
  }
  const bool stream = body_requests_stream(body);
  auto unavailable = [&](bool timeout) {
    if (stream) respond(c, timeout ? 504 : 503, "text/event-stream", timeout ? kBodyTimeoutSse : kBodyUnavailableSse);
    else respond(c, timeout ? 504 : 503, "application/json", timeout ? kBodyTimeoutJson : kBodyUnavailableJson);
  };
  bool available;
  {
    std::lock_guard<std::mutex> g(view_mu_);
    available = view_.attached && view_.runtime_initialized && view_.local_control_ready;
  }
  if (!available || !tok_) { unavailable(false); return; }

  // id allocation: stream ids count from 1, fire-and-forget ids carry the top bit
  uint64_t creq;
  if (stream) {
    creq = next_stream_id_++;
    if (creq == 0 || (creq & kNonstreamRequestBit)) { creq = 1; next_stream_id_ = 2; }
  } else {
    uint64_t id = next_nonstream_id_++;
    if (id == 0 || (id & kNonstreamRequestBit)) { id = 1; next_nonstream_id_ = 2; }
    creq = kNonstreamRequestBit | id;
  }

  svc::CompatRequest cr;
  std::vector<uint32_t> ids;
  svc::SubmitResult res;
  try {
    cr = r == Route::AnthropicMessages ? svc::prepare_anthropic_json(body, cfg_.text_capacity, cfg_.template_style)
                                       : svc::prepare_openai_json(body, cfg_.text_capacity, cfg_.template_style);
    ids = tok_->encode(cr.text, true);
    if (stream && !c.client_id) c.client_id = svc_->register_client(uint64_t(c.fd));
    svc::SubmitRequest sr;
    sr.flags = cr.flags;
    sr.priority = cr.priority;
    sr.thinking_budget = cr.thinking_budget;
    sr.output_budget = cr.output_budget;
    sr.max_prefill_tokens_per_step = cr.max_prefill_tokens_per_step;
    sr.tokenizer_flags = cr.tokenizer_flags;
    sr.client_id = stream ? c.client_id : nonstream_client_;
    sr.client_request_id = creq;
    res = svc_->submit(sr, uint32_t(ids.size()));
  } catch (const StatusError& e) {
    switch (e.status) {
      case Status::Busy: unavailable(true); return;
      case Status::ParseError: case Status::InvalidArgument: case Status::SchemaError:
      case Status::CapacityExceeded:
        respond(c, 400, "application/json", kBodyBadRequest);
        return;
      default: unavailable(false); return;
    }
  }
  EngineWork w;
  w.kind = EngineWork::Submit;
  w.handle = res.serving_request_handle;
  w.token_ids = std::move(ids);
  w.output_budget = res.output_budget;
  w.thinking_budget = res.thinking_budget;
  w.priority = cr.priority;
  w.flags = cr.flags;
  w.client_id = res.client_id;
  w.client_request_id = res.client_request_id;
  if (!stream) {
    push_work(std::move(w));
    respond(c, 202, "application/json", build_submit_accepted_json(res));
    return;
  }
  c.streaming = true;
  c.stream_handle = res.serving_request_handle;
  stream_conn_[c.stream_handle] = c.fd;
  begin_sse(c);
  send_chunk(c, build_submit_accepted_sse(res));
  push_work(std::move(w));
}

bool Gateway::process_frames(Conn& c) {
  while (c.in.size() >= svc::kHeaderBytes) {
    svc::FrameHeader h;
    try {
      h = svc::parse_header(c.in.substr(0, svc::kHeaderBytes));
      svc::validate_header(h);
    } catch (const StatusError& e) {
      c.out += svc::build_error_frame(c.client_id, 0, e.status);
      c.in.clear();
      return false;  // framing is lost: answer and close
    }
    if (c.in.size() < svc::kHeaderBytes + h.body_bytes) return true;
    const std::string body = c.in.substr(svc::kHeaderBytes, h.body_bytes);
    c.in.erase(0, svc::kHeaderBytes + h.body_bytes);
    handle_frame(c, h, body);
  }
  return true;
}

void Gateway::handle_frame(Conn& c, const svc::FrameHeader& h, const std::string& body) {
  try {
    switch (h.kind) {
      case svc::kFramePing: c.out += svc::build_pong_frame(c.client_id, h.client_request_id); return;
      case svc::kFrameCancel: {
        const uint64_t creq = svc::parse_cancel_frame(h, body);
        EngineWork w;
        w.kind = EngineWork::Cancel;
        w.handle = svc_->cancel(c.client_id, creq);
        w.client_id = c.client_id;
        w.client_request_id = creq;
        push_work(std::move(w));
        return;
      }
      case svc::kFrameSubmitText:
      case svc::kFrameSubmitTokenIds: {
        svc::SubmitRequest sr = h.kind == svc::kFrameSubmitText ? svc::parse_submit_text_frame(h, body)
                                                                : svc::parse_submit_tokens_frame(h, body);
        sr.client_id = c.client_id;  // a connection speaks for its own client only
        if (h.kind == svc::kFrameSubmitText) {
          if (!tok_) fail(Status::Unsupported, "gateway: no tokenizer for text submissions");
          sr.token_ids = tok_->encode(sr.text, true);
        }
        const svc::SubmitResult res = svc_->submit(sr, uint32_t(sr.token_ids.size()));
        EngineWork w;
        w.kind = EngineWork::Submit;
        w.handle = res.serving_request_handle;
        w.token_ids = std::move(sr.token_ids);
        w.output_budget = res.output_budget;
        w.thinking_budget = res.thinking_budget;
        w.priority = sr.priority;
        w.flags = sr.flags;
        w.client_id = res.client_id;
        w.client_request_id = res.client_request_id;
        c.out += svc::build_ack_frame(res);
        push_work(std::move(w));
        return;
      }
      default: fail(Status::InvalidArgument, "gateway: frame kind not accepted from clients");
    }
  } catch (const StatusError& e) {
    c.out += svc::build_error_frame(c.client_id, h.client_request_id, e.status);
  }
}

void Gateway::deliver_events() {
  std::vector<int> touched;
  while (true) {
    const std::vector<svc::ServiceEvent> evs = svc_->pop_all(4096);
    if (evs.empty()) break;
    for (const svc::ServiceEvent& e : evs) {
      auto fc = frame_conn_.find(e.client_id);
      if (fc != frame_conn_.end()) {
        auto it = conns_.find(fc->second);
        if (it != conns_.end()) {
          it->second->out += svc::build_event_frame(e);
          touched.push_back(fc->second);
        }
        continue;
      }
      if (e.kind == svc::kEvAccepted || e.kind == svc::kEvClientConnected || e.kind == svc::kEvClientDisconnected)
        continue;
      auto sc = stream_conn_.find(e.serving_request_handle);
      if (sc == stream_conn_.end()) continue;
      auto it = conns_.find(sc->second);
      if (it == conns_.end()) { stream_conn_.erase(sc); continue; }
      Conn& c = *it->second;
      send_chunk(c, build_service_event_frame(e, e.kind == svc::kEvToken ? token_text(e.token_id) : std::string()));
      if (svc::event_is_terminal(e.kind)) {
        c.out += "0\r\n\r\n";
        c.streaming = false;
        stream_conn_.erase(sc);
      }
      touched.push_back(c.fd);
    }
  }
  std::sort(touched.begin(), touched.end());
  touched.erase(std::unique(touched.begin(), touched.end()), touched.end());
  for (int fd : touched) {
    auto it = conns_.find(fd);
    if (it == conns_.end()) continue;
    Conn& c = *it->second;
    if (!c.frames && !c.streaming && c.keep_alive && !c.in.empty()) process_http(c);  // pipelined requests
    if (!conns_.count(fd)) continue;
    if (!c.frames && !c.streaming && !c.keep_alive) c.close_after_flush = true;
    flush(c);
  }
}

}  // namespace gw
}  // namespace spc
