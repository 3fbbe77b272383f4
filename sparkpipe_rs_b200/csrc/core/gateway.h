// HTTP/1.1 + SSE gateway and native frame endpoint, served by one epoll thread.
//
// Routes: GET / (demo page), GET /health (runtime observation JSON), GET
// /metrics (Prometheus text), POST /v1/chat/completions, /v1/completions,
// /v1/messages (OpenAI / Anthropic bodies), OPTIONS * (CORS preflight).
// Bearer-key auth on the completion routes, a byte-scan `"stream": true`
// flag, a request-size cap, keep-alive connections, SSE over chunked
// transfer encoding, client disconnect -> cancel.
//
// The whole request path up to the engine is native: JSON -> chat template
// (service.h compat), tokenization (text.h), id mapping and budgets
// (ServiceRuntime) all run on the gateway thread, which answers 202 at once.
// The engine thread only sees token ids (`poll_work`) and hands back token /
// finish events by serving handle (`publish`); the gateway thread turns them
// into SSE frames (token text decoded here) or binary event frames.
//
// Wire compatibility with the reference gateway
// (crates/spark-serve/src/http_gateway.rs): routes :109-136, stream scan
// :139-175, auth :179-191, escaper :193-230, health body :395-563, accepted /
// event frames :565-649, handler and id allocation :809-956. JSON field names,
// order and error bodies are kept byte-identical so existing clients parse
// them unchanged.
#pragma once

#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <deque>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "service.h"
#include "text.h"

namespace spc {
namespace gw {

constexpr uint64_t kNonstreamRequestBit = 1ull << 63;
constexpr size_t kDefaultMaxUploadBytes = 64ull << 20;
constexpr size_t kDefaultMaxRequestBytes = kDefaultMaxUploadBytes + (1ull << 20);
constexpr uint32_t kBackendFlagDspark = 0x1;
constexpr uint32_t kBackendFlagMtp = 0x2;
constexpr uint32_t kRequestApiFlagJitKvPrefetch = 0x1;

enum class Route { None, DemoUi, Health, Metrics, OpenAiChat, OpenAiCompletions, AnthropicMessages, CorsPreflight };
Route route_request(const std::string& method, const std::string& path);
bool body_requests_stream(const std::string& body);
bool authorization_matches(const std::string* authorization, const std::string& api_key);
std::string escape_json_bytes(const std::string& bytes);  // C-style: \" \\ \n \r \t, other < 0x20 as \u00xx

struct BackendView {
  bool attached = false, runtime_initialized = false, local_control_ready = false;
  std::string release_id, release_git_commit, transport_shared_object_path, first_blocker;
  uint64_t release_generation = 0;
  uint32_t kv_context_limit_tokens = 0, max_active_sequences = 0, adaptive_decode_batch_width = 0;
  uint32_t decode_batch_capacity = 0, prefill_wave_token_count = 0, transport_capability_flags = 0;
  uint32_t request_api_flags = 0, speculation_flags = 0;
};

struct ServingCounters {
  uint32_t queued_requests = 0;
  uint64_t completed_streams = 0, prefill_dispatches = 0, prefill_batch_dispatches = 0, prefill_tokens = 0;
  uint64_t decode_dispatches = 0, decoded_tokens = 0;
  uint32_t max_prefill_active = 0, max_prefill_lanes = 0, max_decode_active = 0, max_decode_lanes = 0;
  uint64_t jit_prefetch_dispatches = 0, jit_prefetch_blocks = 0, async_jit_starts = 0, async_jit_completions = 0;
  uint64_t mtp_draft_tokens = 0, mtp_verify_dispatches = 0, mtp_draft_ready = 0, mtp_accepted_draft_tokens = 0;
  uint64_t mtp_committed_tokens = 0, mtp_rejected_tokens = 0;
};

struct HealthStats {
  uint32_t connected_clients = 0, live_requests = 0, event_backlog = 0, dropped_events = 0;
  ServingCounters serving;
};

std::string build_health_body(bool runtime_initialized, bool local_control_ready);
std::string build_service_health_body(const HealthStats& stats, const BackendView& view);
std::string build_metrics_body(const HealthStats& stats, const BackendView& view);
std::string build_submit_accepted_json(const svc::SubmitResult& r);
std::string build_submit_accepted_sse(const svc::SubmitResult& r);
std::string build_service_event_frame(const svc::ServiceEvent& e, const std::string& token_text);
const char* sse_event_name(uint32_t kind);
const std::string& demo_ui_html();

extern const char* const kBodyUnauthorized;
extern const char* const kBodyNotFound;
extern const char* const kBodyBadRequest;
extern const char* const kBodyUnavailableJson;
extern const char* const kBodyUnavailableSse;
extern const char* const kBodyTimeoutJson;
extern const char* const kBodyTimeoutSse;

struct GatewayConfig {
  std::string host = "127.0.0.1";
  int port = 0;             // 0: any free port
  int frame_port = -1;      // -1: no native frame endpoint; 0: any free port
  std::string api_key;      // empty: no auth
  size_t max_request_bytes = kDefaultMaxRequestBytes;
  size_t text_capacity = kDefaultMaxUploadBytes;  // chat-template text cap
  std::string template_style = "glm";
  uint32_t max_connections = 4096;
};

// Work handed to the engine thread.
struct EngineWork {
  enum Kind : uint32_t { Submit = 1, Cancel = 2 };
  uint32_t kind = Submit;
  uint64_t handle = 0;
  std::vector<uint32_t> token_ids;
  uint32_t output_budget = 0, thinking_budget = 0, priority = 0, flags = 0;
  uint64_t client_id = 0, client_request_id = 0;
};

class Gateway {
 public:
  Gateway(const GatewayConfig& cfg, std::shared_ptr<Tokenizer> tok, std::shared_ptr<svc::ServiceRuntime> service);
  ~Gateway();
  void start();
  void stop();
  int port() const { return port_; }
  int frame_port() const { return frame_port_; }
  bool running() const { return running_.load(); }

  void set_backend_view(const BackendView& v);
  void set_serving_counters(const ServingCounters& c);
  // Blocks up to timeout_ms for work (0: poll); returns at most max_items.
  std::vector<EngineWork> poll_work(int timeout_ms, size_t max_items);
  // Engine events by serving handle -> service ring -> connections.
  uint32_t publish(const std::vector<svc::EngineEvent>& events);
  uint64_t accepted_connections() const { return accepted_.load(); }
  uint64_t cancelled_by_disconnect() const { return disconnect_cancels_.load(); }

 private:
  struct Conn;
  void loop();
  void wake();
  void accept_on(int lfd, bool frames);
  void on_readable(Conn& c);
  void on_writable(Conn& c);
  void close_conn(int fd);
  bool process_http(Conn& c);
  bool process_frames(Conn& c);
  void handle_http(Conn& c, const std::string& method, const std::string& path, const std::string* auth,
                   const std::string& body);
  void handle_submission(Conn& c, Route r, const std::string* auth, const std::string& body);
  void handle_frame(Conn& c, const svc::FrameHeader& h, const std::string& body);
  void respond(Conn& c, int code, const char* ctype, const std::string& body);
  void begin_sse(Conn& c);
  void send_chunk(Conn& c, const std::string& data);
  void flush(Conn& c);
  void deliver_events();
  void push_work(EngineWork&& w);
  HealthStats health_stats();
  std::string token_text(uint32_t id) const;

  GatewayConfig cfg_;
  std::shared_ptr<Tokenizer> tok_;
  std::shared_ptr<svc::ServiceRuntime> svc_;
  int epfd_ = -1, lfd_ = -1, ffd_ = -1, evfd_ = -1;
  int port_ = 0, frame_port_ = -1;
  std::thread th_;
  std::atomic<bool> running_{false}, stop_{false};
  std::atomic<uint64_t> accepted_{0}, disconnect_cancels_{0};
  uint64_t next_stream_id_ = 1, next_nonstream_id_ = 1;
  uint64_t nonstream_client_ = 0;

  std::unordered_map<int, std::unique_ptr<Conn>> conns_;
  std::unordered_map<uint64_t, int> stream_conn_;  // serving handle -> fd (SSE)
  std::unordered_map<uint64_t, int> frame_conn_;   // service client id -> fd (frame endpoint)

  std::mutex view_mu_;
  BackendView view_;
  ServingCounters counters_;

  std::mutex work_mu_;
  std::condition_variable work_cv_;
  std::deque<EngineWork> work_;
};

}  // namespace gw
}  // namespace spc
