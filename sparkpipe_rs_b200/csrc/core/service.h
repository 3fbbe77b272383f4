// Service runtime: client sessions, the client-request-id <-> serving-handle
// maps, the service event ring, the binary frame protocol for native service
// clients, and the OpenAI / Anthropic JSON -> chat-template conversion.
//
// The runtime is engine-agnostic and thread-safe (one mutex): a submission is
// validated and mapped here and gets its serving handle (= serving request id,
// allocated from `request_id_base`) before the engine thread ever sees it, so
// the HTTP gateway answers `202 Accepted` without waiting for a GPU step. The
// engine thread later hands token / finish events in by serving handle; they
// are mapped back to (client, client request) and queued in the event ring.
//
// Reference behaviour: crates/spark-serve/src/serving_engine/service.rs
// (constants :23-88, frame header :350-440, ServiceRuntime :505-1300, event
// frame :1301-1328) and compat.rs:26-451. The frame layout (40-byte header,
// magic 0x35504B53, ABI 1, little-endian fields at fixed offsets, 88-byte
// event body) is kept byte-compatible so native clients interoperate.
#pragma once

#include <cstdint>
#include <deque>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.h"

namespace spc {
namespace svc {

constexpr uint32_t kAbiVersion = 1;
constexpr uint64_t kDefaultRequestIdBase = 5000000000ull;
constexpr uint32_t kFrameMagic = 0x35504B53u;
constexpr uint32_t kMaxFrameBodyBytes = 128u << 20;
constexpr uint32_t kMaxTextBytes = 64u << 20;
constexpr uint32_t kMaxTokenFrameCount = 1u << 20;

constexpr uint32_t kFrameSubmitText = 1;
constexpr uint32_t kFrameSubmitTokenIds = 2;
constexpr uint32_t kFrameCancel = 3;
constexpr uint32_t kFramePing = 4;
constexpr uint32_t kFrameEvent = 100;
constexpr uint32_t kFrameSubmitAck = 101;
constexpr uint32_t kFrameError = 102;
constexpr uint32_t kFramePong = 103;

constexpr uint32_t kSubmitFlagRealtime = 0x1;
constexpr uint32_t kSubmitFlagDisableSpeculation = 0x2;
constexpr uint32_t kSubmitKnownFlags = kSubmitFlagRealtime | kSubmitFlagDisableSpeculation;

constexpr size_t kHeaderBytes = 40;
constexpr size_t kSubmitTextBodyBytes = 40;
constexpr size_t kSubmitTokensBodyBytes = 40;
constexpr size_t kCancelBodyBytes = 24;
constexpr size_t kEventBodyBytes = 88;
constexpr size_t kAckBodyBytes = 72;    // this runtime's SUBMIT_ACK body (ServiceSubmitResult fields)
constexpr size_t kErrorBodyBytes = 16;  // this runtime's ERROR body (abi, bytes, status, reserved)

enum EventKind : uint32_t {
  kEvNone = 0,
  kEvAccepted = 1,
  kEvPrefillProgress = 2,
  kEvToken = 3,
  kEvCompleted = 4,
  kEvCancelled = 5,
  kEvError = 6,
  kEvBackpressure = 7,
  kEvClientConnected = 8,
  kEvClientDisconnected = 9,
  kEvStats = 10,
};
inline bool event_is_terminal(uint32_t kind) {
  return kind == kEvCompleted || kind == kEvCancelled || kind == kEvError;
}

constexpr uint32_t kCfgAutoReleaseCompleted = 0x1;
constexpr uint32_t kCfgDefaultFlags = kCfgAutoReleaseCompleted;

struct FrameHeader {
  uint32_t kind = 0, flags = 0, body_bytes = 0;
  uint64_t client_id = 0, client_request_id = 0;
};
std::string serialize_header(const FrameHeader& h);
FrameHeader parse_header(const std::string& bytes);  // InvalidArgument on bad magic / abi / size
void validate_header(const FrameHeader& h, uint32_t max_body_bytes = 0);

struct ServiceEvent {
  uint32_t kind = 0, flags = 0, status = 0, token_id = 0, token_index = 0, token_count = 0;
  uint32_t prompt_token_offset = 0, prompt_token_count = 0, dispatch_kind = 0, dispatch_flags = 0;
  uint64_t client_id = 0, client_request_id = 0, serving_request_id = 0, sequence_id = 0;
  uint64_t serving_request_handle = 0;
};
std::string build_event_frame(const ServiceEvent& e);  // header + 88-byte body
ServiceEvent parse_event_body(const std::string& body);

struct SubmitRequest {
  uint32_t flags = 0, priority = 0, thinking_budget = 0, output_budget = 0;
  uint32_t max_prefill_tokens_per_step = 0, tokenizer_flags = 0;
  uint64_t client_id = 0, client_request_id = 0, sequence_id = 0;
  std::string text;               // submit-text payload (UTF-8)
  std::vector<uint32_t> token_ids;  // submit-token-ids payload
};
SubmitRequest parse_submit_text_frame(const FrameHeader& h, const std::string& body);
SubmitRequest parse_submit_tokens_frame(const FrameHeader& h, const std::string& body);
uint64_t parse_cancel_frame(const FrameHeader& h, const std::string& body);  // client request id
std::string build_submit_text_frame(const SubmitRequest& r);
std::string build_submit_tokens_frame(const SubmitRequest& r);
std::string build_cancel_frame(uint64_t client_id, uint64_t client_request_id);
std::string build_ping_frame(uint64_t client_id, uint64_t cookie);

struct SubmitResult {
  uint32_t prompt_token_count = 0, required_token_capacity = 0, thinking_budget = 0, output_budget = 0;
  uint64_t client_id = 0, client_request_id = 0, serving_request_id = 0, sequence_id = 0;
  uint64_t serving_request_handle = 0;
};
std::string build_ack_frame(const SubmitResult& r);
SubmitResult parse_ack_body(const std::string& body);
std::string build_error_frame(uint64_t client_id, uint64_t client_request_id, Status s);
std::string build_pong_frame(uint64_t client_id, uint64_t cookie);

// Budget policy the runtime applies to every submission (the engine's limits).
struct BudgetPolicy {
  uint32_t default_output_budget = 256;
  uint32_t max_output_budget = 1u << 20;
  uint32_t max_context_tokens = 1u << 20;  // prompt + output must fit
};

struct ServiceConfig {
  uint32_t flags = kCfgDefaultFlags;
  uint64_t request_id_base = kDefaultRequestIdBase;
  uint32_t client_capacity = 1024;
  uint32_t request_capacity = 4096;
  uint32_t event_capacity = 65536;
  BudgetPolicy budgets;
};

struct ServiceStats {
  uint32_t connected_clients = 0, live_requests = 0, completed_mappings = 0, event_count = 0;
  uint32_t event_capacity = 0, dropped_events = 0;
  uint64_t submitted = 0, accepted = 0, forwarded_events = 0, cancelled = 0;
};

// Event as the engine reports it: keyed by serving handle.
struct EngineEvent {
  uint64_t handle = 0;
  uint32_t kind = 0, status = 0, token_id = 0, token_index = 0, token_count = 1;
  uint32_t prompt_token_offset = 0, prompt_token_count = 0, dispatch_kind = 0, dispatch_flags = 0;
};

class ServiceRuntime {
 public:
  explicit ServiceRuntime(const ServiceConfig& cfg);

  uint64_t register_client(uint64_t cookie);
  // Cancels the client's live requests; returns their serving handles (the
  // engine must abort them).
  std::vector<uint64_t> disconnect_client(uint64_t client_id);
  bool has_client(uint64_t client_id) const;

  // Validates and maps a submission whose prompt is already tokenized
  // (`prompt_tokens` tokens); returns the result with the serving handle.
  SubmitResult submit(const SubmitRequest& r, uint32_t prompt_tokens);
  // Cancel by client request id; returns the serving handle to abort.
  uint64_t cancel(uint64_t client_id, uint64_t client_request_id);

  // Maps engine events to service events. Unknown handles are skipped; with a
  // full ring the event is dropped and counted. Returns events queued.
  uint32_t forward(const std::vector<EngineEvent>& events);
  bool pop(ServiceEvent* out);
  std::vector<ServiceEvent> pop_all(size_t max_events);
  // Routing lookup for a live mapping (false if unknown).
  bool lookup(uint64_t client_id, uint64_t client_request_id, uint64_t* handle) const;
  ServiceStats stats() const;
  const BudgetPolicy& budgets() const { return cfg_.budgets; }

 private:
  enum class MapState : uint8_t { Live, Completed, Cancelled };
  struct Mapping {
    MapState state;
    uint64_t client_id, client_request_id, serving_request_id, sequence_id;
  };
  struct Client {
    uint64_t cookie = 0, accepted = 0, completed = 0;
  };
  static uint64_t key(uint64_t client_id, uint64_t creq) { return client_id * 0x9E3779B97F4A7C15ull ^ creq; }
  void push_locked(const ServiceEvent& e);
  void release_finished_locked();

  ServiceConfig cfg_;
  mutable std::mutex mu_;
  uint64_t next_request_ = 0, next_client_ = 1, next_sequence_ = 1;
  std::unordered_map<uint64_t, Client> clients_;
  std::unordered_map<uint64_t, Mapping> by_handle_;
  std::unordered_multimap<uint64_t, uint64_t> by_client_req_;  // key -> handle
  std::deque<ServiceEvent> ring_;
  std::vector<uint64_t> finished_;  // handles to release after forwarding
  ServiceStats st_;
};

// ------------------------------------------------------------------ compat
constexpr uint32_t kCompatDefaultChatFlags = 0x3;  // add generation prompt | enable thinking

struct CompatRequest {
  uint32_t flags = 0, chat_flags = kCompatDefaultChatFlags, priority = 0;
  uint32_t thinking_budget = 0, output_budget = 0, max_prefill_tokens_per_step = 0, tokenizer_flags = 0;
  std::string text;
};
// OpenAI chat ("messages") or completions ("prompt"); files / attachments are
// folded into the prompt text. ParseError on bad JSON, InvalidArgument on a
// bad shape, CapacityExceeded past `capacity` bytes of text.
CompatRequest prepare_openai_json(const std::string& json, size_t capacity, const std::string& style = "glm");
CompatRequest prepare_anthropic_json(const std::string& json, size_t capacity, const std::string& style = "glm");

}  // namespace svc
}  // namespace spc
