// Bindings of the serving plane: service runtime + frame codec, compat JSON,
// and the HTTP / SSE gateway (submodule `serving`).
#include "gateway.h"
#include "registry.h"
#include "service.h"

namespace py = pybind11;
using namespace spc;

namespace {
std::string as_bytes(const py::object& o) {
  if (py::isinstance<py::bytes>(o)) return std::string(o.cast<py::bytes>());
  return o.cast<std::string>();
}
}  // namespace

static BindRegistrar reg([](py::module_& m) {
  auto s = m.def_submodule("serving", "service runtime, frame codec, compat JSON, HTTP/SSE gateway");
  s.attr("ABI_VERSION") = svc::kAbiVersion;
  s.attr("FRAME_MAGIC") = svc::kFrameMagic;
  s.attr("DEFAULT_REQUEST_ID_BASE") = svc::kDefaultRequestIdBase;
  s.attr("FRAME_HEADER_BYTES") = svc::kHeaderBytes;
  s.attr("EVENT_BODY_BYTES") = svc::kEventBodyBytes;
  s.attr("FRAME_SUBMIT_TEXT") = svc::kFrameSubmitText;
  s.attr("FRAME_SUBMIT_TOKEN_IDS") = svc::kFrameSubmitTokenIds;
  s.attr("FRAME_CANCEL") = svc::kFrameCancel;
  s.attr("FRAME_PING") = svc::kFramePing;
  s.attr("FRAME_EVENT") = svc::kFrameEvent;
  s.attr("FRAME_SUBMIT_ACK") = svc::kFrameSubmitAck;
  s.attr("FRAME_ERROR") = svc::kFrameError;
  s.attr("FRAME_PONG") = svc::kFramePong;
  s.attr("EV_ACCEPTED") = uint32_t(svc::kEvAccepted);
  s.attr("EV_PREFILL_PROGRESS") = uint32_t(svc::kEvPrefillProgress);
  s.attr("EV_TOKEN") = uint32_t(svc::kEvToken);
  s.attr("EV_COMPLETED") = uint32_t(svc::kEvCompleted);
  s.attr("EV_CANCELLED") = uint32_t(svc::kEvCancelled);
  s.attr("EV_ERROR") = uint32_t(svc::kEvError);
  s.attr("EV_BACKPRESSURE") = uint32_t(svc::kEvBackpressure);
  s.attr("EV_CLIENT_CONNECTED") = uint32_t(svc::kEvClientConnected);
  s.attr("EV_CLIENT_DISCONNECTED") = uint32_t(svc::kEvClientDisconnected);
  s.attr("NONSTREAM_REQUEST_BIT") = gw::kNonstreamRequestBit;
  s.attr("BACKEND_FLAG_DSPARK") = gw::kBackendFlagDspark;
  s.attr("BACKEND_FLAG_MTP") = gw::kBackendFlagMtp;
  s.attr("REQUEST_API_FLAG_JIT_KV_PREFETCH") = gw::kRequestApiFlagJitKvPrefetch;

  py::class_<svc::FrameHeader>(s, "FrameHeader")
      .def(py::init<>())
      .def_readwrite("kind", &svc::FrameHeader::kind)
      .def_readwrite("flags", &svc::FrameHeader::flags)
      .def_readwrite("body_bytes", &svc::FrameHeader::body_bytes)
      .def_readwrite("client_id", &svc::FrameHeader::client_id)
      .def_readwrite("client_request_id", &svc::FrameHeader::client_request_id);
  s.def("serialize_header", [](const svc::FrameHeader& h) { return py::bytes(svc::serialize_header(h)); });
  s.def("parse_header", [](py::bytes b) { return svc::parse_header(std::string(b)); });
  s.def("validate_header", &svc::validate_header, py::arg("header"), py::arg("max_body_bytes") = 0);

  py::class_<svc::ServiceEvent>(s, "ServiceEvent")
      .def(py::init<>())
      .def_readwrite("kind", &svc::ServiceEvent::kind)
      .def_readwrite("flags", &svc::ServiceEvent::flags)
      .def_readwrite("status", &svc::ServiceEvent::status)
      .def_readwrite("token_id", &svc::ServiceEvent::token_id)
      .def_readwrite("token_index", &svc::ServiceEvent::token_index)
      .def_readwrite("token_count", &svc::ServiceEvent::token_count)
      .def_readwrite("prompt_token_offset", &svc::ServiceEvent::prompt_token_offset)
      .def_readwrite("prompt_token_count", &svc::ServiceEvent::prompt_token_count)
      .def_readwrite("dispatch_kind", &svc::ServiceEvent::dispatch_kind)
      .def_readwrite("dispatch_flags", &svc::ServiceEvent::dispatch_flags)
      .def_readwrite("client_id", &svc::ServiceEvent::client_id)
      .def_readwrite("client_request_id", &svc::ServiceEvent::client_request_id)
      .def_readwrite("serving_request_id", &svc::ServiceEvent::serving_request_id)
      .def_readwrite("sequence_id", &svc::ServiceEvent::sequence_id)
      .def_readwrite("serving_request_handle", &svc::ServiceEvent::serving_request_handle);
  s.def("build_event_frame", [](const svc::ServiceEvent& e) { return py::bytes(svc::build_event_frame(e)); });
  s.def("parse_event_body", [](py::bytes b) { return svc::parse_event_body(std::string(b)); });

  py::class_<svc::SubmitRequest>(s, "SubmitRequest")
      .def(py::init<>())
      .def_readwrite("flags", &svc::SubmitRequest::flags)
      .def_readwrite("priority", &svc::SubmitRequest::priority)
      .def_readwrite("thinking_budget", &svc::SubmitRequest::thinking_budget)
      .def_readwrite("output_budget", &svc::SubmitRequest::output_budget)
      .def_readwrite("max_prefill_tokens_per_step", &svc::SubmitRequest::max_prefill_tokens_per_step)
      .def_readwrite("tokenizer_flags", &svc::SubmitRequest::tokenizer_flags)
      .def_readwrite("client_id", &svc::SubmitRequest::client_id)
      .def_readwrite("client_request_id", &svc::SubmitRequest::client_request_id)
      .def_readwrite("sequence_id", &svc::SubmitRequest::sequence_id)
      .def_property("text", [](const svc::SubmitRequest& r) { return py::bytes(r.text); },
                    [](svc::SubmitRequest& r, py::object v) { r.text = as_bytes(v); })
      .def_readwrite("token_ids", &svc::SubmitRequest::token_ids);
  s.def("parse_submit_text_frame", [](const svc::FrameHeader& h, py::bytes b) {
    return svc::parse_submit_text_frame(h, std::string(b));
  });
  s.def("parse_submit_tokens_frame", [](const svc::FrameHeader& h, py::bytes b) {
    return svc::parse_submit_tokens_frame(h, std::string(b));
  });
  s.def("parse_cancel_frame", [](const svc::FrameHeader& h, py::bytes b) {
    return svc::parse_cancel_frame(h, std::string(b));
  });
  s.def("build_submit_text_frame", [](const svc::SubmitRequest& r) { return py::bytes(svc::build_submit_text_frame(r)); });
  s.def("build_submit_tokens_frame",
        [](const svc::SubmitRequest& r) { return py::bytes(svc::build_submit_tokens_frame(r)); });
  s.def("build_cancel_frame", [](uint64_t c, uint64_t r) { return py::bytes(svc::build_cancel_frame(c, r)); });
  s.def("build_ping_frame", [](uint64_t c, uint64_t k) { return py::bytes(svc::build_ping_frame(c, k)); });
  s.def("build_error_frame", [](uint64_t c, uint64_t r, uint32_t st) {
    return py::bytes(svc::build_error_frame(c, r, Status(st)));
  });

  py::class_<svc::SubmitResult>(s, "SubmitResult")
      .def(py::init<>())
      .def_readwrite("prompt_token_count", &svc::SubmitResult::prompt_token_count)
      .def_readwrite("required_token_capacity", &svc::SubmitResult::required_token_capacity)
      .def_readwrite("thinking_budget", &svc::SubmitResult::thinking_budget)
      .def_readwrite("output_budget", &svc::SubmitResult::output_budget)
      .def_readwrite("client_id", &svc::SubmitResult::client_id)
      .def_readwrite("client_request_id", &svc::SubmitResult::client_request_id)
      .def_readwrite("serving_request_id", &svc::SubmitResult::serving_request_id)
      .def_readwrite("sequence_id", &svc::SubmitResult::sequence_id)
      .def_readwrite("serving_request_handle", &svc::SubmitResult::serving_request_handle);
  s.def("build_ack_frame", [](const svc::SubmitResult& r) { return py::bytes(svc::build_ack_frame(r)); });
  s.def("parse_ack_body", [](py::bytes b) { return svc::parse_ack_body(std::string(b)); });

  py::class_<svc::BudgetPolicy>(s, "BudgetPolicy")
      .def(py::init<>())
      .def_readwrite("default_output_budget", &svc::BudgetPolicy::default_output_budget)
      .def_readwrite("max_output_budget", &svc::BudgetPolicy::max_output_budget)
      .def_readwrite("max_context_tokens", &svc::BudgetPolicy::max_context_tokens);
  py::class_<svc::ServiceConfig>(s, "ServiceConfig")
      .def(py::init<>())
      .def_readwrite("flags", &svc::ServiceConfig::flags)
      .def_readwrite("request_id_base", &svc::ServiceConfig::request_id_base)
      .def_readwrite("client_capacity", &svc::ServiceConfig::client_capacity)
      .def_readwrite("request_capacity", &svc::ServiceConfig::request_capacity)
      .def_readwrite("event_capacity", &svc::ServiceConfig::event_capacity)
      .def_readwrite("budgets", &svc::ServiceConfig::budgets);
  py::class_<svc::ServiceStats>(s, "ServiceStats")
      .def_readonly("connected_clients", &svc::ServiceStats::connected_clients)
      .def_readonly("live_requests", &svc::ServiceStats::live_requests)
      .def_readonly("completed_mappings", &svc::ServiceStats::completed_mappings)
      .def_readonly("event_count", &svc::ServiceStats::event_count)
      .def_readonly("event_capacity", &svc::ServiceStats::event_capacity)
      .def_readonly("dropped_events", &svc::ServiceStats::dropped_events)
      .def_readonly("submitted", &svc::ServiceStats::submitted)
      .def_readonly("accepted", &svc::ServiceStats::accepted)
      .def_readonly("forwarded_events", &svc::ServiceStats::forwarded_events)
      .def_readonly("cancelled", &svc::ServiceStats::cancelled);
  py::class_<svc::EngineEvent>(s, "EngineEvent")
      .def(py::init([](uint64_t handle, uint32_t kind, uint32_t token_id, uint32_t token_index, uint32_t status) {
             svc::EngineEvent e;
             e.handle = handle;
             e.kind = kind;
             e.token_id = token_id;
             e.token_index = token_index;
             e.status = status;
             return e;
           }),
           py::arg("handle"), py::arg("kind"), py::arg("token_id") = 0, py::arg("token_index") = 0,
           py::arg("status") = 0)
      .def_readwrite("handle", &svc::EngineEvent::handle)
      .def_readwrite("kind", &svc::EngineEvent::kind)
      .def_readwrite("status", &svc::EngineEvent::status)
      .def_readwrite("token_id", &svc::EngineEvent::token_id)
      .def_readwrite("token_index", &svc::EngineEvent::token_index)
      .def_readwrite("token_count", &svc::EngineEvent::token_count)
      .def_readwrite("prompt_token_offset", &svc::EngineEvent::prompt_token_offset)
      .def_readwrite("prompt_token_count", &svc::EngineEvent::prompt_token_count)
      .def_readwrite("dispatch_kind", &svc::EngineEvent::dispatch_kind)
      .def_readwrite("dispatch_flags", &svc::EngineEvent::dispatch_flags);

  py::class_<svc::ServiceRuntime, std::shared_ptr<svc::ServiceRuntime>>(s, "ServiceRuntime")
      .def(py::init<const svc::ServiceConfig&>(), py::arg("config") = svc::ServiceConfig())
      .def("register_client", &svc::ServiceRuntime::register_client, py::arg("cookie") = 0)
      .def("disconnect_client", &svc::ServiceRuntime::disconnect_client)
      .def("has_client", &svc::ServiceRuntime::has_client)
      .def("submit", &svc::ServiceRuntime::submit, py::arg("request"), py::arg("prompt_tokens"))
      .def("cancel", &svc::ServiceRuntime::cancel)
      .def("forward", &svc::ServiceRuntime::forward)
      .def("pop", [](svc::ServiceRuntime& r) -> py::object {
        svc::ServiceEvent e;
        if (!r.pop(&e)) return py::none();
        return py::cast(e);
      })
      .def("pop_all", &svc::ServiceRuntime::pop_all, py::arg("max_events") = size_t(1) << 20)
      .def("lookup", [](const svc::ServiceRuntime& r, uint64_t c, uint64_t q) -> py::object {
        uint64_t h = 0;
        if (!r.lookup(c, q, &h)) return py::none();
        return py::int_(h);
      })
      .def("stats", &svc::ServiceRuntime::stats);

  py::class_<svc::CompatRequest>(s, "CompatRequest")
      .def_readonly("flags", &svc::CompatRequest::flags)
      .def_readonly("chat_flags", &svc::CompatRequest::chat_flags)
      .def_readonly("priority", &svc::CompatRequest::priority)
      .def_readonly("thinking_budget", &svc::CompatRequest::thinking_budget)
      .def_readonly("output_budget", &svc::CompatRequest::output_budget)
      .def_property_readonly("text", [](const svc::CompatRequest& r) { return py::bytes(r.text); });
  s.def("prepare_openai_json", [](py::object body, size_t cap, const std::string& style) {
    return svc::prepare_openai_json(as_bytes(body), cap, style);
  }, py::arg("body"), py::arg("capacity") = size_t(64) << 20, py::arg("style") = "glm");
  s.def("prepare_anthropic_json", [](py::object body, size_t cap, const std::string& style) {
    return svc::prepare_anthropic_json(as_bytes(body), cap, style);
  }, py::arg("body"), py::arg("capacity") = size_t(64) << 20, py::arg("style") = "glm");

  // ---- wire builders
  s.def("route_request", [](const std::string& m, const std::string& p) {
    switch (gw::route_request(m, p)) {
      case gw::Route::DemoUi: return "demo_ui";
      case gw::Route::Health: return "health";
      case gw::Route::Metrics: return "metrics";
      case gw::Route::OpenAiChat: return "openai_chat";
      case gw::Route::OpenAiCompletions: return "openai_completions";
      case gw::Route::AnthropicMessages: return "anthropic_messages";
      case gw::Route::CorsPreflight: return "cors_preflight";
      default: return "none";
    }
  });
  s.def("body_requests_stream", [](py::object b) { return gw::body_requests_stream(as_bytes(b)); });
  s.def("authorization_matches", [](py::object auth, const std::string& key) {
    if (auth.is_none()) return gw::authorization_matches(nullptr, key);
    const std::string a = as_bytes(auth);
    return gw::authorization_matches(&a, key);
  });
  s.def("escape_json_bytes", [](py::object b) { return py::bytes(gw::escape_json_bytes(as_bytes(b))); });
  s.def("sse_event_name", &gw::sse_event_name);
  s.def("build_health_body", &gw::build_health_body);
  s.def("build_submit_accepted_json", &gw::build_submit_accepted_json);
  s.def("build_submit_accepted_sse", &gw::build_submit_accepted_sse);
  s.def("build_service_event_frame", [](const svc::ServiceEvent& e, py::object text) {
    return py::bytes(gw::build_service_event_frame(e, as_bytes(text)));
  }, py::arg("event"), py::arg("token_text") = py::bytes(""));
  s.def("demo_ui_html", &gw::demo_ui_html);
  s.attr("BODY_UNAUTHORIZED") = gw::kBodyUnauthorized;
  s.attr("BODY_NOT_FOUND") = gw::kBodyNotFound;
  s.attr("BODY_BAD_REQUEST") = gw::kBodyBadRequest;
  s.attr("BODY_UNAVAILABLE_JSON") = gw::kBodyUnavailableJson;
  s.attr("BODY_UNAVAILABLE_SSE") = gw::kBodyUnavailableSse;
  s.attr("BODY_TIMEOUT_JSON") = gw::kBodyTimeoutJson;
  s.attr("BODY_TIMEOUT_SSE") = gw::kBodyTimeoutSse;

  py::class_<gw::BackendView>(s, "BackendView")
      .def(py::init<>())
      .def_readwrite("attached", &gw::BackendView::attached)
      .def_readwrite("runtime_initialized", &gw::BackendView::runtime_initialized)
      .def_readwrite("local_control_ready", &gw::BackendView::local_control_ready)
      .def_readwrite("release_id", &gw::BackendView::release_id)
      .def_readwrite("release_git_commit", &gw::BackendView::release_git_commit)
      .def_readwrite("release_generation", &gw::BackendView::release_generation)
      .def_readwrite("transport_shared_object_path", &gw::BackendView::transport_shared_object_path)
      .def_readwrite("first_blocker", &gw::BackendView::first_blocker)
      .def_readwrite("kv_context_limit_tokens", &gw::BackendView::kv_context_limit_tokens)
      .def_readwrite("max_active_sequences", &gw::BackendView::max_active_sequences)
      .def_readwrite("adaptive_decode_batch_width", &gw::BackendView::adaptive_decode_batch_width)
      .def_readwrite("decode_batch_capacity", &gw::BackendView::decode_batch_capacity)
      .def_readwrite("prefill_wave_token_count", &gw::BackendView::prefill_wave_token_count)
      .def_readwrite("transport_capability_flags", &gw::BackendView::transport_capability_flags)
      .def_readwrite("request_api_flags", &gw::BackendView::request_api_flags)
      .def_readwrite("speculation_flags", &gw::BackendView::speculation_flags);
  py::class_<gw::ServingCounters>(s, "ServingCounters")
      .def(py::init<>())
      .def_readwrite("queued_requests", &gw::ServingCounters::queued_requests)
      .def_readwrite("completed_streams", &gw::ServingCounters::completed_streams)
      .def_readwrite("prefill_dispatches", &gw::ServingCounters::prefill_dispatches)
      .def_readwrite("prefill_batch_dispatches", &gw::ServingCounters::prefill_batch_dispatches)
      .def_readwrite("prefill_tokens", &gw::ServingCounters::prefill_tokens)
      .def_readwrite("decode_dispatches", &gw::ServingCounters::decode_dispatches)
      .def_readwrite("decoded_tokens", &gw::ServingCounters::decoded_tokens)
      .def_readwrite("max_prefill_active", &gw::ServingCounters::max_prefill_active)
      .def_readwrite("max_prefill_lanes", &gw::ServingCounters::max_prefill_lanes)
      .def_readwrite("max_decode_active", &gw::ServingCounters::max_decode_active)
      .def_readwrite("max_decode_lanes", &gw::ServingCounters::max_decode_lanes)
      .def_readwrite("jit_prefetch_dispatches", &gw::ServingCounters::jit_prefetch_dispatches)
      .def_readwrite("jit_prefetch_blocks", &gw::ServingCounters::jit_prefetch_blocks)
      .def_readwrite("async_jit_starts", &gw::ServingCounters::async_jit_starts)
      .def_readwrite("async_jit_completions", &gw::ServingCounters::async_jit_completions)
      .def_readwrite("mtp_draft_tokens", &gw::ServingCounters::mtp_draft_tokens)
      .def_readwrite("mtp_verify_dispatches", &gw::ServingCounters::mtp_verify_dispatches)
      .def_readwrite("mtp_draft_ready", &gw::ServingCounters::mtp_draft_ready)
      .def_readwrite("mtp_accepted_draft_tokens", &gw::ServingCounters::mtp_accepted_draft_tokens)
      .def_readwrite("mtp_committed_tokens", &gw::ServingCounters::mtp_committed_tokens)
      .def_readwrite("mtp_rejected_tokens", &gw::ServingCounters::mtp_rejected_tokens);
  py::class_<gw::HealthStats>(s, "HealthStats")
      .def(py::init<>())
      .def_readwrite("connected_clients", &gw::HealthStats::connected_clients)
      .def_readwrite("live_requests", &gw::HealthStats::live_requests)
      .def_readwrite("event_backlog", &gw::HealthStats::event_backlog)
      .def_readwrite("dropped_events", &gw::HealthStats::dropped_events)
      .def_readwrite("serving", &gw::HealthStats::serving);
  s.def("build_service_health_body", &gw::build_service_health_body);
  s.def("build_metrics_body", &gw::build_metrics_body);

  py::class_<gw::GatewayConfig>(s, "GatewayConfig")
      .def(py::init<>())
      .def_readwrite("host", &gw::GatewayConfig::host)
      .def_readwrite("port", &gw::GatewayConfig::port)
      .def_readwrite("frame_port", &gw::GatewayConfig::frame_port)
      .def_readwrite("api_key", &gw::GatewayConfig::api_key)
      .def_readwrite("max_request_bytes", &gw::GatewayConfig::max_request_bytes)
      .def_readwrite("text_capacity", &gw::GatewayConfig::text_capacity)
      .def_readwrite("template_style", &gw::GatewayConfig::template_style)
      .def_readwrite("max_connections", &gw::GatewayConfig::max_connections);
  py::class_<gw::EngineWork>(s, "EngineWork")
      .def_readonly("kind", &gw::EngineWork::kind)
      .def_readonly("handle", &gw::EngineWork::handle)
      .def_readonly("token_ids", &gw::EngineWork::token_ids)
      .def_readonly("output_budget", &gw::EngineWork::output_budget)
      .def_readonly("thinking_budget", &gw::EngineWork::thinking_budget)
      .def_readonly("priority", &gw::EngineWork::priority)
      .def_readonly("flags", &gw::EngineWork::flags)
      .def_readonly("client_id", &gw::EngineWork::client_id)
      .def_readonly("client_request_id", &gw::EngineWork::client_request_id);
  s.attr("WORK_SUBMIT") = uint32_t(gw::EngineWork::Submit);
  s.attr("WORK_CANCEL") = uint32_t(gw::EngineWork::Cancel);
  py::class_<gw::Gateway, std::shared_ptr<gw::Gateway>>(s, "Gateway")
      .def(py::init<const gw::GatewayConfig&, std::shared_ptr<Tokenizer>, std::shared_ptr<svc::ServiceRuntime>>(),
           py::arg("config"), py::arg("tokenizer"), py::arg("service"))
      .def("start", &gw::Gateway::start)
      .def("stop", &gw::Gateway::stop, py::call_guard<py::gil_scoped_release>())
      .def_property_readonly("port", &gw::Gateway::port)
      .def_property_readonly("frame_port", &gw::Gateway::frame_port)
      .def_property_readonly("running", &gw::Gateway::running)
      .def_property_readonly("accepted_connections", &gw::Gateway::accepted_connections)
      .def_property_readonly("cancelled_by_disconnect", &gw::Gateway::cancelled_by_disconnect)
      .def("set_backend_view", &gw::Gateway::set_backend_view)
      .def("set_serving_counters", &gw::Gateway::set_serving_counters)
      .def("poll_work", &gw::Gateway::poll_work, py::arg("timeout_ms") = 0, py::arg("max_items") = 1024,
           py::call_guard<py::gil_scoped_release>())
      .def("publish", &gw::Gateway::publish, py::call_guard<py::gil_scoped_release>());
});
