"""Service runtime, binary frame codec and compat JSON (C++), on CPU.

Compat cases mirror crates/spark-serve/tests/serving_engine.rs:1486-1625;
frame layouts follow crates/spark-serve/src/serving_engine/service.rs:350-440
and :1301-1328."""
import struct

import pytest

from sparkpipe_rs_b200.core import StatusError, core

S = core().serving
CHAT_BEGIN = "[gMASK]<sop><|system|>Reasoning Effort: Max"
CHAT_END = "<|assistant|><think>"
NO_THINK_BEGIN = "[gMASK]<sop>"
NO_THINK_END = "<|assistant|><think></think>"


# ------------------------------------------------------------------ frame codec
def test_frame_header_layout_and_validation():
    h = S.FrameHeader()
    h.kind, h.flags, h.body_bytes, h.client_id, h.client_request_id = S.FRAME_PING, 1, 0, 7, 9
    b = S.serialize_header(h)
    assert len(b) == 40
    assert struct.unpack("<IIIIIIQQ", b) == (0x35504B53, 1, 40, S.FRAME_PING, 1, 0, 7, 9)
    h2 = S.parse_header(b)
    assert (h2.kind, h2.client_id, h2.client_request_id) == (S.FRAME_PING, 7, 9)
    with pytest.raises(StatusError) as e:
        S.parse_header(b"\0" * 40)
    assert e.value.code == 1  # invalid_argument
    h.kind = 55
    with pytest.raises(StatusError):
        S.validate_header(h)
    h.kind, h.body_bytes = S.FRAME_SUBMIT_TEXT, (128 << 20) + 1
    with pytest.raises(StatusError) as e:
        S.validate_header(h)
    assert e.value.code == 2  # capacity_exceeded


def test_submit_frames_roundtrip():
    r = S.SubmitRequest()
    r.flags, r.priority, r.output_budget, r.thinking_budget = 1, 5, 33, 4
    r.client_id, r.client_request_id, r.sequence_id = 3, 44, 99
    r.text = "hello"
    f = S.build_submit_text_frame(r)
    h = S.parse_header(f[:40])
    assert h.kind == S.FRAME_SUBMIT_TEXT and h.body_bytes == 45 and h.flags == 1
    body = f[40:]
    assert struct.unpack("<IIIIIIIIQ", body[:40]) == (1, 40, 5, 4, 33, 0, 0, 5, 99)
    p = S.parse_submit_text_frame(h, body)
    assert (p.text, p.priority, p.output_budget, p.sequence_id, p.client_request_id) == (b"hello", 5, 33, 99, 44)
    r.token_ids = [1, 2, 3]
    f = S.build_submit_tokens_frame(r)
    h = S.parse_header(f[:40])
    p = S.parse_submit_tokens_frame(h, f[40:])
    assert list(p.token_ids) == [1, 2, 3] and p.priority == 5
    with pytest.raises(StatusError):  # size mismatch
        S.parse_submit_tokens_frame(h, f[40:-4])
    c = S.build_cancel_frame(3, 44)
    assert S.parse_cancel_frame(S.parse_header(c[:40]), c[40:]) == 44


def test_event_frame_layout():
    e = S.ServiceEvent()
    e.kind, e.status, e.token_id, e.token_index = S.EV_TOKEN, 0, 321, 12
    e.client_id, e.client_request_id, e.serving_request_id, e.sequence_id, e.serving_request_handle = 1, 2, 3, 4, 5
    f = S.build_event_frame(e)
    assert len(f) == 40 + 88
    h = S.parse_header(f[:40])
    assert h.kind == S.FRAME_EVENT and h.body_bytes == 88 and h.client_id == 1 and h.client_request_id == 2
    vals = struct.unpack("<" + "I" * 12 + "Q" * 5, f[40:])
    assert vals[:6] == (1, 88, S.EV_TOKEN, 0, 0, 321) and vals[6] == 12 and vals[12:] == (1, 2, 3, 4, 5)
    e2 = S.parse_event_body(f[40:])
    assert (e2.token_id, e2.serving_request_handle) == (321, 5)


# ------------------------------------------------------------------ runtime
def _runtime(**budget):
    cfg = S.ServiceConfig()
    b = S.BudgetPolicy()
    b.default_output_budget = budget.get("default", 16)
    b.max_output_budget = budget.get("max_out", 64)
    b.max_context_tokens = budget.get("ctx", 128)
    cfg.budgets = b
    cfg.event_capacity = budget.get("events", 1024)
    return S.ServiceRuntime(cfg)


def _req(client, creq, out=0):
    r = S.SubmitRequest()
    r.client_id, r.client_request_id, r.output_budget = client, creq, out
    return r


def test_submit_maps_ids_and_clamps_budgets():
    rt = _runtime()
    c = rt.register_client(0)
    ev = rt.pop()
    assert ev.kind == S.EV_CLIENT_CONNECTED and ev.client_id == c
    r1 = rt.submit(_req(c, 1), 10)
    assert r1.serving_request_id == S.DEFAULT_REQUEST_ID_BASE and r1.output_budget == 16
    assert r1.required_token_capacity == 26 and r1.serving_request_handle == r1.serving_request_id
    r2 = rt.submit(_req(c, 2, out=1000), 100)
    assert r2.serving_request_id == r1.serving_request_id + 1 and r2.output_budget == 28  # context-limited
    with pytest.raises(StatusError) as e:
        rt.submit(_req(c, 1), 5)
    assert e.value.code == 16  # duplicate
    with pytest.raises(StatusError) as e:
        rt.submit(_req(c + 99, 9), 5)
    assert e.value.code == 3  # not_found
    with pytest.raises(StatusError):
        rt.submit(_req(c, 0), 5)
    with pytest.raises(StatusError) as e:
        rt.submit(_req(c, 3), 128)
    assert e.value.code == 2
    assert rt.stats().live_requests == 2 and rt.lookup(c, 2) == r2.serving_request_handle


def test_forward_routes_events_and_releases_on_terminal():
    rt = _runtime()
    c = rt.register_client(0)
    rt.pop()
    r = rt.submit(_req(c, 5), 4)
    h = r.serving_request_handle
    n = rt.forward([S.EngineEvent(h, S.EV_TOKEN, 11, 4), S.EngineEvent(h, S.EV_TOKEN, 12, 5),
                    S.EngineEvent(999, S.EV_TOKEN, 1, 1), S.EngineEvent(h, S.EV_COMPLETED, 0, 6)])
    assert n == 3
    evs = rt.pop_all()
    assert [e.kind for e in evs] == [S.EV_TOKEN, S.EV_TOKEN, S.EV_COMPLETED]
    assert all(e.client_id == c and e.client_request_id == 5 and e.serving_request_id == h for e in evs)
    assert rt.lookup(c, 5) is None  # auto-released
    rt.submit(_req(c, 5), 4)  # the id is reusable after completion


def test_cancel_keeps_mapping_until_engine_reports():
    rt = _runtime()
    c = rt.register_client(0)
    rt.pop()
    h = rt.submit(_req(c, 7), 4).serving_request_handle
    assert rt.cancel(c, 7) == h
    with pytest.raises(StatusError):
        rt.cancel(c, 7)
    assert rt.forward([S.EngineEvent(h, S.EV_CANCELLED)]) == 1
    e = rt.pop()
    assert e.kind == S.EV_CANCELLED and e.client_request_id == 7


def test_disconnect_returns_live_handles():
    rt = _runtime()
    c = rt.register_client(0)
    h1 = rt.submit(_req(c, 1), 4).serving_request_handle
    h2 = rt.submit(_req(c, 2), 4).serving_request_handle
    assert sorted(rt.disconnect_client(c)) == sorted([h1, h2])
    assert not rt.has_client(c)
    assert rt.forward([S.EngineEvent(h1, S.EV_TOKEN, 1, 1)]) == 0
    kinds = [e.kind for e in rt.pop_all()]
    assert kinds == [S.EV_CLIENT_CONNECTED, S.EV_CLIENT_DISCONNECTED]


def test_full_ring_drops_tokens_not_terminals():
    rt = _runtime(events=2)
    c = rt.register_client(0)
    h = rt.submit(_req(c, 1), 4).serving_request_handle
    rt.forward([S.EngineEvent(h, S.EV_TOKEN, i, i) for i in range(5)] + [S.EngineEvent(h, S.EV_COMPLETED)])
    st = rt.stats()
    assert st.dropped_events == 4
    kinds = [e.kind for e in rt.pop_all()]
    assert kinds == [S.EV_CLIENT_CONNECTED, S.EV_TOKEN, S.EV_COMPLETED]


# ------------------------------------------------------------------ compat
def test_compat_openai_chat():
    body = ('{"model":"glm-5.2","priority":123,"max_tokens":17,"messages":['
            '{"role":"system","content":"You are terse."},{"role":"user","content":"Read this C code."}]}')
    r = S.prepare_openai_json(body, 512)
    assert r.output_budget == 17 and r.priority == 123
    assert r.text.decode() == f"{CHAT_BEGIN}<|system|>You are terse.<|user|>Read this C code.{CHAT_END}"


def test_compat_openai_prompt_and_thinking():
    r = S.prepare_openai_json('{"model":"m","max_completion_tokens":5,"prompt":"plain prompt"}', 64)
    assert r.output_budget == 5 and r.text == b"plain prompt"
    r = S.prepare_openai_json('{"thinking_budget_tokens":0,"messages":[{"role":"user","content":"Answer."}]}', 256)
    assert r.thinking_budget == 0 and r.text.decode() == f"{NO_THINK_BEGIN}<|user|>Answer.{NO_THINK_END}"
    r = S.prepare_openai_json('{"thinking_token_budget":1024,"messages":[{"role":"user","content":"Answer."}]}', 256)
    assert r.thinking_budget == 1024 and r.text.decode() == f"{CHAT_BEGIN}<|user|>Answer.{CHAT_END}"
    with pytest.raises(StatusError) as e:
        S.prepare_openai_json('{"thinking_budget_tokens":0,"thinking_token_budget":1024,'
                              '"messages":[{"role":"user","content":"Answer."}]}', 256)
    assert e.value.code == 1


def test_compat_files_and_anthropic():
    body = ('{"messages":[{"role":"user","content":[{"type":"text","text":"Use the attachment."}]}],'
            '"files":[{"filename":"notes.txt","content":"alpha\\nbeta"}]}')
    t = S.prepare_openai_json(body, 512).text.decode()
    assert t == (f"{CHAT_BEGIN}<|user|>Use the attachment.\n[uploaded file: notes.txt]\nalpha\nbeta"
                 f"\n[/uploaded file]\n{CHAT_END}")
    body = ('{"priority":456,"system":"Stay exact.","max_tokens":9,"messages":['
            '{"role":"user","content":[{"type":"text","text":"First"},{"type":"text","text":" second"}]},'
            '{"role":"assistant","content":"Ack"}]}')
    r = S.prepare_anthropic_json(body, 512)
    assert r.output_budget == 9 and r.priority == 456
    assert r.text.decode() == (f"{CHAT_BEGIN}<|system|>Stay exact.<|user|>First second"
                               f"<|assistant|><think></think>Ack{CHAT_END}")


def test_compat_errors():
    with pytest.raises(StatusError) as e:
        S.prepare_openai_json('{"messages":[{"role":"alien","content":"no"}]}', 256)
    assert e.value.code == 1
    with pytest.raises(StatusError) as e:
        S.prepare_openai_json('{"messages":[{"role":"user","content":"too long for buffer"}]}', 8)
    assert e.value.code == 2
    with pytest.raises(StatusError) as e:
        S.prepare_openai_json('{"messages": [', 256)
    assert e.value.code == 5  # parse_error
    with pytest.raises(StatusError):
        S.prepare_openai_json('{"max_tokens":-1,"prompt":"x"}', 256)
    with pytest.raises(StatusError):
        S.prepare_openai_json('{"files":[{"filename":"a"}],"prompt":"x"}', 256)  # file without content
    with pytest.raises(StatusError):
        S.prepare_anthropic_json('{"system":"x"}', 256)


def test_compat_deepseek_style():
    r = S.prepare_openai_json('{"messages":[{"role":"user","content":"hi"}]}', 256, "deepseek")
    assert r.text.decode() == "<｜begin▁of▁sentence｜><｜User｜>hi<｜Assistant｜>"


# ------------------------------------------------------------------ wire helpers
def test_stream_scan_auth_and_routes():
    assert S.body_requests_stream(b'{"stream":true}')
    assert S.body_requests_stream(b'{"x":1, "stream" \n:\t true}')
    assert not S.body_requests_stream(b'{"stream":false}')
    assert not S.body_requests_stream(b'{"streaming":true}')
    assert S.body_requests_stream(b'{"streamx":1,"stream":true}')
    assert S.authorization_matches(None, "")
    assert not S.authorization_matches(None, "k")
    assert S.authorization_matches(b"Bearer k", "k")
    assert not S.authorization_matches(b"bearer k", "k")
    assert not S.authorization_matches(b"Bearer " + b"x" * 600, "x" * 600)
    assert S.route_request("GET", "/health") == "health"
    assert S.route_request("POST", "/health") == "none"
    assert S.route_request("OPTIONS", "/anything") == "cors_preflight"
    assert S.route_request("POST", "/v1/messages") == "anthropic_messages"
    assert S.escape_json_bytes(b'a"b\\c\n\x01\xff') == b'a\\"b\\\\c\\n\\u0001\xff'


def test_accepted_and_event_bodies_are_byte_exact():
    r = S.SubmitResult()
    r.client_request_id, r.serving_request_id, r.sequence_id = 2, 5000000003, 7
    r.prompt_token_count, r.output_budget = 11, 64
    assert S.build_submit_accepted_json(r) == (
        '{"id":"spreq-5000000003","object":"sparkpipe.request","client_request_id":2,'
        '"serving_request_id":5000000003,"sequence_id":7,"prompt_tokens":11,"output_token_budget":64,'
        '"status":"queued"}\n')
    assert S.build_submit_accepted_sse(r) == (
        'event: accepted\ndata: {"client_request_id":2,"serving_request_id":5000000003,"sequence_id":7,'
        '"prompt_tokens":11,"output_token_budget":64}\n\n')
    e = S.ServiceEvent()
    e.kind, e.client_id, e.client_request_id, e.serving_request_id, e.sequence_id = S.EV_TOKEN, 1, 2, 3, 4
    e.token_id, e.token_index = 65, 9
    assert S.build_service_event_frame(e, b'a"b\nc') == (
        b'event: token\ndata: {"kind":3,"status":0,"client_id":1,"client_request_id":2,'
        b'"serving_request_id":3,"sequence_id":4,"token_id":65,"token_index":9,"text":"a\\"b\\nc"}\n\n')
    e.kind = S.EV_COMPLETED
    assert S.build_service_event_frame(e).startswith(b"event: done\n")
    e.kind = S.EV_PREFILL_PROGRESS
    assert S.build_service_event_frame(e).startswith(b"event: event\n")


def test_health_body_statuses():
    v = S.BackendView()
    st = S.HealthStats()
    body = S.build_service_health_body(st, v)
    assert body.startswith('{"schema":"sparkpipe.runtime_observation.v1","release_identity_status":"NOT_MEASURED",')
    assert '"runtime_initialized":0' in body and '"multi_sequence_batching_status":"NOT_WORKING"' in body
    assert body.endswith('"first_blocker":""}\n')
    v.attached = v.runtime_initialized = v.local_control_ready = True
    v.release_id, v.release_git_commit, v.release_generation = "r1", "abc", 3
    v.max_active_sequences = 64
    v.speculation_flags = S.BACKEND_FLAG_MTP
    v.first_blocker = 'x"y'
    st.serving.completed_streams = 1
    st.serving.decoded_tokens = 10
    st.serving.max_decode_lanes = 8
    st.serving.mtp_verify_dispatches = 2
    body = S.build_service_health_body(st, v)
    for frag in ('"release_identity_status":"OBSERVED"', '"end_to_end_observation_status":"OBSERVED"',
                 '"multi_sequence_batching_status":"OBSERVED"', '"mtp_status":"OBSERVED"',
                 '"dspark_status":"NOT_WORKING"', '"jit_kv_status":"NOT_WORKING"', '"first_blocker":"x\\"y"}'):
        assert frag in body, frag
    assert S.build_health_body(True, False) == (
        '{"schema":"sparkpipe.runtime_observation.v1","runtime_initialized":1,"local_control_ready":0,'
        '"end_to_end_observation_status":"NOT_MEASURED","accuracy_status":"NOT_MEASURED",'
        '"performance_status":"NOT_MEASURED"}\n')
