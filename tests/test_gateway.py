"""HTTP/1.1 + SSE gateway and the binary frame endpoint over real loopback
sockets, with a scripted engine thread (no model). Cases follow the
reference gateway's socket tests (crates/spark-serve/tests/http_gateway.rs:
CORS :277, demo page :294, 404 :306, health :324-425, auth :434, 503 :470,
oversize :545, SSE frames :565, escaping :671, disconnect -> cancel :721,
keep-alive :755)."""
import json
import socket
import threading
import time

import pytest
import _http

from sparkpipe_rs_b200.core import core
from sparkpipe_rs_b200.serving.tokenizers import byte_level_tokenizer

S = core().serving


class ScriptedEngine:
    """Engine thread stand-in: answers each submission with a scripted token list."""

    def __init__(self, gw, tokens=(72, 105), hold=False):
        self.gw = gw
        self.tokens = list(tokens)
        self.hold = hold  # True: emit the first token, then wait (for disconnect tests)
        self.submits, self.cancels = [], []
        self.stop = threading.Event()
        self.t = threading.Thread(target=self.run, daemon=True)
        self.t.start()

    def run(self):
        while not self.stop.is_set():
            for w in self.gw.poll_work(20, 64):
                if w.kind == S.WORK_SUBMIT:
                    self.submits.append(w)
                    n = len(w.token_ids)
                    toks = self.tokens[:1] if self.hold else self.tokens
                    evs = [S.EngineEvent(w.handle, S.EV_TOKEN, t, n + i) for i, t in enumerate(toks)]
                    if not self.hold:
                        evs.append(S.EngineEvent(w.handle, S.EV_COMPLETED, 0, n + len(toks)))
                    self.gw.publish(evs)
                else:
                    self.cancels.append(w.handle)
                    self.gw.publish([S.EngineEvent(w.handle, S.EV_CANCELLED)])

    def close(self):
        self.stop.set()
        self.t.join(5)


@pytest.fixture
def server(request):
    opts = getattr(request, "param", {})
    svc = S.ServiceRuntime()
    gc = S.GatewayConfig()
    gc.api_key = opts.get("api_key", "")
    gc.frame_port = 0
    if "max_request_bytes" in opts:
        gc.max_request_bytes = opts["max_request_bytes"]
    gw = S.Gateway(gc, byte_level_tokenizer(1024), svc)
    v = S.BackendView()
    v.attached = v.runtime_initialized = v.local_control_ready = opts.get("ready", True)
    v.max_active_sequences = 8
    gw.set_backend_view(v)
    gw.start()
    eng = ScriptedEngine(gw, hold=opts.get("hold", False))
    yield gw, eng, svc
    eng.close()
    gw.stop()


def test_cors_demo_404_and_keepalive(server):
    gw, _, _ = server
    sock = _http.connect(gw.port)
    sock.sendall(_http.build("OPTIONS", "/v1/chat/completions"))
    r, rest = _http.read_response(sock)
    assert r.status == 200 and r.header("content-type") == "text/plain" and r.body == b""
    assert r.header("access-control-allow-origin") == "*"
    assert r.header("access-control-allow-headers") == "authorization, content-type"
    assert r.header("access-control-allow-methods") == "GET, POST, OPTIONS"
    assert r.header("cache-control") == "no-cache"
    sock.sendall(_http.build("GET", "/"))  # same connection: keep-alive
    r, rest = _http.read_response(sock, rest)
    assert r.status == 200 and r.header("content-type") == "text/html; charset=utf-8"
    assert r.body.startswith(b"<!doctype html>") and r.body.endswith(b"</html>")
    for method, path in [("GET", "/nope"), ("POST", "/health"), ("GET", "/v1/chat/completions")]:
        sock.sendall(_http.build(method, path))
        r, rest = _http.read_response(sock, rest)
        assert r.status == 404 and r.header("content-type") == "application/json"
        assert r.body.decode() == S.BODY_NOT_FOUND
    sock.close()
    assert gw.accepted_connections == 1


def test_pipelined_requests_on_one_connection(server):
    gw, _, _ = server
    sock = _http.connect(gw.port)
    sock.sendall(_http.build("GET", "/health") + _http.build("GET", "/metrics") + _http.build("GET", "/x"))
    r1, rest = _http.read_response(sock)
    r2, rest = _http.read_response(sock, rest)
    r3, rest = _http.read_response(sock, rest)
    assert (r1.status, r2.status, r3.status) == (200, 200, 404)
    assert b"sparkpipe_backend_attached 1" in r2.body
    sock.close()


@pytest.mark.parametrize("server", [{"ready": False}], indirect=True)
def test_unattached_health_and_503(server):
    gw, _, _ = server
    r = _http.request(gw.port, "GET", "/health")
    body = r.body.decode()
    assert body.startswith('{"schema":"sparkpipe.runtime_observation.v1",') and body.endswith("}\n")
    assert '"runtime_initialized":0' in body and '"mtp_status":"NOT_WORKING"' in body
    r = _http.request(gw.port, "POST", "/v1/chat/completions", "{}")
    assert r.status == 503 and r.header("content-type") == "application/json"
    assert r.body.decode() == S.BODY_UNAVAILABLE_JSON
    r = _http.request(gw.port, "POST", "/v1/chat/completions", '{"stream":true}')
    assert r.status == 503 and r.header("content-type") == "text/event-stream"
    assert r.body.decode() == S.BODY_UNAVAILABLE_SSE


@pytest.mark.parametrize("server", [{"api_key": "sekret"}], indirect=True)
def test_auth_only_on_completion_routes(server):
    gw, _, _ = server
    body = '{"prompt":"hi"}'
    r = _http.request(gw.port, "POST", "/v1/completions", body)
    assert r.status == 401 and r.body.decode() == S.BODY_UNAUTHORIZED
    r = _http.request(gw.port, "POST", "/v1/completions", body, {"authorization": "Bearer wrong"})
    assert r.status == 401
    r = _http.request(gw.port, "POST", "/v1/completions", body, {"authorization": "Bearer sekret"})
    assert r.status == 202
    assert _http.request(gw.port, "GET", "/health").status == 200
    assert _http.request(gw.port, "GET", "/").status == 200


def test_nonstream_submit_is_byte_exact(server):
    gw, eng, _ = server
    r = _http.request(gw.port, "POST", "/v1/completions", '{"prompt":"hello","max_tokens":7}')
    assert r.status == 202 and r.header("content-type") == "application/json"
    j = json.loads(r.body)
    assert j["client_request_id"] & S.NONSTREAM_REQUEST_BIT
    assert j["prompt_tokens"] == 5 and j["output_token_budget"] == 7 and j["status"] == "queued"
    expected = (f'{{"id":"spreq-{j["serving_request_id"]}","object":"sparkpipe.request",'
                f'"client_request_id":{j["client_request_id"]},"serving_request_id":{j["serving_request_id"]},'
                f'"sequence_id":{j["sequence_id"]},"prompt_tokens":5,"output_token_budget":7,"status":"queued"}}\n')
    assert r.body.decode() == expected
    deadline = time.time() + 5
    while not eng.submits and time.time() < deadline:
        time.sleep(0.01)
    w = eng.submits[0]
    assert list(w.token_ids) == list(b"hello") and w.output_budget == 7


@pytest.mark.parametrize("server", [{"max_request_bytes": 256}], indirect=True)
def test_oversized_and_malformed_requests_are_400(server):
    gw, _, _ = server
    r = _http.request(gw.port, "POST", "/v1/chat/completions", '{"prompt":"' + "x" * 400 + '"}')
    assert r.status == 400 and r.body.decode() == S.BODY_BAD_REQUEST
    r = _http.request(gw.port, "POST", "/v1/chat/completions", '{"messages": [')
    assert r.status == 400


def test_sse_stream_frames_are_byte_exact(server):
    gw, eng, _ = server
    body = '{"model":"m","stream":true,"messages":[{"role":"user","content":"hi"}]}'
    sock = _http.connect(gw.port)
    sock.sendall(_http.build("POST", "/v1/chat/completions", body))
    status, headers, rest = _http.read_head(sock)
    h = dict((k.lower(), v) for k, v in headers)
    assert status == 202 and h["content-type"] == "text/event-stream" and h["transfer-encoding"] == "chunked"
    first, rest = _http.read_chunk(sock, rest)
    acc = first.decode()
    assert acc.startswith('event: accepted\ndata: {"client_request_id":1,"serving_request_id":')
    sid = json.loads(acc.split("data: ", 1)[1])["serving_request_id"]
    frames = []
    while True:
        c, rest = _http.read_chunk(sock, rest)
        if c is None:
            break
        frames.append(c.decode())
    client = eng.submits[0].client_id
    seq = json.loads(acc.split("data: ", 1)[1])["sequence_id"]
    n = len(eng.submits[0].token_ids)

    def frame(name, kind, tok, idx, text):
        return (f'event: {name}\ndata: {{"kind":{kind},"status":0,"client_id":{client},"client_request_id":1,'
                f'"serving_request_id":{sid},"sequence_id":{seq},"token_id":{tok},"token_index":{idx},'
                f'"text":"{text}"}}\n\n')
    assert frames == [frame("token", 3, 72, n, "H"), frame("token", 3, 105, n + 1, "i"),
                      frame("done", 4, 0, n + 2, "")]
    # the connection stays usable after the stream ends
    sock.sendall(_http.build("GET", "/health"))
    r, _ = _http.read_response(sock, rest)
    assert r.status == 200 and '"live_requests":0' in r.body.decode()
    sock.close()
    assert eng.cancels == []


def test_sse_token_text_is_escaped(server):
    gw, eng, _ = server
    eng.tokens = [ord('"'), ord("\n"), 1, ord("\\")]
    r = _http.request(gw.port, "POST", "/v1/completions", '{"prompt":"q","stream":true}')
    body = r.body.decode()
    assert '"text":"\\""' in body and '"text":"\\n"' in body and '"text":"\\u0001"' in body
    assert '"text":"\\\\"' in body and "event: done\n" in body


@pytest.mark.parametrize("server", [{"hold": True}], indirect=True)
def test_sse_client_disconnect_cancels_request(server):
    gw, eng, svc = server
    sock = _http.connect(gw.port)
    sock.sendall(_http.build("POST", "/v1/chat/completions", '{"stream":true,"prompt":"abc"}'))
    status, _, rest = _http.read_head(sock)
    assert status == 202
    _, rest = _http.read_chunk(sock, rest)  # accepted
    tok, rest = _http.read_chunk(sock, rest)
    assert tok.startswith(b"event: token\n")
    assert svc.stats().live_requests == 1
    sock.close()
    deadline = time.time() + 5
    while not eng.cancels and time.time() < deadline:
        time.sleep(0.01)
    assert eng.cancels == [eng.submits[0].handle]
    assert gw.cancelled_by_disconnect == 1
    assert svc.stats().live_requests == 0


def _read_frame(sock, buf):
    while len(buf) < 40:
        buf += sock.recv(65536)
    h = S.parse_header(buf[:40])
    while len(buf) < 40 + h.body_bytes:
        buf += sock.recv(65536)
    return h, buf[40:40 + h.body_bytes], buf[40 + h.body_bytes:]


def test_frame_endpoint_submit_ping_cancel(server):
    gw, eng, _ = server
    sock = socket.create_connection(("127.0.0.1", gw.frame_port), timeout=20)
    h, body, buf = _read_frame(sock, b"")
    assert h.kind == S.FRAME_EVENT
    hello = S.parse_event_body(body)
    assert hello.kind == S.EV_CLIENT_CONNECTED
    client = hello.client_id
    sock.sendall(S.build_ping_frame(client, 1234))
    h, body, buf = _read_frame(sock, buf)
    assert h.kind == S.FRAME_PONG and h.client_request_id == 1234
    r = S.SubmitRequest()
    r.client_request_id, r.output_budget = 77, 5
    r.token_ids = [5, 6, 7]
    sock.sendall(S.build_submit_tokens_frame(r))
    h, body, buf = _read_frame(sock, buf)
    assert h.kind == S.FRAME_SUBMIT_ACK
    ack = S.parse_ack_body(body)
    assert ack.client_id == client and ack.client_request_id == 77 and ack.prompt_token_count == 3
    kinds = []
    while not kinds or kinds[-1] != S.EV_COMPLETED:
        h, body, buf = _read_frame(sock, buf)
        e = S.parse_event_body(body)
        assert e.client_request_id == 77 and e.serving_request_handle == ack.serving_request_handle
        kinds.append(e.kind)
    assert kinds == [S.EV_TOKEN, S.EV_TOKEN, S.EV_COMPLETED]
    r.text = "hey"
    r.client_request_id = 78
    sock.sendall(S.build_submit_text_frame(r))
    h, body, buf = _read_frame(sock, buf)
    assert h.kind == S.FRAME_SUBMIT_ACK and S.parse_ack_body(body).prompt_token_count == 3
    sock.sendall(S.build_cancel_frame(client, 999))  # unknown id -> error frame
    while True:
        h, body, buf = _read_frame(sock, buf)
        if h.kind == S.FRAME_ERROR:
            break
    assert h.client_request_id == 999
    sock.close()
