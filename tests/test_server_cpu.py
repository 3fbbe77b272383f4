"""End-to-end server on CPU: HTTP request -> C++ gateway (compat, tokenizer,
service runtime) -> engine thread (C++ scheduler + CPU stage driver) -> SSE
tokens, checked against the fp32 oracle's greedy generation."""
import json
import time

import torch
import _http

from sparkpipe_rs_b200.core import core
from sparkpipe_rs_b200.models import oracle
from sparkpipe_rs_b200.models.config import tiny
from sparkpipe_rs_b200.models.cpu_model import CpuMLAMoEModel
from sparkpipe_rs_b200.serving.engine import EngineConfig, LLMEngine
from sparkpipe_rs_b200.serving.server import ServingServer
from sparkpipe_rs_b200.serving.tokenizers import byte_level_tokenizer

S = core().serving


def _server(**kw):
    cfg = tiny()
    m = CpuMLAMoEModel(cfg, seed=0)
    eng = LLMEngine(cfg, EngineConfig(max_batch=4, block_size=16, max_model_len=256, max_prefill_tokens=64),
                    model=m, device="cpu")
    tok = byte_level_tokenizer(cfg.vocab_size)
    return cfg, m, tok, ServingServer(eng, tok, default_max_tokens=6, **kw)


def _sse_events(body: bytes):
    out = []
    for frame in body.decode("utf-8", "replace").split("\n\n"):
        if not frame:
            continue
        name = frame.split("\n", 1)[0][len("event: "):]
        data = json.loads(frame.split("data: ", 1)[1])
        out.append((name, data))
    return out


def test_stream_chat_matches_oracle():
    cfg, m, tok, srv = _server()
    with srv:
        body = json.dumps({"stream": True, "max_tokens": 5, "messages": [{"role": "user", "content": "hello"}]})
        r = _http.request(srv.port, "POST", "/v1/chat/completions", body)
        assert r.status == 202
        evs = _sse_events(r.body)
        assert evs[0][0] == "accepted" and evs[-1][0] == "done" and evs[-1][1]["kind"] == S.EV_COMPLETED
        toks = [d["token_id"] for n, d in evs if n == "token"]
        prompt = S.prepare_openai_json(body, 1 << 20).text
        ids = tok.encode(prompt)
        assert evs[0][1]["prompt_tokens"] == len(ids)
        ref, _ = oracle.greedy_generate(cfg, m.w, torch.tensor(ids), 5)
        assert toks == ref.tolist()
        idx = [d["token_index"] for n, d in evs if n == "token"]
        assert idx == list(range(len(ids), len(ids) + 5))
        # health reflects the completed stream
        h = _http.request(srv.port, "GET", "/health").body.decode()
        deadline = time.time() + 5
        while '"end_to_end_observation_status":"OBSERVED"' not in h and time.time() < deadline:
            time.sleep(0.06)
            h = _http.request(srv.port, "GET", "/health").body.decode()
        assert '"end_to_end_observation_status":"OBSERVED"' in h
    assert srv.error is None


def test_concurrent_streams_and_nonstream():
    cfg, m, tok, srv = _server()
    with srv:
        socks = []
        for i in range(3):
            s = _http.connect(srv.port)
            s.sendall(_http.build("POST", "/v1/completions",
                                  json.dumps({"stream": True, "prompt": f"prompt number {i}", "max_tokens": 4})))
            socks.append(s)
        r = _http.request(srv.port, "POST", "/v1/completions", json.dumps({"prompt": "fire and forget"}))
        assert r.status == 202 and json.loads(r.body)["output_token_budget"] == 6
        for i, s in enumerate(socks):
            resp, _ = _http.read_response(s)
            evs = _sse_events(resp.body)
            toks = [d["token_id"] for n, d in evs if n == "token"]
            ids = tok.encode(f"prompt number {i}")
            ref, _ = oracle.greedy_generate(cfg, m.w, torch.tensor(ids), 4)
            assert toks == ref.tolist()
            s.close()
        deadline = time.time() + 10
        while srv.engine.has_unfinished_requests() and time.time() < deadline:
            time.sleep(0.02)
        assert not srv.engine.has_unfinished_requests()
    assert srv.error is None


def test_disconnect_aborts_engine_request():
    cfg, m, tok, srv = _server()
    with srv:
        s = _http.connect(srv.port)
        s.sendall(_http.build("POST", "/v1/completions",
                              json.dumps({"stream": True, "prompt": "long one", "max_tokens": 200})))
        status, _, rest = _http.read_head(s)
        assert status == 202
        c, rest = _http.read_chunk(s, rest)
        c, rest = _http.read_chunk(s, rest)  # first token
        assert c.startswith(b"event: token")
        s.close()
        deadline = time.time() + 10
        while srv.engine.has_unfinished_requests() and time.time() < deadline:
            time.sleep(0.02)
        assert not srv.engine.has_unfinished_requests()
        assert srv.gateway.cancelled_by_disconnect == 1
        assert srv.engine.scheduler.stats.cancelled == 1


def test_stream_with_tree_speculation_matches_oracle():
    """Speculative decoding through the HTTP path: MTP-tree verify rounds inside the
    engine thread, tokens equal to the oracle's greedy continuation, MTP counters in
    the health body."""
    from sparkpipe_rs_b200.models.config import mtp_head

    cfg = mtp_head(tiny())
    m = CpuMLAMoEModel(cfg, seed=0)
    g = torch.Generator().manual_seed(99)
    wd = {k: (v + 0.15 * v.std() * torch.randn(v.shape, generator=g)) if k not in ("embed", "lm_head") and v.dim() > 1
          else v.clone() for k, v in m.w.items()}
    eng = LLMEngine(cfg, EngineConfig(max_batch=4, block_size=16, max_model_len=256, max_prefill_tokens=64,
                                      speculation="mtp_tree", spec_force=True),
                    model=m, device="cpu", draft=CpuMLAMoEModel(cfg, weights=wd))
    tok = byte_level_tokenizer(cfg.vocab_size)
    srv = ServingServer(eng, tok, default_max_tokens=6)
    with srv:
        body = json.dumps({"stream": True, "max_tokens": 24, "messages": [{"role": "user", "content": "speculate"}]})
        r = _http.request(srv.port, "POST", "/v1/chat/completions", body)
        evs = _sse_events(r.body)
        toks = [d["token_id"] for n, d in evs if n == "token"]
        ids = tok.encode(S.prepare_openai_json(body, 1 << 20).text)
        ref, _ = oracle.greedy_generate(cfg, m.w, torch.tensor(ids), 24)
        assert toks == ref.tolist()
        assert eng.scheduler.stats.verify_steps > 0
        deadline = time.time() + 5
        h = _http.request(srv.port, "GET", "/health").body.decode()
        while '"mtp_status":"OBSERVED"' not in h and time.time() < deadline:
            time.sleep(0.06)
            h = _http.request(srv.port, "GET", "/health").body.decode()
        assert '"mtp_status":"OBSERVED"' in h
    assert srv.error is None
