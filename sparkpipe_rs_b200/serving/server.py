"""OpenAI / Anthropic-compatible HTTP + SSE server around an ``LLMEngine``.

Threads:

* the C++ gateway thread (``core().serving.Gateway``): epoll over the HTTP
  port (and the optional binary frame port), request parsing, auth, JSON ->
  chat template, tokenization, id mapping and budgets (``ServiceRuntime``),
  SSE / frame writing, disconnect -> cancel;
* the engine thread (here): takes token-id submissions and cancels from
  ``Gateway.poll_work``, runs ``LLMEngine.step()`` (one GPU prefill or
  decode step), and publishes token / finish events by serving handle.

The engine thread never touches JSON, text or sockets, so a decode step is
not delayed by request parsing. Reference: the serving engine pump and the
gateway backend seam (crates/spark-serve/src/serving_engine/engine.rs:1942-2050,
crates/spark-serve/src/http_gateway.rs:371-392).

Run: ``python -m sparkpipe_rs_b200.serving.server --model tiny --device cpu --port 8000``.
"""
from __future__ import annotations

import argparse
import threading
import time
import traceback

from ..core import core
from .engine import EngineConfig, LLMEngine, SamplingParams
from .tokenizers import load_tokenizer

FINISH_TO_EVENT = {"cancelled": "EV_CANCELLED", "error": "EV_ERROR"}
STATUS_INTERNAL_ERROR = 17


class ServingServer:
    def __init__(self, engine: LLMEngine, tokenizer, *, host: str = "127.0.0.1", port: int = 0,
                 frame_port: int = -1, api_key: str = "", template_style: str = "glm",
                 default_max_tokens: int = 256, stop_token_ids: tuple = (), release_id: str = "",
                 release_git_commit: str = "", release_generation: int = 0):
        S = core().serving
        self.S = S
        self.engine = engine
        self.tokenizer = tokenizer
        self.stop_token_ids = tuple(int(t) for t in stop_token_ids)
        ec = engine.ecfg
        cfg = S.ServiceConfig()
        b = S.BudgetPolicy()
        b.default_output_budget = default_max_tokens
        b.max_output_budget = ec.max_model_len
        b.max_context_tokens = ec.max_model_len
        cfg.budgets = b
        self.service = S.ServiceRuntime(cfg)
        gc = S.GatewayConfig()
        gc.host = host
        gc.port = port
        gc.frame_port = frame_port
        gc.api_key = api_key
        gc.template_style = template_style
        self.gateway = S.Gateway(gc, tokenizer, self.service)
        self.view = S.BackendView()
        self.view.attached = True
        self.view.runtime_initialized = True
        self.view.local_control_ready = True
        self.view.release_id = release_id
        self.view.release_git_commit = release_git_commit
        self.view.release_generation = release_generation
        self.view.kv_context_limit_tokens = ec.max_model_len
        self.view.max_active_sequences = ec.max_batch
        self.view.adaptive_decode_batch_width = ec.max_batch
        self.view.decode_batch_capacity = ec.max_batch
        self.view.prefill_wave_token_count = ec.max_prefill_tokens
        if engine.spec:  # draft / verify speculation runs inside the engine
            self.view.speculation_flags = self.view.speculation_flags | S.BACKEND_FLAG_MTP
        self.counters = S.ServingCounters()
        self._published: dict[int, int] = {}
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None
        self.error: BaseException | None = None

    # ------------------------------------------------------------------ lifecycle
    @property
    def port(self) -> int:
        return self.gateway.port

    @property
    def frame_port(self) -> int:
        return self.gateway.frame_port

    def start(self):
        self.gateway.set_backend_view(self.view)
        self.gateway.start()
        self._thread = threading.Thread(target=self._run, name="sparkpipe-engine", daemon=True)
        self._thread.start()
        return self

    def stop(self):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=30)
        self.gateway.stop()

    def __enter__(self):
        return self.start()

    def __exit__(self, *exc):
        self.stop()

    # ------------------------------------------------------------------ engine thread
    def _run(self):
        S, eng = self.S, self.engine
        last_counters = 0.0
        while not self._stop.is_set():
            busy = eng.has_unfinished_requests()
            events = []
            for w in self.gateway.poll_work(0 if busy else 20, 4096):
                if w.kind == S.WORK_SUBMIT:
                    self._submit(w)
                else:
                    events += self._cancel(w.handle)
            # a lockstep (expert-parallel) rank steps every turn: its peers may have work
            if eng.lockstep or eng.has_unfinished_requests():
                try:
                    outs = eng.step()
                except Exception as exc:  # fail every live request, keep serving
                    self.error = exc
                    traceback.print_exc()
                    events += self._fail_all()
                    outs = []
                events += self._events(outs)
            if events:
                self.gateway.publish(events)
            now = time.monotonic()
            if now - last_counters > 0.05:
                self._update_counters()
                last_counters = now

    def _submit(self, w):
        params = SamplingParams(max_tokens=max(1, int(w.output_budget)), temperature=0.0,
                                stop_token_ids=self.stop_token_ids, ignore_eos=not self.stop_token_ids,
                                priority=int(w.priority) or 1_000_000)
        self.engine.add_request(list(w.token_ids), params, request_id=int(w.handle))
        self._published[int(w.handle)] = 0

    def _cancel(self, handle: int):
        handle = int(handle)
        self.engine.abort_request(handle)
        self._forget(handle)
        return [self.S.EngineEvent(handle, self.S.EV_CANCELLED)]

    def _forget(self, handle: int):
        self._published.pop(handle, None)
        self.engine.outputs.pop(handle, None)
        self.engine.params.pop(handle, None)

    def _fail_all(self):
        evs = []
        for h in list(self._published):
            self.engine.abort_request(h)
            self._forget(h)
            evs.append(self.S.EngineEvent(h, self.S.EV_ERROR, status=STATUS_INTERNAL_ERROR))
        return evs

    def _events(self, outs):
        S = self.S
        evs = []
        for o in outs:
            h = int(o.request_id)
            if h not in self._published:
                continue
            n0 = self._published[h]
            for i in range(n0, len(o.token_ids)):
                evs.append(S.EngineEvent(h, S.EV_TOKEN, int(o.token_ids[i]), o.prompt_len + i))
            self._published[h] = len(o.token_ids)
            self.counters.decoded_tokens += len(o.token_ids) - n0
            if o.finished:
                kind = getattr(S, FINISH_TO_EVENT.get(o.finish_reason, "EV_COMPLETED"))
                evs.append(S.EngineEvent(h, kind, 0, o.prompt_len + len(o.token_ids),
                                         STATUS_INTERNAL_ERROR if kind == S.EV_ERROR else 0))
                if kind == S.EV_COMPLETED:
                    self.counters.completed_streams += 1
                self._forget(h)
        return evs

    def _update_counters(self):
        c = self.counters
        log = self.engine.step_log
        for kind, seqs, _secs, _tokens in log:  # consume the engine's step log incrementally
            if kind in ("decode", "verify"):
                c.decode_dispatches += 1
                c.mtp_verify_dispatches += int(kind == "verify")
                c.max_decode_lanes = max(c.max_decode_lanes, seqs)
                c.max_decode_active = c.max_decode_lanes
            else:
                c.prefill_dispatches += 1
                c.prefill_batch_dispatches += int(seqs > 1)
                c.max_prefill_lanes = max(c.max_prefill_lanes, seqs)
                c.max_prefill_active = c.max_prefill_lanes
        log.clear()
        c.queued_requests = int(self.engine.scheduler.waiting_count)
        c.prefill_tokens = int(self.engine.scheduler.stats.prefill_tokens)
        if self.engine.spec:
            t = self.engine.scheduler.spec_totals
            c.mtp_draft_tokens = t["proposed"]
            c.mtp_accepted_draft_tokens = t["accepted"]
            c.mtp_committed_tokens = t["committed"]
            c.mtp_rejected_tokens = t["proposed"] - t["accepted"]
        self.gateway.set_serving_counters(c)


def main(argv=None):
    ap = argparse.ArgumentParser(description="sparkpipe-rs B200 OpenAI/Anthropic-compatible server")
    ap.add_argument("--model", default="tiny", help="model preset (tiny, v2_lite, k2, ...)")
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--frame-port", type=int, default=-1)
    ap.add_argument("--api-key", default="")
    ap.add_argument("--api-key-file", default="")
    ap.add_argument("--tokenizer", default="", help="tokenizer.json or compiled tokenizer; default: byte-level")
    ap.add_argument("--template", default="glm", choices=["glm", "deepseek"])
    ap.add_argument("--max-batch", type=int, default=64)
    ap.add_argument("--max-model-len", type=int, default=4096)
    ap.add_argument("--max-tokens", type=int, default=256)
    ap.add_argument("--stop-token", type=int, action="append", default=[])
    ap.add_argument("--speculation", default="", choices=["", "chain", "mtp_tree"],
                    help="speculative decoding with a one-layer draft head")
    ap.add_argument("--draft-len", type=int, default=3)
    ap.add_argument("--spec-p-accept", type=float, default=0.0, help="> 0: forced acceptance (benchmarks)")
    ap.add_argument("--spec-force", action="store_true", help="verify whenever lanes qualify")
    args = ap.parse_args(argv)
    from ..models.config import get_config
    cfg = get_config(args.model)
    ec = EngineConfig(max_batch=args.max_batch, max_model_len=args.max_model_len, speculation=args.speculation,
                      draft_len=args.draft_len, spec_p_accept=args.spec_p_accept, spec_force=args.spec_force)
    model = None
    if args.device == "cpu":
        from ..models.cpu_model import CpuMLAMoEModel
        model = CpuMLAMoEModel(cfg, seed=0, max_positions=args.max_model_len + 8)
    eng = LLMEngine(cfg, ec, model=model, device=args.device)
    tok = load_tokenizer(args.tokenizer, cfg.vocab_size)
    key = args.api_key
    if args.api_key_file:
        with open(args.api_key_file) as f:
            key = f.read().strip()
    srv = ServingServer(eng, tok, host=args.host, port=args.port, frame_port=args.frame_port, api_key=key,
                        template_style=args.template, default_max_tokens=args.max_tokens,
                        stop_token_ids=tuple(args.stop_token))
    srv.start()
    print(f"serving on http://{args.host}:{srv.port}" +
          (f", frames on {args.host}:{srv.frame_port}" if srv.frame_port >= 0 else ""), flush=True)
    try:
        while True:
            time.sleep(3600)
    except KeyboardInterrupt:
        pass
    finally:
        srv.stop()


if __name__ == "__main__":
    main()
