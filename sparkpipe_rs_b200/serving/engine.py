"""LLMEngine: the serving loop that ties the C++ scheduler to the GPU model.

One engine owns one model replica on one GPU. Each ``step()``:

  1. asks the C++ ``Scheduler`` (continuous batching, chunked prefill, prefix
     cache, KV block tables) for a step plan;
  2. copies the plan's host arrays into pinned buffers and issues one
     host->device copy per array;
  3. runs the model: prefill eagerly (variable shapes), decode by replaying the
     CUDA graph captured for the padded batch bucket;
  4. reads the sampled tokens back (device->host) and hands them to the
     scheduler, which advances every request and reports token / finish events.

Request lifecycle and event names follow the reference's serving engine
(crates/spark-serve/src/serving_engine/engine.rs:1381-2050: invoke_prefill /
invoke_decode / complete_*_dispatch / pump) with the reference's ring dispatch
replaced by one local GPU step.
"""
from __future__ import annotations

import itertools
import statistics
import time
from dataclasses import dataclass, field

import torch

from .. import _ext, ops
from ..models.config import MLAMoEConfig
from ..models.mla_moe import DecodeGraph, ForwardBatch, KVCache, MLAMoEModel


@dataclass
class EngineConfig:
    max_batch: int = 64
    block_size: int = 64
    max_model_len: int = 4096
    num_blocks: int = 0               # 0: enough for max_batch full-length sequences
    max_prefill_tokens: int = 16384
    max_consecutive_prefills: int = 4
    use_cuda_graph: bool = True
    decode_buckets: tuple = (1, 2, 4, 8, 16, 32, 64, 128, 256)
    prefix_caching: bool = True
    chunked_prefill: bool = True
    seed: int = 0


@dataclass
class SamplingParams:
    max_tokens: int = 16
    temperature: float = 0.0
    seed: int = 0
    stop_token_ids: tuple = ()
    ignore_eos: bool = False
    priority: int = 1_000_000


@dataclass
class RequestOutput:
    request_id: int
    prompt_len: int
    token_ids: list = field(default_factory=list)
    finished: bool = False
    finish_reason: str = ""
    arrival: float = 0.0
    first_token_time: float = 0.0
    finish_time: float = 0.0

    @property
    def ttft(self) -> float:
        return self.first_token_time - self.arrival

    @property
    def tpot(self) -> float:
        n = len(self.token_ids)
        return (self.finish_time - self.first_token_time) / (n - 1) if n > 1 else 0.0


@dataclass
class GenerateResult:
    outputs: list
    stats: dict


FINISH_REASONS = {1: "length", 2: "stop", 3: "cancelled", 4: "context_limit", 5: "error"}


class _Pinned:
    """Reusable pinned host buffers for the per-step host->device copies."""

    def __init__(self):
        self.bufs: dict[str, torch.Tensor] = {}

    def get(self, name: str, n: int, dtype=torch.int32) -> torch.Tensor:
        t = self.bufs.get(name)
        if t is None or t.numel() < n:
            t = torch.empty(max(n, 64), dtype=dtype, pin_memory=True)
            self.bufs[name] = t
        return t[:n]


class LLMEngine:
    def __init__(self, cfg: MLAMoEConfig, ecfg: EngineConfig | None = None, model=None, device="cuda",
                 cache: KVCache | None = None):
        """``model`` may be the GPU model, the CPU stage driver or a PipelineModel (rank 0
        of a pipeline); ``cache`` defaults to a full cache on ``device``."""
        self.cfg = cfg
        self.ecfg = ecfg or EngineConfig()
        self.device = torch.device(device)
        self.is_cuda = self.device.type == "cuda"
        if self.is_cuda:
            torch.cuda.set_device(self.device)
        self.core = _ext.core()
        e = self.ecfg
        max_blocks = -(-e.max_model_len // e.block_size)
        num_blocks = e.num_blocks or e.max_batch * max_blocks + 16
        self.model = model or MLAMoEModel(cfg, seed=e.seed, device=self.device, max_positions=e.max_model_len + 8)
        self.cache = cache or KVCache(cfg, num_blocks=num_blocks, block_size=e.block_size, device=self.device)
        self.use_graphs = self.is_cuda and e.use_cuda_graph and isinstance(self.model, MLAMoEModel)
        sc = self.core.SchedulerConfig()
        sc.max_batch = e.max_batch
        sc.max_prefill_tokens = e.max_prefill_tokens
        sc.block_tokens = e.block_size
        sc.num_blocks = num_blocks
        sc.max_model_len = e.max_model_len
        sc.max_consecutive_prefills = e.max_consecutive_prefills
        sc.decode_buckets = [b for b in e.decode_buckets if b <= max(e.max_batch, 1)] + (
            [e.max_batch] if e.max_batch not in e.decode_buckets else [])
        flags = self.core.SCHED_DEFAULT_FLAGS
        if not e.prefix_caching:
            flags &= ~self.core.SCHED_PREFIX_CACHE
        if not e.chunked_prefill:
            flags &= ~self.core.SCHED_CHUNKED_PREFILL
        sc.flags = flags
        self.scheduler = self.core.Scheduler(sc)
        self.max_blocks = self.scheduler.max_blocks_per_seq
        self.graphs: dict[int, DecodeGraph] = {}
        self.pinned = _Pinned()
        self.outputs: dict[int, RequestOutput] = {}
        self.params: dict[int, SamplingParams] = {}
        self._ids = itertools.count(1)
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self.step_log: list[tuple[str, int, float]] = []  # (kind, seqs, seconds)

    # ------------------------------------------------------------------ requests
    def add_request(self, prompt_token_ids, params: SamplingParams | None = None, request_id: int | None = None) -> int:
        params = params or SamplingParams()
        rid = request_id if request_id is not None else next(self._ids)
        spec = self.core.RequestSpec(rid, [int(t) for t in prompt_token_ids], int(params.max_tokens),
                                     int(params.priority), [int(t) for t in params.stop_token_ids],
                                     bool(params.ignore_eos))
        self.scheduler.add_request(spec)
        self.outputs[rid] = RequestOutput(rid, len(prompt_token_ids), arrival=time.perf_counter())
        self.params[rid] = params
        return rid

    def abort_request(self, request_id: int) -> bool:
        ok = self.scheduler.cancel(request_id)
        out = self.outputs.get(request_id)
        if ok and out is not None:
            out.finished = True
            out.finish_reason = "cancelled"
            out.finish_time = time.perf_counter()
        return ok

    def has_unfinished_requests(self) -> bool:
        return self.scheduler.has_work()

    # ------------------------------------------------------------------ GPU steps
    def _h2d(self, name: str, arr) -> torch.Tensor:
        if not self.is_cuda:
            return torch.from_numpy(arr.copy())
        host = self.pinned.get(name, len(arr))
        host.numpy()[:] = arr
        self.h2d_bytes += host.numel() * host.element_size()
        return host.to(self.device, non_blocking=True)

    def _sample(self, logits: torch.Tensor, seq_ids, step_index: int) -> torch.Tensor:
        p0 = self.params.get(seq_ids[0]) if seq_ids else None
        temp = p0.temperature if p0 else 0.0
        if self.is_cuda:
            return ops.sample_tokens(logits, temp, p0.seed if p0 else 0, step_index)
        if temp <= 0:
            return logits.float().argmax(-1).to(torch.int32)
        g = torch.Generator().manual_seed((p0.seed if p0 else 0) * 1_000_003 + step_index)
        u = torch.rand(logits.shape, generator=g).clamp_min(1e-20)
        return (logits.float() / temp - torch.log(-torch.log(u))).argmax(-1).to(torch.int32)

    def _graph(self, bucket: int) -> DecodeGraph:
        g = self.graphs.get(bucket)
        if g is None:
            g = DecodeGraph(self.model, self.cache, bucket, self.max_blocks, self.ecfg.max_model_len,
                            use_graph=self.ecfg.use_cuda_graph)
            self.graphs[bucket] = g
        return g

    def _run_prefill(self, plan) -> torch.Tensor:
        fb = ForwardBatch(
            mode="prefill",
            token_ids=self._h2d("p_ids", plan.token_ids),
            positions=self._h2d("p_pos", plan.positions),
            slot_mapping=self._h2d("p_slots", plan.slot_mapping),
            cu_q=self._h2d("p_cuq", plan.cu_q),
            cu_k=self._h2d("p_cuk", plan.cu_k),
            max_q=plan.max_q,
            ctx_slots=self._h2d("p_ctx", plan.ctx_slots) if plan.has_prefix else None,
            logits_idx=self._h2d("p_lidx", plan.logits_idx),
        )
        logits = self.model.forward(fb, self.cache)
        return self._sample(logits, plan.seq_ids, plan.step_index)

    def _run_decode(self, plan) -> torch.Tensor:
        if not self.use_graphs:
            B = plan.padded_seqs
            fb = ForwardBatch(mode="decode", token_ids=self._h2d("d_ids", plan.token_ids),
                              positions=self._h2d("d_pos", plan.positions),
                              slot_mapping=self._h2d("d_slots", plan.slot_mapping),
                              block_table=self._h2d("d_bt", plan.block_table).view(B, plan.max_blocks),
                              context_lens=self._h2d("d_ctx", plan.context_lens),
                              decode_splits=ops.mla_decode_splits(B, self.cfg.num_heads, plan.max_context)
                              if self.is_cuda else 1)
            logits = self.model.forward(fb, self.cache)
            return self._sample(logits, plan.seq_ids, plan.step_index)
        g = self._graph(plan.padded_seqs)
        B = plan.padded_seqs
        ids = self.pinned.get("d_ids", B)
        pos = self.pinned.get("d_pos", B)
        slots = self.pinned.get("d_slots", B)
        ctx = self.pinned.get("d_ctx", B)
        bt = self.pinned.get(f"d_bt{B}", B * self.max_blocks).view(B, self.max_blocks)
        self.h2d_bytes += plan.write_decode_inputs(ids, pos, slots, ctx, bt)
        g.ids.copy_(ids, non_blocking=True)
        g.pos.copy_(pos, non_blocking=True)
        g.slots.copy_(slots, non_blocking=True)
        g.ctx.copy_(ctx, non_blocking=True)
        g.block_table.copy_(bt, non_blocking=True)
        return g.run()

    def step(self) -> list[RequestOutput]:
        """Runs one scheduler step on the GPU; returns the requests that changed."""
        plan = self.scheduler.schedule()
        if plan.kind == 0:
            return []
        t0 = time.perf_counter()
        try:
            if plan.kind == 1:
                sampled = self._run_prefill(plan)
            else:
                sampled = self._run_decode(plan)
            if self.is_cuda:
                host = self.pinned.get("sampled", sampled.numel())
                host.copy_(sampled, non_blocking=True)
                torch.cuda.current_stream(self.device).synchronize()
                self.d2h_bytes += plan.num_seqs * 4
            else:
                host = sampled.to(torch.int32)
        except Exception:
            self.scheduler.fail_step(plan)
            raise
        now = time.perf_counter()
        self.step_log.append(("prefill" if plan.kind == 1 else "decode", plan.num_seqs, now - t0, plan.num_tokens))
        events = self.scheduler.complete_tensor(plan, host[:plan.num_seqs].contiguous())
        changed = {}
        for ev in events:
            out = self.outputs.get(ev.id)
            if out is None:
                continue
            if ev.kind == 1:  # token
                if not out.token_ids:
                    out.first_token_time = now
                out.token_ids.append(int(ev.token))
                changed[ev.id] = out
            elif ev.kind == 2:  # finished
                out.finished = True
                out.finish_reason = FINISH_REASONS.get(int(ev.reason), "unknown")
                out.finish_time = now
                changed[ev.id] = out
        return list(changed.values())

    # ------------------------------------------------------------------ batch API
    def generate(self, prompts, params: SamplingParams | None = None) -> GenerateResult:
        """Submits every prompt, runs steps until all finish; returns outputs and serving stats."""
        params = params or SamplingParams()
        ids = [self.add_request(p, params) for p in prompts]
        h2d0, d2h0 = self.h2d_bytes, self.d2h_bytes
        log0 = len(self.step_log)
        t0 = time.perf_counter()
        while self.scheduler.has_work():
            self.step()
        wall = time.perf_counter() - t0
        outs = [self.outputs.pop(i) for i in ids]
        for i in ids:
            self.params.pop(i, None)
        log = self.step_log[log0:]
        dec = [s for s in log if s[0] == "decode"]
        dec_tokens = sum(s[1] for s in dec)
        dec_secs = sum(s[2] for s in dec)
        gen = sum(len(o.token_ids) for o in outs)
        ttft = [o.ttft * 1000 for o in outs if o.token_ids]
        tpot = [o.tpot * 1000 for o in outs if len(o.token_ids) > 1]
        steps = max(1, len(log))
        stats = {
            "requests": len(outs),
            "generated_tokens": gen,
            "wall_seconds": wall,
            "throughput_tokens_per_s": gen / wall if wall > 0 else 0.0,
            "decode_tokens": dec_tokens,
            "decode_seconds": dec_secs,
            "decode_tokens_per_s": dec_tokens / dec_secs if dec_secs > 0 else 0.0,
            "decode_steps": len(dec),
            "prefill_steps": len(log) - len(dec),
            "prefill_tokens": sum(s[3] for s in log if s[0] == "prefill"),
            "prefill_seconds": sum(s[2] for s in log if s[0] == "prefill"),
            "ttft_p50_ms": statistics.median(ttft) if ttft else 0.0,
            "tpot_p50_ms": statistics.median(tpot) if tpot else 0.0,
            "h2d_bytes_per_step": (self.h2d_bytes - h2d0) / steps,
            "d2h_bytes_per_step": (self.d2h_bytes - d2h0) / steps,
        }
        return GenerateResult(outs, stats)

    def shutdown(self):
        for g in self.graphs.values():
            g.release()
        self.graphs.clear()
        if hasattr(self.model, "shutdown"):
            self.model.shutdown()
        if self.is_cuda:
            torch.cuda.synchronize(self.device)
