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

Expert-parallel ranks (attention data-parallel, experts split over the GPUs)
each run their own engine, but every forward is a collective over the group. The
engines therefore step in lockstep: each step the ranks agree on the host (a gloo
all-reduce of two flags) whether any of them launches a forward, and a rank
without work of its own launches an idle forward (one row that reads no context
and writes no KV) so the others' dispatch and combine find it.

Decode steps overlap the host with the GPU: while step n runs, the scheduler
plans step n+1 ahead of n's tokens (``Scheduler.schedule_ahead``), its inputs are
copied, and its graph is launched with the token ids gathered on the device from
n's sampled tokens; only then does the host wait for n's tokens. A sequence that
stops at step n gets one discarded extra token. Decode graphs for every batch
bucket are captured when the engine starts.

With speculation on (``EngineConfig.speculation``: "chain" or "mtp_tree"), a draft
model keeps its own KV cache current (its first-layer KV is written for prompts and
plainly decoded tokens inside the same step), and the scheduler turns a decode step
into a verify round whenever its policy grants the lanes draft rows: drafts, one
batched target forward over every lane's rows and the commit kernel run as one CUDA
graph per padded batch (``serving/verify.py``), and each lane commits between one and
(drafts + 1) tokens. Measured device times of plain steps and verify rounds feed the
scheduler's utility comparison.

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

import numpy as np
import torch

from .. import _ext, ops
from ..models.config import MLAMoEConfig
from ..models.mla_moe import DecodeGraph, ForwardBatch, KVCache, MLAMoEModel
from .verify import VerifyRound


@dataclass
class EngineConfig:
    max_batch: int = 64
    block_size: int = 64
    max_model_len: int = 4096
    num_blocks: int = 0               # 0: enough for max_batch full-length sequences
    max_prefill_tokens: int = 16384
    max_consecutive_prefills: int = 4
    # prefill and decode at equal priority: False = a waiting prompt's prefill goes first
    # while KV blocks allow it (the reference's rule: prefill wins at equal priority with
    # resident KV headroom); True = at most max_consecutive_prefills prefill steps while
    # decodes wait (protects TPOT during a burst of arrivals)
    prefill_decode_interleave: bool = False
    use_cuda_graph: bool = True
    decode_buckets: tuple = (1, 2, 4, 8, 16, 32, 64, 128, 256)
    prefix_caching: bool = True
    chunked_prefill: bool = True
    seed: int = 0
    async_decode: bool = True         # plan and launch decode step n+1 before reading step n's tokens
    capture_graphs_at_start: bool = True
    speculation: str = ""             # "", "chain" (draft_len drafts per lane) or "mtp_tree" (5 candidates, 6 rows)
    draft_len: int = 3
    spec_p_accept: float = 0.0        # > 0: forced Bernoulli acceptance of each draft token (benchmarks)
    spec_force: bool = False          # verify whenever the lanes qualify (no utility comparison)
    spec_seed: int = 17
    spec_row_cap: int = 0             # firing rows of a verify round (0: rows per lane x max_batch)
    host_kv_blocks: int = 0           # host KV tier: preempted sequences swap their KV out (0: recompute)
    host_prefix_blocks: int = 0       # host KV tier for prefix blocks evicted from the device (0: drop them)
    host_resident_blocks: int = 0     # pinned buffers behind the host tier's slots (0: one per slot)
    host_drive_path: str = ""         # with fewer resident buffers than slots: the drive file the rest spill to
    kv_cache_dtype: str = "bf16"      # "fp8": e4m3 latent rows with per-128 block scales (CUDA, 576-wide rows)
    warm_prefill: bool = True         # one throwaway prefill of the largest chunk at start (allocator warm-up)
    prefill_graphs: bool = False      # replay repeated prefill chunk shapes (no cached prefix) from CUDA graphs


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


def _default_draft(model, e: EngineConfig):
    """A one-layer MTP-style draft head of ``model`` sharing its embedding and LM head:
    on the GPU model's device, or an fp32 CPU stage driver for the CPU model."""
    from .spec_decode import make_draft

    if isinstance(model, MLAMoEModel):
        return make_draft(model, seed=e.seed + 1, max_positions=e.max_model_len + 8)
    from ..models.config import mtp_head
    from ..models.cpu_model import CpuMLAMoEModel
    from ..models.weights import init_weights

    cfg = mtp_head(model.cfg)
    w = init_weights(cfg, seed=e.seed + 1, device="cpu", dtype=torch.float32,
                     share={"embed": model.w["embed"], "lm_head": model.w["lm_head"]})
    return CpuMLAMoEModel(cfg, weights=w, max_positions=e.max_model_len + 8)


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


class _Lockstep:
    """Host-side agreement of the ranks of one expert-parallel group: per step, does
    any rank launch a forward, and does any rank still have work."""

    def __init__(self, ep_group):
        import torch.distributed as dist

        self.dist = dist
        ranks = dist.get_process_group_ranks(ep_group) if ep_group is not dist.group.WORLD else \
            list(range(dist.get_world_size()))
        self.group = dist.new_group(ranks=ranks, backend="gloo")
        self.buf = torch.zeros(2, dtype=torch.int32)

    def agree(self, has_plan: bool, busy: bool) -> tuple[bool, bool]:
        self.buf[0] = int(has_plan)
        self.buf[1] = int(busy)
        self.dist.all_reduce(self.buf, op=self.dist.ReduceOp.MAX, group=self.group)
        return bool(self.buf[0]), bool(self.buf[1])


@dataclass
class _Launched:
    """A step whose GPU work is enqueued: its sampled tokens land in ``host``
    (``plan`` None: an idle forward of a lockstep rank; a verify round: the host
    tensors (committed, counts, paths))."""
    plan: object
    host: object
    event: object          # CUDA event after the device->host copy (None on CPU)
    out: torch.Tensor      # device tensor of the sampled tokens
    t0: float
    timing: tuple | None = None  # CUDA events around the step's device work (cost model)


class _PrefillGraph:
    """One prefill chunk shape without a cached prefix (tokens, sequences, longest
    query) as a CUDA graph: static device inputs, captured the first time the shape comes
    up after the engine's warm-up prefill (else the second time, after an eager run has
    set every kernel's attributes), replayed from then on. A serving burst of equal prompts repeats one shape, and
    the chunk's ~430 launches then cost one graph launch instead of one host round trip
    each."""

    def __init__(self, model, cache, T: int, nseq: int, max_q: int, dev):
        i32 = dict(dtype=torch.int32, device=dev)
        self.model, self.cache = model, cache
        self.ids = torch.zeros(T, **i32)
        self.pos = torch.zeros(T, **i32)
        self.slots = torch.full((T,), -1, **i32)
        self.cu = torch.zeros(nseq + 1, **i32)
        self.lidx = torch.zeros(nseq, **i32)
        self.fb = ForwardBatch(mode="prefill", token_ids=self.ids, positions=self.pos, slot_mapping=self.slots,
                               cu_q=self.cu, cu_k=self.cu, max_q=max_q, logits_idx=self.lidx)
        cur = torch.cuda.current_stream(dev)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(cur)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side), torch.cuda.graph(self.graph, stream=side, capture_error_mode="thread_local"):
            self.out = model.forward(self.fb, cache)
        cur.wait_stream(side)


class LLMEngine:
    def __init__(self, cfg: MLAMoEConfig, ecfg: EngineConfig | None = None, model=None, device="cuda",
                 cache: KVCache | None = None, draft=None):
        """``model`` may be the GPU model, the CPU stage driver or a PipelineModel (rank 0
        of a pipeline, which runs whole steps through its stages and returns sampled
        tokens); ``cache`` defaults to a full cache on ``device``. ``draft``: the
        draft model of speculation (default: a one-layer MTP-style head of ``model``)."""
        self.cfg = cfg
        self.ecfg = ecfg or EngineConfig()
        self.device = torch.device(device)
        self.is_cuda = self.device.type == "cuda"
        if self.is_cuda and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        if self.is_cuda:
            torch.cuda.set_device(self.device)
        self.core = _ext.core()
        e = self.ecfg
        max_blocks = -(-e.max_model_len // e.block_size)
        num_blocks = e.num_blocks or e.max_batch * max_blocks + 16
        self.model = model or MLAMoEModel(cfg, seed=e.seed, device=self.device, max_positions=e.max_model_len + 8)
        if e.speculation not in ("", "chain", "mtp_tree"):
            raise ValueError(f"unknown speculation mode {e.speculation!r}")
        self.spec = e.speculation
        buckets = [b for b in e.decode_buckets if b <= max(e.max_batch, 1)] + (
            [e.max_batch] if e.max_batch not in e.decode_buckets else [])
        # tree verify: two shadow KV rows per batch row, past the scheduler's blocks
        shadow_blocks = -(-2 * max(buckets) // e.block_size) if self.spec == "mtp_tree" else 0
        if cache is not None and shadow_blocks and cache.num_blocks < num_blocks + shadow_blocks:
            raise ValueError("tree speculation needs a cache with room for the shadow blocks")
        self.cache = cache or KVCache(cfg, num_blocks=num_blocks + shadow_blocks, block_size=e.block_size,
                                      device=self.device, kv_dtype=e.kv_cache_dtype if self.is_cuda else "bf16")
        self.use_graphs = self.is_cuda and e.use_cuda_graph and isinstance(self.model, MLAMoEModel)
        self._pgraphs: dict[tuple, _PrefillGraph] = {}
        self._pseen: dict[tuple, int] = {}
        self._prefill_warmed = False
        self.draft = self.dcache = None
        if self.spec:
            self.draft = draft or _default_draft(self.model, e)
            self.dcache = KVCache(self.draft.cfg, num_blocks=num_blocks, block_size=e.block_size, device=self.device,
                                  layers=1)
        sc = self.core.SchedulerConfig()
        sc.max_batch = e.max_batch
        sc.max_prefill_tokens = e.max_prefill_tokens
        sc.block_tokens = e.block_size
        sc.num_blocks = num_blocks
        sc.max_model_len = e.max_model_len
        sc.max_consecutive_prefills = e.max_consecutive_prefills
        sc.decode_buckets = buckets
        flags = self.core.SCHED_DEFAULT_FLAGS
        if not e.prefix_caching:
            flags &= ~self.core.SCHED_PREFIX_CACHE
        if not e.chunked_prefill:
            flags &= ~self.core.SCHED_CHUNKED_PREFILL
        if e.prefill_decode_interleave:
            flags |= self.core.SCHED_PREFILL_DECODE_INTERLEAVE
        else:
            flags &= ~self.core.SCHED_PREFILL_DECODE_INTERLEAVE
        if self.spec:
            sc.spec_mode = self.core.SPEC_CHAIN if self.spec == "chain" else self.core.SPEC_MTP_TREE
            sc.spec_draft_len = e.draft_len
            sc.spec_row_cap = e.spec_row_cap
            sc.spec_shadow_slot_base = num_blocks * e.block_size
            if e.spec_force:
                flags |= self.core.SCHED_MTP_FORCE_ENABLE
        sc.flags = flags
        sc.host_blocks = e.host_kv_blocks
        sc.host_prefix_blocks = e.host_prefix_blocks if e.prefix_caching else 0
        self.scheduler = self.core.Scheduler(sc)
        self.max_blocks = self.scheduler.max_blocks_per_seq
        self.host_tier = None
        if e.host_kv_blocks or sc.host_prefix_blocks:
            from .kv_offload import HostKvTier

            slots = e.host_kv_blocks + sc.host_prefix_blocks
            drive = None
            if e.host_resident_blocks and e.host_resident_blocks < slots:
                from .kv_offload import DriveSpill

                probe = HostKvTier(self.cache, 1)
                drive = DriveSpill(probe.block_bytes, slots, path=e.host_drive_path or None)
                del probe
            self.host_tier = HostKvTier(self.cache, slots, resident_blocks=e.host_resident_blocks, drive=drive)
        self.graphs: dict[int, DecodeGraph] = {}
        self.verify_rounds: dict[int, VerifyRound] = {}
        self._cost_ema: dict[tuple[int, int], float] = {}
        self._timing = None
        self.tree_paths = [0] * 6  # resolved MTP tree paths over every verified lane
        self.device_ms: dict[int, float] = {}  # CUDA-event time of timed steps by plan kind
        self.pinned = _Pinned()
        self.outputs: dict[int, RequestOutput] = {}
        self.params: dict[int, SamplingParams] = {}
        self._ids = itertools.count(1)
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        # CUDA eager decode reuses one set of pinned input buffers, so it stays synchronous;
        # a pipeline runs whole steps on its stages and needs each step's tokens first
        self.stages = bool(getattr(self.model, "runs_plans", False))
        self.async_decode = e.async_decode and (self.use_graphs or not self.is_cuda) and not self.stages
        if self.stages and self.spec:
            raise ValueError("speculation runs on a single-stage model")
        self._inflight: _Launched | None = None
        self.ahead_steps = 0  # decode steps launched ahead of the previous step's tokens
        self.idle_steps = 0   # idle forwards of a lockstep rank
        ep = getattr(self.model, "ep", None)
        self._lockstep = _Lockstep(ep.group) if ep is not None and getattr(ep, "group", None) is not None \
            and ep.world > 1 else None
        self._more = True     # lockstep: some rank of the group still has work
        self._parity = 0
        self._last_done = 0.0
        self._random: set[int] = set()  # live requests that sample (temperature > 0)
        # lockstep ranks capture every bucket up front: a capture's warm-up forward is a collective
        if self.use_graphs and (e.capture_graphs_at_start or self._lockstep is not None):
            for b in sc.decode_buckets:
                self._graph(b)
                if self.spec:
                    self._verify_round(b)
        if self.spec and self.use_graphs and not e.spec_force:
            self._prime_step_costs()
        if e.warm_prefill and self.is_cuda and isinstance(self.model, MLAMoEModel):
            self._warm_prefill()
        self.step_log: list[tuple[str, int, float, int]] = []  # (kind, seqs, seconds, tokens)

    # ------------------------------------------------------------------ requests
    def add_request(self, prompt_token_ids, params: SamplingParams | None = None, request_id: int | None = None) -> int:
        params = params or SamplingParams()
        rid = request_id if request_id is not None else next(self._ids)
        spec = self.core.RequestSpec(rid, [int(t) for t in prompt_token_ids], int(params.max_tokens),
                                     int(params.priority), [int(t) for t in params.stop_token_ids],
                                     bool(params.ignore_eos), float(params.temperature), int(params.seed))
        self.scheduler.add_request(spec)
        self.outputs[rid] = RequestOutput(rid, len(prompt_token_ids), arrival=time.perf_counter())
        self.params[rid] = params
        if params.temperature > 0:
            self._random.add(rid)
        return rid

    def _draft_kv(self, fb):
        self.draft.write_kv(fb, self.dcache)

    def abort_request(self, request_id: int) -> bool:
        ok = self.scheduler.cancel(request_id)
        self._random.discard(request_id)
        out = self.outputs.get(request_id)
        if ok and out is not None:
            out.finished = True
            out.finish_reason = "cancelled"
            out.finish_time = time.perf_counter()
        return ok

    @property
    def lockstep(self) -> bool:
        """This engine is one rank of an expert-parallel group and must step with it."""
        return self._lockstep is not None

    def has_unfinished_requests(self) -> bool:
        """This engine still has work; for a lockstep rank, some rank of the group has
        (as agreed at the last step), so the caller keeps stepping."""
        local = self.scheduler.has_work() or self._inflight is not None
        return local or (self._lockstep is not None and self._more)

    # ------------------------------------------------------------------ GPU steps
    def _h2d(self, name: str, arr) -> torch.Tensor:
        if not self.is_cuda:
            return torch.from_numpy(arr.copy())
        host = self.pinned.get(name, len(arr))
        host.numpy()[:] = arr
        self.h2d_bytes += host.numel() * host.element_size()
        return host.to(self.device, non_blocking=True)

    def _sampling_rows(self, plan, rows: int, tag: str):
        """Per-row (temperature, noise key) host tensors of a plan, or None when every row is greedy."""
        if not self._random:
            return None
        temps = self.pinned.get(f"t_{tag}", rows, torch.float32) if self.is_cuda else torch.empty(rows)
        keys = self.pinned.get(f"k_{tag}", rows, torch.int64) if self.is_cuda else torch.empty(rows, dtype=torch.int64)
        return (temps, keys) if self.scheduler.sampling_rows(plan, temps, keys) else None

    def _sample(self, logits: torch.Tensor, plan) -> torch.Tensor:
        rows = self._sampling_rows(plan, logits.shape[0], "p")
        if self.is_cuda:
            if rows is None:
                return ops.sample_tokens(logits)
            temps, keys = rows
            self.h2d_bytes += temps.numel() * 12
            return ops.sample_tokens(logits, row_temp=temps.to(self.device, non_blocking=True),
                                     row_key=keys.to(self.device, non_blocking=True))
        out = logits.float().argmax(-1).to(torch.int32)
        if rows is not None:  # Gumbel-max per sampled row, noise seeded by the row's key
            temps, keys = rows
            for i in range(logits.shape[0]):
                if temps[i] > 0:
                    g = torch.Generator().manual_seed(int(keys[i]) & ((1 << 63) - 1))
                    u = torch.rand(logits.shape[1], generator=g).clamp_min(1e-20)
                    out[i] = int((logits[i].float() / float(temps[i]) - torch.log(-torch.log(u))).argmax())
        return out

    def _graph(self, bucket: int) -> DecodeGraph:
        g = self.graphs.get(bucket)
        if g is None:
            g = DecodeGraph(self.model, self.cache, bucket, self.max_blocks, self.ecfg.max_model_len,
                            use_graph=self.ecfg.use_cuda_graph, extra=self._draft_kv if self.spec else None)
            self.graphs[bucket] = g
        return g

    def _verify_round(self, bucket: int) -> VerifyRound:
        v = self.verify_rounds.get(bucket)
        if v is None:
            e = self.ecfg
            v = VerifyRound(self.model, self.draft, self.cache, self.dcache, bucket, self.spec, e.draft_len,
                            self.max_blocks, e.max_model_len, e.spec_p_accept, e.spec_seed,
                            use_graph=self.use_graphs)
            v.capture()
            self.verify_rounds[bucket] = v
        return v

    def _record_cost(self, kind: int, bucket: int, ms: float):
        """Device time of a plain step (kind 2) / verify round (kind 3) into the
        scheduler's cost model, as an exponential average per padded batch."""
        key = (kind, bucket)
        prev = self._cost_ema.get(key)
        ema = ms if prev is None else 0.75 * prev + 0.25 * ms
        self._cost_ema[key] = ema
        self.scheduler.set_step_cost(kind, bucket, int(ema * 1e6))

    def _prime_step_costs(self):
        """One timed replay per captured graph with idle rows: a first estimate of each
        step kind's cost, replaced by the times measured while serving."""
        for b in list(self.graphs):
            for kind, run in ((2, self.graphs[b].run), (3, self.verify_rounds[b].run)):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                run()
                e1.record()
                e1.synchronize()
                self._record_cost(kind, b, e0.elapsed_time(e1))

    def _warm_prefill(self):
        """One prefill forward of the largest chunk on throwaway inputs (token 0, every
        KV slot -1 so nothing is written): the first real chunk then finds its activation
        and workspace memory in the caching allocator's pool instead of paying for fresh
        device allocations inside its time to first token. Lockstep ranks all run it."""
        e = self.ecfg
        T = max(1, e.max_prefill_tokens)
        L = max(1, min(T, e.max_model_len))
        lens = [L] * (T // L) + ([T % L] if T % L else [])
        dev = self.device
        cu = torch.tensor([0] + list(itertools.accumulate(lens)), dtype=torch.int32, device=dev)
        pos = torch.cat([torch.arange(n, dtype=torch.int32) for n in lens]).to(dev)
        fb = ForwardBatch(mode="prefill", token_ids=torch.zeros(T, dtype=torch.int32, device=dev), positions=pos,
                          slot_mapping=torch.full((T,), -1, dtype=torch.int32, device=dev), cu_q=cu, cu_k=cu, max_q=L,
                          logits_idx=(cu[1:] - 1).contiguous())
        self.model.forward(fb, self.cache)
        torch.cuda.synchronize(dev)
        self._prefill_warmed = True

    def _prefill_graph(self, plan):
        """The captured graph of this plan's chunk shape, if it has one (or gets one now:
        second sighting of the shape); None runs the chunk eagerly."""
        if not (self.use_graphs and self.ecfg.prefill_graphs) or plan.has_prefix or self._lockstep is not None:
            return None
        if not np.array_equal(plan.cu_q, plan.cu_k):  # keys beyond the chunk: not this graph's shape
            return None
        sig = (len(plan.token_ids), len(plan.cu_q) - 1, int(plan.max_q))
        g = self._pgraphs.get(sig)
        if g is None:
            seen = self._pseen.get(sig, 0)
            self._pseen[sig] = seen + 1
            # after the warm-up prefill every prefill kernel's attributes are set, so a
            # shape can be captured the first time it comes up
            if (seen == 0 and not self._prefill_warmed) or len(self._pgraphs) >= 4:
                return None
            g = self._pgraphs[sig] = _PrefillGraph(self.model, self.cache, sig[0], sig[1], sig[2], self.device)
        return g

    def _run_prefill(self, plan) -> torch.Tensor:
        g = self._prefill_graph(plan)
        if g is not None:
            for name, buf, arr in (("p_ids", g.ids, plan.token_ids), ("p_pos", g.pos, plan.positions),
                                   ("p_slots", g.slots, plan.slot_mapping), ("p_cuq", g.cu, plan.cu_q),
                                   ("p_lidx", g.lidx, plan.logits_idx)):
                host = self.pinned.get(name, len(arr))
                host.numpy()[:] = arr
                self.h2d_bytes += host.numel() * host.element_size()
                buf.copy_(host, non_blocking=True)
            g.graph.replay()
            if self.spec:
                self._draft_kv(g.fb)
            return self._sample(g.out, plan)
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
        if self.spec:
            self._draft_kv(fb)
        return self._sample(logits, plan)

    def _run_verify(self, plan):
        """Copies a verify plan's rows into its round's device arrays and runs the round."""
        B = plan.padded_seqs
        v = self._verify_round(B)
        R = B * v.rows
        if self.is_cuda:
            par = self._parity
            self._parity ^= 1
            ids = self.pinned.get(f"v_ids{par}", R)
            pos = self.pinned.get(f"v_pos{par}", R)
            slots = self.pinned.get(f"v_slots{par}", R)
            ctx = self.pinned.get(f"v_ctx{par}", R)
            bt = self.pinned.get(f"v_bt{B}_{par}", B * self.max_blocks).view(B, self.max_blocks)
            budget = self.pinned.get(f"v_budget{par}", B)
            keys = self.pinned.get(f"v_keys{par}", B, torch.int64)
            sync = self.pinned.get(f"v_sync{par}", 9 * B) if self.spec == "mtp_tree" else None
            self.h2d_bytes += plan.write_verify_inputs(ids, pos, slots, ctx, bt, budget, keys, sync)
            for dst, src in ((v.tok, ids), (v.pos, pos), (v.slot, slots), (v.ctx, ctx), (v.bt, bt),
                             (v.budget, budget), (v.keys, keys)):
                dst.copy_(src, non_blocking=True)
            if sync is not None:
                v.sync.view(-1).copy_(sync, non_blocking=True)
        else:
            v.tok.copy_(torch.from_numpy(plan.token_ids))
            v.pos.copy_(torch.from_numpy(plan.positions))
            v.slot.copy_(torch.from_numpy(plan.slot_mapping))
            v.ctx.copy_(torch.from_numpy(plan.context_lens))
            v.bt.copy_(torch.from_numpy(plan.block_table).view(B, -1)[:, : v.bt.shape[1]])
            v.budget.copy_(torch.from_numpy(plan.draft_budget))
            v.keys.copy_(torch.from_numpy(plan.accept_keys))
            if self.spec == "mtp_tree":
                v.sync.copy_(torch.stack([torch.from_numpy(plan.sync_token_ids), torch.from_numpy(plan.sync_positions),
                                          torch.from_numpy(plan.sync_slots)]))
        return v.run(timed=True)

    def _run_decode(self, plan, prev: _Launched | None = None) -> torch.Tensor:
        if not self.use_graphs:
            B = plan.padded_seqs
            tok = self._h2d("d_ids", plan.token_ids)
            if plan.flags & self.core.DECISION_SCHEDULED_AHEAD:
                n = plan.num_seqs
                tok[:n] = prev.out.to(tok.device)[tok[:n].long()]
            fb = ForwardBatch(mode="decode", token_ids=tok,
                              positions=self._h2d("d_pos", plan.positions),
                              slot_mapping=self._h2d("d_slots", plan.slot_mapping),
                              block_table=self._h2d("d_bt", plan.block_table).view(B, plan.max_blocks),
                              context_lens=self._h2d("d_ctx", plan.context_lens),
                              decode_splits=ops.mla_decode_splits(B, self.cfg.num_heads, plan.max_context,
                                                                  kv_fp8=getattr(self.cache, "fp8", False))
                              if self.is_cuda else 1)
            logits = self.model.forward(fb, self.cache)
            if self.spec:
                self._draft_kv(fb)
            return self._sample(logits, plan)
        g = self._graph(plan.padded_seqs)
        B = plan.padded_seqs
        # two sets of pinned input buffers: the set written now was last read by the
        # step before the previous one, whose copies have completed
        par = self._parity
        self._parity ^= 1
        ids = self.pinned.get(f"d_ids{par}", B)
        pos = self.pinned.get(f"d_pos{par}", B)
        slots = self.pinned.get(f"d_slots{par}", B)
        ctx = self.pinned.get(f"d_ctx{par}", B)
        bt = self.pinned.get(f"d_bt{B}_{par}", B * self.max_blocks).view(B, self.max_blocks)
        self.h2d_bytes += plan.write_decode_inputs(ids, pos, slots, ctx, bt)
        g.ids.copy_(ids, non_blocking=True)
        g.pos.copy_(pos, non_blocking=True)
        g.slots.copy_(slots, non_blocking=True)
        g.ctx.copy_(ctx, non_blocking=True)
        g.block_table.copy_(bt, non_blocking=True)
        rows = self._sampling_rows(plan, B, f"d{par}")
        if rows is not None or g.sampling_dirty:
            if rows is None:
                g.temps.zero_()
                g.keys.zero_()
            else:
                g.temps.copy_(rows[0], non_blocking=True)
                g.keys.copy_(rows[1], non_blocking=True)
                self.h2d_bytes += B * 12
            g.sampling_dirty = rows is not None
        if plan.flags & self.core.DECISION_SCHEDULED_AHEAD:
            ops.gather_prev_tokens(g.ids, prev.out, plan.num_seqs)
        if self.spec:  # plain-step cost for the speculation utility
            self._timing = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            self._timing[0].record()
            out = g.run()
            self._timing[1].record()
            return out
        return g.run()

    def _launch(self, plan, prev: _Launched | None = None) -> _Launched:
        t0 = time.perf_counter()
        self._timing = None
        try:
            if plan.kind == 3:
                return self._launch_verify(plan, t0)
            if self.stages:
                rows = self._sampling_rows(plan, plan.num_seqs, "s")
                sampled = self.model.run_plan(plan, *(rows if rows is not None else (None, None)))
            elif plan.kind == 1:
                sampled = self._run_prefill(plan)
            else:
                sampled = self._run_decode(plan, prev)
            n = plan.num_seqs
            if self.is_cuda:
                host = self.pinned.get(f"sampled{self._parity}", n)
                host.copy_(sampled[:n], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record()
                self.d2h_bytes += n * 4
            else:
                host, ev = sampled[:n].to(torch.int32).contiguous(), None
        except Exception:
            self.scheduler.fail_step(plan)
            raise
        return _Launched(plan, host, ev, sampled, t0, self._timing)

    def _launch_verify(self, plan, t0: float) -> _Launched:
        committed, counts, paths = self._run_verify(plan)
        v = self.verify_rounds[plan.padded_seqs]
        n, rows = plan.num_seqs, v.rows
        if self.is_cuda:
            par = self._parity
            hc = self.pinned.get(f"vc{par}", n * rows)
            hn = self.pinned.get(f"vn{par}", n)
            hp = self.pinned.get(f"vp{par}", n)
            hc.copy_(committed[:n].reshape(-1), non_blocking=True)
            hn.copy_(counts[:n], non_blocking=True)
            hp.copy_(paths[:n], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record()
            self.d2h_bytes += n * (rows + 2) * 4
        else:
            hc, hn, hp, ev = committed[:n].reshape(-1).clone(), counts[:n].clone(), paths[:n].clone(), None
        return _Launched(plan, (hc, hn, hp), ev, counts, t0, v.timing)

    def _launch_idle(self) -> _Launched:
        """A forward that serves no sequence (one row, no context, no KV write), so
        this rank joins a collective step in which only other ranks have work."""
        t0 = time.perf_counter()
        if self.use_graphs:
            g = self._graph(self.scheduler.bucket_for(1))
            g.ids.zero_()
            g.pos.zero_()
            g.ctx.zero_()
            g.slots.fill_(-1)
            out = g.run()
        elif hasattr(self.model, "idle_forward"):
            out = self.model.idle_forward(self.cache)
        else:
            z = torch.zeros(1, dtype=torch.int32, device=self.device)
            fb = ForwardBatch(mode="decode", token_ids=z, positions=z.clone(), slot_mapping=z - 1,
                              block_table=torch.zeros(1, self.max_blocks, dtype=torch.int32, device=self.device),
                              context_lens=z.clone(), decode_splits=1)
            out = self.model.forward(fb, self.cache)
        ev = None
        if self.is_cuda:
            ev = torch.cuda.Event()
            ev.record()
        self.idle_steps += 1
        return _Launched(None, None, ev, out, t0)

    def _apply_swaps(self, plan):
        """Host-tier copies of a plan, before its step: KV blocks of preempted sequences
        out to their host slots, then restored sequences' slots back into blocks."""
        out, inn = plan.swap_out, plan.swap_in
        if len(out):
            self.host_tier.evict_to(out[0::2].tolist(), out[1::2].tolist())
        if len(inn):
            self.host_tier.restore(inn[0::2].tolist(), inn[1::2].tolist())

    def step(self) -> list[RequestOutput]:
        """One engine step: launches at most one GPU step and completes the step
        before it; returns the requests that changed."""
        changed: dict[int, RequestOutput] = {}
        cur, self._inflight = self._inflight, None
        plan = None
        if cur is not None and cur.plan is not None and self.async_decode and cur.plan.kind == 2:
            a = self.scheduler.schedule_ahead(cur.plan)
            if a.flags & self.core.DECISION_SWAP:
                self._apply_swaps(a)
            if a.kind == 2:
                plan = a
        if plan is None:
            if cur is not None:
                changed.update(self._complete(cur))
                cur = None
            p = self.scheduler.schedule()
            if p.flags & self.core.DECISION_SWAP:
                self._apply_swaps(p)
            plan = p if p.kind != 0 else None
        idle = False
        if self._lockstep is not None:
            busy = plan is not None or cur is not None or self.scheduler.has_work()
            any_plan, self._more = self._lockstep.agree(plan is not None, busy)
            idle = plan is None and any_plan
        launched = None
        try:
            if plan is not None:
                launched = self._launch(plan, cur)
                if plan.flags & self.core.DECISION_SCHEDULED_AHEAD:
                    self.ahead_steps += 1
            elif idle:
                launched = self._launch_idle()
        except Exception:
            if cur is not None:
                self.scheduler.fail_step(cur.plan)
            raise
        try:
            if cur is not None:
                changed.update(self._complete(cur))
        except Exception:
            if launched is not None and launched.plan is not None:
                self.scheduler.fail_step(launched.plan)
            raise
        if launched is not None:
            if self.async_decode and (launched.plan is None or launched.plan.kind == 2):
                self._inflight = launched  # completed by the next step, after it launches its successor
            else:
                changed.update(self._complete(launched))
        return list(changed.values())

    def _complete(self, cur: _Launched) -> dict[int, RequestOutput]:
        plan = cur.plan
        try:
            if cur.event is not None:
                cur.event.synchronize()
        except Exception:
            if plan is not None:
                self.scheduler.fail_step(plan)
            raise
        if plan is None:  # idle forward
            return {}
        now = time.perf_counter()
        # with overlapped steps a step's time is the interval since the previous step ended
        dt = now - max(cur.t0, self._last_done)
        self._last_done = now
        if cur.timing is not None:
            ms = cur.timing[0].elapsed_time(cur.timing[1])
            self.device_ms[plan.kind] = self.device_ms.get(plan.kind, 0.0) + ms
            self._record_cost(plan.kind, plan.padded_seqs, ms)
        if plan.kind == 3:
            hc, hn, hp = cur.host
            n = plan.num_seqs
            counts = hn.numpy()[:n]
            self.step_log.append(("verify", n, dt, int(counts.sum())))
            if self.spec == "mtp_tree":
                for k, c in enumerate(np.bincount(hp.numpy()[:n], minlength=6)[:6]):
                    self.tree_paths[k] += int(c)
            events = self.scheduler.complete_verify(plan, hc.numpy()[: n * plan.rows_per_seq].reshape(n, -1), counts,
                                                    hp.numpy()[:n] if self.spec == "mtp_tree" else None)
        else:
            self.step_log.append(("prefill" if plan.kind == 1 else "decode", plan.num_seqs, dt, plan.num_tokens))
            events = self.scheduler.complete_tensor(plan, cur.host)
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
                self._random.discard(ev.id)
        return changed

    # ------------------------------------------------------------------ batch API
    def generate(self, prompts, params: SamplingParams | None = None) -> GenerateResult:
        """Submits every prompt, runs steps until all finish; returns outputs and serving stats."""
        params = params or SamplingParams()
        ids = [self.add_request(p, params) for p in prompts]
        h2d0, d2h0 = self.h2d_bytes, self.d2h_bytes
        log0 = len(self.step_log)
        t0 = time.perf_counter()
        if self._lockstep is not None:
            # every rank of the group calls generate; all leave at the same agreed step
            while True:
                self.step()
                if not self._more:
                    break
        else:
            while self.has_unfinished_requests():
                self.step()
        wall = time.perf_counter() - t0
        outs = [self.outputs.pop(i) for i in ids]
        for i in ids:
            self.params.pop(i, None)
        log = self.step_log[log0:]
        dec = [s for s in log if s[0] in ("decode", "verify")]
        ver = [s for s in log if s[0] == "verify"]
        dec_tokens = sum(s[3] for s in dec)
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
            "verify_steps": len(ver),
            "verify_lanes": sum(s[1] for s in ver),
            "verify_committed_tokens": sum(s[3] for s in ver),
            "tokens_per_verify_lane": sum(s[3] for s in ver) / max(1, sum(s[1] for s in ver)),
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
        if self._inflight is not None:  # drain a step planned ahead
            cur, self._inflight = self._inflight, None
            self._complete(cur)
        for g in self.graphs.values():
            g.release()
        self.graphs.clear()
        for v in self.verify_rounds.values():
            v.release()
        self.verify_rounds.clear()
        self._pgraphs.clear()
        if hasattr(self.model, "shutdown"):
            self.model.shutdown()
        if self.is_cuda:
            torch.cuda.synchronize(self.device)
