"""Pipeline parallelism driven by the work plane: layer stages on separate ranks,
every step carried to them as work-control packets through each rank's daemon.

Rank 0 runs the serving engine and stage 0. A scheduler step becomes ``chunks``
micro-batch packets (``work_control.build_stage_packets``: contiguous lanes, one
transaction each, with an execution payload: rows' positions and cache slots,
decode block tables and context lengths or prefill query / key offsets, and each
lane's sampling parameters). Each packet enters rank 0's ``RankDaemon`` (ledger
handshake, duplicate check, per-sequence ordering), which forwards it to the next
rank before it runs the local stage (forward-then-submit). Every rank runs its
layers on the packet's rows and hands the residual stream on with a point-to-point
send (NCCL between GPUs, gloo between CPU ranks); the last rank computes the
logits of the packet's sampling rows, samples them (greedy, or Gumbel-max with the
lane's temperature and noise key) and completes the transaction with one final
event per lane, which goes back to rank 0 as one message per packet. Rank 0 turns
the final events into the step's sampled tokens.

Micro-batches overlap stages: while stage s runs micro-batch k + 1, stage s + 1
runs micro-batch k, and each hidden-state send is asynchronous, so a step of two
stages and two micro-batches takes about three stage-halves instead of four.

Control messages (packet wires forward, final-event batches back to rank 0) travel
on a gloo group as a length followed by the bytes; a zero length ends the run.
Every stage owns the paged KV cache of its own layers with the scheduler's block
numbering, so a packet's slots are valid on every stage.

Stage boundaries come from the stage planner (``core.stage_plan``); the reference
cuts its ring the same way (crates/spark-sched/src/stage_plan.rs:404-484). The
packet / ledger / final-event flow follows crates/spark-node/src/rank_daemon/
daemon.rs:987-1128 and backend/decode.rs:144-746, with the hidden-state hand-off of
crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_hidden_transport.h.
"""
from __future__ import annotations

import time

import torch
import torch.distributed as dist

from ..core import core
from ..models.mla_moe import ForwardBatch

FINAL_EVENT_BYTES = 272


def split_layers(num_layers: int, stages: int, first_routed_layer: int = 0) -> list[list[int]]:
    """Balanced contiguous layer ranges (uniform per-layer cost); see core.stage_plan
    for the cost-driven planner."""
    base, extra = divmod(num_layers, stages)
    out, start = [], 0
    for s in range(stages):
        n = base + (1 if s < extra else 0)
        out.append(list(range(start, start + n)))
        start += n
    return out


def layer_costs(cfg, phase: str = "decode") -> tuple[list[int], int]:
    """Relative per-layer costs and the last stage's extra (final norm + LM head):
    decode steps are bound by the weight bytes a layer reads (every routed expert of
    a batch), prefill chunks by the weights each token multiplies (its top-k experts)."""
    H, nh = cfg.hidden_size, cfg.num_heads
    qa = cfg.q_lora_rank or nh * (cfg.qk_nope_head_dim + cfg.qk_rope_head_dim)
    attn = H * (qa + cfg.kv_lora_rank + cfg.qk_rope_head_dim) + cfg.kv_lora_rank * nh * (
        cfg.qk_nope_head_dim + cfg.v_head_dim) + nh * cfg.v_head_dim * H
    if cfg.q_lora_rank:
        attn += cfg.q_lora_rank * nh * (cfg.qk_nope_head_dim + cfg.qk_rope_head_dim)
    expert = 3 * H * cfg.moe_intermediate_size
    routed = cfg.n_routed_experts if phase == "decode" else cfg.num_experts_per_tok
    costs = []
    for i in range(cfg.num_layers):
        ffn = (routed + cfg.n_shared_experts) * expert if cfg.is_moe_layer(i) else 3 * H * cfg.intermediate_size
        costs.append(max(1, (attn + ffn) // 1000))
    return costs, max(1, cfg.vocab_size * H // 1000)


def plan_stages(cfg, stages: int, costs: list[int] | None = None, final_extra: int | None = None,
                phase: str = "decode") -> list[list[int]]:
    """Contiguous layer ranges per stage from the stage planner: the cuts that minimise
    the slowest stage under per-layer costs (measured, or ``layer_costs``), the last
    stage also paying the LM head."""
    if costs is None:
        costs, est_extra = layer_costs(cfg, phase)
        final_extra = est_extra if final_extra is None else final_extra
    sp = core().stage_plan
    first_routed = cfg.first_k_dense_replace if cfg.n_routed_experts else cfg.num_layers
    geo = sp.Geometry(cfg.num_layers, min(first_routed, cfg.num_layers), cfg.num_layers)
    plan = sp.build_balanced(geo, [int(c) for c in costs], int(final_extra or 0), stages)
    return [list(range(st.first_layer, st.first_layer + st.layer_count)) for st in plan.stages]


def work_config(cfg, block_size: int, max_model_len: int, max_lanes: int, max_prefill_tokens: int):
    """Packet geometry the daemons validate against."""
    w = core().work_control.Config()
    w.kv_block_tokens = block_size
    w.maximum_context_tokens = -(-max_model_len // block_size) * block_size
    w.output_vocab_count = cfg.vocab_size
    w.max_lane_count = max(1, max_lanes)
    w.max_prefill_tokens_per_packet = max(1, max_prefill_tokens)
    return w


class _Link:
    """Length-prefixed byte messages on a gloo group; sends are asynchronous and
    complete before the next send to the same peer reuses nothing (each keeps its
    buffers until ``drain``)."""

    def __init__(self, group):
        self.group = group
        self.pending = []

    def send(self, dst: int, payload: bytes):
        n = torch.tensor([len(payload)], dtype=torch.int64)
        self.pending.append((dist.isend(n, dst, group=self.group), n))
        if payload:
            buf = torch.frombuffer(bytearray(payload), dtype=torch.uint8)
            self.pending.append((dist.isend(buf, dst, group=self.group), buf))
        if len(self.pending) > 64:
            self.drain(keep=16)

    def recv(self, src: int) -> bytes:
        n = torch.zeros(1, dtype=torch.int64)
        dist.recv(n, src, group=self.group)
        if int(n) == 0:
            return b""
        buf = torch.empty(int(n), dtype=torch.uint8)
        dist.recv(buf, src, group=self.group)
        return buf.numpy().tobytes()

    def drain(self, keep: int = 0):
        while len(self.pending) > keep:
            w, _ = self.pending.pop(0)
            w.wait()


def sample_rows(logits: torch.Tensor, temps, keys) -> list[int]:
    """Greedy argmax per row, or Gumbel-max for rows with a temperature, the noise
    seeded by the row's key (the engine's sampling, at the last stage)."""
    if logits.is_cuda:
        from .. import ops

        if temps is None or not (temps > 0).any():
            return ops.sample_tokens(logits).tolist()
        t = torch.as_tensor(temps, dtype=torch.float32).to(logits.device)
        k = torch.as_tensor(keys, dtype=torch.int64).to(logits.device)
        return ops.sample_tokens(logits, row_temp=t, row_key=k).tolist()
    out = logits.float().argmax(-1).tolist()
    if temps is not None:
        for i, t in enumerate(temps):
            if t > 0:
                g = torch.Generator().manual_seed(int(keys[i]) & ((1 << 63) - 1))
                u = torch.rand(logits.shape[1], generator=g).clamp_min(1e-20)
                out[i] = int((logits[i].float() / float(t) - torch.log(-torch.log(u))).argmax())
    return out


class _StageGraph:
    """CUDA graph of one stage's decode forward for a padded lane count: static input
    buffers (token ids, positions, slots, block table, context lengths and, past stage
    0, the received hidden rows), captured once after an eager warm-up over idle rows
    (context 0, slot -1: nothing read, no KV written). Rows past a packet's lanes stay
    idle."""

    def __init__(self, rt, lanes: int, cols: int):
        from .. import ops

        dev, m = rt.device, rt.model
        i32 = dict(dtype=torch.int32, device=dev)
        self.lanes = lanes
        self.ids = torch.zeros(lanes, **i32)
        self.pos = torch.zeros(lanes, **i32)
        self.slots = torch.full((lanes,), -1, **i32)
        self.bt = torch.zeros(lanes, cols, **i32)
        self.ctx = torch.zeros(lanes, **i32)
        self.h = torch.zeros(lanes, rt.hidden, dtype=rt.h_dtype, device=dev) if rt.rank > 0 else None
        splits = ops.mla_decode_splits(lanes, m.cfg.num_heads, cols * rt.wcfg.kv_block_tokens,
                                       kv_fp8=getattr(rt.cache, "fp8", False))
        self.fb = ForwardBatch(mode="decode", token_ids=self.ids, positions=self.pos, slot_mapping=self.slots,
                               block_table=self.bt, context_lens=self.ctx, decode_splits=splits)

        def run():
            return m.forward(self.fb, rt.cache, layers=rt.layers, hidden_in=self.h, return_hidden=not rt.last,
                             layer_offset=rt.layers[0])

        run()  # sets kernel attributes and sizes workspaces outside capture
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        cur = torch.cuda.current_stream(dev)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(cur)
        # thread-local capture: the process group's own threads (NCCL watchdog, gloo
        # workers) keep making CUDA calls while this thread captures
        with torch.cuda.stream(side), torch.cuda.graph(self.graph, stream=side, capture_error_mode="thread_local"):
            self.out = run()
        cur.wait_stream(side)

    def load(self, pk, dev):
        """Copies a decode packet's rows into the static inputs; the rest go idle."""
        e = pk.exec
        n = len(e.context_lens)

        def put(dst, a):
            dst[:n].copy_(torch.from_numpy(a).to(dev, non_blocking=True).view(dst[:n].shape))

        put(self.ids, pk.input_token_ids)
        put(self.pos, e.positions)
        put(self.slots, e.slots)
        put(self.ctx, e.context_lens)
        put(self.bt, e.block_table)
        if n < self.lanes:
            self.slots[n:].fill_(-1)
            self.ctx[n:].zero_()
        return n


class StageRuntime:
    """One pipeline rank: its daemon, its layers and KV cache, its links. Decode
    packets replay a per-stage CUDA graph of the padded lane count on GPUs
    (``use_graphs``); prefill packets run eagerly."""

    def __init__(self, model, stage_layers: list[list[int]], cache, wcfg, group=None, control_group=None,
                 device=None, use_graphs: bool = True):
        self.C = core()
        self.model, self.stage_layers, self.cache, self.wcfg = model, stage_layers, cache, wcfg
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if len(stage_layers) != self.world or self.world < 2:
            raise ValueError("one stage per rank, at least two stages")
        self.layers = stage_layers[self.rank]
        self.last = self.rank == self.world - 1
        self.device = torch.device(device) if device is not None else model.device
        ranks = list(range(self.world)) if group is None else dist.get_process_group_ranks(group)
        self.control = control_group or dist.new_group(ranks=ranks, backend="gloo")
        self.link = _Link(self.control)
        self.hidden_sends = []
        R = self.C.rank_daemon
        dc = R.DaemonConfig()
        dc.rank, dc.world, dc.work = self.rank, self.world, wcfg
        self.finals: list[bytes] = []
        self.daemon = R.RankDaemon(dc, self._forward, self._execute, self.finals.append)
        self.h_dtype = torch.float32 if self.device.type == "cpu" else torch.bfloat16
        self.hidden = model.cfg.hidden_size
        self.executed = 0
        self.use_graphs = use_graphs and self.device.type == "cuda"
        self.graphs: dict[tuple[int, int], _StageGraph] = {}
        self.graph_replays = 0
        self.last_logits = None  # last stage: logits of the most recent packet (diagnostics)
        self.after_execute = None  # optional callable(runtime) after each packet (diagnostics)

    # ------------------------------------------------------------------ daemon callbacks
    def _forward(self, wire: bytes):
        self.link.send(self.rank + 1, wire)

    def _batch(self, pk) -> ForwardBatch:
        W = self.C.work_control
        e = pk.exec
        dev = self.device

        def t(a):
            return torch.from_numpy(a).to(dev)

        if pk.flags & W.FLAG_PREFILL:
            return ForwardBatch(mode="prefill", token_ids=t(pk.prefill_tokens), positions=t(e.positions),
                                slot_mapping=t(e.slots), cu_q=t(e.cu_q), cu_k=t(e.cu_k), max_q=int(e.max_q),
                                ctx_slots=t(e.ctx_slots) if len(e.ctx_slots) else None,
                                logits_idx=t(e.logits_rows))
        lanes = len(e.context_lens)
        splits = 1
        if dev.type == "cuda":
            from .. import ops

            splits = ops.mla_decode_splits(lanes, self.model.cfg.num_heads, int(e.context_lens.max()),
                                           kv_fp8=getattr(self.cache, "fp8", False))
        return ForwardBatch(mode="decode", token_ids=t(pk.input_token_ids), positions=t(e.positions),
                            slot_mapping=t(e.slots), block_table=t(e.block_table).view(lanes, e.block_table_cols),
                            context_lens=t(e.context_lens), decode_splits=splits)

    def _graph_for(self, pk):
        """The stage graph for a decode packet (lanes rounded up to a power of two),
        captured on first use; None for prefill packets or without graphs."""
        W = self.C.work_control
        if not self.use_graphs or pk.flags & W.FLAG_PREFILL:
            return None
        lanes = len(pk.exec.context_lens)
        bucket = 1 << max(0, (lanes - 1).bit_length())
        key = (bucket, int(pk.exec.block_table_cols))
        g = self.graphs.get(key)
        if g is None:
            g = self.graphs[key] = _StageGraph(self, bucket, key[1])
        return g

    def _execute(self, wire: bytes):
        t0 = time.perf_counter_ns()
        pk = self.C.work_control.deserialize(wire)
        g = self._graph_for(pk)
        if g is not None:
            rows = g.load(pk, self.device)
            if self.rank > 0:
                dist.irecv(g.h[:rows], self.rank - 1, group=self.group).wait()
            g.graph.replay()
            self.graph_replays += 1
            out = g.out[:rows]
        else:
            fb = self._batch(pk)
            rows = fb.token_ids.numel()
            h = None
            if self.rank > 0:
                h = torch.empty(rows, self.hidden, dtype=self.h_dtype, device=self.device)
                dist.irecv(h, self.rank - 1, group=self.group).wait()
            out = self.model.forward(fb, self.cache, layers=self.layers, hidden_in=h, return_hidden=not self.last,
                                     layer_offset=self.layers[0])
        if not self.last:
            out = out.to(self.h_dtype).clone() if g is not None else out.to(self.h_dtype).contiguous()
            self.hidden_sends.append((dist.isend(out, self.rank + 1, group=self.group), out))
            while len(self.hidden_sends) > 4:
                w, _ = self.hidden_sends.pop(0)
                w.wait()
            self.daemon.complete(pk.identity, self.C.Status.OK, [], time.perf_counter_ns() - t0)
        else:
            self.last_logits = out
            e = pk.exec
            toks = sample_rows(out, e.temperature, e.sample_keys)
            self.finals.clear()
            self.daemon.complete_lanes(pk.identity, self.C.Status.OK, [[t] for t in toks],
                                       time.perf_counter_ns() - t0)
            self.link.send(0, b"".join(self.finals))
        self.executed += 1
        if self.after_execute is not None:
            self.after_execute(self)

    # ------------------------------------------------------------------ stage loop (ranks >= 1)
    def serve(self):
        """Runs packets from the previous rank until it ends the run."""
        while True:
            wire = self.link.recv(self.rank - 1)
            if not wire:
                if not self.last:
                    self.link.send(self.rank + 1, b"")
                break
            self.daemon.submit(wire)
            self.daemon.pump()
        self.close()

    def close(self):
        self.link.drain()
        for w, _ in self.hidden_sends:
            w.wait()
        self.hidden_sends.clear()
        self.graphs.clear()  # graphs release their pools before the process group goes


class PipelineModel(StageRuntime):
    """Rank 0 of a pipeline: the engine hands it whole scheduler steps
    (``runs_plans``) and receives each lane's sampled token from the final events."""

    runs_plans = True

    def __init__(self, model, stage_layers, cache, wcfg, micro_batches: int = 2, group=None, control_group=None,
                 device=None, use_graphs: bool = True):
        super().__init__(model, stage_layers, cache, wcfg, group, control_group, device, use_graphs)
        if self.rank != 0:
            raise ValueError("PipelineModel runs on rank 0")
        self.cfg = model.cfg
        self.micro_batches = max(1, micro_batches)
        self.step = 0
        self.tx = 0
        self.final_events = 0

    def run_plan(self, plan, temps=None, keys=None) -> torch.Tensor:
        """Runs one scheduler step through every stage; returns the sampled token of
        each of the plan's sequences (int32, in plan order)."""
        W, R = self.C.work_control, self.C.rank_daemon
        self.step += 1
        ident = W.Identity()
        ident.control_generation, ident.request_generation = 1, 1
        ident.dispatch_generation = ident.step_generation = self.step
        ident.transaction_id = self.tx + 1
        ident.step_chunk_count = 1
        ident.transaction_phase = W.PHASE_PREFILL
        n = plan.num_seqs
        t = None if temps is None else temps.numpy()[:n]
        k = None if keys is None else keys.numpy()[:n]
        wires = W.build_stage_packets(plan, ident, self.wcfg, self.micro_batches, t, k)
        self.tx += len(wires)
        for wire in wires:
            ack = R.ack_from_wire(self.daemon.submit(wire))
            if ack.status != int(self.C.Status.OK):
                raise RuntimeError(f"pipeline: packet refused by the daemon (status {ack.status})")
            self.daemon.pump()
        tokens: dict[int, int] = {}
        for _ in wires:
            buf = self.link.recv(self.world - 1)
            for off in range(0, len(buf), FINAL_EVENT_BYTES):
                ev = R.final_event_from_wire(buf[off:off + FINAL_EVENT_BYTES])
                if ev.status != int(self.C.Status.OK) or not ev.token_ids:
                    raise RuntimeError("pipeline: a stage failed its packet")
                tokens[int(ev.sequence_id)] = int(ev.token_ids[0])
                self.final_events += 1
        return torch.tensor([tokens[int(s)] for s in plan.seq_ids[:n]], dtype=torch.int32)

    def shutdown(self):
        self.link.send(1, b"")
        self.close()


__all__ = ["split_layers", "layer_costs", "plan_stages", "work_config", "StageRuntime", "PipelineModel", "sample_rows", "FINAL_EVENT_BYTES"]
