"""Pipeline parallelism: layer stages on separate ranks, hidden states handed
off with point-to-point send/recv (NCCL between GPUs, gloo between CPU ranks).

Rank 0 runs the serving engine and stage 0. For every step it broadcasts the
step's batch description (one small int32 tensor: header + token ids,
positions, cache slots, cu_seqlens / block tables) to all stage ranks, runs
its layers and sends the residual stream to stage 1; each stage receives,
runs its layers and forwards; the last stage computes the logits of the
requested rows and sends them back to rank 0. Every stage owns the paged KV
cache of its own layers with the same block numbering, so the scheduler's
slot mapping is valid on every stage.

Stage boundaries come from the stage planner (``core.build_stage_plan``); the
reference cuts its 13-node ring the same way
(crates/spark-sched/src/stage_plan.rs:404-484) and hands hidden states over
its pluggable transport (crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_hidden_transport.h:11-345).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..models.mla_moe import ForwardBatch

HEADER = 16
MODES = {"prefill": 1, "decode": 2}


def pack_batch(fb: ForwardBatch) -> torch.Tensor:
    """Flattens a ForwardBatch into one int32 CPU tensor (header + arrays)."""
    parts = [fb.token_ids, fb.positions, fb.slot_mapping]
    hdr = [0] * HEADER
    hdr[0] = MODES[fb.mode]
    hdr[1] = fb.token_ids.numel()
    if fb.mode == "decode":
        hdr[2], hdr[3] = fb.block_table.shape
        hdr[4] = fb.decode_splits
        parts += [fb.block_table.flatten(), fb.context_lens]
    else:
        hdr[2] = fb.cu_q.numel()
        hdr[3] = fb.max_q
        hdr[5] = fb.ctx_slots.numel() if fb.ctx_slots is not None else -1
        parts += [fb.cu_q, fb.cu_k]
        if fb.ctx_slots is not None:
            parts.append(fb.ctx_slots)
    hdr[6] = fb.logits_idx.numel() if fb.logits_idx is not None else -1
    if fb.logits_idx is not None:
        parts.append(fb.logits_idx)
    body = torch.cat([p.reshape(-1).to("cpu", torch.int32) for p in parts])
    return torch.cat([torch.tensor(hdr, dtype=torch.int32), body])


def unpack_batch(buf: torch.Tensor, device) -> ForwardBatch:
    h = buf[:HEADER].tolist()
    mode = "prefill" if h[0] == 1 else "decode"
    T = h[1]
    off = HEADER

    def take(n):
        nonlocal off
        t = buf[off:off + n].to(device)
        off += n
        return t

    ids, pos, slots = take(T), take(T), take(T)
    fb = ForwardBatch(mode=mode, token_ids=ids, positions=pos, slot_mapping=slots)
    if mode == "decode":
        rows, cols = h[2], h[3]
        fb.block_table = take(rows * cols).view(rows, cols)
        fb.context_lens = take(rows)
        fb.decode_splits = h[4]
    else:
        nb = h[2]
        fb.cu_q, fb.cu_k = take(nb), take(nb)
        fb.max_q = h[3]
        if h[5] >= 0:
            fb.ctx_slots = take(h[5])
    if h[6] >= 0:
        fb.logits_idx = take(h[6])
    return fb


def split_layers(num_layers: int, stages: int, first_routed_layer: int = 0) -> list[list[int]]:
    """Balanced contiguous layer ranges (uniform per-layer cost); see core.build_stage_plan
    for the cost-driven planner."""
    base, extra = divmod(num_layers, stages)
    out, start = [], 0
    for s in range(stages):
        n = base + (1 if s < extra else 0)
        out.append(list(range(start, start + n)))
        start += n
    return out


class PipelineModel:
    """Rank-0 view of a pipelined model: ``forward`` drives every stage and returns
    the last stage's logits (or hidden states)."""

    def __init__(self, local_model, stage_layers: list[list[int]], group=None, device=None):
        self.local = local_model
        self.stage_layers = stage_layers
        self.group = group
        self.world = dist.get_world_size(group)
        self.device = torch.device(device) if device is not None else local_model.device
        self.cfg = local_model.cfg
        assert len(stage_layers) == self.world, "one stage per rank"

    def _bcast(self, buf: torch.Tensor):
        n = torch.tensor([buf.numel()], dtype=torch.int64)
        dev = "cpu" if dist.get_backend(self.group) == "gloo" else self.device
        n = n.to(dev)
        dist.broadcast(n, 0, group=self.group)
        dist.broadcast(buf.to(dev), 0, group=self.group)

    def forward(self, fb: ForwardBatch, cache, **_):
        self._bcast(pack_batch(fb))
        h = self.local.forward(fb, cache, layers=self.stage_layers[0], return_hidden=True, layer_offset=0) \
            if _accepts_offset(self.local) else self.local.forward(fb, cache, layers=self.stage_layers[0],
                                                                   return_hidden=True)
        if self.world == 1:
            raise RuntimeError("PipelineModel needs at least two stages")
        dist.send(h.contiguous(), dst=1, group=self.group)
        n_rows = fb.logits_idx.numel() if fb.logits_idx is not None else fb.token_ids.numel()
        logits = torch.empty(n_rows, self.cfg.vocab_size, dtype=h.dtype, device=h.device)
        dist.recv(logits, src=self.world - 1, group=self.group)
        return logits

    def shutdown(self):
        stop = torch.zeros(HEADER, dtype=torch.int32)
        self._bcast(stop)


def _accepts_offset(model) -> bool:
    import inspect

    return "layer_offset" in inspect.signature(model.forward).parameters


def stage_worker_loop(local_model, stage_layers: list[list[int]], cache, group=None, device=None):
    """Loop of ranks >= 1: receive a batch, run this stage, pass the result on.
    Returns when rank 0 broadcasts an empty batch (``PipelineModel.shutdown``)."""
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    layers = stage_layers[rank]
    device = torch.device(device) if device is not None else local_model.device
    comm_dev = "cpu" if dist.get_backend(group) == "gloo" else device
    hidden = local_model.cfg.hidden_size
    h_dtype = torch.float32 if device.type == "cpu" else torch.bfloat16
    while True:
        n = torch.zeros(1, dtype=torch.int64, device=comm_dev)
        dist.broadcast(n, 0, group=group)
        buf = torch.zeros(int(n.item()), dtype=torch.int32, device=comm_dev)
        dist.broadcast(buf, 0, group=group)
        buf = buf.cpu()
        if int(buf[0]) == 0:
            return
        fb = unpack_batch(buf, device)
        T = fb.token_ids.numel()
        h = torch.empty(T, hidden, dtype=h_dtype, device=device)
        dist.recv(h, src=rank - 1, group=group)
        last = rank == world - 1
        kw = {"layer_offset": layers[0]} if _accepts_offset(local_model) else {}
        out = local_model.forward(fb, cache, layers=layers, hidden_in=h, return_hidden=not last, **kw)
        if last:
            dist.send(out.to(h_dtype).contiguous(), dst=0, group=group)
        else:
            dist.send(out.contiguous(), dst=rank + 1, group=group)
