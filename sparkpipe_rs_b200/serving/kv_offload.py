"""Host-memory tier for paged KV blocks: evict blocks of the device cache into
pinned host memory and restore them (possibly into other physical blocks) ahead of
use, on a side stream.

  evict(blocks)    kv_blocks_copy gathers the blocks' rows of every layer into a
                   device staging buffer, then one device->host copy per batch moves
                   them into pinned host slots; returns the host slot ids.
  prefetch(slots, blocks)  one host->device copy into staging (on the copy stream,
                   overlapping whatever runs on the compute stream), then
                   kv_blocks_copy scatters the rows into the target blocks; an event
                   marks completion and ``wait(handle)`` orders the compute stream
                   after it, so a decode step that needs the blocks waits only for them.

  evict_to / restore  the same with host slots chosen by the caller: the scheduler
                   owns the host tier's slot allocation when it preempts a sequence to
                   host memory and restores it later (StepPlan.swap_out / swap_in).

On a CPU cache (the CPU stage driver) the same calls copy with plain indexing.

The residency bookkeeping (which blocks are resident, eviction order) is the C++
KvArena's / scheduler's; this is the data mover. Batches are capped so the staging buffer stays
small; every copy is one cudaMemcpyAsync (no batched-copy API).

Reference behaviour: the KV cache async prefetch backend declared in
crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_kv_cache.h:227-300 (copy
engine, in-flight capacity) and the tier-3 lookahead design of spark_nvme_tier.h; the
reference ships neither.
"""
from __future__ import annotations

import torch

from .. import ops


class HostKvTier:
    """The cache's arrays move together: one plane for a bf16 (or CPU fp32) cache, two
    for the fp8 cache (its e4m3 rows and their block scales, both as 2-byte units)."""

    def __init__(self, cache, host_blocks: int, max_batch_blocks: int = 64):
        self.cache = cache
        self.planes = cache.planes() if hasattr(cache, "planes") else [cache.data]
        data = self.planes[0]
        self.layers = data.shape[0]
        self.bs = cache.block_size
        self.rows = [p.shape[2] for p in self.planes]
        self.row = self.rows[0]
        self.plane_elems = [self.layers * self.bs * r for r in self.rows]
        self.block_elems = sum(self.plane_elems)
        self.max_batch = max_batch_blocks
        self.is_cuda = data.device.type == "cuda"
        self.evicted_blocks = 0
        self.restored_blocks = 0
        if not self.is_cuda:
            self.host = [torch.empty(host_blocks, self.layers, self.bs, r, dtype=p.dtype)
                         for p, r in zip(self.planes, self.rows)]
            self.free, self.pending = list(range(host_blocks))[::-1], []
            return
        self.host = [torch.empty(host_blocks, e, dtype=p.dtype, pin_memory=True)
                     for p, e in zip(self.planes, self.plane_elems)]
        self.free = list(range(host_blocks))[::-1]
        self.pending = []  # (event, host slots) of restores still reading their slots
        # one staging buffer per direction and plane: evictions run on the compute
        # stream, restores on the copy stream
        self.staging_out = [torch.empty(max_batch_blocks * e, dtype=p.dtype, device=p.device)
                            for p, e in zip(self.planes, self.plane_elems)]
        self.staging_in = [torch.empty(max_batch_blocks * e, dtype=p.dtype, device=p.device)
                           for p, e in zip(self.planes, self.plane_elems)]
        self.stream = torch.cuda.Stream(device=data.device)

    def _ids(self, blocks):
        return torch.as_tensor(blocks, dtype=torch.int32).to(self.planes[0].device, non_blocking=True)

    def _reclaim(self, block: bool = False):
        keep = []
        for ev, slots in self.pending:
            if block:
                ev.synchronize()
            if block or ev.query():
                self.free.extend(slots)
            else:
                keep.append((ev, slots))
        self.pending = keep

    def evict(self, blocks: list[int]) -> list[int]:
        """Copies the blocks to host slots (blocking until the copy is done); the device
        blocks may be reused afterwards. Returns one host slot per block."""
        self._reclaim(block=len(blocks) > len(self.free))
        if len(blocks) > len(self.free):
            raise RuntimeError("host KV tier full")
        slots = [self.free.pop() for _ in blocks]
        self.evict_to(blocks, slots)
        return slots

    def _cpu_views(self):
        return [p.view(self.layers, -1, self.bs, r) for p, r in zip(self.planes, self.rows)]

    def evict_to(self, blocks: list[int], slots: list[int]):
        """Copies device blocks into the given host slots; returns when the copy is done
        (earlier restores reading any host slot are waited for first)."""
        assert len(slots) == len(blocks)
        if not self.is_cuda:
            for v, h in zip(self._cpu_views(), self.host):
                for b, s in zip(blocks, slots):
                    h[s].copy_(v[:, b])
            self.evicted_blocks += len(blocks)
            return
        self._reclaim(block=True)
        for i in range(0, len(blocks), self.max_batch):
            chunk, sl = blocks[i:i + self.max_batch], slots[i:i + self.max_batch]
            n = len(chunk)
            ids = self._ids(chunk)
            for plane, stage, host, e in zip(self.planes, self.staging_out, self.host, self.plane_elems):
                ops.kernels().kv_blocks_copy(plane, ids, stage, self.bs, True)
                st = stage[:n * e].view(n, e)
                # host slots of one batch are copied one contiguous run at a time
                j = 0
                while j < n:
                    k = j
                    while k + 1 < n and sl[k + 1] == sl[k] + 1:
                        k += 1
                    host[sl[j]:sl[k] + 1].copy_(st[j:k + 1], non_blocking=True)
                    j = k + 1
        torch.cuda.current_stream().synchronize()
        self.evicted_blocks += len(blocks)

    def restore(self, slots: list[int], blocks: list[int]):
        """Copies host slots into device blocks; the compute stream waits for the copy."""
        if not self.is_cuda:
            for v, h in zip(self._cpu_views(), self.host):
                for s, b in zip(slots, blocks):
                    v[:, b].copy_(h[s])
            self.restored_blocks += len(blocks)
            return
        self.wait(self.prefetch(slots, blocks, owned=False))

    def prefetch(self, slots: list[int], blocks: list[int], owned: bool = True):
        """Starts restoring host slots into device blocks on the copy stream; returns a
        handle for ``wait``. The host slots return to the free list once the copy that
        reads them has completed (``owned``: slots from ``evict``)."""
        assert len(slots) == len(blocks)
        done = torch.cuda.Event()
        cur = torch.cuda.current_stream()
        self.stream.wait_stream(cur)  # the target blocks may have been in use just before
        with torch.cuda.stream(self.stream):
            for i in range(0, len(blocks), self.max_batch):
                chunk, sl = blocks[i:i + self.max_batch], slots[i:i + self.max_batch]
                n = len(chunk)
                ids = self._ids(chunk)
                for plane, stage, host, e in zip(self.planes, self.staging_in, self.host, self.plane_elems):
                    st = stage[:n * e].view(n, e)
                    for j, s in enumerate(sl):
                        st[j].copy_(host[s], non_blocking=True)
                    ops.kernels().kv_blocks_copy(plane, ids, stage, self.bs, False)
            done.record(self.stream)
        # slots this tier handed out return to its free list once read; caller-owned
        # slots are only waited for before the next eviction
        self.pending.append((done, list(slots) if owned else []))
        self.restored_blocks += len(blocks)
        return done

    def wait(self, handle):
        torch.cuda.current_stream().wait_event(handle)
