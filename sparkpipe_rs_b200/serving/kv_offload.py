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

Drive spill (``resident_blocks`` < ``host_blocks`` with an NVMe ``Tier``): the
scheduler's host slots become virtual. Only ``resident_blocks`` pinned buffers exist;
when a slot needs one and none is free, the least recently used resident slot is
written to the drive tier (two-phase reserve / write / commit under a key unique to the
slot and its write generation) and its buffer reused. A restore of a slot that lives
on the drive asks the tier for it (``request_demand``), pumps the tier until the read
lands in a staging buffer, copies it into a pinned buffer and consumes it. The
scheduler plans swaps exactly as without the drive; the drive is the host tier's
backing store (tier 3 under tier 2).

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


class DriveSpill:
    """The drive under the host tier: an ``nvme_tier.Tier`` over a file (or a given
    block device), one KV block per drive block rounded up to the I/O alignment."""

    def __init__(self, block_bytes: int, blocks: int, path: str | None = None, device=None,
                 staging_buffers: int = 4):
        from ..core import core

        N = core().nvme_tier
        align = int(N.IO_ALIGNMENT)
        self.block_bytes = -(-block_bytes // align) * align
        cfg = N.Config()
        cfg.block_bytes = self.block_bytes
        cfg.budget_bytes = self.block_bytes * max(1, blocks)
        cfg.staging_buffers = max(2, staging_buffers)
        if device is None:
            if path is None:
                raise ValueError("a drive spill needs a file path or a block device")
            device = N.FileDevice(path, cfg.budget_bytes)
        self.device = device
        self.tier = N.Tier(cfg, device)
        self.Demand = N.Demand


class HostKvTier:
    """The cache's arrays move together: one plane for a bf16 (or CPU fp32) cache, two
    for the fp8 cache (its e4m3 rows and their block scales, both as 2-byte units)."""

    def __init__(self, cache, host_blocks: int, max_batch_blocks: int = 64, resident_blocks: int = 0,
                 drive=None, max_demand_polls: int = 1_000_000):
        """``resident_blocks`` (0: all of them) pinned buffers back ``host_blocks`` slots;
        with fewer, ``drive`` (a ``DriveSpill`` of at least one KV block's bytes per
        block) holds the rest."""
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
        # virtual slots: slot -> pinned buffer, or slot -> drive key; LRU order of slots
        n_res = host_blocks if not resident_blocks else min(resident_blocks, host_blocks)
        self.n_res = n_res
        if n_res < host_blocks and drive is None:
            raise ValueError("fewer resident host buffers than slots needs a drive tier")
        self.drive = drive if n_res < host_blocks else None
        self.max_demand_polls = max_demand_polls
        self.buf_of: dict[int, int] = {} if self.drive is not None else {i: i for i in range(host_blocks)}
        self.on_drive: dict[int, int] = {}
        self.lru: dict[int, None] = {}
        self.free_bufs = list(range(n_res))[::-1] if self.drive is not None else []
        self.write_gen = 0
        self.spilled_blocks = self.fetched_blocks = 0
        self.elem_bytes = [p.element_size() for p in self.planes]
        self.block_bytes = sum(e * b for e, b in zip(self.plane_elems, self.elem_bytes))
        if self.drive is not None and self.drive.block_bytes < self.block_bytes:
            raise ValueError("the drive tier's blocks are smaller than a KV block")
        if not self.is_cuda:
            self.host = [torch.empty(n_res, self.layers, self.bs, r, dtype=p.dtype)
                         for p, r in zip(self.planes, self.rows)]
            self.free, self.pending = list(range(host_blocks))[::-1], []
            return
        self.host = [torch.empty(n_res, e, dtype=p.dtype, pin_memory=True)
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

    # ------------------------------------------------------------------ virtual slots
    def _buf_bytes(self, buf: int) -> bytes:
        return b"".join(h[buf].contiguous().view(torch.uint8).numpy().tobytes() for h in self.host)

    def _set_buf_bytes(self, buf: int, data: bytes):
        off = 0
        for h, e, b in zip(self.host, self.plane_elems, self.elem_bytes):
            n = e * b
            src = torch.frombuffer(bytearray(data[off:off + n]), dtype=torch.uint8)
            h[buf].view(-1).view(torch.uint8).copy_(src)
            off += n

    def _touch(self, slot: int):
        self.lru.pop(slot, None)
        self.lru[slot] = None

    def _spill_one(self, keep: set[int]):
        """Writes the least recently used resident slot (not in ``keep``) to the drive and
        frees its buffer."""
        for slot in self.lru:
            if slot in self.buf_of and slot not in keep:
                break
        else:
            raise RuntimeError("host KV tier: every resident buffer is in use by this batch")
        buf = self.buf_of.pop(slot)
        self.lru.pop(slot)
        self.write_gen += 1
        key = (slot << 32) | (self.write_gen & 0xffffffff)
        r = self.drive.tier.reserve_write(key)
        st = self.drive.device.write(r.offset, self._buf_bytes(buf))
        if int(st) != 0:
            self.drive.tier.abort_write(r)
            raise RuntimeError(f"host KV tier: drive write failed ({st})")
        self.drive.tier.commit_write(r)
        self.drive.tier.pin(key, True)  # the slot's only copy: the drive's clock must not take it
        self.on_drive[slot] = key
        self.free_bufs.append(buf)
        self.spilled_blocks += 1

    def _buffer_for(self, slot: int, keep: set[int]) -> int:
        """The pinned buffer of ``slot`` for a write (its old drive copy is dropped)."""
        if self.drive is None:
            return slot
        old = self.on_drive.pop(slot, None)
        if old is not None:
            self.drive.tier.pin(old, False)  # overwritten: the drive copy is stale
        if slot not in self.buf_of:
            if not self.free_bufs:
                self._spill_one(keep)
            self.buf_of[slot] = self.free_bufs.pop()
        self._touch(slot)
        return self.buf_of[slot]

    def _resident(self, slot: int, keep: set[int]) -> int:
        """The pinned buffer holding ``slot``'s bytes, read back from the drive if needed."""
        if self.drive is None:
            return slot
        if slot in self.buf_of:
            self._touch(slot)
            return self.buf_of[slot]
        key = self.on_drive.pop(slot)
        D, tier = self.drive.Demand, self.drive.tier
        data = None
        for step in range(self.max_demand_polls):  # bounded: a read that never lands is an error
            d, payload, _ = tier.request_demand(key, 0)
            if d == D.READY:
                data = payload
                break
            if d == D.MISS:
                raise RuntimeError("host KV tier: a spilled block is no longer on the drive")
            tier.pump(0)
        if data is None:
            raise RuntimeError("host KV tier: drive read did not land")
        tier.consume(key)
        tier.pin(key, False)
        if not self.free_bufs:
            self._spill_one(keep)
        buf = self.buf_of[slot] = self.free_bufs.pop()
        self._set_buf_bytes(buf, data[:self.block_bytes])
        self._touch(slot)
        self.fetched_blocks += 1
        return buf

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
        if self.drive is not None and len(slots) > self.n_res:
            # a batch larger than the pinned buffers goes in pieces: each piece's bytes are
            # on the host (and may spill) before the next piece needs buffers
            for i in range(0, len(slots), self.n_res):
                self.evict_to(blocks[i:i + self.n_res], slots[i:i + self.n_res])
            return
        keep = set(slots)
        if not self.is_cuda:
            bufs = [self._buffer_for(s, keep) for s in slots]
            for v, h in zip(self._cpu_views(), self.host):
                for b, s in zip(blocks, bufs):
                    h[s].copy_(v[:, b])
            self.evicted_blocks += len(blocks)
            return
        self._reclaim(block=True)
        slots = [self._buffer_for(s, keep) for s in slots]
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
        if self.drive is not None and len(slots) > self.n_res:
            for i in range(0, len(slots), self.n_res):
                piece_s, piece_b = slots[i:i + self.n_res], blocks[i:i + self.n_res]
                if self.is_cuda:  # the piece's copy reads its buffers: done before they are reused
                    ev = self.prefetch(piece_s, piece_b, owned=False)
                    ev.synchronize()
                    self.wait(ev)
                else:
                    self.restore(piece_s, piece_b)
            return
        if not self.is_cuda:
            keep = set(slots)
            bufs = [self._resident(s, keep) for s in slots]
            for v, h in zip(self._cpu_views(), self.host):
                for s, b in zip(bufs, blocks):
                    v[:, b].copy_(h[s])
            self.restored_blocks += len(blocks)
            return
        self.wait(self.prefetch(slots, blocks, owned=False))

    def prefetch(self, slots: list[int], blocks: list[int], owned: bool = True):
        """Starts restoring host slots into device blocks on the copy stream; returns a
        handle for ``wait``. The host slots return to the free list once the copy that
        reads them has completed (``owned``: slots from ``evict``)."""
        assert len(slots) == len(blocks)
        if self.drive is not None:
            # drive-resident slots come back into pinned buffers first (host work); the
            # tier's own free list then holds buffer ids, not slot ids
            if owned:
                raise ValueError("prefetch of tier-owned slots is not available with a drive")
            keep = set(slots)
            self._reclaim(block=True)
            slots = [self._resident(s, keep) for s in slots]
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
