"""Per-rank work daemon (C++): wire records, the transaction ledger, the daemon's
dedup / ordering / forward-then-execute pump, and a two-process pipeline over gloo.

Ledger cases follow crates/spark-node/src/rank_daemon/work_ledger.rs; wire sizes
follow its wire.rs."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from sparkpipe_rs_b200.core import StatusError, core

C = core()
RD, WC = C.rank_daemon, C.work_control
OK, DUP, VF, BUSY = 0, 16, 9, 15


def ident(tid=1, gen=1, step=1, phase=2):
    i = WC.Identity()
    i.control_generation, i.transaction_id, i.dispatch_generation = gen, tid, 1
    i.request_generation, i.step_generation = 1, step
    i.step_chunk_count, i.transaction_phase = 1, phase
    return i


def packet(tid, seqs, step=1, gen=1):
    p = WC.Packet()
    p.identity = ident(tid, gen, step)
    lanes = []
    for s in seqs:
        lane = WC.Lane()
        lane.request_id = s
        lane.sequence_id = s
        lane.sequence_position = 10 + step
        lane.context_token_count = 11 + step
        lane.input_token_id = 7
        lanes.append(lane)
    p.lanes = lanes
    p.active_sequence_count = len(seqs)
    p.execution_row_count = len(seqs)
    p.execution_batch_bucket = WC.select_batch_bucket(len(seqs))
    p.block_token_count = 64
    return p


def cfg(rank=0, world=1, **kw):
    c = RD.DaemonConfig()
    c.rank, c.world = rank, world
    for k, v in kw.items():
        setattr(c, k, v)
    w = WC.Config()
    w.output_vocab_count = 1000
    c.work = w
    return c


# ------------------------------------------------------------------ wire records
def test_wire_record_sizes_and_roundtrips():
    i = ident(tid=77, step=3)
    b = RD.identity_to_wire(i)
    assert len(b) == RD.IDENTITY_BYTES == 56
    assert RD.identity_from_wire(b).transaction_id == 77
    a = RD.Ack()
    a.status, a.state, a.identity, a.packet_fingerprint = DUP, RD.STATE_ACCEPTED, i, 123
    w = RD.ack_to_wire(a)
    assert len(w) == RD.ACK_BYTES == 96
    back = RD.ack_from_wire(w)
    assert (back.status, back.state, back.packet_fingerprint, back.identity.step_generation) == (DUP, 2, 123, 3)
    with pytest.raises(StatusError):
        RD.ack_from_wire(b"\0" * 96)
    e = RD.FinalEvent()
    e.token_ids, e.request_id, e.identity, e.service_time_ns = [5, 6, 7], 9, i, 1234
    w = RD.final_event_to_wire(e)
    assert len(w) == RD.FINAL_EVENT_BYTES == 272
    f = RD.final_event_from_wire(w)
    assert list(f.token_ids) == [5, 6, 7] and f.request_id == 9 and f.service_time_ns == 1234
    assert RD.packet_dedup_hash32(b"abc") == 0x1A47E90B  # FNV-1a 32


# ------------------------------------------------------------------ ledger
def test_ledger_observe_replay_conflict_and_transitions():
    L = RD.TransactionLedger(8)
    i = ident(1)
    assert L.observe(i, 42) == RD.Observation.NEW
    assert L.observe(i, 42) == RD.Observation.REPLAY_ACTIVE
    assert L.observe(i, 43) == RD.Observation.CONFLICT
    L.transition(i, RD.STATE_ACCEPTED)
    with pytest.raises(StatusError):
        L.transition(i, RD.STATE_COMMITTED)  # skips EXECUTING
    L.transition(i, RD.STATE_EXECUTING)
    L.transition(i, RD.STATE_COMMITTED)
    assert L.observe(i, 42) == RD.Observation.REPLAY_TERMINAL
    with pytest.raises(StatusError) as e:
        L.transition(i, RD.STATE_COMMITTED)
    assert e.value.code == DUP
    assert (L.entries, L.active, L.terminal) == (1, 0, 1)
    with pytest.raises(StatusError):
        L.observe(i, 0)


def test_ledger_generations_and_recycling():
    L = RD.TransactionLedger(4)
    L.observe(ident(1, gen=2), 1)
    with pytest.raises(StatusError) as e:
        L.observe(ident(2, gen=1), 1)  # stale generation
    assert e.value.code == VF
    with pytest.raises(StatusError) as e:
        L.observe(ident(2, gen=3), 1)  # newer generation while a transaction is active
    assert e.value.code == BUSY
    L.transition(ident(1, gen=2), RD.STATE_CANCELLED)
    assert L.observe(ident(2, gen=3), 1) == RD.Observation.NEW  # reset on the new generation
    assert L.control_generation == 3 and L.entries == 1
    # a full table recycles its oldest terminal entry; an all-active table refuses
    for t in range(3, 6):
        L.observe(ident(t, gen=3), 1)
    for t in (2, 3):
        L.transition(ident(t, gen=3), RD.STATE_FAILED, C.Status.INTERNAL_ERROR)
    assert L.observe(ident(9, gen=3), 1) == RD.Observation.NEW
    assert L.find(ident(2, gen=3)) is None and L.find(ident(3, gen=3)) is not None
    full = RD.TransactionLedger(2)
    full.observe(ident(1), 1)
    full.observe(ident(2), 1)
    with pytest.raises(StatusError) as e:
        full.observe(ident(3), 1)
    assert e.value.code == 2


# ------------------------------------------------------------------ daemon
def test_three_rank_chain_forwards_executes_and_finalises():
    finals, executed = [], {0: [], 1: [], 2: []}
    daemons = []

    def make(r):
        def forward(b):
            ack = RD.ack_from_wire(daemons[r + 1].submit(b))
            assert ack.status == OK

        def execute(b):
            executed[r].append(WC.deserialize(b).identity.transaction_id)
        return RD.RankDaemon(cfg(r, 3), forward if r < 2 else None, execute, finals.append if r == 2 else None)
    daemons.extend(make(r) for r in range(3))
    for tid, seqs in [(1, [10, 11]), (2, [12])]:
        ack = RD.ack_from_wire(daemons[0].submit(packet(tid, seqs).serialize()))
        assert ack.status == OK and ack.state == RD.STATE_ACCEPTED
    for d in daemons:
        d.pump()
    assert executed == {0: [1, 2], 1: [1, 2], 2: [1, 2]}
    for d in daemons:
        for tid in (1, 2):
            d.complete(ident(tid), C.Status.OK, [100 + tid], 500)
    assert len(finals) == 2
    f = RD.final_event_from_wire(finals[0])
    assert f.identity.transaction_id == 1 and list(f.token_ids) == [101]
    for d in daemons:
        s = d.stats()
        assert (s.accepted, s.executed, s.committed, s.inflight) == (2, 2, 2, 0)
        assert d.ledger.find(ident(1)).state == RD.STATE_COMMITTED
    assert daemons[0].stats().forwarded == 2 and daemons[2].stats().forwarded == 0


def test_duplicates_conflicts_and_bad_packets():
    d = RD.RankDaemon(cfg(), None, None, None)
    wire = packet(1, [5]).serialize()
    assert RD.ack_from_wire(d.submit(wire)).status == OK
    dup = RD.ack_from_wire(d.submit(wire))  # retransmission: same bytes
    assert dup.status == DUP and dup.state == RD.STATE_ACCEPTED
    changed = packet(1, [6]).serialize()  # same transaction, different payload
    assert RD.ack_from_wire(d.submit(changed)).status == VF
    bad = bytearray(wire)
    bad[0] ^= 0xFF
    a = RD.ack_from_wire(d.submit(bytes(bad)))
    assert a.status != OK and a.state == RD.STATE_FAILED
    s = d.stats()
    assert (s.accepted, s.duplicates, s.conflicts, s.rejected) == (1, 1, 1, 1)


def test_same_sequence_steps_run_in_order():
    order = []
    d = RD.RankDaemon(cfg(), None, lambda b: order.append(WC.deserialize(b).identity.transaction_id), None)
    d.submit(packet(1, [5, 6], step=1).serialize())
    d.submit(packet(2, [6], step=2).serialize())     # waits for seq 6
    d.submit(packet(3, [7], step=1).serialize())     # independent: may overtake
    d.submit(packet(4, [6, 8], step=3).serialize())  # waits behind packet 2
    assert d.pump() == 2 and order == [1, 3]
    d.complete(ident(1, step=1))
    assert d.pump() == 1 and order == [1, 3, 2]
    d.complete(ident(2, step=2))
    assert d.pump() == 1 and order == [1, 3, 2, 4]


def test_queue_capacity_and_cancel():
    d = RD.RankDaemon(cfg(queue_capacity=2), None, None, None)
    assert RD.ack_from_wire(d.submit(packet(1, [1]).serialize())).status == OK
    assert RD.ack_from_wire(d.submit(packet(2, [2]).serialize())).status == OK
    assert RD.ack_from_wire(d.submit(packet(3, [3]).serialize())).status == BUSY
    d.cancel(ident(2))
    assert d.ledger.find(ident(2)).state == RD.STATE_CANCELLED and d.stats().queued == 1
    assert RD.ack_from_wire(d.submit(packet(3, [3]).serialize())).status == OK
    with pytest.raises(StatusError):
        d.cancel(ident(99))


# ------------------------------------------------------------------ two processes over gloo
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _pipeline_rank(rank, port, q):
    import torch
    import torch.distributed as dist
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2,
                                timeout=datetime.timedelta(seconds=60))

        def send(b, dst):
            dist.send(torch.tensor([len(b)], dtype=torch.int64), dst)
            dist.send(torch.frombuffer(bytearray(b), dtype=torch.uint8), dst)

        def recv(src):
            n = torch.zeros(1, dtype=torch.int64)
            dist.recv(n, src)
            buf = torch.zeros(int(n), dtype=torch.uint8)
            dist.recv(buf, src)
            return bytes(buf.numpy())

        if rank == 0:
            d = RD.RankDaemon(cfg(0, 2), lambda b: send(b, 1), None, None)
            for tid in (1, 2, 3):
                d.submit(packet(tid, [tid]).serialize())
            d.pump()
            finals = [RD.final_event_from_wire(recv(1)) for _ in range(3)]
            q.put(("ok", sorted(f.identity.transaction_id for f in finals), [list(f.token_ids) for f in finals]))
        else:
            finals = []
            d = RD.RankDaemon(cfg(1, 2), None, None, finals.append)
            for _ in range(3):
                assert RD.ack_from_wire(d.submit(recv(0))).status == OK
            d.pump()
            for tid in (1, 2, 3):
                d.complete(ident(tid), C.Status.OK, [tid * 10])
            for f in finals:
                send(f, 0)
            q.put(("ok", d.stats().committed, None))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put(("error", repr(e), None))


def test_two_rank_pipeline_over_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_pipeline_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(r[0] == "ok" for r in res), res
    rank0 = next(r for r in res if isinstance(r[1], list))
    assert rank0[1] == [1, 2, 3] and sorted(rank0[2]) == [[10], [20], [30]]
