"""Work-output plane (C++): bounded queue, non-blocking socket, write / acknowledge
choreography against a real rank daemon on the other end of a socket, duplicate and
hard-negative acknowledgements, resend after a full receiver, reconnect after a
broken connection, and the sequence-release ring.

Behaviour follows crates/spark-node/src/backend/work_output.rs."""
import socket
import struct
import threading
import time

import pytest

from sparkpipe_rs_b200.core import core

C = core()
WO, WC, RD = C.work_output, C.work_control, C.rank_daemon
OK, CAPACITY, BUSY, ROUTE, DUP, VF = 0, 2, 15, 14, 16, 9


def ident(tid, step=1):
    i = WC.Identity()
    i.control_generation, i.transaction_id, i.dispatch_generation = 1, tid, 1
    i.request_generation, i.step_generation = 1, step
    i.step_chunk_count, i.transaction_phase = 1, 2
    return i


def wcfg():
    w = WC.Config()
    w.output_vocab_count = 1000
    return w


def packet(tid, seqs=(1, 2)):
    p = WC.Packet()
    p.identity = ident(tid)
    lanes = []
    for s in seqs:
        lane = WC.Lane()
        lane.request_id = lane.sequence_id = s
        lane.sequence_position, lane.context_token_count, lane.input_token_id = 10, 11, 7
        lanes.append(lane)
    p.lanes = lanes
    p.active_sequence_count = p.execution_row_count = len(seqs)
    p.execution_batch_bucket = WC.select_batch_bucket(len(seqs))
    p.block_token_count = 64
    return p


def read_packet(sock):
    head = b""
    while len(head) < 12:
        chunk = sock.recv(12 - len(head))
        if not chunk:
            return None
        head += chunk
    total = struct.unpack_from("<I", head, 8)[0]
    body = head
    while len(body) < total:
        body += sock.recv(total - len(body))
    return body


class Peer(threading.Thread):
    """The next rank: answers each packet with `answer(bytes) -> ack bytes`."""

    def __init__(self, sock, answer, limit=None):
        super().__init__(daemon=True)
        self.sock, self.answer, self.limit, self.seen = sock, answer, limit, []

    def run(self):
        try:
            while self.limit is None or len(self.seen) < self.limit:
                b = read_packet(self.sock)
                if b is None:
                    return
                self.seen.append(b)
                self.sock.sendall(self.answer(b))
        except OSError:  # the test closed the socket
            return


def fake_ack(status):
    def answer(b):
        a = RD.Ack()
        a.status, a.identity = status, WC.deserialize(b).identity
        a.packet_fingerprint = WC.fingerprint_bytes(b)
        return RD.ack_to_wire(a)
    return answer


def pump_until(out, want=OK, tries=400, **kw):
    for _ in range(tries):
        st = int(out.pump(**kw))
        if st == want:
            return st
        time.sleep(0.005)
    return st


def make(queue=4):
    return WO.WorkOutput(wcfg(), True, "127.0.0.1", 1, 64, queue, 8)


def test_queue_bounds_and_validation():
    out = make(queue=2)
    out.enqueue(packet(1))
    out.enqueue(packet(2))
    with pytest.raises(Exception):
        out.enqueue(packet(3))  # full
    bad = packet(4)
    bad.block_token_count = 32
    with pytest.raises(Exception):
        make().enqueue(bad)
    last = WO.WorkOutput(wcfg(), False, "", 0, 64, 2, 2)  # final stage: nothing to send
    last.enqueue(packet(5))
    assert int(last.pump()) == OK and last.queued == 1


def test_send_to_rank_daemon_and_duplicates():
    a, b = socket.socketpair()
    cfg = RD.DaemonConfig()
    cfg.work = wcfg()
    daemon = RD.RankDaemon(cfg)
    peer = Peer(b, lambda x: daemon.submit(x))
    peer.start()
    out = make()
    out.adopt_socket(a.detach())
    for t in (1, 2, 3):
        out.enqueue(packet(t, seqs=(t,)))
    assert pump_until(out) == OK and out.queued == 0
    s = out.stats
    assert (s.sent, s.acknowledged, s.duplicates, s.hard_failures) == (3, 3, 0, 0)
    assert daemon.ledger.entries == 3
    # the same packet again (a replay after a lost acknowledgement): the daemon says duplicate
    out.enqueue(packet(2, seqs=(2,)))
    assert pump_until(out) == OK and out.stats.duplicates == 1
    out.drop_socket()
    peer.join(5)  # the peer sees end of stream; close its socket only after it stopped reading
    b.close()


def test_hard_negative_and_full_receiver():
    a, b = socket.socketpair()
    answers = iter([fake_ack(CAPACITY), fake_ack(OK), fake_ack(VF)])
    peer = Peer(b, lambda x: next(answers)(x))
    peer.start()
    out = make()
    out.adopt_socket(a.detach())
    out.enqueue(packet(1))
    out.enqueue(packet(2))
    assert int(pump_until(out, want=BUSY)) == BUSY  # receiver full: packet 1 rewinds
    failed = []
    assert pump_until(out, on_hard_failure=lambda p, st: failed.append((p.identity.transaction_id, int(st)))) == OK
    s = out.stats
    assert (s.sent, s.resent, s.acknowledged, s.hard_failures) == (3, 1, 1, 1)
    assert failed == [(2, VF)] and out.queued == 0
    assert peer.seen[0] == peer.seen[1]  # the resend is byte-identical
    out.drop_socket()
    peer.join(5)  # the peer sees end of stream; close its socket only after it stopped reading
    b.close()


def test_broken_connection_then_reconnect_over_tcp():
    srv = socket.socket()
    srv.bind(("127.0.0.1", 0))
    srv.listen(2)
    port = srv.getsockname()[1]
    out = WO.WorkOutput(wcfg(), True, "127.0.0.1", port, 64, 4, 8)
    out.enqueue(packet(1))
    st = int(out.pump())
    assert st in (OK, BUSY)  # connecting or waiting for the acknowledgement
    conn, _ = srv.accept()
    assert read_packet(conn) is not None
    conn.close()  # dies before acknowledging
    assert pump_until(out, want=ROUTE) == ROUTE and not out.has_socket
    # next pump reconnects and resends whole
    out.pump()
    conn2, _ = srv.accept()
    peer = Peer(conn2, fake_ack(OK))
    peer.start()
    assert pump_until(out) == OK and out.stats.acknowledged == 1 and out.stats.socket_drops == 1
    assert len(peer.seen) == 1 and WC.deserialize(peer.seen[0]).identity.transaction_id == 1
    out.drop_socket()
    peer.join(5)
    conn2.close()
    srv.close()


def test_release_ring():
    out = make()
    for i in range(1, 4):
        out.queue_release(WO.ReleaseRecord(100 + i, 1, i, 20 + i))
    with pytest.raises(Exception):
        out.queue_release(WO.ReleaseRecord(1, 1, 1, 0))  # no tokens
    p = out.build_release_packet(ident(9), 2)
    assert p.flags & 0x20 and p.identity.transaction_phase == 4
    assert [lane.sequence_id for lane in p.lanes] == [1, 2] and [lane.context_token_count for lane in p.lanes] == [21, 22]
    out.enqueue(p)  # a valid packet
    out.pop_releases(2)
    assert out.releases == 1 and out.release(0).sequence_id == 3 and out.stats.releases_sent == 2
    with pytest.raises(Exception):
        out.pop_releases(2)
