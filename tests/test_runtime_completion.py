"""Runtime completion (C++): credit ledger, final event queue, transmission window and
the transaction controller (prepare / execute / commit over every participant, cancel
in reverse order on failure, replay answered from the record, conflicts refused).

Participant flags, slot states and the controller surface follow
crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_runtime_completion.h."""
import pytest

from sparkpipe_rs_b200.core import core

C = core()
RC, WC = C.runtime_completion, C.work_control
OK, INVALID, NOT_FOUND, BUSY, DUP, INTERNAL = 0, 1, 3, 15, 16, 17


def ident(tid=1, gen=1, step=1, phase=2):
    i = WC.Identity()
    i.control_generation, i.transaction_id, i.dispatch_generation = gen, tid, 1
    i.request_generation, i.step_generation = 1, step
    i.step_chunk_count, i.transaction_phase = 1, phase
    return i


def request(tid=1, payload=b"step", seq=7):
    r = RC.Request()
    r.identity, r.request_id, r.sequence_id, r.sequence_position, r.payload = ident(tid), 100 + tid, seq, 3, payload
    return r


class Part:
    """Records every call; fails prepare or execute on request."""

    def __init__(self, name, log, fail_prepare=0, fail_execute=0, flags=None):
        self.name, self.log = name, log
        self.fail_prepare, self.fail_execute = fail_prepare, fail_execute
        if flags is not None:
            self.flags = flags

    def prepare(self, r):
        self.log.append((self.name, "prepare", r.identity.transaction_id))
        return self.fail_prepare

    def execute(self, r):
        self.log.append((self.name, "execute", r.identity.transaction_id))
        return self.fail_execute

    def commit(self, r):
        self.log.append((self.name, "commit", r.identity.transaction_id))

    def cancel(self, r, reason):
        self.log.append((self.name, "cancel", int(reason)))


def test_credit_ledger():
    c = RC.CreditLedger([2, 1, 1, 1])
    assert c.acquire(RC.DOMAIN_TRANSPORT_WINDOW, 2) and not c.acquire(RC.DOMAIN_TRANSPORT_WINDOW, 1)
    assert c.available(RC.DOMAIN_TRANSPORT_WINDOW) == 0 and c.in_use(RC.DOMAIN_TRANSPORT_WINDOW) == 2
    c.release(RC.DOMAIN_TRANSPORT_WINDOW, 2)
    with pytest.raises(Exception):
        c.release(RC.DOMAIN_EXECUTION, 1)  # not held
    with pytest.raises(Exception):
        c.acquire(4, 1)  # unknown domain
    with pytest.raises(Exception):
        RC.CreditLedger([1, 0, 1, 1])


def test_final_event_queue_order_and_ack():
    q = RC.FinalEventQueue(2)
    evs = []
    for t in (1, 2):
        e = RC.FinalEvent()
        e.identity, e.payload_fingerprint, e.request_id = ident(t), 50 + t, t
        evs.append(q.push(e))
    assert evs == [1, 2] and q.pending == 2
    with pytest.raises(Exception):
        q.push(e)  # full
    assert q.peek().generation == 1
    assert int(q.acknowledge(ident(1), 1, 999)) == INVALID  # wrong fingerprint
    assert int(q.acknowledge(ident(2), 2, 52)) == OK  # out of order is allowed
    assert int(q.acknowledge(ident(2), 2, 52)) == NOT_FOUND
    assert q.peek().generation == 1 and int(q.acknowledge(ident(1), 1, 51)) == OK and q.peek() is None


def test_transmission_window_reserve_send_ack_replay():
    w = RC.TransmissionWindow(2)
    s1, g1 = w.reserve(ident(1), 11)
    assert w.reserve(ident(1), 11) == (s1, g1)  # idempotent
    with pytest.raises(Exception):
        w.reserve(ident(1), 12)  # same identity, other payload
    s2, g2 = w.reserve(ident(2), 22)
    with pytest.raises(Exception):
        w.reserve(ident(3), 33)  # full
    assert w.next_replay() is None  # nothing sent yet
    with pytest.raises(Exception):
        w.acknowledge(s1, g1, ident(1), 11)  # not sent
    w.mark_sent(s1, g1)
    w.mark_sent(s2, g2)
    assert w.next_replay() == (s1, g1)  # sent longest ago
    w.mark_sent(s1, g1)  # re-sent
    assert w.slot(s1).retry_count == 1 and w.next_replay() == (s2, g2)
    assert int(w.acknowledge(s2, g2, ident(2), 99)) == INVALID
    assert int(w.acknowledge(s2, g2, ident(2), 22)) == OK and w.in_use == 1
    assert int(w.acknowledge(s2, g2, ident(2), 22)) == NOT_FOUND  # stale
    s3, g3 = w.reserve(ident(3), 33)
    assert s3 == s2 and g3 != g2  # reused under a new generation
    with pytest.raises(Exception):
        w.mark_sent(s2, g2)


def test_controller_commit_and_replay():
    log = []
    ctl = RC.Controller([Part("kv", log), Part("sched", log)], final_event_capacity=4)
    res = ctl.run(request(1))
    assert int(res.status) == OK and not res.replayed and res.committed == 2 and res.cancelled == 0
    assert log == [("kv", "prepare", 1), ("sched", "prepare", 1), ("kv", "execute", 1), ("sched", "execute", 1),
                   ("kv", "commit", 1), ("sched", "commit", 1)]
    ev = ctl.peek_final_event()
    assert ev.generation == res.final_event_generation and ev.request_id == 101 and int(ev.status) == OK
    assert ctl.ledger_state(ident(1)) == C.rank_daemon.STATE_COMMITTED
    # an identical replay is answered from the record: no participant runs again
    log.clear()
    again = ctl.run(request(1))
    assert again.replayed and int(again.status) == OK and again.final_event_generation == res.final_event_generation
    assert log == []
    # same identity, another payload: refused
    assert int(ctl.run(request(1, payload=b"other")).status) == DUP
    assert ctl.credits_available(RC.DOMAIN_COMPLETION_OWNERSHIP) == 63
    assert int(ctl.acknowledge_final_event(ident(1), ev.generation, ev.payload_fingerprint)) == OK
    assert ctl.credits_available(RC.DOMAIN_COMPLETION_OWNERSHIP) == 64 and ctl.pending_final_events == 0


def test_controller_prepare_failure_cancels_in_reverse():
    log = []
    ctl = RC.Controller([Part("a", log), Part("b", log, fail_prepare=BUSY), Part("c", log)])
    res = ctl.run(request(2))
    assert int(res.status) == BUSY and res.committed == 0 and res.cancelled == 2
    assert log == [("a", "prepare", 2), ("b", "prepare", 2), ("b", "cancel", BUSY), ("a", "cancel", BUSY)]
    assert ctl.ledger_state(ident(2)) == C.rank_daemon.STATE_CANCELLED
    assert int(ctl.peek_final_event().status) == BUSY


def test_controller_execute_failure_and_throwing_participant():
    log = []
    ctl = RC.Controller([Part("a", log), Part("b", log, fail_execute=INVALID)])
    res = ctl.run(request(3))
    assert int(res.status) == INVALID and res.cancelled == 2
    assert log[-2:] == [("b", "cancel", INVALID), ("a", "cancel", INVALID)]
    assert ctl.ledger_state(ident(3)) == C.rank_daemon.STATE_FAILED

    class Boom(Part):
        def execute(self, r):
            raise RuntimeError("participant crashed")

    ctl2 = RC.Controller([Part("a", log), Boom("b", log)])
    assert int(ctl2.run(request(4)).status) == INTERNAL


def test_controller_bounds_and_validation():
    log = []
    with pytest.raises(Exception):
        RC.Controller([Part("a", log, flags=RC.FLAG_TRANSACTIONAL_STAGING)])  # lacks required guarantees
    with pytest.raises(Exception):
        RC.Controller([Part("a", log), Part("a", log)])  # duplicate names
    with pytest.raises(Exception):
        RC.Controller([])
    ctl = RC.Controller([Part("a", log)], final_event_capacity=1)
    assert int(ctl.run(request(5)).status) == OK
    # the unacknowledged final event holds the only slot: a new transaction waits
    assert int(ctl.run(request(6)).status) == BUSY and ctl.ledger_state(ident(6)) is None
    ev = ctl.peek_final_event()
    ctl.acknowledge_final_event(ident(5), ev.generation, ev.payload_fingerprint)
    assert int(ctl.run(request(6)).status) == OK
    bad = request(7)
    bad.payload = b""
    with pytest.raises(Exception):
        ctl.run(bad)
