"""Host-side expert batching queue (C++), on CPU. Cases follow the behaviour of the
reference's GLM52 expert queue (V/model-families/glm52/src/spark_glm52_expert_queue.c):
configuration validation, threshold and deadline firing, FIFO order, the 1024-row
firing cap, and the sealed-batch mode's seal / drain / unseal cycle."""
import pytest

from sparkpipe_rs_b200.core import StatusError, core

Q = core().expert_queue
LOW, SEALED = Q.Mode.LOW_LATENCY, Q.Mode.SEALED_BATCH
INVALID, CAP, NOT_FOUND, BUSY, UNSUPPORTED = 1, 2, 3, 15, 19


def _q(mode=LOW, layers=2, experts=4, threshold=3, deadline=100):
    return Q.ExpertQueue(Q.Config(layers, experts, threshold, deadline, mode))


@pytest.mark.parametrize("args", [(0, 4, 3, 100, LOW), (9, 4, 3, 100, LOW), (2, 0, 3, 100, LOW),
                                  (2, 257, 3, 100, LOW), (2, 4, 0, 100, LOW), (2, 4, 1025, 100, LOW),
                                  (2, 4, 3, 0, LOW), (2, 4, 3, 100, Q.Mode.INVALID)])
def test_invalid_configurations(args):
    with pytest.raises(StatusError) as e:
        Q.ExpertQueue(Q.Config(*args))
    assert e.value.code == INVALID


def test_threshold_and_deadline_firing_in_fifo_order():
    q = _q()
    q.enqueue(0, 1, 10, 1000)
    q.enqueue(0, 1, 11, 1001)
    assert q.next_firing(1050) is None                  # 2 rows < threshold, deadline not reached
    q.enqueue(1, 3, 30, 1002)
    q.enqueue(0, 1, 12, 1003)
    assert q.next_firing(1050) == (0, 1, [10, 11, 12])  # threshold reached
    assert q.next_firing(1101) is None                  # slot (1,3) is 99 ns old
    assert q.next_firing(1102) == (1, 3, [30])          # deadline
    s = q.stats()
    assert (s.firings, s.fired_rows, s.enqueued) == (2, 4, 0)
    with pytest.raises(StatusError) as e:
        q.enqueue(2, 0, 1, 0)
    assert e.value.code == INVALID


def test_scan_order_and_oldest_arrival_after_partial_firing():
    q = _q(threshold=1)
    q.enqueue(1, 0, 5, 0)
    q.enqueue(0, 3, 6, 0)
    q.enqueue(0, 2, 7, 0)
    assert [q.next_firing(0)[:2] for _ in range(3)] == [(0, 2), (0, 3), (1, 0)]  # layers, then experts
    q.set_firing_threshold(1024)
    for i in range(1000):
        q.enqueue(0, 0, i, 500 + i)
    assert q.next_firing(599) is None                     # below the threshold, oldest row 99 ns old
    assert q.next_firing(600)[2] == list(range(1000))     # deadline: every row, oldest first
    for i in range(1500):
        q.enqueue(0, 0, i, 5000 + i)
    layer, expert, rows = q.next_firing(5000)             # threshold: at most 1024 rows per firing
    assert rows == list(range(1024)) and q.slot_rows(0, 0) == 476
    assert q.next_firing(5000 + 100) is None               # the oldest remaining row arrived at 6024
    assert q.next_firing(6024 + 100)[2] == list(range(1024, 1500))
    with pytest.raises(StatusError):
        q.set_firing_threshold(0)


def test_sealed_batch_mode():
    q = _q(mode=SEALED)
    with pytest.raises(StatusError) as e:
        q.seal(0)
    assert e.value.code == NOT_FOUND
    for i in range(5):
        q.enqueue(0, i % 2, i, 0)
    q.enqueue(1, 3, 99, 0)
    assert q.next_firing(10 ** 12) is None               # nothing fires before the seal
    q.seal(0)
    assert q.sealed(0)
    with pytest.raises(StatusError) as e:
        q.seal(0)
    assert e.value.code == BUSY
    with pytest.raises(StatusError) as e:
        q.enqueue(0, 0, 7, 0)
    assert e.value.code == BUSY
    assert q.next_firing(0) == (0, 0, [0, 2, 4])           # whole slots, regardless of threshold
    assert q.next_firing(0) == (0, 1, [1, 3])
    assert not q.sealed(0) and q.layer_rows(0) == 0        # drained -> unsealed
    assert q.next_firing(0) is None                        # layer 1 is not sealed
    q.enqueue(0, 0, 8, 0)                                  # accepted again
    q.seal(1)
    assert q.next_firing(0) == (1, 3, [99])               # layer 0 holds a row but is not sealed
    assert q.next_firing(0) is None and q.layer_rows(0) == 1


def test_seal_rejects_slots_larger_than_a_firing_and_low_latency_cannot_seal():
    q = _q(mode=SEALED, threshold=1)
    for i in range(1025):
        q.enqueue(0, 0, i, 0)
    with pytest.raises(StatusError) as e:
        q.seal(0)
    assert e.value.code == CAP
    with pytest.raises(StatusError) as e:
        _q().seal(0)
    assert e.value.code == UNSUPPORTED


class _ScanModel:
    """Plain model of the firing rule: scan slots in (layer, expert) order."""

    def __init__(self, layers, experts, threshold, deadline, sealed_mode):
        self.L, self.E, self.t, self.d, self.sm = layers, experts, threshold, deadline, sealed_mode
        self.rows = {}
        self.sealed = [False] * layers

    def enqueue(self, l, e, rid, ts):
        self.rows.setdefault((l, e), []).append((rid, ts))

    def next(self, now):
        for l in range(self.L):
            for e in range(self.E):
                r = self.rows.get((l, e), [])
                if not r:
                    continue
                if self.sm:
                    due = self.sealed[l]
                else:
                    due = len(r) >= self.t or (now >= r[0][1] and now - r[0][1] >= self.d)
                if due:
                    take = len(r) if self.sm else min(len(r), 1024)
                    out, self.rows[(l, e)] = r[:take], r[take:]
                    if self.sm and not any(self.rows.get((l, x)) for x in range(self.E)):
                        self.sealed[l] = False
                    return (l, e, [x[0] for x in out])
        return None


@pytest.mark.parametrize("mode", [LOW, SEALED])
def test_random_operations_match_a_slot_scan(mode):
    import random
    rnd = random.Random(11 if mode == LOW else 12)
    L, E, T, D = 3, 5, 4, 50
    q, m = _q(mode=mode, layers=L, experts=E, threshold=T, deadline=D), _ScanModel(L, E, T, D, mode == SEALED)
    now, rid = 0, 0
    for _ in range(3000):
        op = rnd.random()
        now += rnd.randint(0, 7)
        if op < 0.55:
            l, e = rnd.randrange(L), rnd.randrange(E)
            if mode == SEALED and m.sealed[l]:
                with pytest.raises(StatusError):
                    q.enqueue(l, e, rid, now)
            else:
                q.enqueue(l, e, rid, now)
                m.enqueue(l, e, rid, now)
            rid += 1
        elif op < 0.65 and mode == SEALED:
            l = rnd.randrange(L)
            if not m.sealed[l] and any(m.rows.get((l, x)) for x in range(E)):
                q.seal(l)
                m.sealed[l] = True
        elif op < 0.68 and mode == LOW:
            m.t = rnd.randint(1, 8)
            q.set_firing_threshold(m.t)
        else:
            assert q.next_firing(now) == m.next(now)
    while (f := m.next(10 ** 18)) is not None:
        assert q.next_firing(10 ** 18) == f
