"""KV backing tier and the restore/evict work control (C++), on CPU: fingerprinted
keys, the host-memory store and stage client (explicit enablement, in-flight bound,
completion contract), the pressure-limited restore lookahead, and restore/evict
batches round-tripping real bytes. Behaviour follows the reference's KV-store and
stage-client headers and its Qwen 3.6 work control
(V/model-families/qwen36/src/spark_qwen36_work_control.c)."""
import time

import numpy as np
import pytest

from sparkpipe_rs_b200.core import StatusError, core

K = core().kv_tier
INVALID, CAP, NOT_FOUND, BUSY, PENDING = 1, 2, 3, 15, 18


def _wait(client, bid, timeout=5.0):
    t0 = time.time()
    while time.time() - t0 < timeout:
        r = client.poll(bid)
        if not isinstance(r, int):
            return r
        time.sleep(0.001)
    raise AssertionError("batch did not complete")


def test_keys_bind_every_identity_field():
    a = K.format_key(1, 2, 3, 4, 5)
    assert a.startswith("sp/") and len(a) < K.MAX_KEY_BYTES
    others = [K.format_key(9, 2, 3, 4, 5), K.format_key(1, 9, 3, 4, 5), K.format_key(1, 2, 9, 4, 5),
              K.format_key(1, 2, 3, 9, 5), K.format_key(1, 2, 3, 4, 9), K.format_key(1, 2, 3, 4, K.STATE_BLOCK)]
    assert len({a, *others}) == 7


def test_lookahead_selection():
    assert K.normalize_lookahead(0, 10) == 3 and K.normalize_lookahead(20, 10) == 8
    assert K.normalize_lookahead(5, 2) == 2
    cum = [4, 9, 15, 30]
    assert K.select_lookahead(0, 4, 100, 80, 64, cum) == 3      # 20 free, default lookahead 3: 4, 9, 15 fit
    assert K.select_lookahead(0, 4, 100, 90, 64, cum) == 2      # 10 free: the first two packets (4, 9)
    assert K.select_lookahead(0, 4, 100, 95, 64, cum) == 1      # 5 free: only the first
    assert K.select_lookahead(8, 4, 100, 0, 12, cum) == 2       # staging holds 12 blocks
    assert K.select_lookahead(8, 4, 100, 0, 3, cum) == 0        # not even the first packet fits
    assert K.select_lookahead(8, 2, 1000, 0, 1000, cum) == 2    # bounded by the queue depth


def test_disabled_tier_and_client_bounds():
    off = K.StageKvClient("none", None, 0, 1, 2)
    assert not off.enabled
    with pytest.raises(StatusError) as e:
        off.submit(K.GET, [K.Block(K.GET, "k", 8, 1)], 0)
    assert e.value.code == NOT_FOUND
    with pytest.raises(StatusError):
        K.StageKvClient("", None, 0, 1, 2)
    with pytest.raises(StatusError):
        K.StageKvClient("memory", K.MemoryStore(), 0, 0, 2)    # fingerprints must be non-zero
    store = K.MemoryStore()
    c = K.StageKvClient("memory", store, 0, 1, 2)
    buf = np.zeros(16, np.uint8)
    store.set_paused(True)
    ids = [c.submit(K.PUT, [K.Block(K.PUT, f"k{i}", buf.ctypes.data, 16)], 0) for i in range(K.MAX_INFLIGHT_BATCHES)]
    with pytest.raises(StatusError) as e:
        c.submit(K.PUT, [K.Block(K.PUT, "x", buf.ctypes.data, 16)], 0)
    assert e.value.code == BUSY
    assert c.poll(ids[0]) == PENDING
    store.set_paused(False)
    for i in ids:
        assert _wait(c, i).status == 0
    assert c.inflight == 0 and store.stored_blocks() == K.MAX_INFLIGHT_BATCHES
    with pytest.raises(StatusError):
        c.submit(K.GET, [K.Block(K.PUT, "k0", buf.ctypes.data, 16)], 0)   # block op differs from the batch op
    bid = c.submit(K.GET, [K.Block(K.GET, "never-stored", buf.ctypes.data, 16)], 0)
    assert _wait(c, bid).status == NOT_FOUND                                # outcome travels in the completion


def _plan(**kw):
    p = K.PlanConfig()
    p.model_fp, p.layout_fp, p.rank, p.block_bytes, p.state_bytes = 0xA1, 0xB2, 3, 64, 160
    p.lookahead, p.physical_capacity, p.allocated, p.staging_capacity = 0, 64, 40, 16
    for k, v in kw.items():
        setattr(p, k, v)
    return p


def _mover(client, plan, block_records=8, state_records=2, batch=16):
    bstage = np.zeros((max(block_records, 1), plan.block_bytes), np.uint8)
    sstage = np.zeros((max(state_records, 1), plan.state_bytes), np.uint8)
    m = K.TierMover(plan, client, bstage.ctypes.data, block_records, sstage.ctypes.data, state_records, batch)
    return m, bstage, sstage


def test_cumulative_counts_and_restore_selection():
    eq = K.state_block_equivalents(160, 64)
    assert eq == 3 and K.state_block_equivalents(0, 64) == 0
    lanes = [K.PendingLane(7, [0, 1], True), K.PendingLane(8, [4]), K.PendingLane(9, [2, 3, 5], True)]
    cum = K.cumulative_nonresident(lanes, [2, 1], eq)
    assert cum == [2 + 3 + 1, 6 + 3 + 3]
    plan = _plan()
    c = K.StageKvClient("memory", K.MemoryStore(), plan.rank, plan.model_fp, plan.layout_fp)
    m, _, _ = _mover(c, plan)
    assert m.restore_packets(cum) == 2                            # room min(24 free, 16 staging): 6 and 12 fit
    m.set_pressure(64, 40, 8)
    assert m.restore_packets(cum) == 1
    for bad in ([2, 2], [0, 3], [4]):
        with pytest.raises(StatusError):
            K.cumulative_nonresident(lanes, bad, eq)


def _wait_landed(m, d):
    t0 = time.time()
    while m.channel(d).stage != K.LANDED and time.time() - t0 < 5:
        m.poll()
    return m.channel(d)


def test_evict_then_restore_round_trips_bytes():
    plan = _plan()
    store = K.MemoryStore()
    c = K.StageKvClient("memory", store, plan.rank, plan.model_fp, plan.layout_fp)
    RESTORE, EVICT = K.Direction.RESTORE, K.Direction.EVICT
    rng = np.random.default_rng(0)
    kv = {7: rng.integers(0, 255, (3, 64), dtype=np.uint8), 9: rng.integers(0, 255, (2, 64), dtype=np.uint8)}
    st = {7: rng.integers(0, 255, 160, dtype=np.uint8), 9: rng.integers(0, 255, 160, dtype=np.uint8)}
    m, bstage, sstage = _mover(c, plan)
    for seq in (7, 9):
        blocks = m.plan_evict(seq, list(range(kv[seq].shape[0])), True, kv[seq].ctypes.data, st[seq].ctypes.data)
        assert blocks[0].key.endswith("/state") and [b.op for b in blocks] == [K.PUT] * len(blocks)
        m.start(EVICT, blocks, 0)
        with pytest.raises(StatusError):
            m.start(EVICT, blocks, 0)                               # one batch per channel
        assert _wait_landed(m, EVICT).outcome == 0
        assert m.collect(EVICT) == 0
        assert m.channel(EVICT).stage == K.FREE
    with pytest.raises(StatusError):
        m.collect(EVICT)
    # restore both sequences into staging, lane by lane
    lanes = [K.PendingLane(7, [0, 1, 2], True), K.PendingLane(9, [0, 1], True)]
    rb = m.plan_restore(lanes, [1, 1])
    assert (rb.lanes_built, rb.block_records, rb.state_records, len(rb.blocks)) == (2, 5, 2, 7)
    assert rb.blocks[0].key.endswith("/state") and rb.blocks[4].key.endswith("/state")   # state record first
    m.start(RESTORE, rb.blocks, 1)
    assert _wait_landed(m, RESTORE).outcome == 0
    assert np.array_equal(bstage[:3], kv[7]) and np.array_equal(bstage[3:5], kv[9])
    assert np.array_equal(sstage[0], st[7]) and np.array_equal(sstage[1], st[9])
    assert m.collect(RESTORE) == 0
    # a lane that does not fit ends the batch; the first lane must fit
    m4, _, _ = _mover(c, plan, block_records=4)
    rb = m4.plan_restore(lanes, [1, 1])
    assert rb.lanes_built == 1 and rb.block_records == 3
    m1, _, _ = _mover(c, plan, state_records=1)
    assert m1.plan_restore(lanes, [1, 1]).lanes_built == 1              # one state record of staging
    mb, _, _ = _mover(c, plan, batch=5)
    assert mb.plan_restore(lanes, [1, 1]).lanes_built == 1              # 4 + 3 records > 5
    m2, _, _ = _mover(c, plan, block_records=2)
    with pytest.raises(StatusError) as e:
        m2.plan_restore(lanes, [1, 1])
    assert e.value.code == CAP
    with pytest.raises(StatusError):
        m.plan_evict(7, [], False, bstage.ctypes.data, sstage.ctypes.data)
    with pytest.raises(StatusError) as e:
        m.plan_evict(7, list(range(20)), False, bstage.ctypes.data, sstage.ctypes.data)
    assert e.value.code == CAP


def test_restore_prefix_matches_lane_by_lane_rule():
    """The binary search over prefix sums picks the same lanes as adding lanes one at a
    time until the first one that would overflow a resource."""
    plan = _plan()
    c = K.StageKvClient("memory", K.MemoryStore(), plan.rank, plan.model_fp, plan.layout_fp)
    rng = np.random.default_rng(5)
    for trial in range(200):
        n = int(rng.integers(1, 7))
        spec = [(list(range(int(rng.integers(0, 5)))), bool(rng.integers(0, 2))) for _ in range(n)]
        spec = [(b, st) if (b or st) else ([0], st) for b, st in spec]
        lanes = [K.PendingLane(i + 1, b, st) for i, (b, st) in enumerate(spec)]
        br, sr, batch = int(rng.integers(1, 12)), int(rng.integers(1, 4)), int(rng.integers(1, 14))
        m, _, _ = _mover(c, plan, block_records=br, state_records=sr, batch=batch)
        taken, recs, blks, sts = 0, 0, 0, 0
        for b, st in spec:
            s = 1 if st else 0
            if recs + len(b) + s > batch or blks + len(b) > br or sts + s > sr:
                break
            recs, blks, sts, taken = recs + len(b) + s, blks + len(b), sts + s, taken + 1
        if taken == 0:
            with pytest.raises(StatusError):
                m.plan_restore(lanes, [1] * n)
        else:
            rb = m.plan_restore(lanes, [1] * n)
            assert (rb.lanes_built, rb.block_records, rb.state_records) == (taken, blks, sts)
