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


def test_cumulative_counts_and_restore_selection():
    eq = K.state_block_equivalents(160, 64)
    assert eq == 3 and K.state_block_equivalents(0, 64) == 0
    lanes = [K.PendingLane(7, [0, 1], True), K.PendingLane(8, [4]), K.PendingLane(9, [2, 3, 5], True)]
    cum = K.cumulative_nonresident(lanes, [2, 1], eq)
    assert cum == [2 + 3 + 1, 6 + 3 + 3]
    assert K.select_restore_packets(_plan(), cum) == 2          # room min(24 free, 16 staging): 6 and 12 fit
    assert K.select_restore_packets(_plan(staging_capacity=8), cum) == 1
    for bad in ([2, 2], [0, 3], [4]):
        with pytest.raises(StatusError):
            K.cumulative_nonresident(lanes, bad, eq)


def test_evict_then_restore_round_trips_bytes():
    plan = _plan()
    store = K.MemoryStore()
    c = K.StageKvClient("memory", store, plan.rank, plan.model_fp, plan.layout_fp)
    rng = np.random.default_rng(0)
    kv = {7: rng.integers(0, 255, (3, 64), dtype=np.uint8), 9: rng.integers(0, 255, (2, 64), dtype=np.uint8)}
    st = {7: rng.integers(0, 255, 160, dtype=np.uint8), 9: rng.integers(0, 255, 160, dtype=np.uint8)}
    restore, evict = K.BatchState(), K.BatchState()
    for seq in (7, 9):
        blocks = K.build_evict_batch(plan, seq, list(range(kv[seq].shape[0])), True, kv[seq].ctypes.data,
                                     st[seq].ctypes.data, 16)
        assert blocks[0].key.endswith("/state") and [b.op for b in blocks] == [K.PUT] * len(blocks)
        K.submit_batch(c, evict, K.PUT, blocks, 0)
        with pytest.raises(StatusError):
            K.submit_batch(c, evict, K.PUT, blocks, 0)          # one outstanding batch per kind
        t0 = time.time()
        while evict.phase != K.READY and time.time() - t0 < 5:
            K.progress(c, restore, evict)
        assert evict.status == 0
        K.acknowledge(evict)
    with pytest.raises(StatusError):
        K.acknowledge(evict)
    # restore both sequences into staging, lane by lane
    bstage = np.zeros((8, 64), np.uint8)
    sstage = np.zeros((2, 160), np.uint8)
    lanes = [K.PendingLane(7, [0, 1, 2], True), K.PendingLane(9, [0, 1], True)]
    rb = K.build_restore_batch(plan, lanes, [1, 1], bstage.ctypes.data, 8, sstage.ctypes.data, 2, 16)
    assert (rb.lanes_built, rb.block_records, rb.state_records, len(rb.blocks)) == (2, 5, 2, 7)
    K.submit_batch(c, restore, K.GET, rb.blocks, 1)
    t0 = time.time()
    while restore.phase != K.READY and time.time() - t0 < 5:
        K.progress(c, restore, evict)
    assert restore.status == 0
    assert np.array_equal(bstage[:3], kv[7]) and np.array_equal(bstage[3:5], kv[9])
    assert np.array_equal(sstage[0], st[7]) and np.array_equal(sstage[1], st[9])
    K.acknowledge(restore)
    # a lane that does not fit ends the batch; the first lane must fit
    rb = K.build_restore_batch(plan, lanes, [1, 1], bstage.ctypes.data, 4, sstage.ctypes.data, 2, 16)
    assert rb.lanes_built == 1 and rb.block_records == 3
    with pytest.raises(StatusError) as e:
        K.build_restore_batch(plan, lanes, [1, 1], bstage.ctypes.data, 2, sstage.ctypes.data, 2, 16)
    assert e.value.code == CAP
    with pytest.raises(StatusError):
        K.build_evict_batch(plan, 7, [], False, bstage.ctypes.data, sstage.ctypes.data, 16)
    with pytest.raises(StatusError) as e:
        K.build_evict_batch(plan, 7, list(range(20)), False, bstage.ctypes.data, sstage.ctypes.data, 16)
    assert e.value.code == CAP
