"""Drive-backed just-in-time KV tier: schedule logic against a device that lands a
read after a programmed number of polls, and a real file device."""
import os

import pytest

from sparkpipe_rs_b200 import _ext

BLOCK = 8192


def _nt():
    return _ext.core().nvme_tier


def _tier(nt, slots=16, staging=4, reserve=1, latency=2, step_us=1000, bw=8192 * 1000):
    cfg = nt.Config()
    cfg.budget_bytes = slots * BLOCK
    cfg.block_bytes = BLOCK
    cfg.staging_buffers = staging
    cfg.demand_reserve = reserve
    cfg.device_bytes_per_second = bw   # one block per millisecond
    cfg.step_microseconds = step_us    # one millisecond per step: one step per block
    dev = nt.MockDevice(slots * BLOCK, latency)
    return nt.Tier(cfg, dev), dev


def _put(nt, tier, dev, h, fill):
    r = tier.reserve_write(h)
    assert not r.already_present
    assert dev.write(r.offset, bytes([fill]) * BLOCK) == _ext.core().Status.OK
    tier.commit_write(r)
    return r


def test_write_plan_pump_and_consume():
    nt = _nt()
    tier, dev = _tier(nt)
    assert tier.transfer_steps == 1
    for h in range(1, 4):
        _put(nt, tier, dev, h, h)
    assert tier.offset_of(2) is not None and tier.offset_of(99) is None
    rep = tier.plan_lookahead([nt.Need(1, 5), nt.Need(2, 3), nt.Need(3, 9), nt.Need(42, 4)], 0)
    assert (rep.queued, rep.absent, rep.late_risk) == (3, 1, 0)
    # prefetch may use 3 of the 4 staging buffers (one is kept for demand)
    tier.pump(0)
    assert tier.stats.prefetch_issues == 3 and tier.inflight() == 3
    for step in range(1, 4):
        tier.pump(step)
    st = tier.stats
    assert st.prefetch_landings == 3 and st.prefetch_late == 0 and tier.inflight() == 0
    state, data, addr = tier.request_demand(2, 3)
    assert state == nt.Demand.READY and data == bytes([2]) * BLOCK and addr != 0
    assert tier.consume(2) and not tier.consume(2)
    # the on-drive copy stays: a later demand reads it again
    state, _, _ = tier.request_demand(2, 4)
    assert state == nt.Demand.STARTED
    state, _, _ = tier.request_demand(2, 4)
    assert state == nt.Demand.IN_FLIGHT
    for step in range(5, 8):
        tier.pump(step)
    state, data, _ = tier.request_demand(2, 8)
    assert state == nt.Demand.READY and data == bytes([2]) * BLOCK
    assert tier.request_demand(77, 8)[0] == nt.Demand.MISS
    st = tier.stats
    assert (st.demand_hits, st.demand_loads, st.demand_joins, st.demand_misses) == (2, 1, 1, 1)
    assert st.read_bytes == 4 * BLOCK


def test_clock_eviction_generation_and_pins():
    nt = _nt()
    tier, dev = _tier(nt, slots=4, latency=3)
    for h in range(1, 5):
        _put(nt, tier, dev, h, h)
    assert tier.pin(1, True)
    # a read of block 2 is in flight when its slot is evicted: the landing is stale
    assert tier.request_demand(2, 0)[0] == nt.Demand.STARTED
    r = tier.reserve_write(5)  # full: the clock clears reference bits, skips the pinned slot
    assert tier.stats.evictions == 1 and tier.stats.pinned_skips >= 1
    assert tier.offset_of(1) is not None  # pinned survives
    evicted = [h for h in (2, 3, 4) if tier.offset_of(h) is None]
    assert len(evicted) == 1
    tier.abort_write(r)
    assert tier.stats.write_aborts == 1
    for step in range(1, 6):
        tier.pump(step)
    if evicted[0] == 2:
        assert tier.stats.stale_completions == 1
    # writing an existing block again is a no-op reservation
    assert tier.reserve_write(3 if evicted[0] != 3 else 4).already_present


def test_demand_preempts_prefetch_and_residency():
    nt = _nt()
    tier, dev = _tier(nt, slots=16, staging=2, reserve=0, latency=50)
    for h in range(1, 6):
        _put(nt, tier, dev, h, h)
    tier.plan_lookahead([nt.Need(1, 10), nt.Need(2, 11), nt.Need(3, 12)], 0)
    tier.pump(0)
    assert tier.inflight() == 2
    res = tier.will_be_resident_by([1, 2, 3, 4, 99], 0, 1)
    assert res.inflight_on_time == 2 and res.planned_on_time == 2 and res.absent == 1
    assert res.confidence == nt.Confidence.PARTIAL
    assert tier.will_be_resident_by([1, 2], 0, 1).confidence == nt.Confidence.ALL
    assert tier.will_be_resident_by([99], 0, 1).confidence == nt.Confidence.NONE
    # a demand for block 5 takes an in-flight prefetch's buffer
    assert tier.request_demand(5, 1)[0] == nt.Demand.STARTED
    assert tier.stats.prefetch_preemptions == 1
    for step in range(2, 60):
        tier.pump(step)
    assert tier.request_demand(5, 60)[0] == nt.Demand.READY


def test_io_error_is_counted_and_recovered():
    nt = _nt()
    tier, dev = _tier(nt, latency=0)
    _put(nt, tier, dev, 9, 9)
    dev.fail_next_read()
    assert tier.request_demand(9, 0)[0] == nt.Demand.STARTED
    tier.pump(1)
    assert tier.stats.io_errors == 1 and tier.inflight() == 0
    assert tier.request_demand(9, 2)[0] == nt.Demand.STARTED
    tier.pump(3)
    assert tier.request_demand(9, 3)[0] == nt.Demand.READY


def test_invalid_configurations_rejected():
    nt = _nt()
    cfg = nt.Config()
    cfg.block_bytes = 1000  # not a 4096 multiple
    with pytest.raises(Exception):
        nt.Tier(cfg, nt.MockDevice(1 << 20, 0))
    cfg.block_bytes = BLOCK
    cfg.budget_bytes = 1 << 20
    cfg.staging_buffers = 1
    with pytest.raises(Exception):
        nt.Tier(cfg, nt.MockDevice(1 << 20, 0))


def test_file_device_round_trip(tmp_path):
    nt = _nt()
    path = str(tmp_path / "kv.bin")
    cfg = nt.Config()
    cfg.budget_bytes = 32 * BLOCK
    cfg.block_bytes = BLOCK
    dev = nt.FileDevice(path, 32 * BLOCK, 2)
    tier = nt.Tier(cfg, dev)
    payload = {h: os.urandom(BLOCK) for h in (11, 12, 13)}
    for h, b in payload.items():
        r = tier.reserve_write(h)
        assert dev.write(r.offset, b) == _ext.core().Status.OK
        tier.commit_write(r)
    tier.plan_lookahead([nt.Need(h, 1) for h in payload], 0)
    got = {}
    for step in range(2000):
        tier.pump(step)
        for h in payload:
            if h in got:
                continue
            state, data, _ = tier.request_demand(h, step)
            if state == nt.Demand.READY:
                got[h] = data
                tier.consume(h)
        if len(got) == len(payload):
            break
    assert got == payload
    assert tier.drain(1000) == 0
