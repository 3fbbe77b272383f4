"""Stage planner, long-context policy and topology switch (C++), on CPU.

Scenarios follow crates/spark-sched/tests/{stage_plan,long_context,topology_switch}.rs."""
import itertools
import random

import pytest

from sparkpipe_rs_b200.core import StatusError, core

C = core()
SP, LC, TS = C.stage_plan, C.long_context, C.topology_switch
G78 = SP.Geometry(78, 3)


# ------------------------------------------------------------------ stage plan
def test_valid_ring_and_table_builder():
    p = SP.StagePlan()
    p.stages = [SP.Stage(6 * i, 6, SP.FLAG_INPUT_HIDDEN | SP.FLAG_OUTPUT_HIDDEN) for i in range(13)]
    p.stages[0].flags |= SP.FLAG_DENSE_PREFIX
    p.stages[12].flags = SP.FLAG_INPUT_HIDDEN | SP.FLAG_FINAL_TOKEN
    SP.validate(G78, p)
    counts = [6, 7, 7, 7, 7, 7, 7, 6, 6, 6, 6, 6]
    t = SP.build_from_layer_counts(G78, counts)
    assert t.stage_count == 12 and t.stages[1].first_layer == 6 and t.stages[11].first_layer == 72
    assert t.stages[11].flags & SP.FLAG_FINAL_TOKEN and t.stages[0].flags & SP.FLAG_DENSE_PREFIX
    with pytest.raises(StatusError):
        SP.build_from_layer_counts(G78, counts[:-1] + [5])  # does not cover all layers
    with pytest.raises(StatusError):
        SP.build_from_layer_counts(G78, [2, 76])  # splits the dense prefix
    with pytest.raises(StatusError):
        SP.build_from_layer_counts(G78, [39, 39])  # 36 routed layers > 8 per stage


def test_serialize_roundtrip():
    p = SP.build_uniform(G78, 13)
    b = p.serialize()
    assert len(b) == SP.DESCRIPTOR_BYTES == 16 + 13 * 16
    q = SP.StagePlan.deserialize(b)
    assert q.layer_counts() == p.layer_counts()
    with pytest.raises(StatusError):
        SP.StagePlan.deserialize(b"\0" * len(b))


def _brute_force(g, cost, extra, stages):
    best = None
    L = g.layer_count
    for cuts in itertools.combinations(range(1, L), stages - 1):
        bounds = (0,) + cuts + (L,)
        if not all(SP.range_is_valid(g, a, b - a) for a, b in zip(bounds, bounds[1:])):
            continue
        worst = max(sum(cost[a:b]) + (extra if b == L else 0) for a, b in zip(bounds, bounds[1:]))
        best = worst if best is None else min(best, worst)
    return best


def test_balanced_dp_is_optimal_against_brute_force():
    rng = random.Random(0)
    for trial in range(30):
        L = rng.randint(4, 12)
        g = SP.Geometry(L, rng.randint(0, 2), rng.randint(2, 8))
        cost = [rng.randint(1, 100) for _ in range(L)]
        extra = rng.choice([0, 50])
        stages = rng.randint(1, min(4, L))
        ref = _brute_force(g, cost, extra, stages)
        if ref is None:
            with pytest.raises(StatusError):
                SP.build_balanced(g, cost, extra, stages)
            continue
        p = SP.build_balanced(g, cost, extra, stages)
        assert SP.max_stage_cost(p, cost, extra) == ref


def test_balanced_78_layers_and_final_extra():
    cost = [1000 + i for i in range(78)]
    p = SP.build_balanced(G78, cost, 0, 13)
    assert p.stage_count == 13 and p.total_layers() == 78
    q = SP.build_balanced(G78, cost, 20000, 13)
    assert q.stages[12].layer_count < p.stages[12].layer_count  # the head stage sheds layers


def test_planner_caches_per_bucket_and_scales_profiles():
    g = SP.Geometry(27, 1, 27)
    pl = SP.StagePlanner(g)
    a = pl.plan(64, 2)
    b = pl.plan(64, 2)
    assert a.layer_counts() == b.layer_counts() and pl.plan_builds == 1 and pl.plan_hits == 1
    assert not pl.profile(64).measured
    cost = [100] + [400] * 26
    pl.record_profile(64, cost, 2000)
    assert pl.profile(64).measured and pl.profile(64).layer_cost_ns == cost
    assert pl.profile(128).layer_cost_ns[1] == 800 and pl.profile(128).final_extra_ns == 4000
    assert pl.profile(32).layer_cost_ns[1] == 200
    c = pl.plan(64, 2)
    assert pl.plan_builds == 2  # profile change dropped the cache
    assert SP.max_stage_cost(c, cost, 2000) == min(
        max(sum(cost[:k]), sum(cost[k:]) + 2000) for k in range(1, 27))


# ------------------------------------------------------------------ long context
def _policy():
    return LC.Policy(1 << 20, 2048)


def test_bounded_selection_for_256k():
    d, sel = _policy().decode_selection(262144, 2048)
    assert d.flags & LC.PLAN_BOUNDED and d.flags & LC.PLAN_LONG_CONTEXT and d.flags & LC.PLAN_TRUNCATED
    assert d.selected == 2048 and d.selected_blocks < d.context_blocks
    assert d.avoided_reads > 250000
    assert sel[0] == 0 and 262143 in sel and all(t < 262144 for t in sel)
    assert len(set(sel)) == len(sel)
    assert d.sink == 128 and d.recent == 1536 and d.strided == 384
    assert sel[:128] == list(range(128)) and sel[-1536:] == list(range(262144 - 1536, 262144))
    mid = sel[128:128 + 384]
    assert mid == sorted(mid) and mid[0] > 127 and mid[-1] < 262144 - 1536


def test_prefill_plan_and_full_scan_rules():
    p = _policy().prefill_plan(262144, 256)
    assert p.flags & LC.PREFILL_CHUNKED and p.flags & LC.PREFILL_LONG_CONTEXT
    assert p.chunks == 1024 and p.prompt_blocks == 16384 and p.visits == 262144
    p = _policy().prefill_plan(1000, 300)
    assert p.chunks == 4 and p.final_chunk_tokens == 100
    pol = _policy()
    pol.mode = LC.Mode.FULL_SCAN
    pol.flags &= ~LC.REQUIRE_BOUNDED
    with pytest.raises(StatusError) as e:
        pol.decode_selection(262144, 2048)
    assert e.value.code == 1
    pol.flags |= LC.ALLOW_FULL_SCAN
    with pytest.raises(StatusError) as e:
        pol.decode_selection(262144, 2048)
    assert e.value.code == 2
    d, sel = pol.decode_selection(100, 128)
    assert d.flags & LC.PLAN_FULL_SCAN and d.flags & LC.PLAN_PADDED and sel[99] == 99 and sel[100] == LC.INVALID_TOKEN


def test_lane_batch():
    plans, out = _policy().lane_batch([512, 262144], 2048, 2048)
    assert plans[0].selected == 512 and not plans[0].flags & LC.PLAN_TRUNCATED
    assert out[511] == 511 and out[512] == LC.INVALID_TOKEN
    assert plans[1].selected == 2048 and 262143 in out[2048:]
    with pytest.raises(StatusError):
        _policy().decode_selection(2_000_000, 2048)  # over the context limit


# ------------------------------------------------------------------ topology switch
class MockTier(TS.Tier):
    def __init__(self, present):
        super().__init__()
        self.present = set(present)
        self.pins = {}
        self.records = {}
        self.planned = []
        self.next_off = 4096
        self.busy_reserves = 0

    def pin(self, key, pinned):
        if key not in self.present:
            return C.Status.NOT_FOUND
        self.pins[key] = self.pins.get(key, 0) + (1 if pinned else -1)
        return C.Status.OK

    def offset_of(self, key):
        return 1 if key in self.present else None

    def reserve_write(self, key):
        if self.busy_reserves:
            self.busy_reserves -= 1
            return (_st("Busy"), 0, False)
        off = self.next_off
        self.next_off += 4096
        return (_st("Ok"), off, key in self.records)

    def commit_write(self, r):
        return _st("Ok")

    def abort_write(self, r):
        pass

    def plan_lookahead(self, needs, step):
        self.planned += [n.key for n in needs]
        return _st("Ok")


def _st(name):
    return getattr(C.Status, {"Ok": "OK", "Busy": "BUSY"}[name])


class MockSwap(TS.SwapDevice):
    def __init__(self, polls_busy=1):
        super().__init__()
        self.begun = []
        self.polls_busy = polls_busy

    def begin_swap(self, a, b):
        self.begun.append((a.recipe_id, b.recipe_id))
        return _st("Ok")

    def poll_swap(self):
        if self.polls_busy:
            self.polls_busy -= 1
            return _st("Busy")
        return _st("Ok")


class MockWriter(TS.ManifestWriter):
    def __init__(self):
        super().__init__()
        self.blocks = []

    def write_block(self, off, payload):
        self.blocks.append((off, payload))
        return _st("Ok")


def _cfg():
    c = TS.Config()
    c.kv_namespace = 0xABCDEF
    c.max_sequences, c.max_blocks_per_sequence, c.step_time_us = 8, 16, 20000
    c.manifest_block_bytes = 4096
    c.read_bytes_per_s, c.write_bytes_per_s, c.swap_fixed_us = 10 ** 10, 5 * 10 ** 9, 1_000_000
    c.initial = TS.Recipe(11, 10 ** 10, TS.Strategy.TENSOR_PARALLEL)
    return c


def test_switch_warm_and_recompute():
    ns = 0xABCDEF
    warm_hashes = [101, 102, 103]
    cold_hashes = [201, 202]
    tier = MockTier([TS.kv_key(ns, h) for h in warm_hashes + [201]])  # block 202 was never written back
    swap, writer = MockSwap(), MockWriter()
    sw = TS.TopologySwitch(_cfg(), tier, swap, writer)
    sw.track_sequence(1, 11)
    sw.track_sequence(2, 11)
    sw.track_sequence(3, 11)
    sw.set_sequence_kv(1, 150, warm_hashes)
    sw.set_sequence_kv(2, 100, cold_hashes)
    with pytest.raises(StatusError):
        sw.begin(TS.Recipe(11))  # the running recipe
    sw.begin(TS.Recipe(22, 10 ** 10, TS.Strategy.PIPELINE_PARALLEL))
    assert not sw.admissions_open
    with pytest.raises(StatusError):
        sw.track_sequence(9, 11)
    assert sw.advance(0) == TS.State.QUIESCE  # sequences still mid-step
    sw.sequence_at_boundary(1)
    sw.sequence_at_boundary(2)
    sw.sequence_complete(3)  # finished during the drain: not checkpointed
    assert sw.advance(1) == TS.State.SWAP  # checkpointed, swap polled busy once
    with pytest.raises(StatusError):
        sw.set_sequence_kv(1, 151, warm_hashes)  # frozen by the checkpoint
    assert len(writer.blocks) == 2
    off, rec = writer.blocks[0]
    assert int.from_bytes(rec[0:8], "little") == 1 and int.from_bytes(rec[8:16], "little") == 11
    assert int.from_bytes(rec[16:20], "little") == 150 and int.from_bytes(rec[20:24], "little") == 3
    assert int.from_bytes(rec[24:32], "little") == TS.kv_key(ns, 101)
    assert sw.advance(2) == TS.State.STEADY
    assert sw.current_recipe.recipe_id == 22 and sw.admissions_open
    assert sw.resume_class_of(1) == TS.ResumeClass.WARM
    assert sw.resume_class_of(2) == TS.ResumeClass.RECOMPUTE
    st = sw.stats
    assert (st.switches_completed, st.sequences_checkpointed, st.resumed_warm, st.resumed_recompute) == (1, 2, 1, 1)
    assert st.completed_mid_switch == 1 and st.tier_blocks_found == 4 and st.tier_blocks_absent == 1
    assert sorted(tier.planned) == sorted(TS.kv_key(ns, h) for h in warm_hashes)
    assert all(v == 0 for v in tier.pins.values())  # every pin released at resume
    assert swap.begun == [(11, 22)]


def test_switch_retries_busy_checkpoint():
    tier, swap, writer = MockTier([]), MockSwap(0), MockWriter()
    tier.busy_reserves = 2
    sw = TS.TopologySwitch(_cfg(), tier, swap, writer)
    sw.track_sequence(5, 11)
    sw.sequence_at_boundary(5)
    sw.begin(TS.Recipe(33))
    assert sw.advance(0) == TS.State.CHECKPOINT and sw.last_error != 0
    assert sw.advance(1) == TS.State.CHECKPOINT
    assert sw.advance(2) == TS.State.STEADY and sw.last_error == 0
    assert sw.resume_class_of(5) == TS.ResumeClass.RECOMPUTE  # no blocks: nothing to warm


def test_budget_and_keys():
    c = _cfg()
    b = TS.estimate_budget(c, TS.Recipe(22, 2 * 10 ** 10), 100, 10 ** 9)
    assert b.quiesce_us == 20000 and b.checkpoint_us == 100 * 4096 * 10 ** 6 // (5 * 10 ** 9)
    assert b.swap_stream_us == 2_000_000 and b.resume_warm_us == 100_000
    assert b.total_us == b.quiesce_us + b.checkpoint_us + b.swap_fixed_us + b.swap_stream_us
    k = TS.kv_key(1, 2)
    assert k & 1 and k != TS.kv_key(3, 2) and TS.manifest_key(1, 7) != TS.kv_key(1, 7)
    with pytest.raises(StatusError):
        bad = _cfg()
        bad.manifest_block_bytes = 64  # cannot hold 16 keys
        TS.TopologySwitch(bad, MockTier([]), MockSwap(), MockWriter())
