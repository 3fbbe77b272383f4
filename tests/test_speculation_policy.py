"""Speculative-decode policy of the scheduler, on CPU.

* row allocator: the cases of the reference's crates/spark-core/tests/row_allocator.rs
* lane EMA, suppression and reprobe (request_api/speculation.rs:583-690)
* the MTP tree resolution scenario of the reference's `mtp_tree_resolves_every_path`
  (crates/spark-serve/tests/request_api.rs:2440-2520)
* verify plans: tree rows (shadow slots for the alternate leaves, draft-sync rows),
  chain rows with per-lane budgets, completion with variable committed tokens, stop
  tokens inside a round, the utility gate on measured step costs
"""
import numpy as np
import pytest

from sparkpipe_rs_b200.core import StatusError, core

C = core()
S = C.speculation
MT = C.work_control.mtp_tree


# ------------------------------------------------------------------ row allocator
def _assign(lanes, cap, cost=1000):
    return S.row_allocator_assign(lanes, cap, cost)


def test_row_allocator_reference_cases():
    assert _assign([(2900, 5, 0)] * 8, 8) == (8, [0] * 8)                          # saturated: all real
    assert _assign([(2900, 5, 0), (1300, 5, 0)], 8) == (8, [5, 1])                  # fills by alpha
    assert _assign([(900, 0, 0), (2900, 5, 0)], 16) == (7, [0, 5])                  # suppressed stays plain
    assert _assign([(1000, 5, 1), (2900, 5, 0)], 16) == (9, [2, 5])                 # probe grant first
    assert _assign([(1000, 5, 1), (2900, 5, 0)], 3) == (3, [1, 0])                  # probe is capacity-bounded
    assert _assign([(1000, 5, 0)], 16) == (1, [0])                                  # no value, no drafts
    for _ in range(4):
        assert _assign([(2000, 5, 0)] * 3, 5) == (5, [1, 1, 0])                     # ties to the lower lane
    assert _assign([(2900, 5, 0)] * 4, 2) == (2, [0] * 4)                           # overflow clamps
    assert _assign([(2900, 5, 0), (1300, 5, 0)], 8, 600) == (8, [5, 1])             # cost weighted
    assert _assign([(2900, 5, 0), (1300, 5, 0)], 2, 600) == (2, [0, 0])
    assert _assign([(2900, 5, 0)] * 2, 0)[0] == 0
    assert S.alpha_milli(2900) == 655 and S.alpha_milli(1300) == 230 and S.alpha_milli(1000) == 0


# ------------------------------------------------------------------ lane EMA
def test_commit_ema_suppression_and_reprobe():
    # three one-token rounds: 2900 -> 2425 -> 2069 -> 1802 (int32 division truncates toward zero)
    tr = S.observe(2900, 5, 0, [("v", 1)] * 3, 5)
    assert [t[0] for t in tr] == [2425, 2069, 1802] and all(t[1] == 5 for t in tr)
    tr = S.observe(2900, 5, 0, [("v", 1)] * 9, 5)
    emas = [t[0] for t in tr]
    first = next(i for i, e in enumerate(emas) if e < S.SUPPRESS_MILLI)
    assert first == 8 and emas[7:] == [1192, 1144]
    assert tr[first][1:] == (0, S.REPROBE_INTERVAL)        # suppressed: budget 0, countdown 16
    # plain decode runs the countdown down by committed tokens, then the lane probes again
    tr = S.observe(1100, 0, 16, [("p", 1)] * 15 + [("p", 1)], 5)
    assert tr[14][1:] == (0, 1) and tr[15][1:] == (5, 0)
    tr = S.observe(1100, 0, 16, [("p", 20)], 5)
    assert tr[0][1:] == (5, 0)
    # a four-token round pulls the EMA up: 1100 + (4000 - 1100) / 4 = 1825
    assert S.observe(1100, 5, 0, [("v", 4)], 5)[0] == (1825, 5, 0)
    # utility: E x plain > 1.25 x round
    assert S.outranks_plain(2000, 8, 8, 1000, 1599) and not S.outranks_plain(2000, 8, 8, 1000, 1600)


# ------------------------------------------------------------------ MTP tree scenario
DEPTH1_PRIMARY, DEPTH2_PRIMARY, DEPTH2_ALTERNATE, DEPTH3_PRIMARY, DEPTH3_ALTERNATE = 0, 1, 2, 3, 4
INPUT_ROW, DEPTH1_ROW, DEPTH2_PRIMARY_ROW = 0, 1, 2
RES_DEPTH1, RES_DEPTH2_PRIMARY, RES_DEPTH2_ALTERNATE, RES_DEPTH3_PRIMARY = 1, 2, 3, 4
OUTPUT_VOCAB = 154_880


def _candidates(seed):
    return [seed + i for i in range(5)]


def _verifier(cand, path, seed):
    v = [seed + 100 + r for r in range(6)]
    if path == 0:
        return v
    v[INPUT_ROW] = cand[DEPTH1_PRIMARY]
    if path == RES_DEPTH1:
        return v
    if path == RES_DEPTH2_ALTERNATE:
        v[DEPTH1_ROW] = cand[DEPTH2_ALTERNATE]
        return v
    v[DEPTH1_ROW] = cand[DEPTH2_PRIMARY]
    if path == RES_DEPTH2_PRIMARY:
        return v
    v[DEPTH2_PRIMARY_ROW] = cand[DEPTH3_PRIMARY if path == RES_DEPTH3_PRIMARY else DEPTH3_ALTERNATE]
    return v


def test_mtp_tree_resolves_every_path():
    exp_cand = [DEPTH1_PRIMARY, DEPTH1_PRIMARY, DEPTH2_PRIMARY, DEPTH2_ALTERNATE, DEPTH3_PRIMARY, DEPTH3_ALTERNATE]
    exp_parent = [INPUT_ROW, INPUT_ROW, DEPTH1_ROW, DEPTH1_ROW, DEPTH2_PRIMARY_ROW, DEPTH2_PRIMARY_ROW]
    exp_base = [0, 0, 1, 1, 2, 2]
    cand = _candidates(90_000)
    for path in range(6):
        ver = _verifier(cand, path, 91_000)
        got_path, accepted, committed, fallback = MT.resolve(cand, ver, OUTPUT_VOCAB)
        assert got_path == path
        assert accepted == MT.accepted_token_count(path)
        assert committed == accepted + 1
        assert fallback == MT.fallback_row_index(path)
        assert MT.tail_candidate_index(path) == exp_cand[path]
        assert MT.tail_parent_row_index(path) == exp_parent[path]
        assert MT.tail_base_position_offset(path) == exp_base[path]


# ------------------------------------------------------------------ verify plans
def _sched(mode, force=True, max_batch=4, draft_len=3, row_cap=0, num_blocks=64, max_model_len=512):
    sc = C.SchedulerConfig()
    sc.max_batch, sc.block_tokens, sc.num_blocks, sc.max_model_len = max_batch, 16, num_blocks, max_model_len
    sc.decode_buckets = [1, 2, 4]
    sc.spec_mode = mode
    sc.spec_draft_len = draft_len
    sc.spec_row_cap = row_cap
    sc.spec_shadow_slot_base = num_blocks * 16
    if force:
        sc.flags = C.SCHED_DEFAULT_FLAGS | C.SCHED_MTP_FORCE_ENABLE
    return C.Scheduler(sc)


def _prefill(s, prompts, max_new=32, **kw):
    for i, p in enumerate(prompts):
        r = C.RequestSpec(i + 1, p, max_new)
        for k, v in kw.items():
            setattr(r, k, v)
        s.add_request(r)
    plan = s.schedule()
    assert plan.kind == 1
    s.complete(plan, np.array([500 + i for i in range(plan.num_seqs)], np.int32))


def test_tree_verify_plan_rows_and_completion():
    s = _sched(C.SPEC_MTP_TREE)
    _prefill(s, [list(range(20)), list(range(100, 110))])
    assert s.state(1) == C.SlotState.READY_SPECULATIVE_VERIFY
    v = s.schedule()
    assert v.kind == 3 and v.flags & C.DECISION_MTP_TREE_VERIFY and v.rows_per_seq == 6
    Bp = v.padded_seqs
    assert (v.num_seqs, Bp) == (2, 2)
    pos = v.positions.reshape(6, Bp)
    assert pos[:, 0].tolist() == [20, 21, 22, 22, 23, 23] and pos[:, 1].tolist() == [10, 11, 12, 12, 13, 13]
    assert (v.context_lens.reshape(6, Bp) == pos + 1).all()
    slots = v.slot_mapping.reshape(6, Bp)
    base = 64 * 16
    assert slots[3].tolist() == [base, base + 2] and slots[5].tolist() == [base + 1, base + 3]
    bt = v.block_table.reshape(Bp, -1)
    assert slots[2, 0] == bt[0, 22 // 16] * 16 + 22 % 16 and slots[4, 1] == bt[1, 0] * 16 + 13
    assert v.token_ids.reshape(6, Bp)[0].tolist() == [500, 501]
    sp = v.sync_positions.reshape(3, Bp)
    assert sp[:, 0].tolist() == [17, 18, 19] and v.sync_token_ids.reshape(3, Bp)[:, 0].tolist() == [17, 18, 19]
    assert s.state(1) == C.SlotState.RUNNING_SPECULATIVE_VERIFY
    # lane 0 resolved path 5 (4 tokens), lane 1 path 0 (1 token)
    committed = np.full((2, 6), -1, np.int32)
    committed[0, :4] = [7, 8, 9, 10]
    committed[1, 0] = 11
    ev = s.complete_verify(v, committed, np.array([4, 1], np.int32), np.array([5, 0], np.int32))
    assert [e.token for e in ev if e.kind == 1 and e.id == 1] == [7, 8, 9, 10]
    assert s.output_tokens(1) == [500, 7, 8, 9, 10] and s.output_tokens(2) == [501, 11]
    l1, l2 = s.lane_state(1), s.lane_state(2)
    assert l1["ema_milli"] == 2900 + (4000 - 2900) // 4 and l2["ema_milli"] == 2900 - 1900 // 4
    t = s.spec_totals
    assert (t["rounds"], t["committed"], t["accepted"], t["proposed"]) == (2, 5, 3, 10)
    nxt = s.schedule()
    assert nxt.kind == 3 and nxt.positions.reshape(6, 2)[0].tolist() == [24, 11]
    # an invalid resolution is refused
    with pytest.raises(StatusError):
        s.complete_verify(nxt, committed, np.array([3, 1], np.int32), np.array([5, 0], np.int32))


def test_tree_stop_token_inside_a_round_and_budget_gate():
    s = _sched(C.SPEC_MTP_TREE)
    r = C.RequestSpec(1, list(range(8)), 32, stop_token_ids=[9])
    s.add_request(r)
    s.complete(s.schedule(), np.array([5], np.int32))
    v = s.schedule()
    assert v.kind == 3
    committed = np.array([[7, 9, 8, 6, -1, -1]], np.int32)
    ev = s.complete_verify(v, committed, np.array([4], np.int32), np.array([5], np.int32))
    assert [e.token for e in ev if e.kind == 1] == [7, 9] and ev[-1].kind == 2 and ev[-1].reason == 2
    assert not s.has_work()
    # fewer than 5 tokens left: the tree cannot commit its maximum, so the batch decodes plainly
    s = _sched(C.SPEC_MTP_TREE)
    s.add_request(C.RequestSpec(1, list(range(8)), 4))
    s.complete(s.schedule(), np.array([5], np.int32))
    assert s.schedule().kind == 2


def test_tree_needs_full_grants_and_chain_suppression_reprobe():
    # tree: one-token rounds lower the EMA until the allocator's milli values can no
    # longer grant all five candidates (EMA 1255: alpha 203 -> 203, 41, 8, 1, 0), and
    # from then on the batch decodes plainly
    s = _sched(C.SPEC_MTP_TREE)
    _prefill(s, [list(range(8)), list(range(30, 38))], max_new=200)
    one = np.array([[1, -1, -1, -1, -1, -1], [2, -1, -1, -1, -1, -1]], np.int32)
    rounds = 0
    while True:
        v = s.schedule()
        if v.kind != 3:
            break
        s.complete_verify(v, one, np.array([1, 1], np.int32), np.array([0, 0], np.int32))
        rounds += 1
    assert rounds == 7 and s.lane_state(1)["ema_milli"] == 1255 and s.lane_state(1)["budget"] == 5
    # chain: verify while any draft row is granted, until the EMA falls below 1.15
    # tokens (2900 -> ... -> 1192 -> 1144): suppressed, 16 plain tokens, then a reprobe
    s = _sched(C.SPEC_CHAIN, draft_len=3)
    _prefill(s, [list(range(8)), list(range(30, 38))], max_new=200)
    one = np.array([[1, -1, -1, -1], [2, -1, -1, -1]], np.int32)
    rounds = 0
    while True:
        v = s.schedule()
        if v.kind != 3:
            break
        s.complete_verify(v, one, np.array([1, 1], np.int32))
        rounds += 1
    assert rounds == 9 and s.lane_state(1)["budget"] == 0 and s.spec_totals["suppressed"] == 2
    assert s.lane_state(2)["countdown"] == 16
    plain = 1
    s.complete(v, np.array([3, 4], np.int32))
    while True:
        v = s.schedule()
        if v.kind == 3:
            break
        s.complete(v, np.array([3, 4], np.int32))
        plain += 1
    assert plain == 16 and s.spec_totals["reprobes"] == 2 and v.draft_budget[:2].tolist() == [3, 3]


def test_chain_budgets_from_row_allocator_and_idle_rows():
    # row cap 6 for 2 lanes: base rows 2, 4 draft rows by alpha -> lane with the higher EMA first
    s = _sched(C.SPEC_CHAIN, draft_len=3, row_cap=6)
    _prefill(s, [list(range(8)), list(range(30, 38))], max_new=64)
    v = s.schedule()
    assert v.kind == 3 and v.rows_per_seq == 4 and v.draft_budget[:2].tolist() == [2, 2]
    ctx = v.context_lens.reshape(4, v.padded_seqs)
    assert ctx[:, 0].tolist() == [9, 10, 11, 0] and v.slot_mapping.reshape(4, 2)[3].tolist() == [-1, -1]
    # lane 0 accepts both drafts, lane 1 none: lane 0's EMA rises above lane 1's
    committed = np.array([[40, 41, 42, -1], [43, -1, -1, -1]], np.int32)
    s.complete_verify(v, committed, np.array([3, 1], np.int32))
    assert s.output_tokens(1) == [500, 40, 41, 42]
    l1, l2 = s.lane_state(1), s.lane_state(2)
    assert (l1["ema_milli"], l2["ema_milli"]) == (2925, 2425)
    v = s.schedule()
    want = S.row_allocator_assign([(2925, 3, 0), (2425, 3, 0)], 6, 1000)[1]
    assert v.draft_budget[:2].tolist() == want
    with pytest.raises(StatusError):  # more tokens than a lane's budget allows: nothing is applied
        s.complete_verify(v, committed, np.array([1, want[1] + 2], np.int32))
    assert s.output_tokens(1) == [500, 40, 41, 42]


def test_utility_gate_uses_measured_step_costs():
    s = _sched(C.SPEC_CHAIN, force=False, draft_len=3)
    _prefill(s, [list(range(8)), list(range(30, 38))])
    # unmeasured: 1 ms + 20 us per row -> a 4-row round costs ~1.1x a plain step: 2 tokens beat 1.25x
    s.set_step_cost(2, 2, 1_000_000)
    s.set_step_cost(3, 2, 1_700_000)   # 2.0 x 1.0 > 1.25 x 1.7 is false -> plain decode
    v = s.schedule()
    assert v.kind == 2
    s.complete(v, np.array([1, 2], np.int32))
    s.set_step_cost(3, 2, 1_500_000)   # 2.0 > 1.875 -> verify
    assert s.schedule().kind == 3
    assert s.estimate_step_ns(3, 2) == 1_500_000


def test_sampled_requests_never_speculate():
    s = _sched(C.SPEC_CHAIN)
    s.add_request(C.RequestSpec(1, list(range(8)), 32, temperature=0.7, seed=3))
    s.complete(s.schedule(), np.array([5], np.int32))
    assert s.lane_state(1)["disabled"] and s.schedule().kind == 2


def test_speculation_config_validation():
    sc = C.SchedulerConfig()
    sc.spec_mode = C.SPEC_CHAIN
    sc.spec_draft_len = 8
    with pytest.raises(StatusError):
        C.Scheduler(sc)
    sc.spec_mode = C.SPEC_MTP_TREE
    sc.spec_draft_len = 3
    with pytest.raises(StatusError):  # tree speculation needs shadow slots
        C.Scheduler(sc)
