"""Continuous-batching scheduler (C++): chunked prefill, prefix reuse, decode
padding, preemption and stop conditions."""
import numpy as np
import pytest

from sparkpipe_rs_b200.core import core, StatusError


def make(max_batch=4, budget=64, blocks=64, bt=16, max_len=256, flags=None):
    C = core()
    c = C.SchedulerConfig()
    c.max_batch, c.max_prefill_tokens, c.num_blocks, c.block_tokens, c.max_model_len = max_batch, budget, blocks, bt, max_len
    c.decode_buckets = [1, 2, 4, 8]
    if flags is not None:
        c.flags = flags
    return C.Scheduler(c)


def req(i, n, max_new=4, start=0, **kw):
    return core().RequestSpec(i, list(range(start, start + n)), max_new, **kw)


def drive(s, sample=lambda plan: np.full(plan.num_seqs, 7, np.int32)):
    plans = []
    while s.has_work():
        p = s.schedule()
        if p.kind == 0:
            break
        plans.append(p)
        s.complete(p, sample(p))
    return plans


def test_chunked_prefill_packs_prompts_under_the_budget():
    s = make(budget=40)
    s.add_request(req(1, 30))
    s.add_request(req(2, 30, start=100))
    p = s.schedule()
    assert p.kind == 1 and p.num_tokens == 40 and list(p.cu_q) == [0, 30, 40]
    assert list(p.emits_token) == [1, 0] and list(p.chunk_lens) == [30, 10]
    assert list(p.logits_idx) == [29, 39]
    ev = s.complete(p, np.array([5, 0], np.int32))
    assert [(e.kind, e.id) for e in ev] == [(1, 1), (4, 2)]
    p2 = s.schedule()  # request 2 continues its prompt (interleave cap not reached)
    assert p2.kind == 1 and list(p2.positions[:2]) == [10, 11] and p2.has_prefix
    assert list(p2.cu_k) == [0, 30]


def test_decode_padding_block_tables_and_slots():
    s = make(bt=16)
    for i in range(3):
        s.add_request(req(i + 1, 20, start=i * 50))
    drive_one = s.schedule()
    s.complete(drive_one, np.full(drive_one.num_seqs, 9, np.int32))
    p = s.schedule()
    assert p.kind == 2 and p.num_seqs == 3 and p.padded_seqs == 4
    assert p.flags & core().DECISION_CUDAGRAPH_PADDING
    assert list(p.context_lens) == [21, 21, 21, 0]
    assert list(p.token_ids[:3]) == [9, 9, 9] and list(p.positions[:3]) == [20, 20, 20]
    bt = np.asarray(p.block_table).reshape(4, p.max_blocks)
    for r in range(3):
        assert p.slot_mapping[r] == bt[r, 1] * 16 + 4
    assert p.slot_mapping[3] == -1


def test_stop_length_and_events():
    s = make()
    s.add_request(req(1, 8, max_new=3))
    s.add_request(core().RequestSpec(2, list(range(8)), 10, 1000000, [7], False))
    plans = drive(s)
    assert s.stats.finished == 2
    assert not s.has_work()
    assert s.prefix_cache.sequence_count == 0


def test_prefix_reuse_across_requests():
    s = make(bt=16)
    s.add_request(req(1, 40, max_new=1))
    drive(s)
    s.add_request(req(2, 40, max_new=1))
    p = s.schedule()
    assert p.kind == 1 and p.cached_prefix_tokens == 32 and p.has_prefix
    assert p.num_tokens == 8 and list(p.cu_k) == [0, 40]
    assert p.flags & core().DECISION_PREFIX_CACHE_USED


def test_prefix_cache_disabled_never_reuses():
    C = core()
    s = make(bt=16, flags=C.SCHED_DEFAULT_FLAGS & ~C.SCHED_PREFIX_CACHE)
    s.add_request(req(1, 40, max_new=1))
    drive(s)
    s.add_request(req(2, 40, max_new=1))
    assert s.schedule().cached_prefix_tokens == 0


def test_preemption_when_blocks_run_out():
    s = make(max_batch=4, blocks=6, bt=4, max_len=64, budget=64)
    for i in range(3):
        s.add_request(req(i + 1, 7, max_new=12, start=i * 100))
    plans = drive(s)
    assert s.stats.preemptions > 0
    assert s.stats.finished == 3


def test_rejections_and_cancel():
    s = make(max_len=32)
    with pytest.raises(StatusError):
        s.add_request(req(1, 40))
    s.add_request(req(2, 8))
    with pytest.raises(StatusError):
        s.add_request(req(2, 8))
    assert s.cancel(2) and not s.cancel(2)
    assert not s.has_work()


def test_priority_orders_admission():
    s = make(budget=8)
    s.add_request(req(1, 8, priority=10))
    s.add_request(req(2, 8, priority=99))
    p = s.schedule()
    assert list(p.seq_ids) == [2]
