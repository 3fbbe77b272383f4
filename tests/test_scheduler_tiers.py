"""Scheduler features around the KV cache, on CPU: lookahead protection of queued
prompts' cached blocks, prefix-family cohorting (a family's leader prefills the
shared prefix once, its followers wait and then hit the cache), and preemption to
the host KV tier (swap-out / swap-in copies in the plans, host slot accounting),
end to end through the engine with tokens equal to the fp32 oracle."""
import numpy as np
import torch

from sparkpipe_rs_b200.core import core
from sparkpipe_rs_b200.models import oracle
from sparkpipe_rs_b200.models.config import tiny
from sparkpipe_rs_b200.models.cpu_model import CpuMLAMoEModel
from sparkpipe_rs_b200.serving.engine import EngineConfig, LLMEngine, SamplingParams

C = core()


def test_lookahead_protection_orders_eviction():
    pc = C.PrefixCache(4, 8, 16)
    a, b = list(range(100, 109)), list(range(200, 209))   # 2 full reusable blocks each (+ tail)
    for sid, t in ((1, a), (2, b)):
        pc.reserve_prompt(sid, t)
        pc.commit(sid, 8)
        pc.release_sequence(sid)
    assert pc.warm_blocks == 4
    # a queued prompt will reuse a's blocks: they are evicted last although they are older
    pc.reset_lookahead_protection()
    assert pc.protect_prompt_lookahead(a + [7], 5) == 2 and pc.protected_warm_blocks == 2
    assert pc.trim_warm_blocks(2) == 2
    assert pc.probe_prompt(a + [7]).matched_block_count == 2 and pc.probe_prompt(b + [7]).matched_block_count == 0
    # protected blocks go last, lowest demand first
    pc.reserve_prompt(3, b)
    pc.commit(3, 8)
    pc.release_sequence(3)
    pc.reset_lookahead_protection()
    pc.protect_prompt_lookahead(a + [1], 9)
    pc.protect_prompt_lookahead(b + [1], 2)
    assert pc.trim_warm_blocks(2) == 2
    assert pc.probe_prompt(a + [7]).matched_block_count == 2 and pc.stats.protected_evictions == 2
    # a new epoch clears the marks
    pc.reset_lookahead_protection()
    assert pc.protected_warm_blocks == 0


def _sched(num_blocks=64, host_blocks=0, max_batch=4, bt=16, max_prefill=4096, flags=None):
    sc = C.SchedulerConfig()
    sc.max_batch, sc.block_tokens, sc.num_blocks, sc.max_model_len = max_batch, bt, num_blocks, 1024
    sc.max_prefill_tokens = max_prefill
    sc.decode_buckets = [1, 2, 4]
    sc.host_blocks = host_blocks
    if flags is not None:
        sc.flags = flags
    return C.Scheduler(sc)


def test_prefix_family_leader_first_then_followers_hit():
    s = _sched(max_prefill=128)
    shared = list(range(1000, 1096))                         # 6 blocks of 16
    s.add_request(C.RequestSpec(1, shared + [1, 2, 3], 4))
    s.add_request(C.RequestSpec(2, shared + [4, 5], 4))
    s.add_request(C.RequestSpec(3, shared + [6], 4))
    s.add_request(C.RequestSpec(4, list(range(5000, 5020)), 4))  # unrelated
    p = s.schedule()
    assert p.kind == 1 and p.flags & C.DECISION_PREFIX_FAMILY
    # the leader (earliest) takes its first chunk; the followers wait; the unrelated prompt fills the budget
    assert list(p.seq_ids)[0] == 1 and 2 not in p.seq_ids and 3 not in p.seq_ids
    assert s.state(2) == C.SlotState.WAITING_PREFIX_COHORT
    while s.state(2) != C.SlotState.READY_DECODE:
        p = s.schedule()
        if p.kind == 1:
            for i, sid in enumerate(p.seq_ids):
                if sid in (2, 3):
                    # followers start after the leader's shared blocks are cached
                    assert p.positions[p.cu_q[i]] == 96
        s.complete(p, np.zeros(p.num_seqs, np.int32))
    st = s.stats
    assert st.cached_prompt_tokens >= 2 * 96 and st.family_deferrals > 0


def test_cohorting_off_prefills_the_shared_prefix_twice():
    flags = C.SCHED_DEFAULT_FLAGS & ~C.SCHED_PREFIX_COHORTING
    s = _sched(max_prefill=4096, flags=flags)
    shared = list(range(1000, 1096))
    s.add_request(C.RequestSpec(1, shared + [1], 4))
    s.add_request(C.RequestSpec(2, shared + [2], 4))
    p = s.schedule()
    assert sorted(p.seq_ids) == [1, 2] and p.num_tokens == 2 * 97


def test_swap_preemption_round_trip_in_plans():
    # 8 blocks of 16 tokens; two sequences of 60 prompt tokens need 4 blocks each, the
    # first decode step that crosses a block boundary preempts the newer one
    s = _sched(num_blocks=8, host_blocks=16)
    s.add_request(C.RequestSpec(1, list(range(60)), 20))
    s.add_request(C.RequestSpec(2, list(range(100, 160)), 20))
    p = s.schedule()
    s.complete(p, np.array([1, 2], np.int32))
    outs, ins = [], []
    for _ in range(200):
        p = s.schedule()
        if len(p.swap_out):
            outs.append(p.swap_out.reshape(-1, 2))
            assert s.state(2) == C.SlotState.SWAPPED and s.swapped_count == 1
        if len(p.swap_in):
            ins.append(p.swap_in.reshape(-1, 2))
        if p.kind == 0:
            break
        s.complete(p, np.full(p.num_seqs, 7, np.int32))
    assert outs and ins
    # every restored host slot was written by the swap-out; the restore skips nothing it needs
    assert set(ins[0][:, 0]) <= set(outs[0][:, 1])
    st = s.stats
    assert st.swapped_out >= 1 and st.swapped_in >= 1 and st.swap_in_blocks <= st.swap_out_blocks
    assert not s.has_work() and s.free_host_blocks == 16
    assert len(s.output_tokens(1)) == 0  # finished requests are forgotten


def _engine(**kw):
    cfg = tiny()
    m = CpuMLAMoEModel(cfg, seed=0)
    ec = EngineConfig(max_batch=4, block_size=16, max_model_len=256, max_prefill_tokens=256, **kw)
    return cfg, m, LLMEngine(cfg, ec, model=m, device="cpu")


def test_engine_swapped_sequences_resume_with_identical_tokens():
    # 12 blocks for 4 sequences of 40 prompt + 24 new tokens (4 blocks each at the end):
    # decode runs out of blocks, preempted sequences go to the host tier and come back
    cfg, m, eng = _engine(num_blocks=12, host_kv_blocks=32)
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, cfg.vocab_size, (40,), generator=g).tolist() for _ in range(4)]
    res = eng.generate(prompts, SamplingParams(max_tokens=24, ignore_eos=True))
    st = eng.scheduler.stats
    assert st.swapped_out > 0 and st.swapped_in > 0 and eng.host_tier.restored_blocks > 0
    for p, o in zip(prompts, res.outputs):
        ref, _ = oracle.greedy_generate(cfg, m.w, torch.tensor(p), 24)
        assert o.token_ids == ref.tolist()
    # without the host tier the same load recomputes instead, with the same tokens
    cfg, m, eng2 = _engine(num_blocks=12)
    res2 = eng2.generate(prompts, SamplingParams(max_tokens=24, ignore_eos=True))
    assert eng2.scheduler.stats.swapped_out == 0 and eng2.scheduler.stats.preemptions > 0
    assert [o.token_ids for o in res2.outputs] == [o.token_ids for o in res.outputs]


def test_engine_prefix_family_saves_prefill_tokens():
    cfg, m, eng = _engine(num_blocks=64)
    g = torch.Generator().manual_seed(3)
    shared = torch.randint(0, cfg.vocab_size, (96,), generator=g).tolist()
    prompts = [shared + torch.randint(0, cfg.vocab_size, (5,), generator=g).tolist() for _ in range(3)]
    res = eng.generate(prompts, SamplingParams(max_tokens=6, ignore_eos=True))
    for p, o in zip(prompts, res.outputs):
        ref, _ = oracle.greedy_generate(cfg, m.w, torch.tensor(p), 6)
        assert o.token_ids == ref.tolist()
    assert res.stats["prefill_tokens"] == 101 + 2 * 5 + 2 * 0  # the shared 96 tokens are computed once
    assert eng.scheduler.stats.family_deferrals > 0


def test_prefix_host_tier_demotes_and_promotes():
    pc = C.PrefixCache(4, 6, 16)
    pc.enable_host_tier(100, 3)
    a = list(range(100, 109))                      # 2 reusable blocks + a tail token
    pc.reserve_prompt(1, a)
    pc.commit(1, 8)
    pc.release_sequence(1)                         # a's 2 blocks are warm on the device
    pc.reserve_prompt(2, list(range(500, 524)))    # 6 blocks: both warm blocks are evicted
    out, inn = pc.take_tier_copies()
    assert len(out) == 4 and not inn and sorted(out[1::2]) == [100, 101] and pc.host_entries == 2
    assert pc.stats.demoted_blocks == 2
    # the prompt still hits its prefix: in the host tier
    look = pc.probe_prompt(a + [1])
    assert look.matched_block_count == 2 and look.host_block_count == 2
    pc.release_sequence(2)
    r = pc.reserve_prompt(3, a + [1])
    assert r.reusable_token_count == 8
    out, inn = pc.take_tier_copies()
    # promotion copies land in the reservation's first two blocks; eviction made room first
    assert list(inn[1::2]) == list(r.physical_blocks[:2]) and sorted(inn[0::2]) == [100, 101]
    assert pc.stats.promoted_blocks == 2 and pc.host_entries == len(out) // 2
    # the promoted slots are free again only after the deferred release
    pc.release_deferred_slots()


def test_engine_reuses_a_prefix_from_the_host_tier():
    # 10 device blocks of 16: prompt A's 6 full blocks are pushed out by two other prompts,
    # then A comes back: its prefix is restored from the host tier, not recomputed
    cfg, m, eng = _engine(num_blocks=10, host_prefix_blocks=16)
    g = torch.Generator().manual_seed(5)
    a = torch.randint(0, cfg.vocab_size, (100,), generator=g).tolist()
    first = eng.generate([a], SamplingParams(max_tokens=4, ignore_eos=True))
    for _ in range(2):
        other = torch.randint(0, cfg.vocab_size, (120,), generator=g).tolist()
        eng.generate([other], SamplingParams(max_tokens=4, ignore_eos=True))
    again = eng.generate([a], SamplingParams(max_tokens=4, ignore_eos=True))
    st = eng.scheduler.stats
    assert st.prefix_tier_out_blocks > 0 and st.prefix_tier_in_blocks == 6
    assert again.stats["prefill_tokens"] == 100 - 96
    ref, _ = oracle.greedy_generate(cfg, m.w, torch.tensor(a), 4)
    assert first.outputs[0].token_ids == ref.tolist() == again.outputs[0].token_ids


def test_engine_swaps_through_a_drive_backed_host_tier(tmp_path):
    """The host tier's 32 slots backed by only 2 pinned buffers: swapped-out blocks spill
    to a drive file through the NVMe tier (reserve / write / commit, pinned while they
    are a slot's only copy) and come back by demand reads; tokens stay equal to the
    fp32 oracle."""
    cfg, m, eng = _engine(num_blocks=12, host_kv_blocks=32, host_resident_blocks=2,
                          host_drive_path=str(tmp_path / "kv_spill.bin"))
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, cfg.vocab_size, (40,), generator=g).tolist() for _ in range(4)]
    res = eng.generate(prompts, SamplingParams(max_tokens=24, ignore_eos=True))
    tier = eng.host_tier
    assert eng.scheduler.stats.swapped_in > 0
    assert tier.spilled_blocks > 0 and tier.fetched_blocks > 0
    st = tier.drive.tier.stats
    assert st.publishes == tier.spilled_blocks and st.demand_misses == 0 and st.io_errors == 0
    for p, o in zip(prompts, res.outputs):
        ref, _ = oracle.greedy_generate(cfg, m.w, torch.tensor(p), 24)
        assert o.token_ids == ref.tolist()


def test_drive_spill_round_trip_with_a_mock_device():
    """Virtual host slots over a mock drive (reads land after a few polls): every slot's
    bytes come back after being spilled, whatever the order."""
    from sparkpipe_rs_b200.models.mla_moe import KVCache
    from sparkpipe_rs_b200.serving.kv_offload import DriveSpill, HostKvTier

    cfg = tiny()
    cache = KVCache(cfg, num_blocks=8, block_size=16, device="cpu")
    cache.data.copy_(torch.randn_like(cache.data))
    probe = HostKvTier(cache, 1)
    mock = C.nvme_tier.MockDevice(probe.block_bytes * 64 + 65536, 3)
    drive = DriveSpill(probe.block_bytes, 8, device=mock)
    tier = HostKvTier(cache, 8, resident_blocks=2, drive=drive)
    orig = cache.data.clone()
    tier.evict_to([0, 1, 2, 3, 4, 5], [5, 4, 3, 2, 1, 0])   # 4 of 6 slots spill
    cache.data.zero_()
    tier.restore([0, 3, 5, 1, 4, 2], [5, 2, 0, 4, 1, 3])
    L = cache.data.shape[0]
    got, want = cache.data.view(L, 8, 16, -1), orig.view(L, 8, 16, -1)
    assert torch.equal(got[:, :6], want[:, :6])
    assert tier.spilled_blocks >= 4 and tier.fetched_blocks >= 4 and mock.reads >= 4
