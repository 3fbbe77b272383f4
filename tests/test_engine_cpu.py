"""The serving engine (C++ scheduler + CPU stage driver) against the fp32 oracle."""
import torch

from sparkpipe_rs_b200.models import oracle
from sparkpipe_rs_b200.models.config import tiny
from sparkpipe_rs_b200.models.cpu_model import CpuMLAMoEModel
from sparkpipe_rs_b200.serving.engine import EngineConfig, LLMEngine, SamplingParams


def _engine(**kw):
    cfg = tiny()
    m = CpuMLAMoEModel(cfg, seed=0)
    ec = EngineConfig(max_batch=4, block_size=16, max_model_len=128, max_prefill_tokens=40, **kw)
    return cfg, m, LLMEngine(cfg, ec, model=m, device="cpu")


def test_greedy_generation_matches_oracle():
    cfg, m, eng = _engine()
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab_size, (32,), generator=g).tolist() for _ in range(4)]
    res = eng.generate(prompts, SamplingParams(max_tokens=16, ignore_eos=True))
    for p, o in zip(prompts, res.outputs):
        ref, _ = oracle.greedy_generate(cfg, m.w, torch.tensor(p), 16)
        assert o.token_ids == ref.tolist()
        assert o.finish_reason == "length"
    assert res.stats["prefill_steps"] >= 3  # 128 prompt tokens under a 40-token budget
    assert res.stats["decode_steps"] == 15


def test_prefix_cache_hit_gives_same_tokens():
    cfg, m, eng = _engine()
    g = torch.Generator().manual_seed(1)
    p = torch.randint(0, cfg.vocab_size, (40,), generator=g).tolist()
    a = eng.generate([p], SamplingParams(max_tokens=6, ignore_eos=True))
    b = eng.generate([p], SamplingParams(max_tokens=6, ignore_eos=True))
    assert a.outputs[0].token_ids == b.outputs[0].token_ids
    assert eng.scheduler.stats.cached_prompt_tokens == 32


def test_stop_token_and_abort():
    cfg, m, eng = _engine()
    p = list(range(10, 30))
    ref, _ = oracle.greedy_generate(cfg, m.w, torch.tensor(p), 4)
    stop = ref.tolist()[2]
    res = eng.generate([p], SamplingParams(max_tokens=10, stop_token_ids=(stop,)))
    assert res.outputs[0].finish_reason == "stop"
    assert res.outputs[0].token_ids[-1] == stop
    rid = eng.add_request(p, SamplingParams(max_tokens=50))
    eng.step()
    assert eng.abort_request(rid)
    assert not eng.has_unfinished_requests()


def test_ahead_scheduled_decode_matches_synchronous():
    """Decode steps planned ahead of the previous step's tokens give the same
    outputs as the synchronous loop, with stop tokens, uneven lengths and an abort."""
    cfg, m, sync = _engine(async_decode=False)
    _, _, ahead = _engine(async_decode=True)
    ahead.model = sync.model = m
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (20, 33, 7, 18)]
    ref0, _ = oracle.greedy_generate(cfg, m.w, torch.tensor(prompts[0]), 8)
    stop = ref0.tolist()[4]
    params = [SamplingParams(max_tokens=12, stop_token_ids=(stop,)), SamplingParams(max_tokens=5, ignore_eos=True),
              SamplingParams(max_tokens=9, ignore_eos=True), SamplingParams(max_tokens=1, ignore_eos=True)]
    outs = []
    for eng in (sync, ahead):
        ids = [eng.add_request(p, sp) for p, sp in zip(prompts, params)]
        got = {}
        while eng.has_unfinished_requests():
            for o in eng.step():
                if o.finished:
                    got[o.request_id] = (list(o.token_ids), o.finish_reason)
        outs.append([got[i] for i in ids])
    assert outs[0] == outs[1]
    assert outs[1][0][1] == "stop" and outs[1][0][0][-1] == stop
    assert [len(t) for t, _ in outs[1][1:]] == [5, 9, 1]
    assert ahead.ahead_steps > 0 and sync.ahead_steps == 0


def test_ahead_plan_layout_and_policy():
    cfg, m, eng = _engine(async_decode=False)
    core = eng.core
    sc = eng.scheduler
    for i, n in enumerate((10, 70)):
        sc.add_request(core.RequestSpec(100 + i, list(range(1, n + 1)), 4, ignore_eos=True))
    while sc.waiting_count:
        p = sc.schedule()
        sc.complete(p, [5] * p.num_seqs)
    d = sc.schedule()
    assert d.kind == 2 and list(d.positions[:2]) == [10, 70]
    a = sc.schedule_ahead(d)
    assert a.kind == 2 and a.flags & core.DECISION_SCHEDULED_AHEAD
    assert list(a.src_rows[:2]) == [0, 1] and list(a.token_ids[:2]) == [0, 1]
    assert list(a.positions[:2]) == [11, 71] and list(a.context_lens[:2]) == [12, 72]
    bt = a.block_table.reshape(a.padded_seqs, a.max_blocks)
    assert a.slot_mapping[1] == bt[1][71 // 16] * 16 + 71 % 16
    # a waiting prompt with a free seat means the policy runs a prefill next
    sc.complete(d, [7, 7])
    sc.add_request(core.RequestSpec(200, [1, 2, 3], 4))
    assert sc.schedule_ahead(a).kind == 0
    sc.complete(a, [8, 8])
    # a sequence whose last token is due at the in-flight step is left out
    p = sc.schedule()
    assert p.kind == 1
    sc.complete(p, [9])
    d = sc.schedule()
    a = sc.schedule_ahead(d)
    assert a.kind == 2 and a.num_seqs == 1 and a.seq_ids == [200] and a.src_rows[0] == 2


def test_sampling_is_seeded_per_request_not_per_batch():
    cfg, m, eng = _engine()
    g = torch.Generator().manual_seed(5)
    p = torch.randint(0, cfg.vocab_size, (24,), generator=g).tolist()
    others = [torch.randint(0, cfg.vocab_size, (30,), generator=g).tolist() for _ in range(2)]
    sp = SamplingParams(max_tokens=10, temperature=1.5, seed=11, ignore_eos=True)
    alone = eng.generate([p], sp).outputs[0].token_ids
    batched = eng.generate(others[:1] + [p] + others[1:], sp).outputs[1].token_ids
    greedy = eng.generate([p], SamplingParams(max_tokens=10, ignore_eos=True)).outputs[0].token_ids
    other_seed = eng.generate([p], SamplingParams(max_tokens=10, temperature=1.5, seed=12,
                                                  ignore_eos=True)).outputs[0].token_ids
    assert alone == batched
    assert alone != greedy and alone != other_seed
