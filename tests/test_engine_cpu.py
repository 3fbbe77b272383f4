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
