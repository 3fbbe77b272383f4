"""Speculative decoding through the serving engine (``LLMEngine.generate``), on CPU.

Greedy verification must not change a request's tokens: with chain drafts and with
the MTP tree (alternate leaves in shadow KV slots, an accepted alternate's KV moved
into place), every request's output equals the fp32 oracle's greedy continuation.
The draft is a perturbed copy of a one-layer target, so drafts are often right and
every tree path occurs. Forced Bernoulli acceptance commits tokens at the expected
rate. Also: the commit kernels' plain statements against the host tree resolution.
"""
import numpy as np
import pytest
import torch

from sparkpipe_rs_b200.core import core
from sparkpipe_rs_b200.models import oracle
from sparkpipe_rs_b200.models.config import mtp_head, tiny
from sparkpipe_rs_b200.models.cpu_model import CpuMLAMoEModel
from sparkpipe_rs_b200.serving import verify
from sparkpipe_rs_b200.serving.engine import EngineConfig, LLMEngine, SamplingParams

MT = core().work_control.mtp_tree


def _models(noise=0.15, seed=0):
    cfg = mtp_head(tiny())
    target = CpuMLAMoEModel(cfg, seed=seed)
    g = torch.Generator().manual_seed(99)
    w = {k: (v + noise * v.std() * torch.randn(v.shape, generator=g)) if k not in ("embed", "lm_head") and v.dim() > 1
         else v.clone() for k, v in target.w.items()}
    return cfg, target, CpuMLAMoEModel(cfg, weights=w)


def _engine(cfg, target, draft, mode, **kw):
    ec = EngineConfig(max_batch=4, block_size=16, max_model_len=256, max_prefill_tokens=64, speculation=mode,
                      spec_force=True, **kw)
    return LLMEngine(cfg, ec, model=target, device="cpu", draft=draft)


def _prompts(cfg, n, length, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, cfg.vocab_size, (length,), generator=g).tolist() for _ in range(n)]


@pytest.mark.parametrize("mode", ["chain", "mtp_tree"])
def test_greedy_speculation_keeps_the_target_tokens(mode):
    cfg, target, draft = _models()
    eng = _engine(cfg, target, draft, mode, draft_len=3)
    prompts = _prompts(cfg, 4, 24, 5)
    res = eng.generate(prompts, SamplingParams(max_tokens=40, ignore_eos=True))
    for p, o in zip(prompts, res.outputs):
        ref, _ = oracle.greedy_generate(cfg, target.w, torch.tensor(p), 40)
        assert o.token_ids == ref.tolist()
        assert o.finish_reason == "length"
    st = res.stats
    assert st["verify_steps"] > 0 and st["tokens_per_verify_lane"] > 1.5
    assert st["generated_tokens"] == 160
    if mode == "mtp_tree":
        assert all(c > 0 for c in eng.tree_paths[1:]), eng.tree_paths   # every accepted path occurred
        assert eng.tree_paths[3] + eng.tree_paths[5] > 0                  # alternate leaves committed


def test_tree_with_an_unrelated_draft_and_a_two_layer_target():
    cfg = tiny()
    target = CpuMLAMoEModel(cfg, seed=0)
    eng = LLMEngine(cfg, EngineConfig(max_batch=4, block_size=16, max_model_len=256, max_prefill_tokens=64,
                                      speculation="mtp_tree", spec_force=True), model=target, device="cpu")
    prompts = _prompts(cfg, 3, 20, 7)
    res = eng.generate(prompts, SamplingParams(max_tokens=12, ignore_eos=True))
    for p, o in zip(prompts, res.outputs):
        ref, _ = oracle.greedy_generate(cfg, target.w, torch.tensor(p), 12)
        assert o.token_ids == ref.tolist()


def test_forced_acceptance_commits_at_the_expected_rate():
    cfg, target, draft = _models()
    eng = _engine(cfg, target, draft, "chain", draft_len=3, spec_p_accept=0.7)
    res = eng.generate(_prompts(cfg, 4, 16, 3), SamplingParams(max_tokens=120, ignore_eos=True))
    # E[committed per round] = 1 + 0.7 + 0.49 + 0.343 = 2.533 (lanes near their length cap draft less)
    assert 2.1 < res.stats["tokens_per_verify_lane"] < 2.8
    assert all(len(o.token_ids) == 120 for o in res.outputs)


def test_sampled_requests_and_stop_tokens_under_speculation():
    cfg, target, draft = _models()
    eng = _engine(cfg, target, draft, "mtp_tree")
    prompts = _prompts(cfg, 2, 16, 9)
    ref, _ = oracle.greedy_generate(cfg, target.w, torch.tensor(prompts[0]), 20)
    stop = int(ref[9])
    res = eng.generate([prompts[0]], SamplingParams(max_tokens=20, stop_token_ids=(stop,)))
    first = ref.tolist().index(stop)
    assert res.outputs[0].token_ids == ref.tolist()[:first + 1] and res.outputs[0].finish_reason == "stop"
    # a sampled request never speculates, a greedy one beside it still matches the oracle
    a = eng.add_request(prompts[1], SamplingParams(max_tokens=10, temperature=0.8, seed=4, ignore_eos=True))
    b = eng.add_request(prompts[0], SamplingParams(max_tokens=10, ignore_eos=True))
    while eng.has_unfinished_requests():
        eng.step()
    assert eng.outputs[b].token_ids == ref.tolist()[:10]
    assert len(eng.outputs[a].token_ids) == 10


def test_commit_statements_match_the_host_tree_resolution():
    g = torch.Generator().manual_seed(0)
    B = 8
    for trial in range(30):
        cand = torch.randint(0, 6, (5, B), generator=g, dtype=torch.int32)
        tok = torch.cat([torch.randint(0, 6, (1, B), generator=g, dtype=torch.int32), cand]).flatten()
        tgt = torch.randint(0, 6, (6 * B,), generator=g, dtype=torch.int32)
        ctx = torch.ones(B, dtype=torch.int32)
        slots = torch.arange(6 * B, dtype=torch.int32)
        cache = torch.randn(2, 6 * B, 4)
        before = cache.clone()
        committed, counts, paths = verify.tree_commit_reference(tok, tgt, ctx, slots, B, cache)
        for b in range(B):
            c = [int(tok[(r + 1) * B + b]) for r in range(5)]
            v = [int(tgt[r * B + b]) for r in range(6)]
            path, acc, com, _ = MT.resolve(c, v, 16)
            assert (int(paths[b]), int(counts[b])) == (path, com)
            want = [c[MT.tail_candidate_index(r)] for r in _path_rows(path)] + [v[path]]
            assert committed[b, :com].tolist() == want
            if path in (3, 5):
                dst = int(slots[(2 if path == 3 else 4) * B + b])
                assert torch.equal(cache[:, dst], before[:, int(slots[path * B + b])])
    # chain statement: agreement within budget
    tok = torch.tensor([5, 6, 7, 8, 9, 1, 2, 3], dtype=torch.int32)     # L = 3, B = 2: rows j * 2 + b
    tgt = torch.tensor([7, 8, 9, 2, 4, 0, 0, 0], dtype=torch.int32)
    c, n = verify.chain_commit_reference(tok, tgt, torch.ones(2, dtype=torch.int32), torch.zeros(2, dtype=torch.int32),
                                         torch.tensor([3, 1]), torch.zeros(2, dtype=torch.int64), 2, 3)
    assert n.tolist() == [3, 2] and c[0].tolist() == [7, 9, 4, -1] and c[1].tolist() == [8, 2, -1, -1]


def _path_rows(path):
    rows = []
    r = path
    parent = (0, 0, 1, 1, 2, 2)
    while r != 0:
        rows.append(r)
        r = parent[r]
    return rows[::-1]
