"""Speculation in the serving engine on the GPU: the verify kernels against their plain
statements, the MLA decode kernel's explicit last-token slot, and ``LLMEngine``
verify rounds (chain and MTP tree, CUDA graphs) whose every committed token is the
target's (near-)argmax given the tokens before it."""
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _small(layers=1, vocab=2048):
    from sparkpipe_rs_b200.models.config import v2_lite

    return v2_lite().replace(name="small-spec-engine", num_layers=layers, hidden_size=1024, n_routed_experts=16,
                             num_experts_per_tok=4, moe_intermediate_size=256, intermediate_size=1408,
                             n_shared_experts=1, vocab_size=vocab, first_k_dense_replace=1, init_std=0.05)


def test_top2_rows_matches_torch():
    from sparkpipe_rs_b200 import ops

    g = torch.Generator(device=DEV).manual_seed(0)
    for V in (4096, 102400, 1000):
        x = torch.randn(37, V, device=DEV, generator=g).to(torch.bfloat16)
        o0 = torch.empty(37, dtype=torch.int32, device=DEV)
        o1 = torch.empty(37, dtype=torch.int32, device=DEV)
        ops.top2_rows(x, o0, o1)
        xf = x.float()
        # reference with ties to the lower id: sort by (-value, id)
        for r in range(37):
            vals = xf[r]
            order = sorted(range(V), key=lambda i: (-vals[i].item(), i))[:2] if V <= 4096 else None
            if order is None:
                top = torch.topk(vals, 2)
                assert o0[r].item() == top.indices[0].item() or vals[o0[r]].item() == top.values[0].item()
                assert vals[o1[r]].item() == top.values[1].item() and o1[r].item() != o0[r].item()
            else:
                assert [o0[r].item(), o1[r].item()] == order


def test_commit_kernels_match_statements():
    from sparkpipe_rs_b200 import ops
    from sparkpipe_rs_b200.serving import verify

    g = torch.Generator().manual_seed(1)
    B, L = 24, 3
    for trial in range(6):
        tok = torch.randint(0, 4, ((L + 1) * B,), generator=g, dtype=torch.int32)
        tgt = torch.randint(0, 4, ((L + 1) * B,), generator=g, dtype=torch.int32)
        ctx = torch.randint(0, 3, (B,), generator=g, dtype=torch.int32)
        pos = torch.randint(0, 1000, (B,), generator=g, dtype=torch.int32)
        budget = torch.randint(0, L + 1, (B,), generator=g, dtype=torch.int32)
        keys = torch.randint(0, 1 << 62, (B,), generator=g, dtype=torch.int64)
        p = 0.0 if trial % 2 == 0 else 0.7
        want_c, want_n = verify.chain_commit_reference(tok, tgt, ctx, pos, budget, keys, B, L, p, 17)
        c = torch.empty(B, L + 1, dtype=torch.int32, device=DEV)
        n = torch.empty(B, dtype=torch.int32, device=DEV)
        d = [t.to(DEV) for t in (tok, tgt, ctx, pos, budget, keys)]
        ops.spec_chain_commit(*d, L, c, n, p, 17)
        assert torch.equal(c.cpu(), want_c) and torch.equal(n.cpu(), want_n)
    # tree: paths, commits and the KV move of accepted alternates in a [layers, slots, 576] bf16 cache
    B = 40
    for trial in range(4):
        tok = torch.randint(0, 3, (6 * B,), generator=g, dtype=torch.int32)
        tgt = torch.randint(0, 3, (6 * B,), generator=g, dtype=torch.int32)
        ctx = (torch.rand(B, generator=g) > 0.1).int()
        slots = torch.randperm(8 * B, generator=g)[: 6 * B].int()
        cache = torch.randn(3, 8 * B, 576, generator=g).to(torch.bfloat16)
        ref_cache = cache.clone()
        want = verify.tree_commit_reference(tok, tgt, ctx, slots, B, ref_cache)
        dc = cache.to(DEV)
        out = [torch.empty(B, 6, dtype=torch.int32, device=DEV), torch.empty(B, dtype=torch.int32, device=DEV),
               torch.empty(B, dtype=torch.int32, device=DEV)]
        ops.mtp_tree_commit(tok.to(DEV), tgt.to(DEV), ctx.to(DEV), slots.to(DEV), dc, *out)
        for got, w in zip(out, want):
            assert torch.equal(got.cpu(), w)
        assert torch.equal(dc.cpu(), ref_cache)


def test_mla_decode_last_slot_equals_substituted_cache():
    from sparkpipe_rs_b200 import ops

    g = torch.Generator(device=DEV).manual_seed(2)
    B, H, nblk = 6, 16, 6
    cache = (torch.randn(nblk * B * 64 + 64, 576, device=DEV, generator=g) * 0.5).to(torch.bfloat16)
    bt = torch.arange(B * nblk, dtype=torch.int32, device=DEV).view(B, nblk)
    ctx = torch.tensor([1, 63, 64, 65, 200, 384], dtype=torch.int32, device=DEV)
    q = (torch.randn(B, H, 576, device=DEV, generator=g) * 0.5).to(torch.bfloat16)
    shadow = nblk * B * 64  # the spare block's rows
    last = torch.tensor([shadow, -1, shadow + 2, bt[3, 1].item() * 64 + 0, shadow + 5, shadow + 9],
                        dtype=torch.int32, device=DEV)
    # reference: the same kernel over a cache whose last-token rows hold the shadow rows
    sub = cache.clone()
    for b in range(B):
        if last[b] >= 0:
            t = int(ctx[b]) - 1
            sub[int(bt[b, t // 64]) * 64 + t % 64] = cache[int(last[b])]
    for splits in (1, 3):
        o = torch.empty(B, H, 512, dtype=torch.bfloat16, device=DEV)
        r = torch.empty_like(o)
        ops.mla_decode(q, cache, bt, ctx, o, splits, 0.07, impl="mma", last_slot=last)
        ops.mla_decode(q, sub, bt, ctx, r, splits, 0.07, impl="mma")
        torch.cuda.synchronize()
        assert torch.equal(o, r), (o.float() - r.float()).abs().max()
    assert ops.status_word() == 0


def _perturbed_pair(cfg, noise):
    from sparkpipe_rs_b200.models.mla_moe import MLAMoEModel
    from sparkpipe_rs_b200.models.weights import init_weights

    w = init_weights(cfg, seed=0, device=DEV)
    g = torch.Generator(device=DEV).manual_seed(7)
    wd = {k: ((v.float() + noise * v.float().std() * torch.randn(v.shape, device=DEV, generator=g)).to(v.dtype)
              if k not in ("embed", "lm_head") and v.dim() > 1 else v) for k, v in w.items()}
    target = MLAMoEModel(cfg, weights=w, device=DEV, max_positions=1024)
    draft = MLAMoEModel(cfg, weights=wd, device=DEV, max_positions=1024)
    return target, draft


def _check_near_argmax(model, prompts, outputs, tol=0.1):
    from sparkpipe_rs_b200.models.mla_moe import ForwardBatch, KVCache

    for p, o in zip(prompts, outputs):
        seq = torch.tensor(p + o[:-1], dtype=torch.int32, device=DEV)
        n = seq.shape[0]
        cache = KVCache(model.cfg, num_blocks=(n + 63) // 64 + 1, block_size=64, device=DEV)
        cu = torch.tensor([0, n], dtype=torch.int32, device=DEV)
        ar = torch.arange(n, dtype=torch.int32, device=DEV)
        fb = ForwardBatch(mode="prefill", token_ids=seq, positions=ar, slot_mapping=ar, cu_q=cu, cu_k=cu, max_q=n)
        logits = model.forward(fb, cache).float()[len(p) - 1:]
        got = logits.gather(1, torch.tensor(o, device=DEV)[:, None])[:, 0]
        gap = logits.max(-1).values - got
        assert gap.max().item() <= tol, (gap.max().item(), int(gap.argmax()))


@pytest.mark.parametrize("mode", ["chain", "mtp_tree"])
def test_engine_verify_rounds_commit_the_targets_tokens(mode):
    from sparkpipe_rs_b200 import ops
    from sparkpipe_rs_b200.serving.engine import EngineConfig, LLMEngine, SamplingParams

    cfg = _small(layers=1)
    # chain: an unperturbed copy drafts exactly what the target decodes, so nearly every
    # draft is accepted unless the draft's KV (prefill, plain steps, rounds) is wrong;
    # tree: a perturbed copy, so the alternate leaves win now and then
    target, draft = _perturbed_pair(cfg, 0.0 if mode == "chain" else 0.05)
    ec = EngineConfig(max_batch=8, block_size=64, max_model_len=512, max_prefill_tokens=512,
                      decode_buckets=(1, 2, 4, 8), speculation=mode, draft_len=3, spec_force=True)
    eng = LLMEngine(cfg, ec, model=target, device=DEV, draft=draft)
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (20, 63, 64, 90, 130, 7)]
    res = eng.generate(prompts, SamplingParams(max_tokens=48, ignore_eos=True))
    outs = [o.token_ids for o in res.outputs]
    assert all(len(o) == 48 for o in outs)
    st = res.stats
    assert st["verify_steps"] > 5, st
    assert st["tokens_per_verify_lane"] > (3.5 if mode == "chain" else 1.1), st
    if mode == "mtp_tree":
        assert eng.tree_paths[3] + eng.tree_paths[5] > 0 and eng.tree_paths[4] > 0, eng.tree_paths
    _check_near_argmax(target, prompts, outs)
    assert ops.status_word() == 0
    eng.shutdown()


def test_engine_tree_with_default_draft_on_a_two_layer_target():
    from sparkpipe_rs_b200.models.mla_moe import MLAMoEModel
    from sparkpipe_rs_b200.serving.engine import EngineConfig, LLMEngine, SamplingParams

    cfg = _small(layers=2, vocab=512)
    target = MLAMoEModel(cfg, seed=1, device=DEV, max_positions=1024)
    ec = EngineConfig(max_batch=4, block_size=64, max_model_len=512, max_prefill_tokens=512,
                      decode_buckets=(1, 2, 4), speculation="mtp_tree", spec_force=True)
    eng = LLMEngine(cfg, ec, model=target, device=DEV)
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (33, 70, 5)]
    res = eng.generate(prompts, SamplingParams(max_tokens=24, ignore_eos=True))
    _check_near_argmax(target, prompts, [o.token_ids for o in res.outputs])
    eng.shutdown()


def test_engine_forced_acceptance_rate():
    from sparkpipe_rs_b200.models.mla_moe import MLAMoEModel
    from sparkpipe_rs_b200.serving.engine import EngineConfig, LLMEngine, SamplingParams

    cfg = _small(layers=2)
    target = MLAMoEModel(cfg, seed=1, device=DEV, max_positions=1024)
    ec = EngineConfig(max_batch=16, block_size=64, max_model_len=1024, max_prefill_tokens=2048,
                      decode_buckets=(1, 2, 4, 8, 16), speculation="chain", draft_len=3, spec_p_accept=0.7,
                      spec_force=True)
    eng = LLMEngine(cfg, ec, model=target, device=DEV)
    g = torch.Generator().manual_seed(6)
    prompts = [torch.randint(0, cfg.vocab_size, (64,), generator=g).tolist() for _ in range(16)]
    res = eng.generate(prompts, SamplingParams(max_tokens=200, ignore_eos=True))
    assert 2.3 < res.stats["tokens_per_verify_lane"] < 2.75, res.stats   # E = 1 + 0.7 + 0.49 + 0.343
    eng.shutdown()
