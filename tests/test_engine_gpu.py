"""The serving engine on the GPU: CUDA-graph decode with steps scheduled ahead of
the previous step's tokens against the synchronous loop, and per-request sampling."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _cfg():
    from sparkpipe_rs_b200.models.config import v2_lite

    return v2_lite().replace(name="small-mla-moe", num_layers=3, hidden_size=1024, n_routed_experts=16,
                             num_experts_per_tok=4, moe_intermediate_size=256, intermediate_size=2048,
                             n_shared_experts=1, vocab_size=4096, first_k_dense_replace=1, init_std=0.05)


def _engine(model, cfg, **kw):
    from sparkpipe_rs_b200.serving.engine import EngineConfig, LLMEngine

    kw = {"max_batch": 8, "block_size": 64, "max_model_len": 512, "max_prefill_tokens": 256,
          "decode_buckets": (1, 2, 4, 8), **kw}
    ec = EngineConfig(**kw)
    return LLMEngine(cfg, ec, model=model, device="cuda")


def _run(eng, prompts, params):
    ids = [eng.add_request(p, sp) for p, sp in zip(prompts, params)]
    got = {}
    while eng.has_unfinished_requests():
        for o in eng.step():
            if o.finished:
                got[o.request_id] = (list(o.token_ids), o.finish_reason)
    return [got[i] for i in ids]


def test_ahead_decode_matches_synchronous_graph_loop():
    from sparkpipe_rs_b200.models.mla_moe import MLAMoEModel
    from sparkpipe_rs_b200.serving.engine import SamplingParams

    cfg = _cfg()
    model = MLAMoEModel(cfg, seed=0, device="cuda", max_positions=1024)
    sync = _engine(model, cfg, async_decode=False)
    ahead = _engine(model, cfg, async_decode=True)
    assert sorted(sync.graphs) == [1, 2, 4, 8]  # captured when the engine starts
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (40, 65, 17, 90, 33, 128, 9)]
    probe = _run(sync, prompts[:1], [SamplingParams(max_tokens=12, ignore_eos=True)])[0][0]
    stop = probe[5]
    params = [SamplingParams(max_tokens=24, stop_token_ids=(stop,))]
    params += [SamplingParams(max_tokens=n, ignore_eos=True) for n in (20, 7, 31, 3)]
    params += [SamplingParams(max_tokens=16, temperature=0.8, seed=s, ignore_eos=True) for s in (1, 2)]
    a = _run(sync, prompts, params)
    b = _run(ahead, prompts, params)
    assert ahead.ahead_steps > 0 and sync.ahead_steps == 0
    assert a == b
    assert b[0][1] == "stop" and b[0][0][-1] == stop and len(b[0][0]) == 6
    assert [len(t) for t, _ in b[1:5]] == [20, 7, 31, 3]
    assert b[5][0] != b[6][0]  # two seeds, two samples
    for e in (sync, ahead):
        e.shutdown()


def test_swapped_sequences_resume_from_the_host_tier():
    """Decode runs out of KV blocks: the scheduler swaps the newest sequences' KV to
    pinned host memory (caller-chosen slots) and restores it into fresh blocks later.
    The tier's round trip is bit-exact, and every committed token is the target's
    (near-)argmax given the tokens before it; a run with room for everything gives the
    same tokens."""
    from sparkpipe_rs_b200.models.mla_moe import KVCache, MLAMoEModel
    from sparkpipe_rs_b200.serving.engine import SamplingParams
    from sparkpipe_rs_b200.serving.kv_offload import HostKvTier

    cfg = _cfg()
    cache = KVCache(cfg, num_blocks=12, block_size=64, device="cuda")
    cache.data.normal_()
    tier = HostKvTier(cache, host_blocks=6, max_batch_blocks=2)
    before = [cache.data[:, b * 64:(b + 1) * 64].clone() for b in (1, 4, 7)]
    tier.evict_to([1, 4, 7], [5, 0, 3])
    cache.data.zero_()
    tier.restore([5, 0, 3], [8, 2, 11])
    for want, b in zip(before, (8, 2, 11)):
        assert torch.equal(cache.data[:, b * 64:(b + 1) * 64], want)

    model = MLAMoEModel(cfg, seed=0, device="cuda", max_positions=1024)
    g = torch.Generator().manual_seed(8)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (100, 120, 90, 110)]
    params = SamplingParams(max_tokens=60, ignore_eos=True)
    # 4 sequences end at 160-180 tokens (3 blocks each): 8 blocks force preemption
    tight = _engine(model, cfg, num_blocks=8, host_kv_blocks=16)
    res = tight.generate(prompts, params)
    st = tight.scheduler.stats
    assert st.swapped_out > 0 and st.swapped_in > 0 and tight.host_tier.restored_blocks > 0
    roomy = _engine(model, cfg)
    ref = roomy.generate(prompts, params)
    same = sum(a.token_ids == b.token_ids for a, b in zip(res.outputs, ref.outputs))
    assert same >= 3, [(a.token_ids[:8], b.token_ids[:8]) for a, b in zip(res.outputs, ref.outputs)]
    from test_spec_engine_gpu import _check_near_argmax

    # a preempted sequence decodes in other batches than the teacher-forced prefill, so a
    # near-tie may go either way: allow two bf16 ulps of logits of magnitude 16-32
    _check_near_argmax(model, prompts, [o.token_ids for o in res.outputs], tol=0.25)
    tight.shutdown()
    roomy.shutdown()


@pytest.mark.parametrize("kv_dtype", ["bf16", "fp8"])
def test_drive_backed_host_tier_round_trip_on_the_gpu_cache(tmp_path, kv_dtype):
    """Host slots over 2 pinned buffers and a drive file: device blocks evicted in
    pieces spill through the NVMe tier and come back bit-exact into other blocks (the
    fp8 cache moves its block scales with its rows)."""
    from sparkpipe_rs_b200.models.mla_moe import KVCache
    from sparkpipe_rs_b200.serving.kv_offload import DriveSpill, HostKvTier

    cfg = _cfg()
    cache = KVCache(cfg, num_blocks=12, block_size=64, device="cuda", kv_dtype=kv_dtype)
    for t in cache.planes():
        t.view(torch.uint8).copy_(torch.randint(0, 120, t.view(torch.uint8).shape, dtype=torch.uint8))
    probe = HostKvTier(cache, 1)
    drive = DriveSpill(probe.block_bytes, 8, path=str(tmp_path / "spill.bin"))
    tier = HostKvTier(cache, 8, max_batch_blocks=2, resident_blocks=2, drive=drive)
    src, dst = [1, 4, 7, 9, 10], [8, 2, 11, 0, 3]
    before = [[t[:, b * 64:(b + 1) * 64].clone() for t in cache.planes()] for b in src]
    tier.evict_to(src, [5, 0, 3, 6, 1])
    for t in cache.planes():
        t.zero_()
    tier.restore([5, 0, 3, 6, 1], dst)
    torch.cuda.synchronize()
    for want, b in zip(before, dst):
        for w, t in zip(want, cache.planes()):
            assert torch.equal(t[:, b * 64:(b + 1) * 64], w)
    assert tier.spilled_blocks >= 3 and tier.fetched_blocks >= 3


def test_prefill_graphs_replay_repeated_chunk_shapes():
    """Six 100-token prompts in 200-token chunks: the chunk shape repeats, so one prefill
    graph is captured (at the first chunk after the engine's warm-up prefill) and replayed
    for the others; tokens equal an engine that runs every chunk eagerly."""
    from sparkpipe_rs_b200.models.mla_moe import MLAMoEModel
    from sparkpipe_rs_b200.serving.engine import SamplingParams

    cfg = _cfg()
    model = MLAMoEModel(cfg, seed=0, device="cuda", max_positions=1024)
    g = torch.Generator().manual_seed(11)
    prompts = [torch.randint(0, cfg.vocab_size, (100,), generator=g).tolist() for _ in range(6)]
    params = SamplingParams(max_tokens=8, ignore_eos=True)
    outs = {}
    for graphs in (False, True):
        eng = _engine(model, cfg, max_prefill_tokens=200, prefill_graphs=graphs, prefix_caching=False)
        res = eng.generate(prompts, params)
        outs[graphs] = [o.token_ids for o in res.outputs]
        if graphs:
            assert len(eng._pgraphs) == 1 and list(eng._pgraphs) == [(200, 2, 100)]
        eng.shutdown()
    assert outs[True] == outs[False]
