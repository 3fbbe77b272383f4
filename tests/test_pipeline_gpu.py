"""The work-plane pipeline on two GPUs (one process per GPU, NCCL for hidden states,
gloo for packets and final events): a 4-layer MLA-MoE split 2 / 2. With one
micro-batch per step the greedy tokens equal a single-GPU engine's; with one or two
micro-batches the last stage's prefill logits are bitwise equal to a single-GPU
forward of the same batch (the hand-off between stages is exact). With two
micro-batches the decode packets replay per-stage CUDA graphs (padded lane buckets,
their own split-KV factor), so tokens match the single-GPU engine's up to near-ties."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cfg():
    from sparkpipe_rs_b200.models.config import v2_lite

    return v2_lite().replace(name="pp-mla-moe", num_layers=4, hidden_size=1024, n_routed_experts=16,
                             num_experts_per_tok=4, moe_intermediate_size=256, intermediate_size=2048,
                             n_shared_experts=1, vocab_size=4096, first_k_dense_replace=1, init_std=0.05)


def _prompts(cfg):
    g = torch.Generator().manual_seed(1)
    return [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (40, 70, 100, 33)]


def _engine_cfg(**kw):
    from sparkpipe_rs_b200.serving.engine import EngineConfig

    return EngineConfig(max_batch=4, block_size=64, max_model_len=256, max_prefill_tokens=512,
                        decode_buckets=(1, 2, 4), use_cuda_graph=False, async_decode=False, **kw)


def _worker(rank, port, micro, graphs, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        from sparkpipe_rs_b200.models.mla_moe import KVCache, MLAMoEModel
        from sparkpipe_rs_b200.parallel.pipeline import PipelineModel, StageRuntime, split_layers, work_config
        from sparkpipe_rs_b200.serving.engine import LLMEngine, SamplingParams

        cfg = _cfg()
        stages = split_layers(cfg.num_layers, 2)
        model = MLAMoEModel(cfg, seed=0, device=dev, max_positions=512)
        nblocks = 4 * 4 + 16
        cache = KVCache(cfg, num_blocks=nblocks, block_size=64, device=dev, layers=2)
        wcfg = work_config(cfg, 64, 256, 4, 512)
        if rank == 0:
            pm = PipelineModel(model, stages, cache, wcfg, micro_batches=micro, use_graphs=graphs)
            eng = LLMEngine(cfg, _engine_cfg(num_blocks=nblocks), model=pm, device=dev, cache=cache)
            res = eng.generate(_prompts(cfg), SamplingParams(max_tokens=24, ignore_eos=True))
            eng.shutdown()
            out_q.put(("rank0", [o.token_ids for o in res.outputs], pm.final_events, pm.graph_replays))
        else:
            rt = StageRuntime(model, stages, cache, wcfg, use_graphs=graphs)
            first = []
            rt.after_execute = lambda r: first.append(r.last_logits.float().cpu()) if not first else None
            rt.serve()
            out_q.put(("rank1", first[0], rt.graph_replays))
        torch.cuda.synchronize()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("micro,graphs", [(1, False), (2, True)])
def test_two_gpu_pipeline_matches_single_gpu(micro, graphs):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, micro, graphs, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(2):
        item = q.get(timeout=600)
        got[item[0]] = item[1:]
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    tokens, finals, replays0 = got["rank0"]
    pp_logits, replays1 = got["rank1"]
    # every decode packet (23 steps x micro-batches) replayed a graph on both stages
    assert (replays0, replays1) == ((23 * micro, 23 * micro) if graphs else (0, 0))

    # single-GPU reference: the same model and the same batches in one process
    from sparkpipe_rs_b200.models.mla_moe import ForwardBatch, KVCache, MLAMoEModel
    from sparkpipe_rs_b200.serving.engine import LLMEngine, SamplingParams

    cfg = _cfg()
    model = MLAMoEModel(cfg, seed=0, device="cuda", max_positions=512)
    eng = LLMEngine(cfg, _engine_cfg(num_blocks=32), model=model, device="cuda")
    ref = eng.generate(_prompts(cfg), SamplingParams(max_tokens=24, ignore_eos=True))
    eng.shutdown()
    ref_tokens = [o.token_ids for o in ref.outputs]
    if micro == 1:  # the same batches in the same order: the same tokens
        assert tokens == ref_tokens
    else:           # half batches per packet: a near-tie may round the other way
        assert sum(a == b for a, b in zip(tokens, ref_tokens)) >= 3
    assert finals == 4 + 23 * 4
    # the first packet's logits: the prefill of the first micro-batch's prompts
    prompts = _prompts(cfg)[: pp_logits.shape[0]]
    lens = [len(p) for p in prompts]
    cache = KVCache(cfg, num_blocks=16, block_size=64, device="cuda")
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device="cuda")
    pos = torch.cat([torch.arange(n, dtype=torch.int32) for n in lens]).cuda()
    slots = torch.cat([torch.arange(n, dtype=torch.int32) + 128 * i for i, n in enumerate(lens)]).cuda()
    fb = ForwardBatch(mode="prefill", token_ids=torch.tensor(sum(prompts, []), dtype=torch.int32, device="cuda"),
                      positions=pos, slot_mapping=slots, cu_q=cu, cu_k=cu, max_q=max(lens),
                      logits_idx=(cu[1:] - 1).contiguous())
    single = model.forward(fb, cache).float().cpu()
    assert torch.equal(pp_logits, single)
