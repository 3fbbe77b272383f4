"""GPU-free plumbing run: tiny MLA-MoE (2 layers, hidden 256, 4 heads, q_lora 96,
kv_lora 64, nope 32 / rope 16 / v 32, 8 experts top-2 + 1 shared, FFN 128,
vocab 1024, fp32 weights N(0, 0.02), seed 0) served by a 2-stage pipeline over
two gloo ranks; 4 prompts of 32 uniform ids, greedy 16 tokens each, checked
against a plain PyTorch CPU forward (logits and tokens)."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        from sparkpipe_rs_b200.models import oracle
        from sparkpipe_rs_b200.models.config import tiny
        from sparkpipe_rs_b200.models.cpu_model import CpuMLAMoEModel
        from sparkpipe_rs_b200.parallel.pipeline import PipelineModel, split_layers, stage_worker_loop

        cfg = tiny()
        stages = split_layers(cfg.num_layers, world)
        model = CpuMLAMoEModel(cfg, seed=0)
        block, max_len = 16, 64
        nblocks = 4 * (max_len // block) + 4
        if rank == 0:
            from sparkpipe_rs_b200.serving.engine import EngineConfig, LLMEngine, SamplingParams

            cache = model.new_cache(nblocks, block, layers=len(stages[0]))
            pm = PipelineModel(model, stages)
            captured = []
            orig = pm.forward

            def fwd(fb, c, **kw):
                lg = orig(fb, c, **kw)
                captured.append((fb.mode, lg.clone()))
                return lg

            pm.forward = fwd
            eng = LLMEngine(cfg, EngineConfig(max_batch=4, block_size=block, max_model_len=max_len,
                                              num_blocks=nblocks, max_prefill_tokens=256),
                            model=pm, device="cpu", cache=cache)
            g = torch.Generator().manual_seed(0)
            prompts = [torch.randint(0, 1024, (32,), generator=g).tolist() for _ in range(4)]
            res = eng.generate(prompts, SamplingParams(max_tokens=16, ignore_eos=True))
            eng.shutdown()
            ok_tokens, max_err = True, 0.0
            first_logits = captured[0][1]  # prefill logits of the 4 prompts' last tokens
            for i, (p, o) in enumerate(zip(prompts, res.outputs)):
                ref_tokens, ref_logits = oracle.greedy_generate(cfg, model.w, torch.tensor(p), 16)
                ok_tokens &= o.token_ids == ref_tokens.tolist()
                max_err = max(max_err, (first_logits[i] - ref_logits[0]).abs().max().item())
            out_q.put((ok_tokens, max_err, res.stats["decode_steps"]))
        else:
            cache = model.new_cache(nblocks, block, layers=len(stages[rank]))
            stage_worker_loop(model, stages, cache)
    finally:
        dist.destroy_process_group()


def test_two_stage_gloo_pipeline_matches_cpu_forward():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    ok_tokens, max_err, decode_steps = q.get(timeout=5)
    assert ok_tokens
    assert max_err < 1e-4
    assert decode_steps == 15
