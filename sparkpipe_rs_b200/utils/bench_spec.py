"""Speculative-decoding benchmark: a 1-layer MTP-style draft head (same hidden size,
one MLA layer, one dense FFN of width 1408, sharing the target's embedding and LM
head) drafts 3 tokens per sequence, the MLA-MoE target (DeepSeek-V2-Lite shape,
bf16, random N(0, 0.02) weights) verifies all of them in one batched forward, and
acceptance is forced by a seeded Bernoulli(0.7) per draft token so the result does
not depend on the weights. Load: 128 concurrent requests over the box, 512-token
prompts, 512 output tokens.

Reported (one JSON line, rank 0; device time, CUDA events, max over ranks):
  * accepted tokens/s  — committed tokens (accepted drafts + verifier tokens) per second
  * verify tokens/s    — target rows verified per second (B * (L + 1) per round)
  * the spec_finish kernel's device time per round

    python -m sparkpipe_rs_b200.utils.bench_spec [--rounds K] [--warmup W]
    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 -m sparkpipe_rs_b200.utils.bench_spec

``--engine`` serves the same load through the public serving API instead:
``LLMEngine.generate`` with chain speculation (the scheduler's verify plans, one
CUDA graph per verify round, forced acceptance), prompts prefilled by the engine.
It reports committed tokens/s over the decode phase on the device (CUDA events of
every verify round, max over ranks) and end to end (host wall clock of the decode
steps, including the per-round host->device plan copies and the device->host read
of the committed tokens).

With several ranks attention is data-parallel (each rank owns 128 / N requests)
and the target's routed experts are split over the ranks.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="v2_lite")
    ap.add_argument("--requests", type=int, default=128, help="concurrent requests over the box")
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--output", type=int, default=512)
    ap.add_argument("--draft-len", type=int, default=3)
    ap.add_argument("--p-accept", type=float, default=0.7)
    ap.add_argument("--rounds", type=int, default=0, help="timed rounds (default: enough for --output tokens)")
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--engine", action="store_true", help="serve through LLMEngine.generate")
    args = ap.parse_args()
    if args.engine:
        return engine_main(args)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    from sparkpipe_rs_b200 import ops
    from sparkpipe_rs_b200.models.config import get_config
    from sparkpipe_rs_b200.models.mla_moe import ForwardBatch, KVCache, MLAMoEModel
    from sparkpipe_rs_b200.parallel.expert_parallel import ExpertParallel
    from sparkpipe_rs_b200.serving.spec_decode import SpecDecoder, make_draft
    from sparkpipe_rs_b200.utils.clocks import ClockSampler

    cfg = get_config(args.model)
    B = max(1, args.requests // world)
    L, P = args.draft_len, args.prompt
    # expected committed tokens per round under forced acceptance: 1 + p + p^2 + ... + p^L
    per_round = sum(args.p_accept ** i for i in range(L + 1))
    rounds = args.rounds or max(1, math.ceil(args.output / per_round))
    max_ctx = P + (L + 1) * (args.warmup + rounds + 2) + 1
    bs = 64
    bps = math.ceil(max_ctx / bs)
    ep = None
    if world > 1 and cfg.n_routed_experts % world == 0:
        ep = ExpertParallel(cfg, rank, world, max(B * (L + 1), B * P), dev, group=dist.group.WORLD)
    target = MLAMoEModel(cfg, seed=0, device=dev, max_positions=max_ctx + 64, ep=ep)
    draft = make_draft(target, seed=1, max_positions=max_ctx + 64)
    tc = KVCache(cfg, num_blocks=B * bps, block_size=bs, device=dev)
    dc = KVCache(draft.cfg, num_blocks=B * bps, block_size=bs, device=dev)
    bt = torch.arange(B * bps, dtype=torch.int32, device=dev).view(B, bps)
    g = torch.Generator().manual_seed(rank)
    prompts = torch.randint(0, cfg.vocab_size, (B, P), generator=g, dtype=torch.int32)
    ids = prompts.flatten().to(dev)
    pos = torch.arange(P, dtype=torch.int32, device=dev).repeat(B)
    slots = (bt[:, :, None] * bs + torch.arange(bs, device=dev, dtype=torch.int32)).view(B, -1)[:, :P]
    cu = torch.arange(0, (B + 1) * P, P, dtype=torch.int32, device=dev)
    fb = ForwardBatch(mode="prefill", token_ids=ids, positions=pos, slot_mapping=slots.flatten().contiguous(),
                      cu_q=cu, cu_k=cu, max_q=P, logits_idx=(cu[1:] - 1).contiguous())
    first = ops.sample_tokens(target.forward(fb, tc))
    draft.forward(fb, dc)
    sd = SpecDecoder(target, draft, tc, dc, B, L, bps, max_ctx, p_accept=args.p_accept, seed=17,
                     use_graph=not args.no_graph)
    sd.start(first, torch.full((B,), P, dtype=torch.int32), bt)
    c0 = ops.launch_count()
    sd.round()  # eager round (+ graph capture)
    launches_per_round = ops.launch_count() - c0
    for _ in range(args.warmup):
        sd.round()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    before = sd.committed_tokens()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record()
        for _ in range(rounds):
            sd.round()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    committed = sd.committed_tokens() - before
    # spec_finish alone, timed on the same stream (state it advances is discarded after)
    fin_ms = 0.0
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    saved = [t.clone() for t in (sd.tok, sd.pos, sd.ctx, sd.slot)]
    f0.record()
    for _ in range(20):
        ops.kernels().spec_finish(sd.tok, sd.tgt, L, args.p_accept, 17, sd.pos, sd.ctx, sd.slot, sd.bt, bs,
                                  sd.accepted, sd.committed, None)
    f1.record()
    torch.cuda.synchronize()
    fin_ms = f0.elapsed_time(f1) / 20
    for t, v in zip((sd.tok, sd.pos, sd.ctx, sd.slot), saved):
        t.copy_(v)
    vals = torch.tensor([ms, float(committed), fin_ms], dtype=torch.float64, device=dev)
    if dist:
        mx = vals[[0, 2]].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        tot = vals[1:2].clone()
        dist.all_reduce(tot)
        vals = torch.stack([mx[0], tot[0], mx[1]])
    ms_max, committed_all, fin_max = (float(v) for v in vals)
    status = ops.status_word()
    if rank == 0:
        print(json.dumps({
            "metric": "speculative decode accepted tokens/s (box, max over ranks)",
            "value": committed_all / (ms_max / 1000.0),
            "unit": "tokens/s",
            "verify_tokens_per_s": B * world * (L + 1) * rounds / (ms_max / 1000.0),
            "spec_finish_us": fin_max * 1000.0,
            "ms_per_round": ms_max / rounds,
            "accepted_per_round": committed_all / (rounds * B * world),
            "n_gpus": world, "rounds": rounds, "warmup": args.warmup,
            "higher_is_better": True, "dtype": "bf16",
            "data": "synthetic: seeded uniform-random prompt ids, random-init N(0,0.02) weights, forced "
                    f"Bernoulli({args.p_accept}) acceptance",
            "config": {"target": cfg.name, "draft": draft.cfg.name, "draft_len": L, "requests": B * world,
                       "prompt": P, "output": args.output,
                       "parallelism": f"dp{world}-ep{world}" if ep is not None else f"dp{world}"},
            "clocks": clk.summary(), "gpu_launches": launches_per_round * rounds, "kernel_status": status,
        }), flush=True)
    sd.release()
    if dist:
        dist.barrier()
        if ep is not None:
            ep.close()
        dist.destroy_process_group()


def engine_main(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    from sparkpipe_rs_b200 import ops
    from sparkpipe_rs_b200.models.config import get_config
    from sparkpipe_rs_b200.models.mla_moe import MLAMoEModel
    from sparkpipe_rs_b200.parallel.expert_parallel import ExpertParallel
    from sparkpipe_rs_b200.serving.engine import EngineConfig, LLMEngine, SamplingParams
    from sparkpipe_rs_b200.utils.clocks import ClockSampler

    cfg = get_config(args.model)
    B = max(1, args.requests // world)
    L, P = args.draft_len, args.prompt
    max_len = P + args.output + L + 8
    ep = None
    if world > 1 and cfg.n_routed_experts % world == 0:
        ep = ExpertParallel(cfg, rank, world, max(B * (L + 1), B * P), dev, group=dist.group.WORLD)
    model = MLAMoEModel(cfg, seed=0, device=dev, max_positions=max_len + 64, ep=ep)
    buckets = tuple(sorted({b for b in (1, 2, 4, 8, 16, 32, 64, 128) if b < B} | {B}))
    ec = EngineConfig(max_batch=B, block_size=64, max_model_len=max_len, max_prefill_tokens=max(B * P // 4, P),
                      decode_buckets=buckets, speculation="chain", draft_len=L, spec_p_accept=args.p_accept,
                      spec_force=True, use_cuda_graph=not args.no_graph)
    eng = LLMEngine(cfg, ec, model=model, device=dev)
    g = torch.Generator().manual_seed(rank)
    prompts = [torch.randint(0, cfg.vocab_size, (P,), generator=g).tolist() for _ in range(B)]
    # warm-up: a short generation through the same graphs
    eng.generate(prompts[: min(B, 4)], SamplingParams(max_tokens=8, ignore_eos=True))
    eng.device_ms.clear()
    c0 = ops.launch_count()
    with ClockSampler(local) as clk:
        res = eng.generate(prompts, SamplingParams(max_tokens=args.output, ignore_eos=True))
    launches = ops.launch_count() - c0
    st = res.stats
    dev_ms = eng.device_ms.get(3, 0.0) + eng.device_ms.get(2, 0.0)
    vals = torch.tensor([dev_ms, st["decode_seconds"] * 1000.0, float(st["decode_tokens"]), st["ttft_p50_ms"],
                         st["tpot_p50_ms"]], dtype=torch.float64, device=dev)
    if dist:
        mx = vals.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        tot = vals.clone()
        dist.all_reduce(tot)
        vals = torch.stack([mx[0], mx[1], tot[2], mx[3], mx[4]])
    dev_ms, wall_ms, tokens, ttft, tpot = (float(v) for v in vals)
    if rank == 0:
        print(json.dumps({
            "metric": "speculative decode accepted tokens/s through LLMEngine.generate (box, max over ranks)",
            "value": tokens / (dev_ms / 1000.0),
            "unit": "tokens/s",
            "e2e": {"value": tokens / (wall_ms / 1000.0), "unit": "tokens/s",
                    "h2d_bytes_per_step": st["h2d_bytes_per_step"], "d2h_bytes_per_step": st["d2h_bytes_per_step"]},
            "tokens_per_verify_lane": st["tokens_per_verify_lane"], "verify_steps": st["verify_steps"],
            "decode_steps": st["decode_steps"], "ttft_p50_ms": ttft, "tpot_p50_ms": tpot,
            "n_gpus": world, "higher_is_better": True, "dtype": "bf16",
            "data": "synthetic: seeded uniform-random prompt ids, random-init N(0,0.02) weights, forced "
                    f"Bernoulli({args.p_accept}) acceptance",
            "config": {"target": cfg.name, "draft_len": L, "requests": B * world, "prompt": P, "output": args.output,
                       "parallelism": f"dp{world}-ep{world}" if ep is not None else f"dp{world}"},
            "clocks": clk.summary(), "gpu_launches": launches, "kernel_status": ops.status_word(),
        }), flush=True)
    eng.shutdown()
    if dist:
        dist.barrier()
        if ep is not None:
            ep.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
