#!/usr/bin/env python
"""Decode-throughput benchmark of the MLA-MoE serving engine on B200.

Workload (one replica per GPU, weak scaling): DeepSeek-V2-Lite-shape MLA-MoE in
bf16 with random N(0, 0.02) weights; 64 concurrent requests per GPU with
1024-token synthetic prompts (seeded uniform ids), greedy decoding, paged
latent KV in 64-token blocks.

Two numbers are reported:
  * ``value`` — device-timed decode throughput: K decode steps of the whole
    batch (one CUDA graph per step: 27 layers + lm_head + sampling + input
    advance), CUDA events on the launching stream, max over ranks.
  * ``e2e`` — the same metric end to end through the public engine API
    (``LLMEngine.generate``): every step copies its inputs host->device from
    pinned memory and reads the sampled tokens back, plus p50 TTFT / TPOT.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
For N > 1 launch one process per GPU with torch.distributed.run.

``--model k2`` runs the 1T Kimi-K2-shape workload instead: block-scaled fp8
weights (128x128 e4m3 blocks, fp32 scales), 256 concurrent requests over the
box, 2048-token prompts, 512 output tokens, attention data-parallel and the 384
routed experts split over the GPUs (8 GPUs hold the 1T parameters).
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import sys
import time

METRIC = "decode tokens/s (box, max over ranks)"
PUBLISHED_BASELINE = None  # the reference publishes no B200 (or comparable) number


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default="v2_lite")
    ap.add_argument("--batch", type=int, default=0,
                    help="concurrent requests per GPU (default: 64 for v2_lite; 256 over the box for k2)")
    ap.add_argument("--prompt", type=int, default=0, help="prompt tokens (default 1024; 2048 for k2)")
    ap.add_argument("--output", type=int, default=0, help="output tokens (default 256; 512 for k2)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--parallel", default="auto", choices=["auto", "dp", "ep"],
                    help="N>1: dp = replicated model per GPU; ep = data-parallel attention + experts split "
                         "over the GPUs (auto: ep when the experts divide evenly)")
    ap.add_argument("--layers", type=int, default=0,
                    help="diagnostic only: run the first N layers (a result with it is not the named workload)")
    ap.add_argument("--prefill-chunk", type=int, default=0,
                    help="max tokens per prefill forward (default 8192; 2048 for k2)")
    ap.add_argument("--weights-pack", default="",
                    help="load the model's weights from this stage-pack checkpoint directory (written first, "
                         "from the seeded random init, when it has no index yet)")
    return ap.parse_args()


def reference_arm(args):
    print(json.dumps({
        "impl": "reference",
        "unavailable": "the reference is a Rust Cargo workspace: pip reports it is not installable (no setup.py or "
                       "pyproject.toml), this image has no Rust toolchain, and its GPU kernels are not in its tree",
        "metric": METRIC, "n_gpus": args.gpus,
    }))


def load_weights_pack(root, cfg, dev, ep, rank, world):
    """This rank's weights from a stage pack (an expert-parallel rank reads only its
    experts); rank 0 writes the pack from the seeded random init if it has none."""
    import os as _os

    import torch
    import torch.distributed as dist

    from sparkpipe_rs_b200.core import core
    from sparkpipe_rs_b200.models.checkpoint import load_pack, save_pack
    from sparkpipe_rs_b200.models.weights import init_weights

    index = _os.path.join(root, core().stagepack.INDEX_FILE)
    if rank == 0 and not _os.path.exists(index):
        save_pack(root, cfg, init_weights(cfg, seed=0, device=dev, dtype=torch.bfloat16))
        torch.cuda.empty_cache()
    if world > 1:
        dist.barrier()
    return load_pack(root, cfg, device=dev, experts=ep.local_expert_range() if ep is not None else None)


def main():
    args = parse_args()
    if args.impl == "reference":
        reference_arm(args)
        return 0

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    from sparkpipe_rs_b200 import ops
    from sparkpipe_rs_b200.models.config import get_config
    from sparkpipe_rs_b200.models.mla_moe import DecodeGraph, ForwardBatch, KVCache, MLAMoEModel
    from sparkpipe_rs_b200.parallel.expert_parallel import ExpertParallel
    from sparkpipe_rs_b200.utils.clocks import ClockSampler

    cfg = get_config(args.model)
    if args.layers:
        cfg = cfg.replace(num_layers=args.layers)
    big = cfg.weight_dtype == "fp8_block"  # the 1T fp8 workload: 256 requests over the box, 2048 in / 512 out
    args.batch = args.batch or (max(1, 256 // world) if big else 64)
    args.prompt = args.prompt or (2048 if big else 1024)
    args.output = args.output or (512 if big else 256)
    args.prefill_chunk = args.prefill_chunk or (2048 if big else 8192)
    B, P = args.batch, args.prompt
    bs = 64
    par = args.parallel
    if par == "auto":
        par = "ep" if world > 1 and cfg.n_routed_experts % world == 0 else "dp"
    seqs_per_chunk = max(1, min(B, args.prefill_chunk // P))
    ep = None
    if par == "ep" and world > 1:
        ep = ExpertParallel(cfg, rank, world, max(B, seqs_per_chunk * P), dev, group=dist.group.WORLD)
    torch.manual_seed(1234 + rank)
    weights = None
    if args.weights_pack:
        weights = load_weights_pack(args.weights_pack, cfg, dev, ep, rank, world)
    model = MLAMoEModel(cfg, weights=weights, seed=0, device=dev,
                        max_positions=P + args.output + args.warmup + args.steps + 64, ep=ep)
    del weights
    def _nbytes(t):
        if isinstance(t, ops.Fp8Weight):
            return t.q.numel() + t.s.numel() * 4
        return t.numel() * t.element_size()

    weight_gb = sum(_nbytes(t) for t in model.w.values()) / 1e9
    parallelism = f"dp{world}-ep{world}" if ep is not None else f"dp{world}"

    # ------------------------------------------------------------ device-timed decode
    # the timed steps start at context P; a second timed window runs at mid-output context
    mid_start = max(P + args.warmup + args.steps, P + args.output // 2)
    total_ctx = mid_start + args.steps + 2
    bps = math.ceil(total_ctx / bs)
    cache = KVCache(cfg, num_blocks=B * bps, block_size=bs, device=dev)
    block_table = torch.arange(B * bps, dtype=torch.int32, device=dev).view(B, bps)
    g = torch.Generator(device="cpu").manual_seed(rank)
    prompts = torch.randint(0, cfg.vocab_size, (B, P), generator=g, dtype=torch.int32)
    slots = (block_table[:, :, None] * bs + torch.arange(bs, device=dev, dtype=torch.int32)).view(B, -1)[:, :P]
    first = torch.empty(B, dtype=torch.int32, device=dev)
    for b0 in range(0, B, seqs_per_chunk):  # prefill in chunks of whole prompts
        nb = min(seqs_per_chunk, B - b0)
        ids = prompts[b0:b0 + nb].flatten().to(dev)
        pos = torch.arange(P, dtype=torch.int32, device=dev).repeat(nb)
        cu = torch.arange(0, (nb + 1) * P, P, dtype=torch.int32, device=dev)
        fb = ForwardBatch(mode="prefill", token_ids=ids, positions=pos,
                          slot_mapping=slots[b0:b0 + nb].flatten().contiguous(), cu_q=cu, cu_k=cu, max_q=P,
                          logits_idx=(cu[1:] - 1).contiguous())
        logits = model.forward(fb, cache)
        first[b0:b0 + nb] = ops.sample_tokens(logits)
        del logits, fb
    torch.cuda.synchronize()

    graph = DecodeGraph(model, cache, B, bps, total_ctx, use_graph=not args.no_graph, self_advance=True)
    # inputs of the first decode step
    graph.ids.copy_(first)
    graph.pos.fill_(P)
    graph.ctx.fill_(P + 1)
    graph.block_table.copy_(block_table)
    graph.slots.copy_(block_table[:, P // bs] * bs + P % bs)
    # count this package's kernels of one step (eager replay of the same ops)
    c0 = ops.launch_count()
    graph._step()
    per_step_launches = ops.launch_count() - c0
    # reset to the first step's inputs after the counting step
    graph.ids.copy_(first)
    graph.pos.fill_(P)
    graph.ctx.fill_(P + 1)
    graph.slots.copy_(block_table[:, P // bs] * bs + P % bs)
    for _ in range(args.warmup):
        graph.run()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record()
        for _ in range(args.steps):
            graph.run()
        e1.record()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    status = ops.status_word()
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    value = B * world * args.steps / (ms_max / 1000.0)
    # the same steps at mid-output context (untimed advance, then one more timed window)
    for _ in range(mid_start - (P + args.warmup + args.steps)):
        graph.run()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    m0, m1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    m0.record()
    for _ in range(args.steps):
        graph.run()
    m1.record()
    torch.cuda.synchronize()
    tm = torch.tensor([m0.elapsed_time(m1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
    ms_mid = float(tm.item())
    mid = {"context": mid_start + 1, "ms_per_step": ms_mid / args.steps,
           "value": B * world * args.steps / (ms_mid / 1000.0)}
    graph.release()
    del graph, cache
    torch.cuda.empty_cache()

    # ------------------------------------------------------------ end to end (public API)
    e2e = None
    if not args.no_e2e:
        from sparkpipe_rs_b200.serving.engine import EngineConfig, LLMEngine, SamplingParams

        engine = LLMEngine(cfg, EngineConfig(max_batch=B, block_size=bs, max_model_len=P + args.output + 64,
                                             num_blocks=B * math.ceil((P + args.output + 64) / bs) + 64,
                                             max_prefill_tokens=seqs_per_chunk * P,
                                             use_cuda_graph=not args.no_graph),
                           model=model, device=dev)
        prompts_l = [p.tolist() for p in prompts]
        res = engine.generate(prompts_l, SamplingParams(max_tokens=args.output, temperature=0.0,
                                                        ignore_eos=True))
        stats = res.stats
        vals = torch.tensor([stats["decode_tokens"], stats["decode_seconds"], stats["ttft_p50_ms"],
                             stats["tpot_p50_ms"]], dtype=torch.float64, device=dev)
        if world > 1:
            tok = vals[0:1].clone()
            dist.all_reduce(tok)
            mx = vals[1:].clone()
            dist.all_reduce(mx, op=dist.ReduceOp.MAX)
            vals = torch.cat([tok, mx])
        e2e = {"value": float(vals[0] / vals[1]), "unit": "tokens/s",
               "h2d_bytes_per_step": stats["h2d_bytes_per_step"], "d2h_bytes_per_step": stats["d2h_bytes_per_step"],
               "ttft_p50_ms": float(vals[2]), "tpot_p50_ms": float(vals[3]),
               "requests": B * world, "prompt_len": P, "output_len": args.output,
               "api": "LLMEngine.generate",
               "prefill_steps": stats["prefill_steps"], "prefill_ms_per_step":
                   1000.0 * stats["prefill_seconds"] / max(1, stats["prefill_steps"]),
               "prefill_tokens_per_s": stats["prefill_tokens"] / max(1e-9, stats["prefill_seconds"])}
        engine.shutdown()

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_max / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": (value / PUBLISHED_BASELINE) if PUBLISHED_BASELINE else None,
            "dtype": ("fp8 (e4m3 128x128-block weights, 1x128-block activations, fp32 accumulate; bf16 attention "
                      "and KV)") if cfg.weight_dtype == "fp8_block" else "bf16",
            "data": "synthetic: seeded uniform-random prompt ids, random-init N(0,0.02) weights",
            "config": {
                "model": f"{cfg.name} ({cfg.num_layers} layers, hidden {cfg.hidden_size}, "
                         f"{cfg.n_routed_experts} experts top-{cfg.num_experts_per_tok} + {cfg.n_shared_experts} shared)",
                "global_batch": B * world,
                "seq_len": P,
                "output_len": args.output,
                "kv_block": bs,
                "parallelism": parallelism,
                "l2": f"inputs larger than L2: each decode step streams {weight_gb:.1f} GB of weights per GPU",
            },
            "clocks": clk.summary(),
            "gpu_launches": per_step_launches * args.steps,
            "kernel_status": status,
            "impl": "ours",
        }
        if e2e is not None:
            line["e2e"] = e2e
        line["mid_output"] = mid
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        if ep is not None:
            ep.close()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
