"""Per-kernel device-time breakdown of one MLA-MoE decode step.

Runs the kernel-backed model eagerly for a few decode steps of a batch with a
given context length and prints, per kernel name, the summed device time per
step (from the CUDA activity trace of torch.profiler) and its share. This is a
diagnostic: the benchmark numbers come from CUDA-event timing without any
profiler attached.

    python -m sparkpipe_rs_b200.utils.profile_decode --batch 64 --ctx 1024

Launched with torch.distributed.run (N processes, one GPU each) it profiles the
expert-parallel model: attention data-parallel, experts split over the ranks,
and every rank prints its own breakdown.
"""
from __future__ import annotations

import argparse
import collections
import datetime
import math
import os

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="v2_lite")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--ctx", type=int, default=1024)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--layers", type=int, default=0, help="override layer count (0 = model default)")
    ap.add_argument("--routed-experts", type=int, default=0,
                    help="override the routed expert count: E / N with the per-GPU batch reproduces the expert "
                         "load and weight bytes of one rank of an N-way expert-parallel run")
    ap.add_argument("--no-trace", action="store_true", help="run the steps without the profiler (for ncu)")
    ap.add_argument("--graph", action="store_true", help="replay the step as one CUDA graph")
    ap.add_argument("--phase-clock", action="store_true",
                    help="report device phase clocks (attention / MLP-MoE / LM head) of the timed replays")
    ap.add_argument("--time", type=int, default=0,
                    help="also time this many graph replays with CUDA events (device ms per step)")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))

    from sparkpipe_rs_b200.models.config import get_config
    from sparkpipe_rs_b200.models.mla_moe import DecodeGraph, KVCache, MLAMoEModel

    cfg = get_config(args.model)
    if args.layers:
        cfg = cfg.replace(num_layers=args.layers)
    if args.routed_experts:
        cfg = cfg.replace(n_routed_experts=args.routed_experts, n_group=1, topk_group=1)
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    ep = None
    if world > 1:
        import torch.distributed as dist
        from sparkpipe_rs_b200.parallel.expert_parallel import ExpertParallel
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        ep = ExpertParallel(cfg, rank, world, args.batch, dev, group=dist.group.WORLD)
    horizon = args.ctx + 2 + args.steps + (args.time + 3 if args.time else 0) + 16  # every position a step reaches
    model = MLAMoEModel(cfg, seed=0, device=dev, max_positions=horizon + 64, ep=ep)
    B, bs = args.batch, 64
    bps = math.ceil(horizon / bs)
    cache = KVCache(cfg, num_blocks=B * bps, block_size=bs, device=dev)
    cache.data.normal_(0, 1)
    bt = torch.arange(B * bps, dtype=torch.int32, device=dev).view(B, bps)

    def start(g):
        # distinct tokens per row, so routing spreads over the experts as in serving
        g.ids.copy_(torch.randint(0, cfg.vocab_size, (B,), generator=torch.Generator().manual_seed(0),
                                  dtype=torch.int32))
        g.block_table.copy_(bt)
        g.pos.fill_(args.ctx)
        g.ctx.fill_(args.ctx + 1)
        g.slots.copy_(bt[:, args.ctx // bs] * bs + args.ctx % bs)

    dg = DecodeGraph(model, cache, B, bps, horizon, use_graph=args.graph, self_advance=True)
    start(dg)
    for _ in range(2):
        dg.run()
    torch.cuda.synchronize()
    if args.time:
        if args.phase_clock:
            from sparkpipe_rs_b200.models.mla_moe import PhaseClock
            model.phase_clock = PhaseClock(dev)
        tg = dg if args.graph else DecodeGraph(model, cache, B, bps, horizon, use_graph=True, self_advance=True)
        start(tg)
        for _ in range(3):
            tg.run()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.time):
            tg.run()
        e1.record()
        torch.cuda.synchronize()
        print(f"[rank {rank}/{world}] graph replay: {e0.elapsed_time(e1) / args.time:.3f} ms per decode step "
              f"(batch {B}, context {args.ctx}, {cfg.num_layers} layers)", flush=True)
        if model.phase_clock is not None:
            # warm-up replays (3) + timed replays, all through the same graph
            rep = model.phase_clock.report(3 + args.time)
            print(f"[rank {rank}/{world}] phase clocks, us per step: " +
                  ", ".join(f"{k} {v:.1f}" for k, v in rep.items()), flush=True)
            model.phase_clock = None
        start(dg)
        if tg is not dg:
            tg.release()
    if args.no_trace:
        for _ in range(args.steps):
            dg.run()
        torch.cuda.synchronize()
        print("ran", args.steps, "decode steps")
    else:
        _trace(args, dg, rank, world, cfg, B)
    if world > 1:  # every path: graphs holding collectives go before the process group
        dg.release()
        torch.distributed.barrier()
        ep.close()
        torch.distributed.destroy_process_group()


def _trace(args, dg, rank, world, cfg, B):
    """Per-kernel device time of ``args.steps`` decode steps from torch.profiler."""
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(args.steps):
            dg.run()
        torch.cuda.synchronize()
    tot = collections.defaultdict(float)
    cnt = collections.defaultdict(int)
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA:
            name = ev.name.split("(")[0].split("<")[0][:60]
            if "gemm_bf16_kernel" in ev.name:
                name = ev.name.split("(")[0][:80]
            tot[name] += ev.device_time_total
            cnt[name] += 1
    all_us = sum(tot.values()) / args.steps
    print(f"[rank {rank}/{world}] decode step: batch {B}, context {args.ctx}, layers {cfg.num_layers}: "
          f"{all_us / 1000:.3f} ms of kernel time per step")
    print(f"{'kernel':80s} {'us/step':>10s} {'share':>7s} {'launches/step':>14s}")
    for name, us in sorted(tot.items(), key=lambda kv: -kv[1]):
        print(f"{name:80s} {us / args.steps:10.1f} {100 * us / args.steps / all_us:6.1f}% "
              f"{cnt[name] / args.steps:14.1f}")


if __name__ == "__main__":
    main()
