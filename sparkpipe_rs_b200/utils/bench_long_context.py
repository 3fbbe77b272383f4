"""Long-context benchmark through the public engine API (``LLMEngine.generate``).

Request A: one 131072-token prompt of seeded uniform-random ids, chunked prefill in
8192-token chunks (each chunk attends to every earlier chunk through the paged
latent KV cache), then 256 greedy decode tokens at ~131K context. Request B: a
prompt that shares A's first 65536 tokens (then 65536 new ones), submitted after A
finished, so its shared prefix comes from the prefix cache (64-token blocks) and
only the new half is prefilled.

Reported (one JSON line): TTFT of A and B, prefill tokens actually computed for
each (B's shows the prefix-cache hit), prefill throughput, decode TPOT at long
context, and the per-step host<->device bytes. Wall-clock timing of the engine
(host loop included), as a serving user sees it.

    python -m sparkpipe_rs_b200.utils.bench_long_context [--model v2_lite] [--prompt 131072]

Under torchrun (one process per GPU) the model runs expert-parallel (attention
data-parallel, routed experts split over the ranks): rank 0 serves both requests and
the other ranks step in lockstep with idle forwards, supplying their experts. The
1T Kimi-K2-shape config runs this way on 8 GPUs:

    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \
        -m sparkpipe_rs_b200.utils.bench_long_context --model k2
"""
from __future__ import annotations

import argparse
import json
import math

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="v2_lite")
    ap.add_argument("--prompt", type=int, default=131072)
    ap.add_argument("--shared", type=int, default=65536)
    ap.add_argument("--output", type=int, default=256)
    ap.add_argument("--chunk", type=int, default=8192)
    args = ap.parse_args()
    from sparkpipe_rs_b200.models.config import get_config
    from sparkpipe_rs_b200.models.mla_moe import MLAMoEModel
    from sparkpipe_rs_b200.serving.engine import EngineConfig, LLMEngine, SamplingParams
    from sparkpipe_rs_b200.utils.clocks import ClockSampler

    import datetime
    import os

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    cfg = get_config(args.model)
    P, S, out = args.prompt, args.shared, args.output
    max_len = P + out + 64
    bs = 64
    ep = None
    if world > 1:
        import torch.distributed as dist
        from sparkpipe_rs_b200.parallel.expert_parallel import ExpertParallel

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
        ep = ExpertParallel(cfg, rank, world, args.chunk, dev, group=dist.group.WORLD)
    model = MLAMoEModel(cfg, seed=0, device=dev, max_positions=max_len + 64, ep=ep)
    # request A's whole context plus request B's new part: B reuses A's prefix blocks
    # from the prefix cache, and A's other cached blocks are evicted as B needs room
    blocks = math.ceil(max_len / bs) + math.ceil((P - S + out) / bs) + 64
    engine = LLMEngine(cfg, EngineConfig(max_batch=2, block_size=bs, max_model_len=max_len, num_blocks=blocks,
                                         max_prefill_tokens=args.chunk, use_cuda_graph=True, prefix_caching=True),
                       model=model, device=dev)
    g = torch.Generator().manual_seed(0)
    a = torch.randint(0, cfg.vocab_size, (P,), generator=g, dtype=torch.int32).tolist()
    b = a[:S] + torch.randint(0, cfg.vocab_size, (P - S,), generator=g, dtype=torch.int32).tolist()
    params = SamplingParams(max_tokens=out, temperature=0.0, ignore_eos=True)
    mine = rank == 0  # rank 0 serves the requests; the others run idle lockstep forwards
    with ClockSampler(dev.index or 0) as clk:
        ra = engine.generate([a] if mine else [], params)
        rb = engine.generate([b] if mine else [], params)
    if not mine:
        engine.shutdown()
        _finish(world, ep)
        return
    sa, sb = ra.stats, rb.stats
    print(json.dumps({
        "metric": "long-context serving (TTFT ms, prefill tokens/s, TPOT ms)",
        "model": cfg.name, "prompt": P, "shared_prefix": S, "output": out, "prefill_chunk": args.chunk,
        "request_a": {"ttft_ms": sa["ttft_p50_ms"], "tpot_ms": sa["tpot_p50_ms"],
                      "prefill_tokens_computed": sa["prefill_tokens"],
                      "prefill_tokens_per_s": sa["prefill_tokens"] / max(sa["prefill_seconds"], 1e-9),
                      "decode_tokens_per_s": sa["decode_tokens_per_s"]},
        "request_b": {"ttft_ms": sb["ttft_p50_ms"], "tpot_ms": sb["tpot_p50_ms"],
                      "prefill_tokens_computed": sb["prefill_tokens"],
                      "prefill_tokens_per_s": sb["prefill_tokens"] / max(sb["prefill_seconds"], 1e-9)},
        "prefix_cache_tokens_reused_by_b": P - sb["prefill_tokens"],
        "h2d_bytes_per_step": sa["h2d_bytes_per_step"], "d2h_bytes_per_step": sa["d2h_bytes_per_step"],
        "dtype": "bf16" if cfg.weight_dtype != "fp8_block" else "fp8",
        "data": "synthetic: seeded uniform-random prompt ids, random-init N(0,0.02) weights",
        "timing": "wall clock around LLMEngine.generate (host scheduling included)",
        "clocks": clk.summary(),
        "n_gpus": world, "parallelism": f"dp{world}-ep{world}" if world > 1 else "1 GPU",
    }), flush=True)
    engine.shutdown()
    _finish(world, ep)


def _finish(world, ep):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        ep.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
