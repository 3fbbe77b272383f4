"""Per-phase and per-kernel device time of one MLA-MoE prefill chunk.

One chunk of ``--seqs`` prompts of ``--len`` tokens (default 8 x 1,024 = 8,192
tokens, the V2-Lite shape) runs eagerly through the kernel-backed model:

  * the chunk's device time (CUDA events around the forward, after warm-up) and
    tokens/s;
  * device phase clocks (embedding, attention, MLP / MoE, LM head), summed over
    layers;
  * per kernel name, the summed device time from the CUDA activity trace of
    torch.profiler (a diagnostic run after the timed ones), with the algorithmic
    FLOPs and TFLOP/s of the GEMM families against the measured sustained bf16 peak
    (``--peak-tflops``, default the driver-measured 1,385.6).

    python -m sparkpipe_rs_b200.utils.profile_prefill --seqs 8 --len 1024

(the model in the profiled process is the only one on the device; ``--layers 2`` keeps
an ncu capture small: one dense and one MoE layer)
"""
from __future__ import annotations

import argparse
import collections
import json
import os

import torch


def gemm_flops(cfg, tokens: int, seq_len: int) -> dict:
    """Algorithmic FLOPs of one prefill chunk by family (2 per multiply-add)."""
    H, nh = cfg.hidden_size, cfg.num_heads
    dn, dr, dv, kvl = cfg.qk_nope_head_dim, cfg.qk_rope_head_dim, cfg.v_head_dim, cfg.kv_lora_rank
    qa = cfg.q_lora_rank or nh * (dn + dr)
    attn_proj = H * (qa + kvl + dr) + (cfg.q_lora_rank * nh * (dn + dr) if cfg.q_lora_rank else 0) \
        + kvl * nh * (dn + dv) + nh * dv * H
    moe_layers = sum(1 for i in range(cfg.num_layers) if cfg.is_moe_layer(i))
    dense_layers = cfg.num_layers - moe_layers
    inter = cfg.moe_intermediate_size
    routed = cfg.num_experts_per_tok * 3 * H * inter
    shared = cfg.n_shared_experts * 3 * H * inter
    dense = 3 * H * cfg.intermediate_size
    # causal attention over each sequence: QK^T (dn + dr) and PV (dv) per head, half the square
    attn_core = nh * (dn + dr + dv) * seq_len / 2
    return {
        "attention projections": 2 * tokens * attn_proj * cfg.num_layers,
        "attention (causal QK^T, PV)": 2 * tokens * attn_core * cfg.num_layers,
        "routed experts": 2 * tokens * routed * moe_layers,
        "shared experts": 2 * tokens * shared * moe_layers,
        "dense FFN": 2 * tokens * dense * dense_layers,
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="v2_lite")
    ap.add_argument("--seqs", type=int, default=8)
    ap.add_argument("--len", type=int, default=1024)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (small ncu cases)")
    ap.add_argument("--peak-tflops", type=float, default=1385.6)
    ap.add_argument("--no-trace", action="store_true", help="skip the profiler pass (for ncu)")
    args = ap.parse_args()
    from sparkpipe_rs_b200.models.config import get_config
    from sparkpipe_rs_b200.models.mla_moe import ForwardBatch, KVCache, MLAMoEModel, PhaseClock

    cfg = get_config(args.model)
    if args.layers:
        cfg = cfg.replace(num_layers=args.layers)
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    S, L = args.seqs, args.len
    T = S * L
    model = MLAMoEModel(cfg, seed=0, device=dev, max_positions=L + 64)
    bps = -(-L // 64)
    cache = KVCache(cfg, num_blocks=S * bps, block_size=64, device=dev)
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, cfg.vocab_size, (T,), generator=g, dtype=torch.int32).to(dev)
    pos = torch.arange(L, dtype=torch.int32, device=dev).repeat(S)
    slots = (torch.arange(S, dtype=torch.int32, device=dev)[:, None] * (bps * 64) + torch.arange(L, device=dev,
                                                                                                  dtype=torch.int32))
    cu = torch.arange(0, T + 1, L, dtype=torch.int32, device=dev)
    fb = ForwardBatch(mode="prefill", token_ids=ids, positions=pos, slot_mapping=slots.flatten().contiguous(),
                      cu_q=cu, cu_k=cu, max_q=L, logits_idx=(cu[1:] - 1).contiguous())
    for _ in range(2):
        model.forward(fb, cache)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.iters):
        model.forward(fb, cache)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.iters
    model.phase_clock = PhaseClock(dev)
    for _ in range(args.iters):
        model.forward(fb, cache)
    torch.cuda.synchronize()
    phases = model.phase_clock.report(args.iters)
    model.phase_clock = None
    fl = gemm_flops(cfg, T, L)
    total = sum(fl.values())
    out = {"chunk_tokens": T, "seqs": S, "seq_len": L, "layers": cfg.num_layers, "ms": ms,
           "tokens_per_s": T / (ms / 1e3), "algorithmic_tflop": total / 1e12,
           "achieved_tflops": total / (ms / 1e3) / 1e12,
           "fraction_of_sustained_peak": total / (ms / 1e3) / 1e12 / args.peak_tflops,
           "phase_us": phases, "family_gflop": {k: v / 1e9 for k, v in fl.items()}}
    print(json.dumps(out), flush=True)
    if args.no_trace:
        return
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        model.forward(fb, cache)
        torch.cuda.synchronize()
    tot = collections.defaultdict(float)
    cnt = collections.defaultdict(int)
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA:
            name = ev.name.split("(")[0][:90]
            tot[name] += ev.device_time_total
            cnt[name] += 1
    all_us = sum(tot.values())
    print(f"prefill chunk {T} tokens: {all_us / 1000:.3f} ms of kernel time (profiler)")
    print(f"{'kernel':90s} {'us':>10s} {'share':>7s} {'launches':>9s}")
    for name, us in sorted(tot.items(), key=lambda kv: -kv[1])[:40]:
        print(f"{name:90s} {us:10.1f} {100 * us / all_us:6.1f}% {cnt[name]:9d}")


if __name__ == "__main__":
    main()
