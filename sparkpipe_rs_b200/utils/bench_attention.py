"""Micro-benchmark of the MLA paged decode attention kernel.

Captures `iters` launches (attention + split-KV combine) into a CUDA graph and
times the replay with CUDA events: device time per call, achieved KV-cache
bandwidth against the bytes that must be read (context x 576 x 2 bytes per
sequence). Sweeps the split-KV factor.

    python -m sparkpipe_rs_b200.utils.bench_attention --batch 64 --heads 16 --ctx 1024 --splits 1,2,3,4,6,8
"""
from __future__ import annotations

import argparse
import math

import torch

from .bench_gemm import time_fn


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--heads", type=int, default=16)
    ap.add_argument("--ctx", type=int, default=1024)
    ap.add_argument("--splits", default="0,1,2,3,4,5,6,8")
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--trace", action="store_true",
                    help="sk only: print the kernel's device event trace of four CTAs (one eager launch)")
    ap.add_argument("--impl", default="sk,mma", help="kernels to time: sk (stream-K), tc (tcgen05 split-KV), "
                                                      "mma (mma.sync split-KV), fp8 (split-KV over the fp8 e4m3 "
                                                      "cache with per-128 block scales)")
    args = ap.parse_args()
    from sparkpipe_rs_b200 import ops

    dev = torch.device("cuda", 0)
    B, H, L = args.batch, args.heads, args.ctx
    bpseq = math.ceil(L / 64)
    # several cache copies so consecutive launches stream from HBM, not L2
    n_caches = max(1, min(8, (1 << 30) // (B * bpseq * 64 * 576 * 2)))
    caches = [torch.randn(B * bpseq * 64, 576, device=dev).bfloat16() for _ in range(n_caches)]
    bt = torch.randperm(B * bpseq, device=dev).int().view(B, bpseq)
    ctx = torch.full((B,), L, device=dev, dtype=torch.int32)
    q = torch.randn(B, H, 576, device=dev).bfloat16()
    out = torch.empty(B, H, 512, device=dev, dtype=torch.bfloat16)
    nbytes = B * L * 576 * 2
    scale = 1 / math.sqrt(192)
    impls = args.impl.split(",")
    if "fp8" in impls:  # the same rows quantised: e4m3 values, amax / 448 per 128-element block
        caches8 = []
        for c in caches:
            xp = torch.zeros(c.shape[0], 640, device=dev)
            xp[:, :576] = c.float()
            amax = xp.view(-1, 5, 128).abs().amax(-1)
            inv = torch.where(amax > 0, 448.0 / amax, torch.zeros_like(amax))
            q8 = (xp.view(-1, 5, 128) * inv[..., None]).view(-1, 640)[:, :576].to(torch.float8_e4m3fn)
            caches8.append((q8.view(torch.uint8).contiguous(), (amax / 448.0).contiguous()))
            del xp
    for impl in impls:
        if impl == "fp8":
            nb8 = B * L * (576 + 20)
            for sp in [int(s) for s in args.splits.split(",")]:
                splits = sp or ops.mla_decode_splits(B, H, L, ops.kernels().num_sms(), kv_fp8=True)
                o_part = torch.empty(B, splits, H, 512, device=dev, dtype=torch.float32)
                lse = torch.empty(B, splits, H, device=dev, dtype=torch.float32)
                us = time_fn(lambda i: ops.mla_decode(q, caches8[i % n_caches][0], bt, ctx, out, splits, scale, o_part,
                                                      lse, kv_scales=caches8[i % n_caches][1]), args.iters)
                print(f"mla_decode[fp8] B={B} H={H} ctx={L} splits={splits}{' (auto)' if sp == 0 else ''}: "
                      f"{us:8.2f} us  {nb8 / us / 1e6:6.2f} TB/s of KV ({nbytes / us / 1e6:6.2f} bf16-equivalent)")
            continue
        if impl == "sk":  # one schedule over all SMs: no split factor
            ops.mla_decode(q, caches[0], bt, ctx, out, 1, scale, impl="sk")  # sizes the scratch outside capture
            us = time_fn(lambda i: ops.mla_decode(q, caches[i % n_caches], bt, ctx, out, 1, scale, impl="sk"),
                         args.iters)
            print(f"mla_decode[sk] B={B} H={H} ctx={L}: {us:8.2f} us  {nbytes / us / 1e6:6.2f} TB/s of KV")
            if args.trace:
                tr = torch.zeros(4 * 64, dtype=torch.int64, device=dev)
                ops.mla_decode(q, caches[0], bt, ctx, out, 1, scale, impl="sk")
                ops.mla_decode(q, caches[-1], bt, ctx, out, 1, scale, impl="sk", trace=tr)
                torch.cuda.synchronize()
                t = tr.view(4, 64).cpu()
                t0 = int(t[t > 0].min())
                names = {0: "start", 1: "sched", 2: "dep", 60: "merge0", 61: "merge1", 63: "end"}
                for c in range(4):
                    row = []
                    for i in range(64):
                        if int(t[c, i]) > 0:
                            nm = names.get(i, f"q{(i - 3) // 2}" if 3 <= i < 19 and i % 2 == 1 else
                                           f"p{(i - 4) // 2}" if 4 <= i < 20 else f"s{i - 20}")
                            row.append(f"{nm}:{(int(t[c, i]) - t0) / 1000:.1f}")
                    print(f"  trace cta#{c}: " + " ".join(row))
            continue
        for sp in [int(s) for s in args.splits.split(",")]:
            splits = sp or ops.mla_decode_splits(B, H, L, ops.kernels().num_sms(), impl=impl)
            o_part = torch.empty(B, splits, H, 512, device=dev, dtype=torch.float32)
            lse = torch.empty(B, splits, H, device=dev, dtype=torch.float32)
            us = time_fn(lambda i: ops.mla_decode(q, caches[i % n_caches], bt, ctx, out, splits, scale, o_part, lse,
                                                  impl=impl), args.iters)
            print(f"mla_decode[{impl}] B={B} H={H} ctx={L} splits={splits}{' (auto)' if sp == 0 else ''}: "
                  f"{us:8.2f} us  {nbytes / us / 1e6:6.2f} TB/s of KV")


if __name__ == "__main__":
    main()
