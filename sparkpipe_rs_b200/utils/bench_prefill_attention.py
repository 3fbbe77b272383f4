"""Micro-benchmark of the chunked MLA prefill attention kernels.

One query chunk of `--q` tokens of `--heads` heads (q_nope 128 + rope 64, v 128)
against Tk keys (a cached prefix plus the chunk; causal on the diagonal), for each
Tk in `--k`. CUDA-event time per call after a warm-up call, and TFLOP/s counted as
(query-key pairs) x heads x (2 x 192 + 2 x 128).

    python -m sparkpipe_rs_b200.utils.bench_prefill_attention --q 8192 --k 8192,32768,131072 --impl tc,mma
"""
from __future__ import annotations

import argparse
import math

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--q", type=int, default=8192)
    ap.add_argument("--k", default="8192,32768,131072")
    ap.add_argument("--heads", type=int, default=16)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--impl", default="tc,mma")
    args = ap.parse_args()
    from sparkpipe_rs_b200 import ops

    dev = torch.device("cuda", 0)
    H, Tq = args.heads, args.q
    for Tk in [int(x) for x in args.k.split(",")]:
        q = torch.randn(Tq, H, 192, device=dev).bfloat16()
        kv = torch.randn(Tk, H, 256, device=dev).bfloat16()
        kpe = torch.randn(Tk, 576, device=dev).bfloat16()[:, 512:]
        o = torch.empty(Tq, H, 128, device=dev, dtype=torch.bfloat16)
        cu_q = torch.tensor([0, Tq], device=dev, dtype=torch.int32)
        cu_k = torch.tensor([0, Tk], device=dev, dtype=torch.int32)
        pairs = Tq * Tk - Tq * (Tq - 1) / 2
        for impl in args.impl.split(","):
            def run():
                ops.prefill_attention(q, kv[:, :, :128], kpe, kv[:, :, 128:], o, cu_q, cu_k, Tq, 1 / math.sqrt(192),
                                      impl=impl)
            run()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(args.iters):
                run()
            b.record()
            torch.cuda.synchronize()
            ms = a.elapsed_time(b) / args.iters
            print(f"prefill_attention[{impl}] Tq={Tq} Tk={Tk} H={H}: {ms:8.2f} ms  "
                  f"{pairs * H * 640 / ms / 1e9:7.1f} TFLOP/s", flush=True)
        del q, kv, kpe, o
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
