"""Micro-benchmark of the tcgen05 linear op on decode / prefill shapes.

Captures `iters` back-to-back launches of ``ops.linear`` (and torch.matmul as a
cuBLAS reference) into one CUDA graph and times its replay with CUDA events,
so the figures are device time per launch (host launch overhead excluded, as
in the graph-replayed decode step). Prints achieved weight bandwidth (TB/s)
and TFLOP/s for each (tokens, out_features, in_features) shape and split-K
setting. Weight matrices are cycled from a pool larger than L2 so every launch
streams its weights from HBM.

    python -m sparkpipe_rs_b200.utils.bench_gemm --shapes 64x2048x2048,64x3648x2048 --splits 0,1,2,4,8
"""
from __future__ import annotations

import argparse

import torch


def parse_shapes(s: str):
    out = []
    for part in s.split(","):
        t, o, k = (int(x) for x in part.lower().split("x"))
        out.append((t, o, k))
    return out


def time_fn(fn, iters: int) -> float:
    for i in range(3):
        fn(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for i in range(iters):
                fn(i)
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) / iters * 1e3  # us


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default="64x2048x2048,64x3648x2048,64x64x2048,64x2048x10944,64x102400x2048")
    ap.add_argument("--splits", default="0,1,2,4,8")
    ap.add_argument("--iters", type=int, default=100)
    ap.add_argument("--pool-mb", type=int, default=512, help="weight pool size (> L2) cycled across launches")
    args = ap.parse_args()
    from sparkpipe_rs_b200 import ops

    dev = torch.device("cuda", 0)
    for (T, O, K) in parse_shapes(args.shapes):
        wbytes = O * K * 2
        n_pool = max(1, min(64, (args.pool_mb << 20) // wbytes))
        ws = [torch.randn(O, K, device=dev).mul_(0.02).bfloat16() for _ in range(n_pool)]
        x = torch.randn(T, K, device=dev).bfloat16()
        out = torch.empty(T, O, device=dev, dtype=torch.bfloat16)
        flops = 2.0 * T * O * K
        for sp in [int(v) for v in args.splits.split(",")]:
            us = time_fn(lambda i: ops.linear(x, ws[i % n_pool], out=out, splits=sp), args.iters)
            print(f"linear T={T:5d} O={O:6d} K={K:6d} splits={sp}: {us:8.2f} us  "
                  f"{wbytes / us / 1e6:6.2f} TB/s  {flops / us / 1e6:8.1f} TFLOP/s")
        # the model's form at decode: partial slabs left for the consuming kernel (one launch)
        us = time_fn(lambda i: ops.linear_slabs(x, ws[i % n_pool], out_dtype=torch.float32), args.iters)
        print(f"linear_slabs T={T:5d} O={O:6d} K={K:6d}: {us:8.2f} us  {wbytes / us / 1e6:6.2f} TB/s")
        us = time_fn(lambda i: torch.matmul(x, ws[i % n_pool].t(), out=out), args.iters)
        print(f"torch.matmul (cuBLAS) T={T:5d} O={O:6d} K={K:6d}: {us:8.2f} us  {wbytes / us / 1e6:6.2f} TB/s  "
              f"{flops / us / 1e6:8.1f} TFLOP/s")
        del ws
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
