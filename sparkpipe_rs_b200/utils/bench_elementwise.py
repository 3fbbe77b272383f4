"""Bandwidth of the memory-bound kernels against the measured HBM copy bandwidth.

Each kernel runs on prefill-sized inputs (8,192 rows by default) rotated over four
copies so consecutive launches stream from HBM, not L2; 50 launches per CUDA graph,
CUDA events around a replay. Bytes are the algorithmic ones (every input read once,
every output written once):

  * add_rmsnorm       residual += x; out = rmsnorm(residual) * gamma   (hidden 2,048)
  * mla_kv_write      latent RMSNorm + rope-key RoPE -> paged cache rows and bf16 rows (576)
  * mla_kv_write fp8  the same into the fp8 cache (e4m3 rows + 5 block scales)
  * quant_fp8_block   bf16 activations -> e4m3 + one scale per 128 (hidden 7,168)
  * rope_q            query RoPE in place (16 heads x 64 rope dims of 192)

    python -m sparkpipe_rs_b200.utils.bench_elementwise [--rows 8192] [--hbm-gbs 6545.3]
"""
from __future__ import annotations

import argparse

import torch

from .bench_gemm import time_fn


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=8192)
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--hbm-gbs", type=float, default=6545.3, help="measured HBM copy bandwidth (GB/s)")
    args = ap.parse_args()
    from sparkpipe_rs_b200 import ops
    from sparkpipe_rs_b200.models.config import v2_lite
    from sparkpipe_rs_b200.models.rope import cos_sin_table

    dev = torch.device("cuda", 0)
    T, R = args.rows, 4
    cfg = v2_lite()

    def report(name, us, nbytes):
        gbs = nbytes / us / 1e3
        print(f"{name:24s} rows={T:6d}: {us:8.2f} us  {gbs:8.1f} GB/s  {gbs / args.hbm_gbs:5.2f} of measured HBM",
              flush=True)

    H = 2048
    xs = [torch.randn(T, H, device=dev).bfloat16() for _ in range(R)]
    rs = [torch.randn(T, H, device=dev).bfloat16() for _ in range(R)]
    outs = [torch.empty(T, H, device=dev, dtype=torch.bfloat16) for _ in range(R)]
    gamma = torch.ones(H, device=dev, dtype=torch.bfloat16)
    us = time_fn(lambda i: ops.add_rmsnorm(xs[i % R], rs[i % R], gamma, outs[i % R], 1e-6), args.iters)
    report("add_rmsnorm", us, 4 * T * H * 2)
    del xs, rs, outs

    tab = cos_sin_table(cfg, 4096, device=dev)
    kv = [torch.randn(T, 576, device=dev).bfloat16() for _ in range(R)]
    nw = torch.ones(512, device=dev, dtype=torch.bfloat16)
    pos = torch.randint(0, 4096, (T,), device=dev, dtype=torch.int32)
    slots = torch.randperm(T * R, device=dev)[:T].int()
    cache = torch.zeros(T * R, 576, device=dev, dtype=torch.bfloat16)
    lat = [torch.empty(T, 576, device=dev, dtype=torch.bfloat16) for _ in range(R)]
    us = time_fn(lambda i: ops.mla_kv_write(kv[i % R], nw, pos, tab, slots, cache, lat[i % R], 512, 64, 1e-6),
                 args.iters)
    report("mla_kv_write", us, 3 * T * 576 * 2)
    c8 = torch.zeros(T * R, 576, device=dev, dtype=torch.uint8)
    sc = torch.zeros(T * R, 5, device=dev)
    us = time_fn(lambda i: ops.mla_kv_write(kv[i % R], nw, pos, tab, slots, c8, None, 512, 64, 1e-6, sc), args.iters)
    report("mla_kv_write fp8", us, T * 576 * 2 + T * (576 + 20))
    del kv, lat, cache, c8, sc

    Hq = 7168
    xq = [torch.randn(T, Hq, device=dev).bfloat16() for _ in range(R)]
    us = time_fn(lambda i: ops.quant_fp8_block(xq[i % R]), args.iters)
    report("quant_fp8_block", us, T * Hq * 2 + T * Hq + T * (Hq // 128) * 4)
    del xq

    q = [torch.randn(T, 16, 192, device=dev).bfloat16() for _ in range(R)]
    us = time_fn(lambda i: ops.rope_q(q[i % R], 128, q[i % R], 128, pos, tab, 64), args.iters)
    report("rope_q", us, 2 * T * 16 * 64 * 2)


if __name__ == "__main__":
    main()
