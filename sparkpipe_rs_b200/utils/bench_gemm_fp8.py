"""Micro-benchmark of the block-scaled fp8 tcgen05 GEMMs.

Dense: ``ops.linear_fp8`` (128x128-block e4m3 weights, 1x128-block e4m3
activations, fp32 scales) at (tokens, out_features, in_features) shapes, against
cuBLAS bf16 (torch.matmul) on the same shape. Grouped: the MoE expert GEMM
(``ops.grouped_gemm_fp8`` with fused SwiGLU, the gate/up projection) with
`--experts` local experts, `--rows` routed rows spread uniformly, hidden `--k`
and expert FFN `--ffn`. CUDA-graph replays timed with CUDA events; weights
cycled from a pool larger than L2. FLOPs count 2 x M x N x K; the fp8 dense peak
is 4.5 PFLOP/s nominal (no measured fp8 reference on this machine).

    python -m sparkpipe_rs_b200.utils.bench_gemm_fp8 --shapes 64x7168x2048,8192x7168x2048 \\
        --experts 48 --rows 16384 --k 7168 --ffn 2048
"""
from __future__ import annotations

import argparse

import torch

from .bench_gemm import parse_shapes, time_fn


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default="64x7168x2048,64x24576x1536,8192x7168x2048,8192x4096x7168")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--pool-mb", type=int, default=512)
    ap.add_argument("--experts", type=int, default=48)
    ap.add_argument("--rows", type=int, default=16384)
    ap.add_argument("--k", type=int, default=7168)
    ap.add_argument("--ffn", type=int, default=2048)
    ap.add_argument("--splits", default="0", help="split-K settings of the dense GEMMs (0 = automatic)")
    ap.add_argument("--no-grouped", action="store_true")
    args = ap.parse_args()
    from sparkpipe_rs_b200 import ops

    dev = torch.device("cuda", 0)
    for (T, O, K) in parse_shapes(args.shapes):
        wbytes = O * K + O * K // 16384 * 4
        n_pool = max(1, min(32, (args.pool_mb << 20) // wbytes))
        ws = [ops.quant_weight_fp8(O, K, seed=i, device=dev) for i in range(n_pool)]
        x = torch.randn(T, K, device=dev).bfloat16()
        xq = ops.quant_act_fp8(x)
        out = torch.empty(T, O, device=dev, dtype=torch.bfloat16)
        flops = 2.0 * T * O * K
        for sp in [int(v) for v in args.splits.split(",")]:
            us = time_fn(lambda i: ops.linear_fp8(xq, ws[i % n_pool], out=out, splits=sp), args.iters)
            print(f"linear_fp8 T={T:5d} O={O:6d} K={K:6d} splits={sp}: {us:9.2f} us  "
                  f"{wbytes / us / 1e6:6.2f} TB/s of weights  {flops / us / 1e6:8.1f} TFLOP/s", flush=True)
        wb = [torch.randn(O, K, device=dev).mul_(0.02).bfloat16() for _ in range(max(1, n_pool // 2))]
        us = time_fn(lambda i: torch.matmul(x, wb[i % len(wb)].t(), out=out), args.iters)
        print(f"torch.matmul bf16 (cuBLAS) T={T:5d} O={O:6d} K={K:6d}: {us:9.2f} us  "
              f"{flops / us / 1e6:8.1f} TFLOP/s", flush=True)
        del ws, wb
        torch.cuda.empty_cache()
    if args.no_grouped:
        return
    # grouped expert gate/up GEMM with fused SwiGLU
    E, R, K, F = args.experts, args.rows, args.k, args.ffn
    flat = ops.quant_weight_fp8(E * 2 * F, K, seed=1, device=dev)
    w13 = ops.interleave_gate_up_fp8(ops.Fp8Weight(flat.q.view(E, 2 * F, K), flat.s.view(E, 2 * F // 128, K // 128)))
    ids = torch.randint(0, E, (R,), device=dev, dtype=torch.int32).view(R, 1)
    bn = 128
    grp_rows, grp_tiles, sorted_tok, _ = ops.moe_align(ids, E, bn)
    x = torch.randn(R, K, device=dev).bfloat16()
    xq = ops.quant_act_fp8(x, sorted_tok)
    act = torch.empty(R, F, device=dev, dtype=torch.bfloat16)
    us = time_fn(lambda i: ops.grouped_gemm_fp8(w13, xq, act, grp_rows, grp_tiles, E, bn, swiglu=True), args.iters)
    flops = 2.0 * R * 2 * F * K
    wbytes = E * 2 * F * K
    print(f"grouped_gemm_fp8 (gate/up + SwiGLU) experts={E} rows={R} K={K} 2F={2 * F}: {us:9.2f} us  "
          f"{flops / us / 1e6:8.1f} TFLOP/s ({flops / us / 1e6 / 4500:.2f} of 4.5 PF nominal)  "
          f"{wbytes / us / 1e6:6.2f} TB/s of weights", flush=True)


if __name__ == "__main__":
    main()
