"""Micro-benchmark of the NVFP4 expansion kernel (``ops.nvfp4.dequant_nvfp4``):
NVFP4 weights (4.5 bits per element) expanded to bf16, timed with CUDA events over
CUDA-graph-free back-to-back launches cycling through a pool of weights larger than
L2. Bandwidth counts the bytes the kernel must move: packed values + block scales in,
bf16 out.

    python -m sparkpipe_rs_b200.utils.bench_nvfp4 --shapes 7168x2048,2048x7168 --pool-mb 1024
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path

import torch

from ..ops.nvfp4 import dequant_nvfp4, quant_nvfp4


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default="7168x2048,2048x7168,4096x4096")
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--pool-mb", type=int, default=1024)
    args = ap.parse_args()
    peaks = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    hbm = json.loads(peaks.read_text()).get("hbm_gbs", 6650.0) if peaks.exists() else 6650.0
    dev = torch.device("cuda", 0)
    for shp in args.shapes.split(","):
        N, K = (int(v) for v in shp.split("x"))
        moved = N * K // 2 + N * K // 16 + N * K * 2
        pool = max(2, min(64, (args.pool_mb << 20) // moved))
        ws = [quant_nvfp4(torch.randn(N, K, device=dev)) for _ in range(pool)]
        outs = [torch.empty(N, K, device=dev, dtype=torch.bfloat16) for _ in range(pool)]
        for i in range(5):
            dequant_nvfp4(ws[i % pool], outs[i % pool])
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(args.iters):
            dequant_nvfp4(ws[i % pool], outs[i % pool])
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / args.iters
        gbs = moved / us / 1e3
        print(f"dequant_nvfp4 {N}x{K}: {us:8.2f} us  {gbs:7.1f} GB/s  ({gbs / hbm:.2f} of measured HBM copy)", flush=True)
        del ws, outs
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
