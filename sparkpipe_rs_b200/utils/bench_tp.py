"""Tensor-parallel collective+GEMM microbenchmark: the fused peer-memory paths
against their NCCL baselines, on one box (launch one process per GPU).

Workload (decode-shaped, sequence parallel): T = 256 tokens over the group, hidden
H = 7168 (Kimi-K2 shape). One iteration is one tensor-parallel block, as between
two attention layers:

  row-parallel GEMM (o_proj-like, Kl = 8192 / W inputs per rank) -> reduce-scatter
  over tokens -> residual add + RMSNorm -> all-gather of the normed rows ->
  column-parallel GEMM (q/kv-like, O = 3072 outputs per rank)

    fused:  rs_gemm (epilogue sends fp32 partials to the token owners) +
            rs_add_rmsnorm (sums them, adds, norms, all-gathers as tagged words) +
            ag_gemm (B polled from the tagged words)            -> 3 kernels
    NCCL:   GEMM (fp32) + reduce_scatter_tensor + add_rmsnorm + all_gather_into_tensor
            + GEMM                                              -> the baseline

Timing: CUDA events around K iterations after warm-up, max over ranks. Roofline
per rank: the slower of the weight stream (both shards' bytes / measured HBM copy
bandwidth) and the bf16-equivalent bytes this rank exchanges over NVLink
(partials of the peers' rows out, its normed rows out; / 770 GB/s measured peer
copy).

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        -m sparkpipe_rs_b200.utils.bench_tp
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch

HBM_GBS = 6417.3      # measured STREAM-style copy (MEASURED_PEAKS.json hbm_gbs)
NVLINK_GBS = 770.0    # measured peer copy per direction per GPU


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=256)
    ap.add_argument("--hidden", type=int, default=7168)
    ap.add_argument("--col-out", type=int, default=3072)
    ap.add_argument("--row-in", type=int, default=8192)
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    args = ap.parse_args()

    import torch.distributed as dist
    from sparkpipe_rs_b200 import ops
    from sparkpipe_rs_b200.parallel.tensor_parallel import TensorParallel

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    T, H = args.tokens, args.hidden
    rows = T // world
    Kl = args.row_in // world
    g = torch.Generator(device=dev).manual_seed(rank)
    tp = TensorParallel(world, rank, rows, H, dev, group=dist.group.WORLD)
    wc = (torch.randn(args.col_out, H, device=dev, generator=g) * 0.02).bfloat16()
    wr = (torch.randn(H, Kl, device=dev, generator=g) * 0.02).bfloat16()
    z = torch.randn(T, Kl, device=dev, generator=g).bfloat16()
    res0 = torch.randn(rows, H, device=dev, generator=g).bfloat16()
    gamma = torch.ones(H, device=dev, dtype=torch.bfloat16)
    out = torch.empty(rows, H, device=dev, dtype=torch.bfloat16)
    y = torch.empty(T, args.col_out, device=dev, dtype=torch.bfloat16)

    res = res0.clone()

    def fused_block():
        slots = tp.rs_gemm(0, z, wr)
        tp.rs_add_rmsnorm(0, slots, res, gamma, out, 1e-6, ag_layer=1)
        tp.ag_gemm(1, wc, out=y)
        tp.end_step()

    def nccl_block():
        mine = tp.nccl_rs_gemm(z, wr)
        ops.add_rmsnorm(mine.bfloat16(), res, gamma, out, 1e-6)
        return tp.nccl_ag_gemm(out, wc)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / args.iters * 1000.0], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # correctness: one block each way from the same residual
    ops.clear_status()
    fused_block()
    y_f, o_f = y.clone(), out.clone()
    res.copy_(res0)
    y_n = nccl_block()
    torch.cuda.synchronize()
    o_err = float((out.float() - o_f.float()).abs().max())
    y_err = float((y_n.float() - y_f.float()).abs().max() / y_n.float().abs().max())
    res.copy_(res0)
    t = {"fused_block_us": timed(fused_block), "nccl_block_us": timed(nccl_block)}
    w_bytes = (args.col_out * H + H * Kl) * 2
    link_bytes = (world - 1) * rows * H * 2 * 2  # bf16-equivalent: peers' partials out + own rows out
    roof_us = max(w_bytes / (HBM_GBS * 1e3), link_bytes / (NVLINK_GBS * 1e3))  # bytes / (GB/s) -> us
    status = ops.status_word()
    if rank == 0:
        print(json.dumps({
            "metric": "tensor-parallel block latency (us, max over ranks)", "n_gpus": world, "tokens": T,
            "hidden": H, "col_out_per_rank": args.col_out, "row_in_per_rank": Kl, **t,
            "roofline_us": roof_us, "fused_frac_of_roofline": roof_us / t["fused_block_us"],
            "speedup_vs_nccl": t["nccl_block_us"] / t["fused_block_us"],
            "normed_rows_max_abs_diff_vs_nccl": o_err, "col_gemm_max_rel_diff_vs_nccl": y_err,
            "kernel_status": status,
            "note": "roofline = max(weight bytes / measured HBM copy 6417 GB/s, bf16 bytes over NVLink / 770 GB/s)",
        }), flush=True)
    dist.barrier()
    tp.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
