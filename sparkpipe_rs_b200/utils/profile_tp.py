"""One tensor-parallel block on emulated ranks (one GPU), for kernel profiling and
quick device timing of the fused TP kernels without a multi-GPU box.

W ranks live in this process (``TensorParallel.emulated``) and every phase runs
rank by rank in dependency order, so no kernel waits on one that has not run:

    rs_gemm (row-parallel GEMM, partials -> owners) for every rank
    rs_add_rmsnorm (+ all-gather of the normed rows) for every rank
    ag_gemm (column-parallel GEMM over the gathered rows) for every rank

Each phase is timed with CUDA events over --iters repetitions (the per-rank time is
the phase time / W). Peer stores land in this GPU's own memory here, so the numbers
show the kernels' local cost; NVLink adds the wire time on a real box.

    python -m sparkpipe_rs_b200.utils.profile_tp --world 2 --tokens 256 --hidden 7168
"""
from __future__ import annotations

import argparse
import json

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--world", type=int, default=2)
    ap.add_argument("--tokens", type=int, default=256)
    ap.add_argument("--hidden", type=int, default=7168)
    ap.add_argument("--col-out", type=int, default=3072)
    ap.add_argument("--row-in", type=int, default=8192)
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()
    from sparkpipe_rs_b200 import ops
    from sparkpipe_rs_b200.parallel.tensor_parallel import TensorParallel

    dev = torch.device("cuda")
    W, T, H = args.world, args.tokens, args.hidden
    rows, Kl = T // W, args.row_in // W
    ranks = TensorParallel.emulated(W, rows, H, dev)
    g = torch.Generator(device=dev).manual_seed(0)
    wc = [(torch.randn(args.col_out, H, device=dev, generator=g) * 0.02).bfloat16() for _ in range(W)]
    wr = [(torch.randn(H, Kl, device=dev, generator=g) * 0.02).bfloat16() for _ in range(W)]
    z = [torch.randn(T, Kl, device=dev, generator=g).bfloat16() for _ in range(W)]
    res = [torch.randn(rows, H, device=dev, generator=g).bfloat16() for _ in range(W)]
    gamma = torch.ones(H, device=dev, dtype=torch.bfloat16)
    out = [torch.empty(rows, H, device=dev, dtype=torch.bfloat16) for _ in range(W)]
    y = [torch.empty(T, args.col_out, device=dev, dtype=torch.bfloat16) for _ in range(W)]
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    tot = [0.0, 0.0, 0.0]
    ops.clear_status()
    for it in range(args.iters + 2):
        ev[0].record()
        slots = [ranks[r].rs_gemm(0, z[r], wr[r]) for r in range(W)]
        ev[1].record()
        for r in range(W):
            ranks[r].rs_add_rmsnorm(0, slots[r], res[r], gamma, out[r], 1e-6, ag_layer=1)
        ev[2].record()
        for r in range(W):
            ranks[r].ag_gemm(1, wc[r], out=y[r])
        ev[3].record()
        for rk in ranks:
            rk.end_step()
        torch.cuda.synchronize()
        if it >= 2:
            for i in range(3):
                tot[i] += ev[i].elapsed_time(ev[i + 1]) * 1000.0 / W
    n = args.iters
    print(json.dumps({"world": W, "tokens": T, "hidden": H, "col_out": args.col_out, "row_in_per_rank": Kl,
                      "rs_gemm_us_per_rank": tot[0] / n, "rs_add_rmsnorm_ag_us_per_rank": tot[1] / n,
                      "ag_gemm_us_per_rank": tot[2] / n, "kernel_status": ops.status_word()}), flush=True)


if __name__ == "__main__":
    main()
