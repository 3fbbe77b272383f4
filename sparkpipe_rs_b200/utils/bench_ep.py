"""Latency of each expert-parallel kernel, on one GPU with emulated ranks.

W ranks live in one process on one GPU (their "peer" buffers are local), one
MoE layer of the given shape is run once phase by phase so every tagged word of
the epoch has arrived, and then each phase kernel of rank 0 is replayed alone
in a CUDA graph (the epoch is not advanced, so every poll succeeds at once) and
timed with CUDA events. The numbers are the in-kernel cost of each phase
without NVLink transfer time or peer skew.

    python -m sparkpipe_rs_b200.utils.bench_ep --world 2 --tokens 64
"""
from __future__ import annotations

import argparse

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="v2_lite")
    ap.add_argument("--world", type=int, default=2)
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--iters", type=int, default=200)
    args = ap.parse_args()

    from sparkpipe_rs_b200 import ops
    from sparkpipe_rs_b200.models.config import get_config
    from sparkpipe_rs_b200.models.mla_moe import _moe_block_n
    from sparkpipe_rs_b200.parallel.expert_parallel import ExpertParallel

    cfg = get_config(args.model).replace(num_layers=2, first_k_dense_replace=0)
    dev = torch.device("cuda", 0)
    W, T = args.world, args.tokens
    E, S, H = cfg.n_routed_experts, cfg.n_shared_experts, cfg.hidden_size
    kk = cfg.num_experts_per_tok + S
    ranks = ExpertParallel.emulated(cfg, W, T, dev)
    El = E // W
    F = cfg.moe_intermediate_size
    w13 = (torch.randn(El + S, 2 * F, H, device=dev) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(El + S, H, F, device=dev) * 0.02).to(torch.bfloat16)
    layer = ranks[0].moe_layers[0]
    g = torch.Generator(device=dev).manual_seed(0)
    xs = [torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16) for _ in range(W)]
    ids = []
    for _ in range(W):
        routed = torch.stack([torch.randperm(E, device=dev, generator=g)[:cfg.num_experts_per_tok] for _ in range(T)])
        shared = torch.arange(E, E + S, device=dev).expand(T, S)
        ids.append(torch.cat([routed, shared], 1).to(torch.int32).contiguous())
    wts = torch.ones(T, kk, device=dev)
    bn = _moe_block_n(T * kk, ranks[0].n_local)
    for r in ranks:
        r.dispatch(layer, xs[ranks.index(r)], ids[ranks.index(r)])
        if r.shared_local:
            r.shared(xs[ranks.index(r)], w13, w2)
    for r in ranks:
        r.receive(layer, bn)
    for r in ranks:
        r.experts(w13, w2, bn, layer=layer)  # the down projection sends the rows to their sources
    res = torch.zeros(T, H, dtype=torch.bfloat16, device=dev)
    out = torch.empty_like(res)
    gamma = torch.ones(H, dtype=torch.bfloat16, device=dev)
    torch.cuda.synchronize()
    assert ops.status_word() == 0, "setup round failed"
    r0 = ranks[0]
    K = r0.K
    j = r0.moe_index[layer]
    phases = {
        "dispatch": lambda: K.ep_dispatch(xs[0], ids[0], r0.args(), r0.epoch, j),
        "shared experts on local tokens": lambda: r0.shared(xs[0], w13, w2),
        "recv_align": lambda: K.ep_recv_align(r0.args(), r0.epoch, j, bn, r0.grp_rows, r0.grp_tiles, r0.src_row,
                                              r0.comb_dst, r0.budget),
        "gather": lambda: K.ep_gather(r0.args(), r0.epoch, j, r0.grp_rows[r0.n_local:], r0.src_row, r0.xs, r0.budget),
        "experts (2 grouped GEMMs)": lambda: r0.experts(w13, w2, bn),
        "experts, down GEMM sends to sources": lambda: r0.experts(w13, w2, bn, layer=layer),
        "combine_send (unfused path)": lambda: K.ep_combine_send(r0.y, r0.grp_rows[r0.n_local:], r0.comb_dst,
                                                                 r0.args(), r0.epoch, j),
        "ep_combine_add_rmsnorm": lambda: r0.combine_add_rmsnorm(layer, wts, res, gamma, out, cfg.rms_norm_eps),
        "combine_add_rmsnorm (local)": lambda: ops.combine_add_rmsnorm(r0.y, r0.src_row, wts, res, gamma, out, kk,
                                                                       cfg.rms_norm_eps),
    }
    print(f"expert-parallel phase latency, emulated world {W}, {T} tokens per rank, {cfg.name}")
    for name, fn in phases.items():
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            fn()
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                for _ in range(20):
                    fn()
            graph.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            for _ in range(args.iters // 20):
                graph.replay()
            e1.record(s)
            torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1000 / (args.iters // 20 * 20)
        print(f"  {name:32s} {us:8.2f} us")
    assert ops.status_word() == 0


if __name__ == "__main__":
    main()
