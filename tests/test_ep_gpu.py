"""Expert-parallel MoE over peer memory (csrc/kernels/ep.cu).

* emulated ranks on one GPU: W ExpertParallel ranks in one process, driven
  phase by phase (every rank's dispatch, then every rank's receive, ...), so no
  kernel waits on a kernel that has not finished; the combined output of every
  rank must equal the single-GPU MoE path bit for bit;
* the bounded wait: a flag that nothing sets ends the receive with the peer
  timeout status, an empty expert schedule and a usable context;
* two real ranks on two GPUs (skipped with fewer GPUs): the expert-parallel
  model's logits equal the single-GPU model's.
"""
import os
import socket

import pytest
import torch

from sparkpipe_rs_b200 import ops
from sparkpipe_rs_b200.models.config import tiny, v2_lite
from sparkpipe_rs_b200.models.mla_moe import _moe_block_n
from sparkpipe_rs_b200.models.weights import init_weights
from sparkpipe_rs_b200.parallel.expert_parallel import ExpertParallel

pytestmark = pytest.mark.gpu


def _cfg():
    return tiny().replace(num_layers=3, hidden_size=512, n_routed_experts=16, num_experts_per_tok=4,
                          n_shared_experts=1, moe_intermediate_size=128, scoring_func="sigmoid",
                          norm_topk_prob=True, routed_scaling_factor=2.5)


def _model_cfg():
    # MLA dims the GPU attention kernels support (kv_lora 512), small everything else
    return v2_lite().replace(name="small-mla-moe", num_layers=4, hidden_size=1024, n_routed_experts=16,
                             num_experts_per_tok=4, moe_intermediate_size=256, intermediate_size=2048,
                             n_shared_experts=1, vocab_size=4096, first_k_dense_replace=1, init_std=0.05)


def _local_moe(cfg, xn, w13, w2, ids, wts, res, gamma, eps):
    E, S = cfg.n_routed_experts, cfg.n_shared_experts
    kk = cfg.num_experts_per_tok + S
    T = xn.shape[0]
    bn = _moe_block_n(T * kk, E + S)
    grp_rows, grp_tiles, sorted_tok, inv_pos = ops.moe_align(ids, E + S, bn)
    xs = ops.gather_rows(xn, sorted_tok)
    act = torch.empty(T * kk, cfg.moe_intermediate_size, dtype=torch.bfloat16, device=xn.device)
    ops.grouped_gemm(w13, xs, act, grp_rows, grp_tiles, E + S, bn, swiglu=True)
    y = torch.empty(T * kk, cfg.hidden_size, dtype=torch.bfloat16, device=xn.device)
    ops.grouped_gemm(w2, act, y, grp_rows, grp_tiles, E + S, bn)
    out = torch.empty_like(xn)
    ops.combine_add_rmsnorm(y, inv_pos, wts, res, gamma, out, kk, eps)
    return out


@pytest.mark.parametrize("world,fused,shared_local,tm", [(2, False, False, False), (4, False, False, False),
                                                        (2, True, True, False), (4, True, True, False),
                                                        (4, True, False, False), (2, True, True, True),
                                                        (4, True, False, True)])
def test_emulated_ranks_match_single_gpu(world, fused, shared_local, tm):
    """fused: the down-projection GEMM's epilogue sends its rows to the source ranks
    (no combine-send kernel); shared_local: the shared experts run on each rank's own
    tokens instead of being dispatched. Every variant must equal the single-GPU MoE
    bit for bit, except tm (the prefill layout: 128-row tiles, token-major gate/up
    GEMMs), whose tiles sum in another order: within bf16 rounding of it."""
    torch.manual_seed(0)
    dev = torch.device("cuda")
    cfg = _cfg()
    E, S, H = cfg.n_routed_experts, cfg.n_shared_experts, cfg.hidden_size
    kk = cfg.num_experts_per_tok + S
    full = init_weights(cfg, seed=3, device=dev)
    for k in list(full):
        if k.endswith("e_w13"):
            full[k] = ops.interleave_gate_up(full[k])
    ranks = ExpertParallel.emulated(cfg, world, cap_tokens=48, device=dev, shared_local=shared_local)
    El = E // world
    local = [{k: torch.cat([v[r * El:(r + 1) * El], v[E:]]).contiguous() for k, v in full.items()
              if k.endswith("e_w13") or k.endswith("e_w2")} for r in range(world)]
    tokens = [7, 0, 48, 21][:world]
    gamma = torch.rand(H, device=dev, dtype=torch.bfloat16) + 0.5
    ops.clear_status()
    for step in range(2):
        for layer in ranks[0].moe_layers:
            p = f"l{layer}."
            xs, ids, wts, res = [], [], [], []
            for r in range(world):
                x = (torch.randn(tokens[r], H, device=dev) * 0.5).to(torch.bfloat16)
                logits = (x.float() @ full[p + "gate"].float().t()).contiguous()
                bias = torch.randn(E, device=dev) * 0.1
                i, w_ = ops.moe_topk(logits, bias, cfg.num_experts_per_tok, 1, True, 2.5, n_shared=S)
                xs.append(x); ids.append(i); wts.append(w_)
                res.append((torch.randn(tokens[r], H, device=dev)).to(torch.bfloat16))
            bn = 128 if tm else _moe_block_n(max(tokens) * kk, ranks[0].n_local)
            for r in range(world):
                ranks[r].dispatch(layer, xs[r], ids[r])
                if shared_local:
                    ranks[r].shared(xs[r], local[r][p + "e_w13"], local[r][p + "e_w2"], token_major=tm)
            for r in range(world):
                ranks[r].receive(layer, bn)
            for r in range(world):
                ranks[r].experts(local[r][p + "e_w13"], local[r][p + "e_w2"], bn, layer=layer if fused else None,
                                 token_major=tm)
            if not fused:
                for r in range(world):
                    ranks[r].combine_send(layer)
            for r in range(world):
                res_ep = res[r].clone()
                out_ep = torch.empty_like(xs[r])
                # reads the returned rows as they arrive (all have: every send ran first)
                ranks[r].combine_add_rmsnorm(layer, wts[r], res_ep, gamma, out_ep, cfg.rms_norm_eps)
                if tokens[r] == 0:
                    continue
                res_ref = res[r].clone()
                out_ref = _local_moe(cfg, xs[r], full[p + "e_w13"], full[p + "e_w2"], ids[r], wts[r], res_ref,
                                     gamma, cfg.rms_norm_eps)
                torch.cuda.synchronize()
                assert ops.status_word() == 0
                if tm:
                    torch.testing.assert_close(res_ep.float(), res_ref.float(), atol=3e-2, rtol=2e-2)
                    torch.testing.assert_close(out_ep.float(), out_ref.float(), atol=6e-2, rtol=3e-2)
                    continue
                assert torch.equal(res_ep, res_ref), (step, layer, r, (res_ep.float() - res_ref.float()).abs().max())
                assert torch.equal(out_ep, out_ref)
        for r in ranks:
            r.end_step()
    torch.cuda.synchronize()
    assert ops.status_word() == 0


def _fp8_slice(w, lo, hi, E):
    """Routed experts lo..hi-1 plus the shared ones of a 3-D Fp8Weight."""
    q = torch.cat([w.q[lo:hi].view(torch.uint8), w.q[E:].view(torch.uint8)]).view(torch.float8_e4m3fn)
    return ops.Fp8Weight(q.contiguous(), torch.cat([w.s[lo:hi], w.s[E:]]).contiguous(), w.sa_rows)


def _local_moe_fp8(cfg, xn, w13i, w2, ids, wts, res, gamma, eps, bn):
    E, S = cfg.n_routed_experts, cfg.n_shared_experts
    kk = cfg.num_experts_per_tok + S
    T = xn.shape[0]
    grp_rows, grp_tiles, sorted_tok, inv_pos = ops.moe_align(ids, E + S, bn)
    xq = ops.quant_act_fp8(xn, sorted_tok)
    act = torch.empty(T * kk, cfg.moe_intermediate_size, dtype=torch.bfloat16, device=xn.device)
    ops.grouped_gemm_fp8(w13i, xq, act, grp_rows, grp_tiles, E + S, bn, swiglu=True)
    y = torch.empty(T * kk, cfg.hidden_size, dtype=torch.bfloat16, device=xn.device)
    ops.grouped_gemm_fp8(w2, ops.quant_act_fp8(act), y, grp_rows, grp_tiles, E + S, bn)
    out = torch.empty_like(xn)
    ops.combine_add_rmsnorm(y, inv_pos, wts, res, gamma, out, kk, eps)
    return out


@pytest.mark.parametrize("world,fused", [(2, False), (4, True)])
def test_emulated_ranks_fp8_transport_match_single_gpu(world, fused):
    """fp8 experts: rows cross as e4m3 + 128-column scales, quantised in the dispatch
    kernel with the same quantiser as the local path, so EP equals local bit for bit."""
    torch.manual_seed(1)
    dev = torch.device("cuda")
    cfg = _cfg().replace(weight_dtype="fp8_block")
    E, S, H = cfg.n_routed_experts, cfg.n_shared_experts, cfg.hidden_size
    kk = cfg.num_experts_per_tok + S
    full = init_weights(cfg, seed=4, device=dev)
    layers = [i for i in range(cfg.num_layers) if cfg.is_moe_layer(i)]
    w13i = {i: ops.interleave_gate_up_fp8(full[f"l{i}.e_w13"]) for i in layers}
    ranks = ExpertParallel.emulated(cfg, world, cap_tokens=48, device=dev, shared_local=fused)
    assert ranks[0].fp8
    El = E // world
    local = [{i: (ops.interleave_gate_up_fp8(_fp8_slice(full[f"l{i}.e_w13"], r * El, (r + 1) * El, E)),
                  _fp8_slice(full[f"l{i}.e_w2"], r * El, (r + 1) * El, E)) for i in layers} for r in range(world)]
    tokens = [9, 0, 48, 30][:world]
    gamma = torch.rand(H, device=dev, dtype=torch.bfloat16) + 0.5
    ops.clear_status()
    for layer in layers:
        p = f"l{layer}."
        xs, ids, wts, res = [], [], [], []
        for r in range(world):
            x = (torch.randn(tokens[r], H, device=dev) * 0.5).to(torch.bfloat16)
            logits = (x.float() @ full[p + "gate"].float().t()).contiguous()
            i, w_ = ops.moe_topk(logits, torch.randn(E, device=dev) * 0.1, cfg.num_experts_per_tok, 1, True, 2.5,
                                 n_shared=S)
            xs.append(x); ids.append(i); wts.append(w_)
            res.append(torch.randn(tokens[r], H, device=dev).to(torch.bfloat16))
        bn = max(32, min(128, _moe_block_n(max(tokens) * kk, ranks[0].n_local)))
        for r in range(world):
            ranks[r].dispatch(layer, xs[r], ids[r])
            if fused:  # the shared experts run locally too
                ranks[r].shared(xs[r], local[r][layer][0], local[r][layer][1])
        for r in range(world):
            ranks[r].receive(layer, bn)
        for r in range(world):
            ranks[r].experts(local[r][layer][0], local[r][layer][1], bn, layer=layer if fused else None)
        if not fused:
            for r in range(world):
                ranks[r].combine_send(layer)
        for r in range(world):
            res_ep = res[r].clone()
            out_ep = torch.empty_like(xs[r])
            ranks[r].combine_add_rmsnorm(layer, wts[r], res_ep, gamma, out_ep, cfg.rms_norm_eps)
            if tokens[r] == 0:
                continue
            res_ref = res[r].clone()
            out_ref = _local_moe_fp8(cfg, xs[r], w13i[layer], full[p + "e_w2"], ids[r], wts[r], res_ref, gamma,
                                     cfg.rms_norm_eps, 32)
            torch.cuda.synchronize()
            assert ops.status_word() == 0
            assert torch.equal(res_ep, res_ref), (layer, r, (res_ep.float() - res_ref.float()).abs().max())
            assert torch.equal(out_ep, out_ref)
    for r in ranks:
        r.end_step()
    torch.cuda.synchronize()
    assert ops.status_word() == 0


def test_receive_wait_times_out_with_status():
    dev = torch.device("cuda")
    cfg = _cfg()
    ranks = ExpertParallel.emulated(cfg, 2, cap_tokens=8, device=dev, budget_cycles=2_000_000,  # ~1 ms
                                    shared_local=False)
    ops.clear_status()
    x = torch.randn(4, cfg.hidden_size, device=dev).to(torch.bfloat16)
    ids = torch.zeros(4, ranks[0].kk, dtype=torch.int32, device=dev)
    layer = ranks[0].moe_layers[0]
    ranks[0].dispatch(layer, x, ids)  # rank 1 never dispatches: its flag stays unset
    ranks[0].grp_rows.fill_(7)
    ranks[0].receive(layer, 16)
    torch.cuda.synchronize()
    assert ops.status_word() == 4  # peer wait timeout
    assert int(ranks[0].grp_rows.sum()) == 0  # empty schedule: downstream kernels do nothing
    ops.clear_status()
    # combine side: nobody returned rows for rank 1's tokens this epoch, so its
    # combine polls run out of budget
    res = torch.zeros(2, cfg.hidden_size, dtype=torch.bfloat16, device=dev)
    out = torch.empty_like(res)
    gamma = torch.ones(cfg.hidden_size, dtype=torch.bfloat16, device=dev)
    ranks[1].combine_add_rmsnorm(layer, torch.ones(2, ranks[1].kk, device=dev), res, gamma, out, 1e-6)
    torch.cuda.synchronize()
    assert ops.status_word() == 4
    ops.clear_status()
    torch.cuda.synchronize()
    assert ops.status_word() == 0
    y = torch.ones(4, device=dev) + 1  # the context is still usable
    assert float(y.sum()) == 8.0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_rank_worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    from sparkpipe_rs_b200.models.mla_moe import ForwardBatch, KVCache, MLAMoEModel
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        cfg = _model_cfg()
        ep = ExpertParallel(cfg, rank, world, cap_tokens=64, device=dev, group=dist.group.WORLD)
        m_ep = MLAMoEModel(cfg, seed=5, device=dev, ep=ep)
        m_ref = MLAMoEModel(cfg, seed=5, device=dev)
        T = 12 + 5 * rank
        g = torch.Generator().manual_seed(rank)
        ids = torch.randint(0, cfg.vocab_size, (T,), generator=g).to(torch.int32).to(dev)
        pos = torch.arange(T, dtype=torch.int32, device=dev)
        outs = []
        for m in (m_ep, m_ref):
            cache = KVCache(cfg, num_blocks=4, block_size=64, device=dev)
            cu = torch.tensor([0, T], dtype=torch.int32, device=dev)
            fb = ForwardBatch(mode="prefill", token_ids=ids, positions=pos, slot_mapping=pos.clone(), cu_q=cu,
                              cu_k=cu, max_q=T)
            dist.barrier()
            outs.append(m.forward(fb, cache).float())
            torch.cuda.synchronize()
        ok = torch.equal(outs[0], outs[1])
        q.put((rank, ok, float((outs[0] - outs[1]).abs().max()), ops.status_word()))
        dist.barrier()
        ep.close()
        dist.destroy_process_group()
    except Exception as e:  # report, never hang the parent
        q.put((rank, False, repr(e), -1))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_expert_parallel_model_matches_single_gpu():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=600) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    for rank, ok, diff, status in sorted(results, key=lambda r: r[0]):
        assert ok and status == 0, (rank, diff, status)


def _lockstep_engine_worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    from sparkpipe_rs_b200.models.mla_moe import MLAMoEModel
    from sparkpipe_rs_b200.serving.engine import EngineConfig, LLMEngine, SamplingParams
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        cfg = _model_cfg()
        ep = ExpertParallel(cfg, rank, world, cap_tokens=128, device=dev, group=dist.group.WORLD)
        ec = dict(max_batch=4, block_size=64, max_model_len=256, max_prefill_tokens=128, decode_buckets=(1, 2, 4))
        eng = LLMEngine(cfg, EngineConfig(**ec), model=MLAMoEModel(cfg, seed=5, device=dev, ep=ep), device=dev)
        ref = LLMEngine(cfg, EngineConfig(**ec), model=MLAMoEModel(cfg, seed=5, device=dev), device=dev)
        g = torch.Generator().manual_seed(20 + rank)
        # rank 0: three requests; rank 1: one short one, so it idles while rank 0 decodes
        reqs = [(40, 12), (70, 20), (9, 5)] if rank == 0 else [(30, 3)]
        prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n, _ in reqs]
        ids = [eng.add_request(p, SamplingParams(max_tokens=k, ignore_eos=True)) for p, (_, k) in zip(prompts, reqs)]
        eng.generate([], SamplingParams())
        got = [eng.outputs.pop(i).token_ids for i in ids]
        want = [ref.generate([p], SamplingParams(max_tokens=k, ignore_eos=True)).outputs[0].token_ids
                for p, (_, k) in zip(prompts, reqs)]
        q.put((rank, got == want, eng.idle_steps, ops.status_word()))
        eng.shutdown()
        ref.shutdown()
        dist.barrier()
        ep.close()
        dist.destroy_process_group()
    except Exception as e:  # report, never hang the parent
        q.put((rank, False, repr(e), -1))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_engines_step_in_lockstep():
    """Expert-parallel engines with uneven work: the rank that runs out of requests
    keeps joining the other's steps with idle forwards; both ranks' tokens equal a
    single-GPU engine's."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_lockstep_engine_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted([q.get(timeout=600) for _ in procs], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=120)
    for rank, ok, idle, status in results:
        assert ok and status == 0, (rank, idle, status)
    assert results[1][2] > 0 and results[0][2] == 0
