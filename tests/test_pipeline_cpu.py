"""GPU-free plumbing run through the work plane: tiny MLA-MoE (2 layers, hidden 256,
4 heads, q_lora 96, kv_lora 64, nope 32 / rope 16 / v 32, 8 experts top-2 + 1
shared, FFN 128, vocab 1024, fp32 weights N(0, 0.02), seed 0) served by a pipeline
of gloo ranks. Every step reaches the stages as work-control packets (two
micro-batches, execution payload) through each rank's RankDaemon ledger; the last
rank samples and sends one final event per lane back to rank 0. 4 prompts of 32
uniform ids, greedy 16 tokens each: tokens equal a plain PyTorch CPU forward, the
last stage's prefill logits match it, and the daemons' ledgers and counters show
every packet forwarded, executed, committed and answered."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _prompts():
    g = torch.Generator().manual_seed(0)
    return [torch.randint(0, 1024, (32,), generator=g).tolist() for _ in range(4)]


def _worker(rank, world, port, micro, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        from sparkpipe_rs_b200.models.config import tiny
        from sparkpipe_rs_b200.models.cpu_model import CpuMLAMoEModel
        from sparkpipe_rs_b200.parallel.pipeline import PipelineModel, StageRuntime, split_layers, work_config

        cfg = tiny()
        stages = split_layers(cfg.num_layers, world)
        model = CpuMLAMoEModel(cfg, seed=0)
        block, max_len = 16, 64
        nblocks = 4 * (max_len // block) + 4
        wcfg = work_config(cfg, block, max_len, 4, 256)
        cache = model.new_cache(nblocks, block, layers=len(stages[rank]))
        if rank == 0:
            from sparkpipe_rs_b200.serving.engine import EngineConfig, LLMEngine, SamplingParams

            pm = PipelineModel(model, stages, cache, wcfg, micro_batches=micro)
            eng = LLMEngine(cfg, EngineConfig(max_batch=4, block_size=block, max_model_len=max_len,
                                              num_blocks=nblocks, max_prefill_tokens=256),
                            model=pm, device="cpu", cache=cache)
            res = eng.generate(_prompts(), SamplingParams(max_tokens=16, ignore_eos=True))
            st = pm.daemon.stats()
            led = pm.daemon.ledger
            eng.shutdown()
            out_q.put(("rank0", [o.token_ids for o in res.outputs], res.stats["decode_steps"],
                       (st.submitted, st.accepted, st.forwarded, st.executed, st.committed, st.duplicates),
                       (led.terminal, led.active), pm.final_events, pm.tx))
        else:
            rt = StageRuntime(model, stages, cache, wcfg)
            first = []

            def keep_first(r):
                if r.last and not first:
                    first.append(r.last_logits.clone())  # the prefill's (first packet's) logits

            rt.after_execute = keep_first
            rt.serve()
            st = rt.daemon.stats()
            out_q.put((f"rank{rank}", (st.submitted, st.forwarded, st.executed, st.committed, st.final_events),
                       first[0] if first else None))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,micro", [(2, 2), (2, 1)])
def test_pipeline_through_packets_ledger_and_final_events(world, micro):
    from sparkpipe_rs_b200.models import oracle
    from sparkpipe_rs_b200.models.config import tiny
    from sparkpipe_rs_b200.models.cpu_model import CpuMLAMoEModel

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, micro, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        item = q.get(timeout=300)
        got[item[0]] = item[1:]
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    tokens, decode_steps, st0, ledger0, finals, packets = got["rank0"]
    cfg = tiny()
    model = CpuMLAMoEModel(cfg, seed=0)
    refs = [oracle.greedy_generate(cfg, model.w, torch.tensor(p), 16) for p in _prompts()]
    assert tokens == [r[0].tolist() for r in refs]
    assert decode_steps == 15
    # every packet was accepted once, forwarded, run and committed on rank 0; one final
    # event per lane per step came back (4 prefill lanes + 15 steps x 4 decode lanes)
    submitted, accepted, forwarded, executed, committed, dups = st0
    assert submitted == accepted == forwarded == executed == committed == packets and dups == 0
    assert ledger0 == (packets, 0) and finals == 4 + 15 * 4
    last = got[f"rank{world - 1}"]
    sub, fwd, exe, com, fin = last[0]
    assert sub == exe == com == packets and fwd == 0 and fin == finals
    logits = last[1]   # first packet: the prefill of its lanes (micro-batch 0)
    for i in range(logits.shape[0]):
        assert (logits[i] - refs[i][1][0]).abs().max().item() < 1e-4


def test_cost_driven_stage_cuts():
    from sparkpipe_rs_b200.models.config import k2, v2_lite
    from sparkpipe_rs_b200.parallel.pipeline import layer_costs, plan_stages

    cfg = v2_lite()
    costs, head = layer_costs(cfg)
    assert costs[0] < costs[1] and head > 0          # the dense first layer reads far fewer bytes
    cuts = plan_stages(cfg, 2)
    assert [len(c) for c in cuts] == [14, 13] and sum(cuts, []) == list(range(27))
    # the slowest stage is no slower than under the uniform split
    uni = [list(range(14)), list(range(14, 27))]
    worst = lambda st: max(sum(costs[i] for i in s) + (head if k == len(st) - 1 else 0) for k, s in enumerate(st))
    assert worst(cuts) <= worst(uni)
    # measured costs move the cut: an expensive last layer pulls the boundary forward
    costs2 = list(costs)
    costs2[-1] *= 6
    assert len(plan_stages(cfg, 2, costs2, head)[1]) < 13
    assert [len(c) for c in plan_stages(k2(), 4)] == [16, 15, 15, 15]
