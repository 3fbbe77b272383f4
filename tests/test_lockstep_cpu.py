"""Expert-parallel ranks step their engines in lockstep: two gloo ranks, each with
its own requests (uneven counts and lengths, then one rank without any), and a model
whose every forward is a collective, as the expert dispatch/combine is on the GPU.
A rank without work must run idle forwards, or its peer's collective never returns
(the process group's short timeout turns that into a failure)."""
import datetime
import os
import socket
from types import SimpleNamespace

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class _CollectiveModel:
    """The CPU model, with one all-reduce per forward standing in for the expert all-to-all."""

    def __init__(self, inner, world):
        self.inner = inner
        self.cfg, self.device = inner.cfg, inner.device
        self.ep = SimpleNamespace(group=dist.group.WORLD, world=world)
        self.forwards = 0
        self.idle = 0

    def _collective(self):
        t = torch.ones(1)
        dist.all_reduce(t)
        assert int(t.item()) == self.ep.world
        self.forwards += 1

    def forward(self, fb, cache):
        self._collective()
        return self.inner.forward(fb, cache)

    def idle_forward(self, cache):
        self._collective()
        self.idle += 1
        return torch.zeros(1, dtype=torch.int32)


def _worker(rank, world, port, out_q, spec=""):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        from sparkpipe_rs_b200.models import oracle
        from sparkpipe_rs_b200.models.config import tiny
        from sparkpipe_rs_b200.models.cpu_model import CpuMLAMoEModel
        from sparkpipe_rs_b200.serving.engine import EngineConfig, LLMEngine, SamplingParams

        cfg = tiny()
        inner = CpuMLAMoEModel(cfg, seed=0)
        model = _CollectiveModel(inner, world)
        draft = None
        if spec:  # verify rounds are one collective target forward each; the draft is local
            from sparkpipe_rs_b200.models.config import mtp_head

            draft = CpuMLAMoEModel(mtp_head(cfg), seed=3)
        eng = LLMEngine(cfg, EngineConfig(max_batch=4, block_size=16, max_model_len=128, max_prefill_tokens=48,
                                          speculation=spec, spec_force=bool(spec)),
                        model=model, device="cpu", draft=draft)
        assert eng.lockstep
        g = torch.Generator().manual_seed(10 + rank)
        results = []
        # phase 1: rank 0 has three requests, rank 1 one short one; phase 2: only rank 1 has work
        first = {0: [(40, 9), (25, 14), (7, 3)], 1: [(12, 2)]}[rank]
        phases = [first, [] if rank == 0 else [(30, 6), (18, 11)]]
        for reqs in phases:  # (prompt length, tokens to generate)
            prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n, _ in reqs]
            ids = [eng.add_request(p, SamplingParams(max_tokens=k, ignore_eos=True))
                   for p, (_, k) in zip(prompts, reqs)]
            res = eng.generate([], SamplingParams())  # steps with the group until every rank is done
            ok = True
            for i, (p, (_, k)) in enumerate(zip(prompts, reqs)):
                ref, _ = oracle.greedy_generate(cfg, inner.w, torch.tensor(p), k)
                ok &= eng.outputs.pop(ids[i]).token_ids == ref.tolist()
            results.append((ok, len(res.outputs)))
        out_q.put((rank, results, model.forwards, model.idle, eng.idle_steps))
        eng.shutdown()
    finally:
        dist.destroy_process_group()


import pytest


@pytest.mark.parametrize("spec", ["", "mtp_tree"])
def test_expert_parallel_engines_step_in_lockstep(spec):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, spec)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = dict((r, (res, fw, idle, eidle)) for r, res, fw, idle, eidle in (q.get(timeout=5) for _ in range(2)))
    for r in (0, 1):
        res, fw, idle, eidle = got[r]
        assert all(ok for ok, _ in res), (r, res)
        assert idle == eidle
    assert got[0][1] == got[1][1]  # the same number of collective forwards on both ranks
    assert got[0][2] > 0 and got[1][2] > 0  # each rank idled while only the other had work
