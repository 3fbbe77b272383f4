"""Tensor parallelism over peer memory (csrc/kernels/tp.cu + the tensor-parallel
operands of the tcgen05 GEMM).

Emulated ranks on one GPU: W TensorParallel ranks in one process, driven phase by
phase (every rank's all-gather send, then every rank's column-parallel GEMM, ...),
so no kernel waits on a kernel that has not finished. Checks:

* AG -> GEMM: each rank's column-parallel output over all T tokens equals the same
  GEMM on the gathered rows (bit for bit: same tiles, same K order);
* GEMM -> RS -> residual + RMSNorm (+ AG of the normed rows): the owner's rows match
  the fp32 sum of every rank's partial products (fixed summation order), and the
  next layer's all-gathered operand equals the normed rows;
* the bounded wait: an all-gather that nobody sent ends with the peer-timeout status.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _tp(world, rows, H, **kw):
    from sparkpipe_rs_b200.parallel.tensor_parallel import TensorParallel

    return TensorParallel.emulated(world, rows, H, torch.device(DEV), **kw)


@pytest.mark.parametrize("world,rows,splits", [(2, 8, 1), (4, 16, 2), (8, 4, 4)])
def test_emulated_tp_block(world, rows, splits):
    from sparkpipe_rs_b200 import ops

    H, Ml, Kl = 1024, 384, 512
    T = world * rows
    g = torch.Generator(device=DEV).manual_seed(world * 10 + rows)
    ranks = _tp(world, rows, H)
    ops.clear_status()
    x = [(torch.randn(rows, H, device=DEV, generator=g) * 0.5).bfloat16() for _ in range(world)]
    wc = [(torch.randn(Ml, H, device=DEV, generator=g) * 0.03).bfloat16() for _ in range(world)]
    wr = [(torch.randn(H, Kl, device=DEV, generator=g) * 0.03).bfloat16() for _ in range(world)]
    z = [(torch.randn(T, Kl, device=DEV, generator=g)).bfloat16() for _ in range(world)]
    res = [(torch.randn(rows, H, device=DEV, generator=g)).bfloat16() for _ in range(world)]
    gamma = (torch.rand(H, device=DEV, generator=g) + 0.5).bfloat16()
    for step in range(2):
        # layer 0: all-gather x, column-parallel GEMM
        for r in range(world):
            ranks[r].ag_send(0, x[r])
        xfull = torch.cat(x)
        for r in range(world):
            y = ranks[r].ag_gemm(0, wc[r])
            ref = ops.linear(xfull, wc[r], splits=1)
            torch.cuda.synchronize()
            assert ops.status_word() == 0
            assert torch.equal(y, ref), (step, r, (y.float() - ref.float()).abs().max())
        # layer 1: row-parallel GEMM -> reduce-scatter -> residual + RMSNorm, all-gathering
        # the normed rows under layer 0 of the next step... here under layer 1's tag
        for r in range(world):
            slots = ranks[r].rs_gemm(1, z[r], wr[r], splits=splits)
        full = sum(z[r].float() @ wr[r].float().t() for r in range(world))  # [T, H]
        outs = []
        for r in range(world):
            rr = res[r].clone()
            out = torch.empty(rows, H, dtype=torch.bfloat16, device=DEV)
            ranks[r].rs_add_rmsnorm(1, slots, rr, gamma, out, 1e-6, ag_layer=1)
            torch.cuda.synchronize()
            assert ops.status_word() == 0
            part = full[r * rows:(r + 1) * rows]
            s_ref = (part.bfloat16().float() + res[r].float()).bfloat16().float()
            torch.testing.assert_close(rr.float(), s_ref, atol=3e-2, rtol=3e-2)
            n_ref = s_ref * torch.rsqrt(s_ref.pow(2).mean(-1, keepdim=True) + 1e-6) * gamma.float()
            torch.testing.assert_close(out.float(), n_ref, atol=3e-2, rtol=3e-2)
            outs.append(out)
        # the normed rows arrived in every rank's AG region: a GEMM reading them
        # equals the GEMM on the concatenated rows
        for r in range(world):
            y = ranks[r].ag_gemm(1, wc[r])
            ref = ops.linear(torch.cat(outs), wc[r], splits=1)
            torch.cuda.synchronize()
            assert torch.equal(y, ref)
        for rk in ranks:
            rk.end_step()
    torch.cuda.synchronize()
    assert ops.status_word() == 0


def test_ag_gemm_times_out_with_status():
    from sparkpipe_rs_b200 import ops

    ranks = _tp(2, 8, 512, budget_cycles=2_000_000)  # ~1 ms
    ops.clear_status()
    w = (torch.randn(128, 512, device=DEV) * 0.02).bfloat16()
    ranks[0].ag_send(0, torch.randn(8, 512, device=DEV).bfloat16())  # rank 1 never sends
    ranks[0].ag_gemm(0, w)
    torch.cuda.synchronize()
    assert ops.status_word() == 4
    ops.clear_status()
    assert (torch.ones(4, device=DEV) + 1).sum().item() == 8  # the context is still usable
