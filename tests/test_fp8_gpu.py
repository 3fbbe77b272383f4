"""Block-scaled fp8 kernels (weight / activation quantisation, the tcgen05 fp8 GEMM
in its split-K, dense and grouped forms) against plain PyTorch fp32 references of
the same dequantised operands."""
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _ops():
    from sparkpipe_rs_b200 import ops

    return ops


def _status_ok():
    assert _ops().status_word() == 0


def _deq_act(a):
    """fp32 view of an Fp8Act: q[r, k] * s[k // 128, r]."""
    R, K = a.q.shape
    return a.q.float() * a.s[:, :R].t().repeat_interleave(128, 1)[:, :K]


def test_quant_weight_from_bf16_and_seeded():
    ops = _ops()
    g = torch.Generator(device=DEV).manual_seed(1)
    src = (torch.randn(300, 512, device=DEV, generator=g) * 0.05).bfloat16()
    w = ops.quant_weight_fp8(300, 512, src=src)
    assert w.s.shape == (3, 4)
    x = src.float()
    blk = x.new_zeros(3, 4)
    for i in range(3):
        for j in range(4):
            blk[i, j] = x[i * 128:(i + 1) * 128, j * 128:(j + 1) * 128].abs().max() / 448
    torch.testing.assert_close(w.s, blk, rtol=1e-6, atol=0)
    d = w.dequant()
    scale = blk.repeat_interleave(128, 0)[:300].repeat_interleave(128, 1)
    assert ((d - x).abs() <= x.abs() / 16 + scale / 64).all()  # e4m3: 3 mantissa bits
    # seeded samples: statistics, determinism, and shards that match the whole
    a = ops.quant_weight_fp8(1024, 2048, seed=7, std=0.02, device=DEV)
    b = ops.quant_weight_fp8(1024, 2048, seed=7, std=0.02, device=DEV)
    assert torch.equal(a.q.view(torch.uint8), b.q.view(torch.uint8)) and torch.equal(a.s, b.s)
    da = a.dequant()
    assert abs(da.mean().item()) < 2e-4 and abs(da.std().item() - 0.02) < 1e-3
    shard = ops.quant_weight_fp8(256, 2048, seed=7, std=0.02, flat0=512 * 2048, device=DEV)
    assert torch.equal(shard.q.view(torch.uint8), a.q[512:768].view(torch.uint8))
    _status_ok()


def test_quant_act_gathered():
    ops = _ops()
    g = torch.Generator(device=DEV).manual_seed(2)
    x = torch.randn(40, 1024, device=DEV, generator=g).bfloat16()
    idx = torch.randint(0, 40 * 3, (77,), device=DEV, generator=g).int()
    a = ops.quant_act_fp8(x, idx, 3)
    src = x.float()[idx.long() // 3]
    torch.testing.assert_close(a.s.t(), src.view(77, 8, 128).abs().amax(-1) / 448, rtol=1e-6, atol=0)
    d = _deq_act(a)
    assert ((d - src).abs() <= src.abs() / 16 + 1e-6 + a.s.t().repeat_interleave(128, 1) / 64).all()
    _status_ok()


@pytest.mark.parametrize("T,O,K,slab", [(32, 576, 7168, False), (32, 1536, 7168, True), (7, 12288, 1536, False),
                                        (200, 1024, 1024, False), (64, 7168, 8192, False), (300, 384, 512, False)])
def test_linear_fp8(T, O, K, slab):
    ops = _ops()
    g = torch.Generator(device=DEV).manual_seed(T + O)
    w = ops.quant_weight_fp8(O, K, seed=T * 131 + O, std=0.02, device=DEV)
    x = torch.randn(T, K, device=DEV, generator=g).bfloat16()
    a = ops.quant_act_fp8(x)
    ref = _deq_act(a) @ w.dequant().t()
    y = ops.linear_fp8(a, w, out_dtype=torch.float32, slab_out=slab)
    if isinstance(y, ops.Slabs):
        y = y.ws[: y.splits * y.stride].view(y.splits, T, O).sum(0)
    torch.testing.assert_close(y, ref, rtol=2e-3, atol=2e-3 * ref.abs().max().item())
    yb = ops.linear_fp8(a, w)  # bf16 output
    torch.testing.assert_close(yb.float(), ref, rtol=1e-2, atol=1e-2 * ref.abs().max().item())
    _status_ok()


@pytest.mark.parametrize("T,E,k,bn,swiglu", [(32, 9, 8, 32, False), (32, 9, 8, 32, True), (500, 17, 4, 64, False),
                                             (700, 6, 3, 128, True)])
def test_grouped_gemm_fp8(T, E, k, bn, swiglu):
    ops = _ops()
    H, F = 1024, 256
    g = torch.Generator(device=DEV).manual_seed(T + E + k)
    x = torch.randn(T, H, device=DEV, generator=g).bfloat16()
    ids = torch.stack([torch.randperm(E, device=DEV, generator=g)[:k] for _ in range(T)]).int()
    grp_rows, grp_tiles, sorted_tok, inv_pos = ops.moe_align(ids, E, bn)
    a = ops.quant_act_fp8(x, sorted_tok)  # gathered straight into the sorted layout
    q = torch.empty(E, 2 * F, H, dtype=torch.float8_e4m3fn, device=DEV)
    s = torch.empty(E, 2 * F // 128, H // 128, device=DEV)
    for e in range(E):
        we = ops.quant_weight_fp8(2 * F, H, seed=100 + e, std=0.03, device=DEV)
        q[e], s[e] = we.q, we.s
    w13 = ops.Fp8Weight(q, s, 128)
    xd = _deq_act(a)
    wd = w13.dequant()
    rows = grp_rows.cpu().tolist()
    if swiglu:
        out = torch.empty(T * k, F, device=DEV, dtype=torch.bfloat16)
        ops.grouped_gemm_fp8(ops.interleave_gate_up_fp8(w13), a, out, grp_rows, grp_tiles, E, bn, swiglu=True)
        ref = torch.zeros(T * k, F, device=DEV)
    else:
        out = torch.empty(T * k, 2 * F, device=DEV, dtype=torch.bfloat16)
        ops.grouped_gemm_fp8(w13, a, out, grp_rows, grp_tiles, E, bn)
        ref = torch.zeros(T * k, 2 * F, device=DEV)
    for e in range(E):
        r0, r1 = rows[e], rows[e + 1]
        if r1 > r0:
            h = xd[r0:r1] @ wd[e].t()
            ref[r0:r1] = torch.nn.functional.silu(h[:, :F]) * h[:, F:] if swiglu else h
    torch.testing.assert_close(out.float(), ref, rtol=1e-2, atol=1e-2 * ref.abs().max().item())
    _status_ok()
