"""Numerics of every sm_100a kernel against a plain PyTorch fp32 reference."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _ops():
    from sparkpipe_rs_b200 import ops

    return ops


def _close(out, ref, atol=3e-2, rtol=3e-2):
    torch.testing.assert_close(out.float(), ref.float(), atol=atol, rtol=rtol)


def _status_ok():
    ops = _ops()
    assert ops.status_word() == 0, f"kernel status word {ops.status_word()}"


# ------------------------------------------------------------------ GEMM
@pytest.mark.parametrize("T,O,K", [(1, 3648, 2048), (7, 2048, 2048), (64, 2048, 1408), (64, 64, 2048),
                                   (200, 5632, 2048), (33, 1000, 576)])
def test_linear_swap_ab(T, O, K):
    ops = _ops()
    g = torch.Generator(device=DEV).manual_seed(T * 7 + O)
    x = torch.randn(T, K, device=DEV, generator=g).bfloat16()
    w = (torch.randn(O, K, device=DEV, generator=g) * 0.02).bfloat16()
    out = ops.linear(x, w)
    _close(out, x.float() @ w.float().t())
    _status_ok()


@pytest.mark.parametrize("splits", [1, 2, 4, 8])
def test_linear_split_k_cluster(splits):
    ops = _ops()
    g = torch.Generator(device=DEV).manual_seed(splits)
    x = torch.randn(48, 2048, device=DEV, generator=g).bfloat16()
    w = (torch.randn(1000, 2048, device=DEV, generator=g) * 0.02).bfloat16()
    out = ops.linear(x, w, splits=splits)
    _close(out, x.float() @ w.float().t())
    _status_ok()


@pytest.mark.parametrize("T,O,K", [(64, 9792, 2048),    # 77 tiles: units spread over every SM
                                   (64, 2048, 8192),    # 16 tiles, long K: many partial slots per tile
                                   (64, 64, 2048),      # one tile
                                   (16, 1408, 1000),    # ragged last K block
                                   (128, 3648, 128)])   # two K blocks per tile
def test_linear_stream_k_split(T, O, K):
    """Decode GEMMs with fewer tiles than SMs use the stream-K split: partial sums
    reduced here (linear) or left as slabs (linear_slabs) must both equal the fp32
    product, also on a second call through the same workspace."""
    ops = _ops()
    g = torch.Generator(device=DEV).manual_seed(T + O + K)
    x = torch.randn(T, K, device=DEV, generator=g).bfloat16()
    w = (torch.randn(O, K, device=DEV, generator=g) * 0.02).bfloat16()
    ref = x.float() @ w.float().t()
    for _ in range(2):
        _close(ops.linear(x, w), ref)
        sl = ops.linear_slabs(x, w, out_dtype=torch.float32)
        if isinstance(sl, ops.Slabs):
            got = sl.ws[: sl.splits * sl.stride].view(sl.splits, T, O).sum(0)
        else:
            got = sl
        _close(got, ref)
    _status_ok()


@pytest.mark.parametrize("T,O,K", [(1000, 3648, 2048), (4096, 2048, 2048), (300, 102400 // 8, 2048), (513, 4096, 512)])
def test_linear_prefill(T, O, K):
    ops = _ops()
    g = torch.Generator(device=DEV).manual_seed(T + O)
    x = torch.randn(T, K, device=DEV, generator=g).bfloat16()
    w = (torch.randn(O, K, device=DEV, generator=g) * 0.02).bfloat16()
    out = ops.linear(x, w)
    _close(out, x.float() @ w.float().t())
    _status_ok()


def test_linear_fp32_out_and_strided_input():
    ops = _ops()
    g = torch.Generator(device=DEV).manual_seed(3)
    base = torch.randn(64, 3000, device=DEV, generator=g).bfloat16()
    x = base[:, 128:128 + 2048]  # row pitch 3000, offset 128 elements (256 B)
    w = (torch.randn(64, 2048, device=DEV, generator=g) * 0.02).bfloat16()
    out = ops.linear(x, w, out_dtype=torch.float32)
    assert out.dtype == torch.float32
    _close(out, x.float() @ w.float().t(), atol=1e-3, rtol=1e-3)


def test_batched_absorb_gemm():
    """q_lat[t, h, :512] = q_nope[t, h] @ W_UK[h] and the W_UV un-absorb product."""
    ops = _ops()
    T, nh, dn, dr, dv, kvl = 37, 16, 128, 64, 128, 512
    g = torch.Generator(device=DEV).manual_seed(5)
    q = torch.randn(T, nh * (dn + dr), device=DEV, generator=g).bfloat16()
    wkvb = (torch.randn(nh * (dn + dv), kvl, device=DEV, generator=g) * 0.02).bfloat16()
    wuk_t = wkvb.view(nh, dn + dv, kvl)[:, :dn].transpose(1, 2).contiguous().view(nh * kvl, dn)
    q_lat = torch.zeros(T, nh, kvl + dr, device=DEV, dtype=torch.bfloat16)
    ops.batched_gemm(wuk_t, q, q_lat.view(T, nh * (kvl + dr)), M=kvl, N=T, K=dn, batch=nh, a_batch_rows=kvl,
                     b_batch_k=dn + dr, ldd=nh * (kvl + dr), d_batch_stride=kvl + dr)
    qn = q.float().view(T, nh, dn + dr)[..., :dn]
    ref = torch.einsum("thd,hdc->thc", qn, wkvb.float().view(nh, dn + dv, kvl)[:, :dn])
    _close(q_lat[..., :kvl], ref)
    o_lat = torch.randn(T, nh, kvl, device=DEV, generator=g).bfloat16()
    attn = torch.empty(T, nh * dv, device=DEV, dtype=torch.bfloat16)
    ops.batched_gemm(wkvb, o_lat.view(T, nh * kvl), attn, M=dv, N=T, K=kvl, batch=nh, a_row0=dn,
                     a_batch_rows=dn + dv, b_batch_k=kvl, ldd=nh * dv, d_batch_stride=dv)
    ref2 = torch.einsum("thc,hvc->thv", o_lat.float(), wkvb.float().view(nh, dn + dv, kvl)[:, dn:]).reshape(T, -1)
    _close(attn, ref2)
    _status_ok()


@pytest.mark.parametrize("T,E,k,bn", [(64, 64, 6, 16), (64, 64, 6, 32), (512, 16, 4, 64), (3000, 64, 6, 256)])
def test_grouped_gemm_moe(T, E, k, bn):
    ops = _ops()
    H, F = 512, 384
    g = torch.Generator(device=DEV).manual_seed(T + E)
    x = torch.randn(T, H, device=DEV, generator=g).bfloat16()
    ids = torch.stack([torch.randperm(E, device=DEV, generator=g)[:k] for _ in range(T)]).int()
    w13 = (torch.randn(E, 2 * F, H, device=DEV, generator=g) * 0.02).bfloat16()
    grp_rows, grp_tiles, sorted_tok, inv_pos = ops.moe_align(ids, E, bn)
    counts = torch.bincount(ids.flatten().long(), minlength=E)
    assert torch.equal(grp_rows[1:].cpu() - grp_rows[:-1].cpu(), counts.int().cpu())
    xs = ops.gather_rows(x, sorted_tok)
    out = torch.empty(T * k, 2 * F, device=DEV, dtype=torch.bfloat16)
    ops.grouped_gemm(w13, xs, out, grp_rows, grp_tiles, E, bn)
    # reference: row r belongs to the expert whose row range holds it
    rows = grp_rows.cpu().tolist()
    ref = torch.empty_like(out, dtype=torch.float32)
    for e in range(E):
        r0, r1 = rows[e], rows[e + 1]
        if r1 > r0:
            ref[r0:r1] = xs[r0:r1].float() @ w13[e].float().t()
    _close(out, ref)
    # inv_pos maps (t, j) to a row holding token t
    st = sorted_tok.cpu()
    ip = inv_pos.cpu().view(T, k)
    assert torch.equal(st[ip.flatten().long()].view(T, k), torch.arange(T).view(T, 1).expand(T, k).int())
    _status_ok()


@pytest.mark.parametrize("T,E,k,bn", [(64, 66, 8, 16), (700, 18, 5, 128)])
def test_grouped_gemm_fused_swiglu(T, E, k, bn):
    ops = _ops()
    H, F = 512, 192
    g = torch.Generator(device=DEV).manual_seed(T * 3 + E)
    x = torch.randn(T, H, device=DEV, generator=g).bfloat16()
    ids = torch.stack([torch.randperm(E, device=DEV, generator=g)[:k] for _ in range(T)]).int()
    w13 = (torch.randn(E, 2 * F, H, device=DEV, generator=g) * 0.05).bfloat16()
    grp_rows, grp_tiles, sorted_tok, inv_pos = ops.moe_align(ids, E, bn)
    xs = ops.gather_rows(x, sorted_tok)
    act = torch.empty(T * k, F, device=DEV, dtype=torch.bfloat16)
    ops.grouped_gemm(ops.interleave_gate_up(w13), xs, act, grp_rows, grp_tiles, E, bn, swiglu=True)
    rows = grp_rows.cpu().tolist()
    ref = torch.empty(T * k, F, device=DEV)
    for e in range(E):
        r0, r1 = rows[e], rows[e + 1]
        if r1 > r0:
            h = xs[r0:r1].float() @ w13[e].float().t()
            ref[r0:r1] = torch.nn.functional.silu(h[:, :F]) * h[:, F:]
    _close(act, ref)
    _status_ok()


@pytest.mark.parametrize("T,E,k,F,swiglu", [(3000, 66, 8, 1408, True), (3000, 66, 8, 1408, False),
                                             (700, 18, 5, 192, True), (257, 9, 3, 256, False)])
def test_grouped_gemm_token_major(T, E, k, F, swiglu):
    """Prefill-shaped expert GEMM with the tokens as M tiles: against an fp32 loop over
    the groups (empty and one-row groups included by the routing), SwiGLU paired in
    registers from the interleaved weights."""
    ops = _ops()
    H = 512
    g = torch.Generator(device=DEV).manual_seed(T + 7 * E + F)
    x = torch.randn(T, H, device=DEV, generator=g).bfloat16()
    # skewed routing: a few hot experts, some experts idle
    logits = torch.randn(T, E, device=DEV, generator=g) + torch.linspace(3, -3, E, device=DEV)
    ids = logits.topk(k, dim=-1).indices.int()
    N = 2 * F if swiglu else F
    w = (torch.randn(E, N, H, device=DEV, generator=g) * 0.05).bfloat16()
    grp_rows, grp_tiles, sorted_tok, inv_pos = ops.moe_align(ids, E, 128)
    xs = ops.gather_rows(x, sorted_tok)
    out = torch.empty(T * k, F if swiglu else N, device=DEV, dtype=torch.bfloat16)
    ops.grouped_gemm_tm(ops.interleave_gate_up(w) if swiglu else w, xs, out, grp_rows, grp_tiles, E, swiglu=swiglu)
    rows = grp_rows.cpu().tolist()
    ref = torch.empty(T * k, out.shape[1], device=DEV)
    for e in range(E):
        r0, r1 = rows[e], rows[e + 1]
        if r1 > r0:
            h = xs[r0:r1].float() @ w[e].float().t()
            ref[r0:r1] = torch.nn.functional.silu(h[:, :F]) * h[:, F:] if swiglu else h
    _close(out, ref)
    _status_ok()


# ------------------------------------------------------------------ norms / rope
@pytest.mark.parametrize("rows,H", [(1, 2048), (64, 2048), (300, 7168), (17, 512)])
def test_add_rmsnorm(rows, H):
    ops = _ops()
    g = torch.Generator(device=DEV).manual_seed(rows)
    x = torch.randn(rows, H, device=DEV, generator=g).bfloat16()
    r = torch.randn(rows, H, device=DEV, generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(H, device=DEV, generator=g)).bfloat16()
    r0 = r.clone()
    out = torch.empty_like(x)
    ops.add_rmsnorm(x, r, w, out, 1e-6)
    s = (x.float() + r0.float()).bfloat16().float()
    _close(r, s, atol=1e-2, rtol=1e-2)
    ref = s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    _close(out, ref)
    out2 = torch.empty_like(x)
    ops.add_rmsnorm(x, None, w, out2, 1e-6)
    ref2 = x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    _close(out2, ref2)


def test_mla_kv_write_and_rope_q():
    ops = _ops()
    from sparkpipe_rs_b200.models.config import v2_lite
    from sparkpipe_rs_b200.models.rope import apply_rope, cos_sin_table

    cfg = v2_lite()
    T, nh = 19, 16
    g = torch.Generator(device=DEV).manual_seed(9)
    tab = cos_sin_table(cfg, 4096, device=DEV)
    kv = torch.randn(T, 3072 + 576, device=DEV, generator=g).bfloat16()
    kv_a = kv[:, 3072:]
    nw = (1 + 0.1 * torch.randn(512, device=DEV, generator=g)).bfloat16()
    pos = torch.randint(0, 4000, (T,), device=DEV, generator=g).int()
    slots = torch.randperm(256, device=DEV, generator=g)[:T].int()
    slots[3] = -1
    cache = torch.zeros(256, 576, device=DEV, dtype=torch.bfloat16)
    lat = torch.empty(T, 576, device=DEV, dtype=torch.bfloat16)
    ops.mla_kv_write(kv_a, nw, pos, tab, slots, cache, lat, 512, 64, 1e-6)
    x = kv_a.float()
    ref_lat = x[:, :512] * torch.rsqrt(x[:, :512].pow(2).mean(-1, keepdim=True) + 1e-6) * nw.float()
    ref_pe = apply_rope(x[:, 512:], pos, tab)
    _close(lat[:, :512], ref_lat)
    _close(lat[:, 512:], ref_pe)
    keep = slots >= 0
    _close(cache[slots[keep].long()], lat[keep], atol=0, rtol=0)
    q = torch.randn(T, nh, 192, device=DEV, generator=g).bfloat16()
    q_lat = torch.zeros(T, nh, 576, device=DEV, dtype=torch.bfloat16)
    ops.rope_q(q, 128, q_lat, 512, pos, tab, 64)
    _close(q_lat[..., 512:], apply_rope(q.float()[..., 128:], pos, tab))


def test_quant_fp8_block():
    ops = _ops()
    x = torch.randn(33, 1024, device=DEV).bfloat16() * 3
    q, s = ops.quant_fp8_block(x)
    deq = q.float().view(33, 8, 128) * s.view(33, 8, 1)
    _close(deq.view(33, 1024), x.float(), atol=0.1, rtol=0.07)
    amax = x.float().view(33, 8, 128).abs().amax(-1)
    _close(s, amax / 448.0, atol=1e-6, rtol=1e-5)


# ------------------------------------------------------------------ attention
def _mla_ref(q, cache, bt, ctx, scale):
    B, H, _ = q.shape
    out = torch.empty(B, H, 512, device=q.device)
    for b in range(B):
        L = int(ctx[b])
        if L == 0:  # an idle row reads nothing and yields zeros
            out[b] = 0
            continue
        blocks = bt[b, : (L + 63) // 64].long()
        rows = (blocks[:, None] * 64 + torch.arange(64, device=q.device)).flatten()[:L]
        kv = cache[rows].float()
        s = (q[b].float() @ kv.t()) * scale
        out[b] = s.softmax(-1) @ kv[:, :512]
    return out


@pytest.mark.parametrize("impl", ["tc", "mma", "sk"])
@pytest.mark.parametrize("H,splits", [(16, 1), (16, 3), (32, 2), (64, 1), (128, 4)])
def test_mla_decode(H, splits, impl):
    ops = _ops()
    g = torch.Generator(device=DEV).manual_seed(H + splits)
    B, nblocks, maxb = 7, 64, 10
    cache = torch.randn(nblocks * 64, 576, device=DEV, generator=g).bfloat16()
    ctx = torch.tensor([1, 63, 64, 65, 300, 640, 0][:B], device=DEV, dtype=torch.int32)
    bt = torch.stack([torch.randperm(nblocks, device=DEV, generator=g)[:maxb] for _ in range(B)]).int()
    q = torch.randn(B, H, 576, device=DEV, generator=g).bfloat16()
    out = torch.empty(B, H, 512, device=DEV, dtype=torch.bfloat16)
    scale = 1.0 / math.sqrt(192)
    ops.mla_decode(q, cache, bt, ctx, out, splits, scale, impl=impl)
    _close(out, _mla_ref(q, cache, bt, ctx, scale), atol=2e-2, rtol=2e-2)
    _status_ok()


@pytest.mark.parametrize("H", [16, 64])
def test_mla_decode_stream_k_balanced_schedule_graph_replay(H):
    """Stream-K decode on a decode-shaped batch (many sequences split over several
    CTAs, short ones kept whole, an idle row), three launches in a row (the arrival
    counters must come back to zero) and a CUDA-graph replay, where the kernel loads
    earlier-position KV before its dependency wait."""
    ops = _ops()
    g = torch.Generator(device=DEV).manual_seed(100 + H)
    B, maxb = 48, 20
    nblocks = B * maxb
    cache = torch.randn(nblocks * 64, 576, device=DEV, generator=g).bfloat16()
    lens = [int(x) for x in torch.randint(1, maxb * 64, (B,), generator=g, device=DEV)]
    lens[3], lens[7], lens[11] = 0, 1, maxb * 64
    ctx = torch.tensor(lens, device=DEV, dtype=torch.int32)
    bt = torch.randperm(nblocks, device=DEV, generator=g).int().view(B, maxb)
    q = torch.randn(B, H, 576, device=DEV, generator=g).bfloat16()
    scale = 1.0 / math.sqrt(192)
    ref = _mla_ref(q, cache, bt, ctx, scale)
    for _ in range(3):
        out = torch.full((B, H, 512), 7.0, device=DEV, dtype=torch.bfloat16)
        ops.mla_decode(q, cache, bt, ctx, out, 1, scale, impl="sk")
        _close(out, ref, atol=2e-2, rtol=2e-2)
    _status_ok()
    out = torch.empty(B, H, 512, device=DEV, dtype=torch.bfloat16)
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s), torch.cuda.graph(graph, stream=s):
        ops.mla_decode(q, cache, bt, ctx, out, 1, scale, impl="sk")
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(2):
        out.fill_(7.0)
        graph.replay()
        torch.cuda.synchronize()
        _close(out, ref, atol=2e-2, rtol=2e-2)
    del graph
    _status_ok()


def _prefill_ref(q, k, kpe, v, cu_q, cu_k, scale):
    out = torch.empty(q.shape[0], q.shape[1], v.shape[2], device=q.device)
    for b in range(len(cu_q) - 1):
        q0, q1, k0, k1 = int(cu_q[b]), int(cu_q[b + 1]), int(cu_k[b]), int(cu_k[b + 1])
        Lq, Lk = q1 - q0, k1 - k0
        if Lq == 0:
            continue
        H = q.shape[1]
        kk = torch.cat([k[k0:k1].float(), kpe[k0:k1].float()[:, None, :].expand(Lk, H, -1)], -1)
        s = torch.einsum("qhd,khd->hqk", q[q0:q1].float(), kk) * scale
        mask = torch.arange(Lk, device=q.device)[None, :] <= (Lk - Lq + torch.arange(Lq, device=q.device))[:, None]
        s = s.masked_fill(~mask[None], float("-inf"))
        out[q0:q1] = torch.einsum("hqk,khd->qhd", s.softmax(-1), v[k0:k1].float())
    return out


@pytest.mark.parametrize("impl", ["tc", "mma"])
@pytest.mark.parametrize("qlens,klens", [([100, 64, 1], [100, 130, 50]), ([1024], [1024]), ([7, 200], [7, 333]),
                                         ([300], [1000])])
def test_prefill_attention(qlens, klens, impl):
    ops = _ops()
    H = 4
    g = torch.Generator(device=DEV).manual_seed(sum(qlens))
    Tq, Tk = sum(qlens), sum(klens)
    q = torch.randn(Tq, H, 192, device=DEV, generator=g).bfloat16()
    kv = torch.randn(Tk, H, 256, device=DEV, generator=g).bfloat16()
    kpe = torch.randn(Tk, 576, device=DEV, generator=g).bfloat16()[:, 512:]
    cu_q = torch.tensor([0] + list(torch.tensor(qlens).cumsum(0)), device=DEV, dtype=torch.int32)
    cu_k = torch.tensor([0] + list(torch.tensor(klens).cumsum(0)), device=DEV, dtype=torch.int32)
    o = torch.empty(Tq, H, 128, device=DEV, dtype=torch.bfloat16)
    scale = 1.0 / math.sqrt(192)
    ops.prefill_attention(q, kv[:, :, :128], kpe, kv[:, :, 128:], o, cu_q, cu_k, max(qlens), scale, impl=impl)
    ref = _prefill_ref(q, kv[:, :, :128], kpe, kv[:, :, 128:], cu_q.cpu(), cu_k.cpu(), scale)
    _close(o, ref, atol=2e-2, rtol=2e-2)


# ------------------------------------------------------------------ MoE routing
@pytest.mark.parametrize("scoring,renorm,E,k,groups", [(0, False, 64, 6, None), (1, True, 384, 8, None),
                                                        (0, True, 8, 2, None), (1, True, 256, 8, (8, 4, "noaux_tc")),
                                                        (0, False, 160, 6, (8, 3, "group_limited_greedy")),
                                                        (0, False, 66, 4, None),
                                                        (1, True, 128, 8, (8, 4, "noaux_tc"))])
@pytest.mark.parametrize("T", [77, 2048])  # a CTA per token / a warp per token (E <= 128)
def test_moe_topk(scoring, renorm, E, k, groups, T):
    ops = _ops()
    from sparkpipe_rs_b200.models import oracle
    from sparkpipe_rs_b200.models.config import MLAMoEConfig
    g = torch.Generator(device=DEV).manual_seed(E)
    logits = torch.randn(T, E, device=DEV, generator=g)
    bias = torch.randn(E, device=DEV, generator=g) * 0.1 if scoring == 1 else None
    ng, tg, method = groups or (1, 1, "greedy")
    ids, w = ops.moe_topk(logits, bias, k, scoring, renorm, 2.5, n_shared=2, n_group=ng, topk_group=tg,
                          group_top2=method == "noaux_tc")
    assert torch.equal(ids[:, k:].cpu(), torch.tensor([[E, E + 1]] * T, dtype=torch.int32))
    assert torch.equal(w[:, k:].cpu(), torch.ones(T, 2))
    ids, w = ids[:, :k].contiguous(), w[:, :k].contiguous()
    cfg = MLAMoEConfig(n_routed_experts=E, num_experts_per_tok=k, scoring_func=["softmax", "sigmoid"][scoring],
                       norm_topk_prob=renorm, routed_scaling_factor=2.5, n_group=ng, topk_group=tg, topk_method=method)
    eye = torch.eye(E, device=DEV)
    ref_ids, ref_w, _ = oracle.route(cfg, logits, eye, bias)  # x @ I.T = the logits
    assert torch.equal(ids.long().sort(-1).values, ref_ids.sort(-1).values)
    sc = logits.softmax(-1) if scoring == 0 else logits.sigmoid()
    rw = sc.gather(-1, ids.long())
    if renorm:
        rw = rw / rw.sum(-1, keepdim=True)
    _close(w, rw * 2.5, atol=1e-5, rtol=1e-5)


def test_moe_topk_many_slabs():
    """Router logits left as 8 split-K slabs: the fused slab sum selects like fp32."""
    ops = _ops()
    T, E, S = 64, 64, 8
    g = torch.Generator(device=DEV).manual_seed(5)
    slabs = torch.randn(S, T, E, device=DEV, generator=g)
    lg = ops.Slabs.__new__(ops.Slabs)
    lg.splits, lg.rows, lg.cols, lg.ws, lg.stride = S, T, E, slabs, T * E
    ids, w = ops.moe_topk(lg, None, 6, 0, False, 1.0, n_shared=2)
    full = slabs.sum(0)
    assert torch.equal(ids[:, :6].long().sort(-1).values, full.softmax(-1).topk(6, -1).indices.sort(-1).values)
    _close(w[:, :6], full.softmax(-1).gather(-1, ids[:, :6].long()), atol=1e-5, rtol=1e-5)


def test_silu_mul_and_combine():
    ops = _ops()
    g = torch.Generator(device=DEV).manual_seed(11)
    h = torch.randn(50, 2 * 1408, device=DEV, generator=g).bfloat16()
    a = ops.silu_mul(h)
    ref = torch.nn.functional.silu(h.float()[:, :1408]) * h.float()[:, 1408:]
    _close(a, ref)
    T, k, H = 20, 6, 2048
    y = torch.randn(T * k, H, device=DEV, generator=g).bfloat16()
    inv = torch.randperm(T * k, device=DEV, generator=g).int()
    w = torch.rand(T, k, device=DEV, generator=g)
    add = torch.randn(T, H, device=DEV, generator=g).bfloat16()
    out = torch.empty(T, H, device=DEV, dtype=torch.bfloat16)
    ops.moe_combine(y, inv, w, add, out, k)
    ref = add.float() + (w[..., None] * y.float()[inv.long()].view(T, k, H)).sum(1)
    _close(out, ref)


# ------------------------------------------------------------------ sampling / embedding / verify
def test_sampling_greedy_and_seeded():
    ops = _ops()
    g = torch.Generator(device=DEV).manual_seed(13)
    logits = torch.randn(9, 102400, device=DEV, generator=g).bfloat16()
    ids = ops.sample_tokens(logits)
    assert torch.equal(ids.long(), logits.float().argmax(-1))
    a = ops.sample_tokens(logits, temperature=1.0, seed=7, offset=3)
    b = ops.sample_tokens(logits, temperature=1.0, seed=7, offset=3)
    c = ops.sample_tokens(logits, temperature=1.0, seed=8, offset=3)
    assert torch.equal(a, b) and not torch.equal(a, c)
    # odd vocabulary exercises the scalar path
    ids2 = ops.sample_tokens(logits[:, :1001].contiguous())
    assert torch.equal(ids2.long(), logits[:, :1001].float().argmax(-1))


def test_embedding():
    ops = _ops()
    table = torch.randn(1000, 2048, device=DEV).bfloat16()
    ids = torch.tensor([0, 5, 999, 5], device=DEV, dtype=torch.int32)
    assert torch.equal(ops.embedding(table, ids), table[ids.long()])


def test_spec_verify():
    ops = _ops()
    draft = torch.tensor([[1, 2, 3], [1, 9, 3], [7, 7, 7]], device=DEV, dtype=torch.int32)
    target = torch.tensor([[1, 2, 3, 4], [1, 2, 3, 4], [8, 0, 0, 0]], device=DEV, dtype=torch.int32)
    acc, com = ops.spec_verify(draft, target)
    assert acc.tolist() == [3, 1, 0]
    assert com.tolist() == [[1, 2, 3, 4], [1, 2, -1, -1], [8, -1, -1, -1]]
    acc2, _ = ops.spec_verify(torch.zeros(4096, 3, device=DEV, dtype=torch.int32),
                              torch.ones(4096, 4, device=DEV, dtype=torch.int32), p_accept=0.7, seed=1)
    # E[accepted] for a Bernoulli(0.7) chain of 3 = 0.7 + 0.49 + 0.343
    assert abs(acc2.float().mean().item() - 1.533) < 0.08


# ------------------------------------------------------------------ fused decode kernels
def test_linear_slabs_and_slab_add_rmsnorm():
    ops = _ops()
    g = torch.Generator(device=DEV).manual_seed(21)
    x = torch.randn(64, 2048, device=DEV, generator=g).bfloat16()
    w = (torch.randn(2048, 2048, device=DEV, generator=g) * 0.02).bfloat16()
    res = torch.randn(64, 2048, device=DEV, generator=g).bfloat16()
    gamma = (1 + 0.1 * torch.randn(2048, device=DEV, generator=g)).bfloat16()
    r0 = res.clone()
    out = torch.empty_like(res)
    sl = ops.linear_slabs(x, w)
    assert isinstance(sl, ops.Slabs) and sl.splits > 1
    ops.slab_add_rmsnorm(sl, res, gamma, out, 1e-6)
    y = (x.float() @ w.float().t()).bfloat16().float()
    s = (y + r0.float()).bfloat16().float()
    _close(res, s, atol=3e-2, rtol=3e-2)
    _close(out, s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + 1e-6) * gamma.float())
    # router logits left as slabs feed the top-k kernel directly
    gate = (torch.randn(64, 2048, device=DEV, generator=g) * 0.02).bfloat16()
    lg = ops.linear_slabs(x, gate, out_dtype=torch.float32)
    ids, wts = ops.moe_topk(lg, None, 6, 0, False, 1.0, n_shared=2)
    ref = (x.float() @ gate.float().t()).softmax(-1)
    assert torch.equal(ids[:, :6].long().sort(-1).values, ref.topk(6, -1).indices.sort(-1).values)


def test_mla_decode_prep_matches_unfused_ops():
    ops = _ops()
    from sparkpipe_rs_b200.models.config import v2_lite
    from sparkpipe_rs_b200.models.rope import cos_sin_table

    cfg = v2_lite()
    T, nh = 40, 16
    g = torch.Generator(device=DEV).manual_seed(31)
    tab = cos_sin_table(cfg, 2048, device=DEV)
    qkv = torch.randn(T, 3072 + 576, device=DEV, generator=g).bfloat16()
    nw = (1 + 0.1 * torch.randn(512, device=DEV, generator=g)).bfloat16()
    pos = torch.randint(0, 2000, (T,), device=DEV, generator=g).int()
    slots = torch.randperm(512, device=DEV, generator=g)[:T].int()
    c1 = torch.zeros(512, 576, device=DEV, dtype=torch.bfloat16)
    c2 = torch.zeros_like(c1)
    qn = torch.empty(T, nh * 128, device=DEV, dtype=torch.bfloat16)
    ql1 = torch.zeros(T, nh, 576, device=DEV, dtype=torch.bfloat16)
    ql2 = torch.zeros_like(ql1)
    ops.mla_decode_prep(qkv, nw, pos, tab, slots, c1, qn, ql1, 128, 0, 3072, 1e-6)
    ops.mla_kv_write(qkv[:, 3072:], nw, pos, tab, slots, c2, None, 512, 64, 1e-6)
    q3 = qkv[:, :3072].reshape(T, nh, 192)
    ops.rope_q(q3, 128, ql2, 512, pos, tab, 64)
    _close(c1, c2, atol=2e-2, rtol=2e-2)
    _close(ql1[..., 512:], ql2[..., 512:], atol=2e-2, rtol=2e-2)
    assert torch.equal(qn.view(T, nh, 128), q3[..., :128])


def test_combine_add_rmsnorm_matches_unfused():
    ops = _ops()
    g = torch.Generator(device=DEV).manual_seed(41)
    T, k, H = 64, 8, 2048
    y = torch.randn(T * k, H, device=DEV, generator=g).bfloat16()
    inv = torch.randperm(T * k, device=DEV, generator=g).int()
    w = torch.rand(T, k, device=DEV, generator=g)
    res = torch.randn(T, H, device=DEV, generator=g).bfloat16()
    gamma = (1 + 0.1 * torch.randn(H, device=DEV, generator=g)).bfloat16()
    r1, r2 = res.clone(), res.clone()
    o1, o2, comb = torch.empty_like(res), torch.empty_like(res), torch.empty_like(res)
    ops.combine_add_rmsnorm(y, inv, w, r1, gamma, o1, k, 1e-6)
    ops.moe_combine(y, inv, w, None, comb, k)
    ops.add_rmsnorm(comb, r2, gamma, o2, 1e-6)
    _close(r1, r2, atol=2e-2, rtol=2e-2)
    _close(o1, o2)


@pytest.mark.parametrize("scoring,E,k,groups", [(0, 64, 6, None), (1, 256, 8, (8, 4, "noaux_tc"))])
def test_moe_route_fused_matches_gemm_router(scoring, E, k, groups):
    """The router with its logits computed inside the top-k kernel selects like the
    gate GEMM + top-k path, with the same weights."""
    ops = _ops()
    g = torch.Generator(device=DEV).manual_seed(E + k)
    T, H = 64, 2048
    x = torch.randn(T, H, device=DEV, generator=g).bfloat16()
    gate = (torch.randn(E, H, device=DEV, generator=g) * 0.05).bfloat16()
    bias = torch.randn(E, device=DEV, generator=g) * 0.1 if scoring == 1 else None
    ng, tg, method = groups or (1, 1, "greedy")
    kw = dict(n_shared=2, n_group=ng, topk_group=tg, group_top2=method == "noaux_tc")
    ids, w = ops.moe_route(x, gate, bias, k, scoring, True, 2.5, **kw)
    logits = x.float() @ gate.float().t()
    ids2, w2 = ops.moe_topk(logits, bias, k, scoring, True, 2.5, **kw)
    assert torch.equal(ids[:, :k].sort(-1).values, ids2[:, :k].sort(-1).values)
    assert torch.equal(ids[:, k:], ids2[:, k:])
    order = ids[:, :k].sort(-1).indices
    order2 = ids2[:, :k].sort(-1).indices
    _close(w[:, :k].gather(1, order), w2[:, :k].gather(1, order2), atol=1e-4, rtol=1e-3)
    _status_ok()



@pytest.mark.parametrize("T,E,k", [(64, 66, 8), (8192, 66, 8), (3000, 384, 9)])
def test_moe_align_layout(T, E, k):
    """Expert-sorted layout (one-CTA path for decode sizes, sliced histogram path above
    16,384 pairs): rows grouped by expert in grp_rows order, inv_pos its inverse, tile
    prefix counts from the row counts."""
    ops = _ops()
    g = torch.Generator(device=DEV).manual_seed(T + E)
    logits = torch.randn(T, E, device=DEV, generator=g) + torch.linspace(2, -2, E, device=DEV)
    ids = logits.topk(k, dim=-1).indices.int().contiguous()
    bn = 64
    grp_rows, grp_tiles, sorted_tok, inv_pos = ops.moe_align(ids, E, bn)
    torch.cuda.synchronize()
    counts = torch.bincount(ids.flatten().long(), minlength=E).cpu()
    rows = grp_rows.cpu()
    assert rows[0] == 0 and torch.equal(rows[1:] - rows[:-1], counts.int())
    tiles = grp_tiles.cpu()
    assert torch.equal(tiles[1:] - tiles[:-1], ((counts + bn - 1) // bn).int())
    inv = inv_pos.cpu().long()
    assert torch.equal(torch.sort(inv).values, torch.arange(T * k))
    flat = ids.flatten().cpu().long()
    st = sorted_tok.cpu().long()
    for i in torch.randint(0, T * k, (500,), generator=torch.Generator().manual_seed(1)).tolist():
        p = int(inv[i])
        e = int(flat[i])
        assert int(rows[e]) <= p < int(rows[e + 1]) and int(st[p]) == i // k
    _status_ok()
