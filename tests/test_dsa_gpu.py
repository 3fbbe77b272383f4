"""DeepSeek sparse attention selection and sparse MLA decode against fp32 PyTorch."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _setup(B=5, Hi=32, H=16, lens=(40, 700, 2048, 2100, 5000), seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    maxb = math.ceil(max(lens) / 64)
    nblk = B * maxb + 8
    bt = torch.stack([torch.randperm(nblk, device=DEV, generator=g)[:maxb] for _ in range(B)]).int()
    ctx = torch.tensor(lens[:B], device=DEV, dtype=torch.int32)
    kcache = torch.randn(nblk * 64, 128, device=DEV, generator=g).bfloat16()
    cache = torch.randn(nblk * 64, 576, device=DEV, generator=g).bfloat16()
    q_idx = torch.randn(B, Hi, 128, device=DEV, generator=g).bfloat16()
    w_idx = torch.rand(B, Hi, device=DEV, generator=g)
    q_lat = torch.randn(B, H, 576, device=DEV, generator=g).bfloat16()
    return bt, ctx, kcache, cache, q_idx, w_idx, q_lat


def _rows(bt, b, L):
    return (bt[b, : (L + 63) // 64].long()[:, None] * 64 + torch.arange(64, device=DEV)).flatten()[:L]


def test_dsa_select_matches_torch_topk():
    from sparkpipe_rs_b200 import ops
    bt, ctx, kcache, _, q_idx, w_idx, _ = _setup()
    topk = 2048
    pos, cnt = ops.dsa_select(q_idx, w_idx, kcache, bt, ctx, max_context=int(ctx.max()), topk=topk)
    torch.cuda.synchronize()
    assert ops.status_word() == 0
    for b in range(bt.shape[0]):
        L = int(ctx[b])
        k = kcache[_rows(bt, b, L)].float()
        score = (torch.relu(q_idx[b].float() @ k.t()) * w_idx[b, :, None]).sum(0)
        want = torch.arange(L, device=DEV) if L <= topk else score.topk(topk).indices.sort().values
        got = pos[b, : int(cnt[b])].long()
        assert int(cnt[b]) == min(L, topk)
        assert torch.equal(got, got.sort().values)  # ascending
        if L <= topk:
            assert torch.equal(got, want) and (pos[b, L:] == -1).all()
        else:
            # the selected scores are the topk largest (ties at the threshold may swap)
            thr = score.topk(topk).values[-1]
            assert (score[got] >= thr - 1e-3 * thr.abs()).all()
            assert len(set(got.tolist()) & set(want.tolist())) >= topk - 2


def test_dsa_sparse_decode_matches_reference():
    from sparkpipe_rs_b200 import ops
    bt, ctx, kcache, cache, q_idx, w_idx, q_lat = _setup(seed=3)
    topk = 1024
    scale = 1 / math.sqrt(192)
    pos, cnt = ops.dsa_select(q_idx, w_idx, kcache, bt, ctx, max_context=int(ctx.max()), topk=topk)
    out = torch.empty(q_lat.shape[0], q_lat.shape[1], 512, device=DEV, dtype=torch.bfloat16)
    ops.dsa_sparse_decode(q_lat, cache, bt, pos, cnt, out, scale)
    torch.cuda.synchronize()
    assert ops.status_word() == 0
    for b in range(bt.shape[0]):
        sel = pos[b, : int(cnt[b])].long()
        kv = cache[_rows(bt, b, int(ctx[b]))[sel]].float()
        ref = ((q_lat[b].float() @ kv.t()) * scale).softmax(-1) @ kv[:, :512]
        err = (out[b].float() - ref).abs().max() / ref.abs().max()
        assert err < 3e-2, (b, float(err))
