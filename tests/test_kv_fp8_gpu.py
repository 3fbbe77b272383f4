"""fp8 (e4m3) latent KV cache: per-128-element block scales written by the KV-write
kernels, the fp8 split-KV MLA decode kernel and the dequantising row gather, each
against a plain PyTorch fp32 reference of the same op (the reference decodes the
stored e4m3 bytes times their scales)."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _ops():
    from sparkpipe_rs_b200 import ops

    return ops


def _status_ok():
    ops = _ops()
    torch.cuda.synchronize()
    assert ops.status_word() == 0
    ops.clear_status()


def quant_rows(x):
    """fp32 [n, 576] -> (uint8 e4m3 [n, 576], fp32 scales [n, 5]): scale = amax / 448 of
    each 128-element block (block 4: the 64 rope dims)."""
    n = x.shape[0]
    xp = torch.zeros(n, 640, device=x.device)
    xp[:, :576] = x
    amax = xp.view(n, 5, 128).abs().amax(-1)
    inv = torch.where(amax > 0, 448.0 / amax, torch.zeros_like(amax))
    q = (xp.view(n, 5, 128) * inv[..., None]).clamp(-448, 448).view(n, 640)[:, :576]
    return q.to(torch.float8_e4m3fn).view(torch.uint8).contiguous(), (amax / 448.0).contiguous()


def dequant_rows(q8, scales):
    v = q8.view(torch.float8_e4m3fn).float()
    return v * scales.repeat_interleave(128, dim=-1)[..., :576]


def _mla_ref(q, rows_f32, bt, ctx, scale):
    B, H, _ = q.shape
    out = torch.empty(B, H, 512, device=q.device)
    for b in range(B):
        L = int(ctx[b])
        if L == 0:
            out[b] = 0
            continue
        blocks = bt[b, : (L + 63) // 64].long()
        rows = (blocks[:, None] * 64 + torch.arange(64, device=q.device)).flatten()[:L]
        kv = rows_f32[rows]
        s = (q[b].float() @ kv.t()) * scale
        out[b] = s.softmax(-1) @ kv[:, :512]
    return out


@pytest.mark.parametrize("stages", ["2", "4"])
@pytest.mark.parametrize("H,splits", [(16, 1), (16, 3), (32, 2), (64, 1), (128, 4)])
def test_fp8_mla_decode_matches_fp32_reference(H, splits, stages, monkeypatch):
    ops = _ops()
    if stages == "4" and (H, splits) not in ((16, 3), (64, 1)):
        pytest.skip("deep-stage variant: two shapes")
    monkeypatch.setenv("SPARKPIPE_MLA8_STAGES", stages)
    g = torch.Generator(device=DEV).manual_seed(H * 10 + splits)
    B, nblocks, maxb = 7, 64, 10
    # rows with a spread of block magnitudes, so the per-block scales matter
    raw = torch.randn(nblocks * 64, 576, device=DEV, generator=g)
    raw *= torch.exp(torch.randn(nblocks * 64, 1, device=DEV, generator=g))
    raw[:, 512:] *= 3.0
    q8, sc = quant_rows(raw)
    rows = dequant_rows(q8, sc)
    ctx = torch.tensor([1, 63, 64, 65, 300, 640, 0][:B], device=DEV, dtype=torch.int32)
    bt = torch.stack([torch.randperm(nblocks, device=DEV, generator=g)[:maxb] for _ in range(B)]).int()
    qv = torch.randn(B, H, 576, device=DEV, generator=g).bfloat16()
    out = torch.empty(B, H, 512, device=DEV, dtype=torch.bfloat16)
    scale = 1.0 / math.sqrt(192)
    ops.mla_decode(qv, q8, bt, ctx, out, splits, scale, kv_scales=sc)
    ref = _mla_ref(qv, rows, bt, ctx, scale)
    err = (out.float() - ref).abs().max().item()
    assert err <= 2e-2 * max(1.0, ref.abs().max().item()), err
    _status_ok()


def test_fp8_mla_decode_last_slot_override():
    """Row b's last context token read from another cache row (a tree verify's shadow
    slot) equals a cache in which that row was copied into place."""
    ops = _ops()
    g = torch.Generator(device=DEV).manual_seed(5)
    B, H, nblocks, maxb = 4, 16, 32, 6
    q8, sc = quant_rows(torch.randn(nblocks * 64, 576, device=DEV, generator=g))
    ctx = torch.tensor([70, 128, 5, 300], device=DEV, dtype=torch.int32)
    # disjoint block tables: a substituted row belongs to one sequence only
    bt = torch.randperm(nblocks - 2, device=DEV, generator=g)[:B * maxb].int().view(B, maxb)
    shadow = torch.tensor([(nblocks - 1) * 64 + b for b in range(B)], device=DEV, dtype=torch.int32)
    shadow[2] = -1  # this row keeps its own last token
    qv = torch.randn(B, H, 576, device=DEV, generator=g).bfloat16()
    scale = 1.0 / math.sqrt(192)
    out = torch.empty(B, H, 512, device=DEV, dtype=torch.bfloat16)
    ops.mla_decode(qv, q8, bt, ctx, out, 2, scale, last_slot=shadow, kv_scales=sc)
    q8b, scb = q8.clone(), sc.clone()
    for b in range(B):
        if int(shadow[b]) < 0:
            continue
        t = int(ctx[b]) - 1
        dst = int(bt[b, t // 64]) * 64 + t % 64
        q8b[dst], scb[dst] = q8[int(shadow[b])], sc[int(shadow[b])]
    ref = torch.empty_like(out)
    ops.mla_decode(qv, q8b, bt, ctx, ref, 2, scale, kv_scales=scb)
    assert torch.equal(out, ref)
    _status_ok()


def test_fp8_kv_writers_quantise_the_bf16_rows():
    """mla_kv_write and mla_decode_prep into the fp8 cache: the block scales are the
    blocks' amax / 448 and the dequantised rows equal the bf16 cache's rows within e4m3
    rounding (half an e4m3 step: 2^-4 of the value, plus bf16 rounding of the
    reference)."""
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
    ref = torch.zeros(512, 576, device=DEV, dtype=torch.bfloat16)
    ops.mla_kv_write(qkv[:, 3072:], nw, pos, tab, slots, ref, None, 512, 64, 1e-6)
    want = ref[slots.long()].float()
    for writer in ("kv_write", "prep"):
        c8 = torch.zeros(512, 576, device=DEV, dtype=torch.uint8)
        sc = torch.zeros(512, 5, device=DEV)
        if writer == "kv_write":
            ops.mla_kv_write(qkv[:, 3072:], nw, pos, tab, slots, c8, None, 512, 64, 1e-6, sc)
        else:
            qn = torch.empty(T, nh * 128, device=DEV, dtype=torch.bfloat16)
            ql = torch.zeros(T, nh, 576, device=DEV, dtype=torch.bfloat16)
            ops.mla_decode_prep(qkv, nw, pos, tab, slots, c8, qn, ql, 128, 0, 3072, 1e-6, sc)
        torch.cuda.synchronize()
        got = dequant_rows(c8[slots.long()], sc[slots.long()])
        wp = torch.zeros(T, 640, device=DEV)
        wp[:, :576] = want
        amax = wp.view(T, 5, 128).abs().amax(-1)
        assert torch.allclose(sc[slots.long()], amax / 448.0, rtol=1e-2, atol=1e-8), writer
        tol = want.abs() * 2.0 ** -4 + amax.repeat_interleave(128, -1)[:, :576] * 2.0 ** -9 + 1e-6
        assert bool(((got - want).abs() <= tol * 1.05).all()), writer
        # untouched rows stay zero
        mask = torch.ones(512, dtype=torch.bool, device=DEV)
        mask[slots.long()] = False
        assert int(c8[mask].count_nonzero()) == 0 and int(sc[mask].count_nonzero()) == 0
    _status_ok()


def test_kv8_gather_dequantises_rows():
    ops = _ops()
    g = torch.Generator(device=DEV).manual_seed(9)
    q8, sc = quant_rows(torch.randn(256, 576, device=DEV, generator=g) * 3)
    idx = torch.randperm(256, device=DEV, generator=g)[:77].int()
    out = ops.kv8_gather(q8, sc, idx)
    ref = dequant_rows(q8[idx.long()], sc[idx.long()]).bfloat16()
    assert torch.equal(out, ref)
    _status_ok()


def test_fp8_cache_model_decode_tracks_bf16_cache():
    """Two V2-Lite-shape layers: a prefill then decode steps with the fp8 cache give
    logits close to the bf16 cache's (cosine > 0.995 per row), through the model's
    prefill KV write, prep kernel, fp8 decode kernel and a chunked prefill that reads
    the earlier chunk back through the dequantising gather."""
    from sparkpipe_rs_b200.models.config import v2_lite
    from sparkpipe_rs_b200.models.mla_moe import ForwardBatch, KVCache, MLAMoEModel

    cfg = v2_lite().replace(num_layers=2)
    dev = torch.device(DEV)
    model = MLAMoEModel(cfg, seed=0, device=dev, max_positions=512)
    S, L = 4, 96
    caches = {k: KVCache(cfg, num_blocks=S * 4, block_size=64, device=dev, kv_dtype=k) for k in ("bf16", "fp8")}
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, cfg.vocab_size, (S, L), generator=g, dtype=torch.int32)
    logits = {}
    for k, cache in caches.items():
        outs = []
        # chunk 1: first 64 tokens of each prompt; chunk 2: the rest with the first as context
        for lo, hi in ((0, 64), (64, L)):
            n = hi - lo
            tok = ids[:, lo:hi].reshape(-1).to(dev)
            pos = torch.arange(lo, hi, dtype=torch.int32).repeat(S).to(dev)
            slots = (torch.arange(S, dtype=torch.int32)[:, None] * 256 + torch.arange(lo, hi, dtype=torch.int32)).reshape(-1).to(dev)
            cu_q = torch.arange(0, S * n + 1, n, dtype=torch.int32, device=dev)
            cu_k = torch.arange(0, S * hi + 1, hi, dtype=torch.int32, device=dev)
            ctx_slots = None
            if lo:
                ctx_slots = (torch.arange(S, dtype=torch.int32)[:, None] * 256 + torch.arange(hi, dtype=torch.int32)).reshape(-1).to(dev)
            fb = ForwardBatch(mode="prefill", token_ids=tok, positions=pos, slot_mapping=slots, cu_q=cu_q, cu_k=cu_k,
                              max_q=n, ctx_slots=ctx_slots, logits_idx=(cu_q[1:] - 1).contiguous())
            outs.append(model.forward(fb, cache).float())
        bt = (torch.arange(S, dtype=torch.int32)[:, None] * 4 + torch.arange(4, dtype=torch.int32)).to(dev)
        nxt = ids[:, L - 1].to(dev)  # the same decode inputs for both caches (no argmax near-ties)
        for step in range(3):
            p = L + step
            fb = ForwardBatch(mode="decode", token_ids=nxt, positions=torch.full((S,), p, dtype=torch.int32, device=dev),
                              slot_mapping=(torch.arange(S, dtype=torch.int32, device=dev) * 256 + p),
                              block_table=bt, context_lens=torch.full((S,), p + 1, dtype=torch.int32, device=dev),
                              decode_splits=2)
            lg = model.forward(fb, cache).float()
            outs.append(lg)
            nxt = ids[:, step].to(dev)  # the same inputs for both caches
        logits[k] = outs
    for a, b in zip(logits["bf16"], logits["fp8"]):
        cos = torch.nn.functional.cosine_similarity(a, b, dim=-1)
        assert float(cos.min()) > 0.995, cos
    _status_ok()
