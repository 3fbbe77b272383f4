"""A model served from a stage-pack checkpoint on the GPU: weights written from the
seeded random init, read back through pinned host buffers onto the device (whole,
and as one expert-parallel rank's experts), equal bit for bit, and a prefill +
decode step of the model built from them yields the same tokens."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _cfg():
    from sparkpipe_rs_b200.models.config import v2_lite

    return v2_lite().replace(num_layers=2, hidden_size=1024, n_routed_experts=16, num_experts_per_tok=4,
                             moe_intermediate_size=256, intermediate_size=2048, vocab_size=4096)


def _tokens(model, cfg):
    from sparkpipe_rs_b200 import ops
    from sparkpipe_rs_b200.models.mla_moe import DecodeGraph, ForwardBatch, KVCache

    cache = KVCache(cfg, num_blocks=8, block_size=64, device=DEV)
    B, P = 2, 40
    bt = torch.arange(B * 4, dtype=torch.int32, device=DEV).view(B, 4)
    ids = torch.randint(0, cfg.vocab_size, (B * P,), dtype=torch.int32, device=DEV,
                        generator=torch.Generator(device=DEV).manual_seed(5))
    pos = torch.arange(P, dtype=torch.int32, device=DEV).repeat(B)
    slots = (bt[:, :1] * 64 + torch.arange(P, dtype=torch.int32, device=DEV)).flatten().contiguous()
    cu = torch.tensor([0, P, 2 * P], dtype=torch.int32, device=DEV)
    fb = ForwardBatch(mode="prefill", token_ids=ids, positions=pos, slot_mapping=slots, cu_q=cu, cu_k=cu, max_q=P,
                      logits_idx=(cu[1:] - 1).contiguous())
    first = ops.sample_tokens(model.forward(fb, cache))
    dg = DecodeGraph(model, cache, B, 4, 128, use_graph=True)
    dg.ids.copy_(first)
    dg.pos.fill_(P)
    dg.ctx.fill_(P + 1)
    dg.block_table.copy_(bt)
    dg.slots.copy_(bt[:, 0] * 64 + P)
    out = dg.run().clone()
    torch.cuda.synchronize()
    dg.release()
    return first.tolist(), out.tolist()


def test_model_from_stage_pack_on_gpu(tmp_path):
    from sparkpipe_rs_b200.models.checkpoint import load_pack, save_pack
    from sparkpipe_rs_b200.models.mla_moe import MLAMoEModel
    from sparkpipe_rs_b200.models.weights import init_weights

    cfg = _cfg()
    w = init_weights(cfg, seed=0, device=DEV, dtype=torch.bfloat16)
    save_pack(tmp_path / "pack", cfg, w)
    got = load_pack(tmp_path / "pack", cfg, device=DEV, verify=True)
    for k in w:
        assert got[k].device == DEV and torch.equal(got[k], w[k]), k
    ep = load_pack(tmp_path / "pack", cfg, device=DEV, experts=(4, 8))
    ref = init_weights(cfg, seed=0, device=DEV, dtype=torch.bfloat16, experts=(4, 8))
    assert torch.equal(ep["l1.e_w13"], ref["l1.e_w13"]) and torch.equal(ep["l1.e_w2"], ref["l1.e_w2"])
    a = _tokens(MLAMoEModel(cfg, weights={k: v.clone() for k, v in w.items()}, device=DEV, max_positions=1024), cfg)
    b = _tokens(MLAMoEModel(cfg, weights=got, device=DEV, max_positions=1024), cfg)
    assert a == b
