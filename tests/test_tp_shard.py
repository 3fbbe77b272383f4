"""Tensor-parallel shard views and node-config derivation (C++), on CPU.

The node-config hashes are golden values of the reference's shape derivation
(crates/spark-node/src/rank_daemon/shape.rs tests); the shard views are checked by
reassembling the full tensors from every rank's slices and by exact equality of a
TP-sharded matmul against the unsharded one."""
import pytest
import torch

from sparkpipe_rs_b200.core import StatusError, core
from sparkpipe_rs_b200.models.config import tiny, v2_lite
from sparkpipe_rs_b200.models.weights import init_weights
from sparkpipe_rs_b200.parallel.tensor_parallel import geometry, node_config, shard_tensor, shard_weights

T = core().tp
GLM_GEO = T.Geometry(64, 192 + 64, 192 + 256, 256)
GLM_IN = T.ModelInputs(78, 6144, 2048, 12288, 512 + 64, 1)


def test_node_config_matches_reference_hashes():
    c = T.derive_node_config(T.Shape(1, 0, 13, 5), GLM_GEO, GLM_IN)
    assert c.configuration_hash == 2005884353472861467
    assert (c.first_layer_index, c.layer_count, c.kv_bytes_per_token) == (30, 6, 3456)
    c = T.derive_node_config(T.Shape(2, 1, 6, 3), GLM_GEO, GLM_IN)
    assert c.configuration_hash == 9169625037557488130
    assert (c.first_layer_index, c.layer_count, c.heads_per_rank, c.moe_intermediate_per_rank,
            c.kv_bytes_per_token) == (39, 13, 32, 1024, 7488)
    c = T.derive_node_config(T.Shape(16, 0, 13, 0), GLM_GEO, GLM_IN)
    assert (c.heads_per_rank, c.moe_intermediate_per_rank) == (4, 128)


@pytest.mark.parametrize("shape", [(3, 0, 13, 0), (2, 2, 13, 0), (1, 0, 13, 13), (1, 0, 0, 0), (1, 0, 5, 0)])
def test_node_config_rejects_invalid_shapes(shape):
    with pytest.raises(StatusError) as e:
        T.derive_node_config(T.Shape(*shape), GLM_GEO, GLM_IN)
    assert e.value.code == 1


def test_classification_and_views():
    geo = GLM_GEO
    assert T.classify("l3.w_qkv_a") == T.ShardClass.REPLICATED
    assert T.classify("model.layers.3.self_attn.q_b_proj.weight") == T.ShardClass.OUTPUT_DIM_HEADS
    assert T.classify("l3.w_o") == T.ShardClass.INPUT_DIM_HEADS
    assert T.classify("l0.w13") == T.ShardClass.CONCAT_OUTPUT
    assert T.classify("l5.e_w2") == T.ShardClass.INPUT_DIM
    assert T.classify("mystery") == T.ShardClass.UNKNOWN
    v = T.compute_view(T.TensorSpec("l1.w_q_b", [64 * 256, 2048]), T.Shape(4, 2), geo)
    assert v.split_dimension == 0 and v.ranges == [(2 * 16 * 256, 16 * 256)]
    assert v.shard_bytes == 16 * 256 * 2048 * 2
    v = T.compute_view(T.TensorSpec("l1.w_o", [6144, 64 * 256]), T.Shape(8, 7), geo)
    assert v.split_dimension == 1 and v.ranges == [(7 * 8 * 256, 8 * 256)]
    v = T.compute_view(T.TensorSpec("l1.e_w13", [10, 4096, 6144]), T.Shape(4, 1), geo)
    assert v.split_dimension == 1 and v.ranges == [(512, 512), (2048 + 512, 512)]
    v = T.compute_view(T.TensorSpec("mystery", [8, 8]), T.Shape(1, 0), geo)
    assert v.shard_class == T.ShardClass.REPLICATED  # degree one: everything whole
    with pytest.raises(StatusError):
        T.compute_view(T.TensorSpec("mystery", [8, 8]), T.Shape(2, 0), geo)
    with pytest.raises(StatusError):
        T.compute_view(T.TensorSpec("l1.w_q_b", [100, 8]), T.Shape(2, 0), geo)  # not whole heads
    h0 = T.geometry_hash(T.TensorSpec("l1.w_o", [6144, 16384]), T.Shape(8, 7),
                         T.compute_view(T.TensorSpec("l1.w_o", [6144, 16384]), T.Shape(8, 7), geo))
    h1 = T.geometry_hash(T.TensorSpec("l1.w_o", [6144, 16384]), T.Shape(8, 6),
                         T.compute_view(T.TensorSpec("l1.w_o", [6144, 16384]), T.Shape(8, 6), geo))
    assert h0 != h1


@pytest.mark.parametrize("degree", [2, 4])
def test_sharded_mlp_and_attention_projections_reassemble(degree):
    cfg = tiny().replace(num_heads=8)
    w = init_weights(cfg, seed=2, dtype=torch.float32)
    shards = [shard_weights(cfg, w, degree, r) for r in range(degree)]
    x = torch.randn(5, cfg.hidden_size)
    # dense/expert MLP: column-parallel [gate; up], row-parallel down; sum of partials == full
    for name13, name2 in [("l0.e_w13", "l0.e_w2")]:
        full13, full2 = w[name13][0], w[name2][0]
        F = full13.shape[0] // 2
        ref = (torch.nn.functional.silu(x @ full13[:F].t()) * (x @ full13[F:].t())) @ full2.t()
        acc = torch.zeros_like(ref)
        for s in shards:
            w13, w2_ = s[name13][0], s[name2][0]
            f = w13.shape[0] // 2
            acc += (torch.nn.functional.silu(x @ w13[:f].t()) * (x @ w13[f:].t())) @ w2_.t()
        assert torch.allclose(acc, ref, atol=1e-5)
    # q_b: concatenating the ranks' output rows restores the full projection
    full = w["l0.w_q_b"]
    cat = torch.cat([s["l0.w_q_b"] for s in shards], 0)
    assert torch.equal(cat, full)
    # w_o: input-split partial sums add up to the full projection
    attn = torch.randn(5, cfg.num_heads * cfg.v_head_dim)
    per = cfg.num_heads * cfg.v_head_dim // degree
    acc = sum(attn[:, r * per:(r + 1) * per] @ shards[r]["l0.w_o"].t() for r in range(degree))
    assert torch.allclose(acc, attn @ w["l0.w_o"].t(), atol=1e-5)
    # replicated tensors are the same object on every rank
    assert all(s["l0.w_qkv_a"] is w["l0.w_qkv_a"] for s in shards)


def test_node_config_of_v2_lite():
    c = node_config(v2_lite(), 2, 1, 1, 0)
    assert c.heads_per_rank == 8 and c.moe_intermediate_per_rank == 704 and c.layer_count == 27
    assert c.kv_bytes_per_token == 27 * 576 * 2
