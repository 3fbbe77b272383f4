"""Tensor-parallel weight sharding of the MLA-MoE model.

``shard_weights(cfg, weights, tp_degree, tp_rank)`` returns this rank's slices of
the model's weights as computed by the C++ shard engine (``core().tp``): the MLA
latent projections, norms, router and embedding replicate; q_b / kv_b split their
output dimension on whole heads, o_proj its input dimension; dense and expert MLPs
split their intermediate dimension ([gate; up] stacks split each half).
``node_config(cfg, ...)`` gives the per-rank dimensions and the configuration hash
of a (TP, PP) shape.
"""
from __future__ import annotations

import torch

from ..core import core
from ..models.config import MLAMoEConfig


def geometry(cfg: MLAMoEConfig):
    T = core().tp
    return T.Geometry(cfg.num_heads, cfg.qk_nope_head_dim + cfg.qk_rope_head_dim,
                      cfg.qk_nope_head_dim + cfg.v_head_dim, cfg.v_head_dim)


def shard_tensor(name: str, t: torch.Tensor, shape, geo) -> torch.Tensor:
    T = core().tp
    view = T.compute_view(T.TensorSpec(name, list(t.shape), t.element_size()), shape, geo)
    if view.shard_class == T.ShardClass.REPLICATED:
        return t
    parts = [t.narrow(view.split_dimension, off, ext) for off, ext in view.ranges]
    out = parts[0] if len(parts) == 1 else torch.cat(parts, view.split_dimension)
    return out.contiguous()


def shard_weights(cfg: MLAMoEConfig, weights: dict, tp_degree: int, tp_rank: int, pp_stage_count: int = 1,
                  pp_stage_index: int = 0) -> dict:
    T = core().tp
    shape = T.Shape(tp_degree, tp_rank, pp_stage_count, pp_stage_index)
    geo = geometry(cfg)
    return {k: shard_tensor(k, v, shape, geo) for k, v in weights.items()}


def node_config(cfg: MLAMoEConfig, tp_degree: int, tp_rank: int, pp_stage_count: int, pp_stage_index: int,
                kv_bytes_per_element: int = 2):
    T = core().tp
    inputs = T.ModelInputs(cfg.num_layers, cfg.hidden_size, cfg.moe_intermediate_size, cfg.intermediate_size,
                           cfg.kv_cache_dim, kv_bytes_per_element)
    return T.derive_node_config(T.Shape(tp_degree, tp_rank, pp_stage_count, pp_stage_index), geometry(cfg), inputs)
