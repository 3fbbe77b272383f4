"""Device arenas of a DeepSeek-V4 KV cache plan and per-layer views into them.

``build_plan`` (C++, ``core().dsv4_cache_plan``) sizes and places every layer's
sliding window, compressed history (with the indexer keys of ratio-4 layers) and
compressor state; ``Dsv4CacheArena`` allocates the three arenas once on a device and
hands out per-layer byte views: ``[sequences, bytes]`` for the per-sequence regions
(sliding window, compressor state) and ``[bytes]`` for the shared history. Every
view starts on the plan's alignment (256 B by default), so a TMA tensor map over it
meets the 16-byte base rule.

Reference behaviour: crates/spark-abi/vendor/sparkpipe/model-families/dsv4/include/sparkpipe/
spark_dsv4_cache_arena.h:13-40 (arena allocation and layer views).
"""
from __future__ import annotations

import torch

from ..core import core


def _mod():
    return core().dsv4_cache_plan


def plan_config(variant: str = "flash", first_layer: int = 0, layers: int | None = None, mtp: bool = False,
                sequences: int = 64, max_context: int = 131072, aggregate_context: int | None = None, **bits):
    """PlanConfig with the given layer range and capacities (aggregate defaults to
    sequences x max_context); ``bits`` sets content_bits / rope_bits / indexer_bits /
    state_bits / page_entries / alignment."""
    m = _mod()
    v = m.Variant.FLASH if variant == "flash" else m.Variant.PRO
    c = m.PlanConfig()
    c.variant = v
    c.first_backbone_layer = first_layer
    c.backbone_layer_count = layers if layers is not None else m.geometry(v).backbone_layers - first_layer
    c.include_mtp_layer = mtp
    c.active_sequence_capacity = sequences
    c.max_context_tokens_per_sequence = max_context
    c.aggregate_context_token_capacity = aggregate_context if aggregate_context is not None else sequences * max_context
    for k, val in bits.items():
        setattr(c, k, val)
    return c


def build_plan(cfg):
    return _mod().build_plan(cfg)


def _packed(elements: int, bits: int) -> int:
    return (elements * bits + 7) // 8


class Dsv4CacheArena:
    """The three arenas of one plan on ``device``, zero-filled."""

    def __init__(self, plan, device):
        self.plan = plan
        self.geometry = _mod().geometry(plan.config.variant)
        mk = lambda n: torch.zeros(max(int(n), 1), dtype=torch.uint8, device=device)  # noqa: E731
        self.sliding = mk(plan.sliding_arena_bytes)
        self.history = mk(plan.history_arena_bytes)
        self.state = mk(plan.state_arena_bytes)

    @property
    def nbytes(self) -> int:
        return self.sliding.numel() + self.history.numel() + self.state.numel()

    def layer_view(self, i: int) -> dict:
        L, c, g = self.plan.layers[i], self.plan.config, self.geometry
        S = c.active_sequence_capacity
        content_dim = g.head_dim - g.rope_dim

        def per_seq(arena, base, stride, off, nbytes):
            return torch.as_strided(arena, (S, nbytes), (stride, 1), base + off)

        def shared(arena, base, off, nbytes):
            return arena[base + off: base + off + nbytes]

        v = {
            "layer": L.absolute_layer, "ratio": L.ratio, "class": L.attn_class,
            "sliding_content": per_seq(self.sliding, L.sliding_arena_offset, L.sliding_sequence_stride,
                                       L.sliding_content_offset, _packed(L.sliding_entries_per_sequence * content_dim, c.content_bits)),
            "sliding_rope": per_seq(self.sliding, L.sliding_arena_offset, L.sliding_sequence_stride,
                                    L.sliding_rope_offset, _packed(L.sliding_entries_per_sequence * g.rope_dim, c.rope_bits)),
        }
        if L.ratio == 0:
            return v
        E = L.compressed_entries
        v["compressed_content"] = shared(self.history, L.history_arena_offset, L.compressed_content_offset,
                                         _packed(E * content_dim, c.content_bits))
        v["compressed_rope"] = shared(self.history, L.history_arena_offset, L.compressed_rope_offset,
                                      _packed(E * g.rope_dim, c.rope_bits))
        csa = L.ratio == 4
        cw = (2 if csa else 1) * g.head_dim
        st = lambda off, tokens, width: per_seq(self.state, L.state_arena_offset, L.state_sequence_stride,  # noqa: E731
                                                off, _packed(tokens * width, c.state_bits))
        v["compressor_kv"] = st(L.compressor_kv_offset, L.compressor_buffer_tokens, cw)
        v["compressor_gate"] = st(L.compressor_gate_offset, L.compressor_buffer_tokens, cw)
        if csa:
            v["indexer_history"] = shared(self.history, L.history_arena_offset, L.indexer_history_offset,
                                          _packed(E * g.index_head_dim, c.indexer_bits))
            iw = 2 * g.index_head_dim
            v["indexer_kv"] = st(L.indexer_kv_offset, L.indexer_buffer_tokens, iw)
            v["indexer_gate"] = st(L.indexer_gate_offset, L.indexer_buffer_tokens, iw)
            v["compressor_overlap_kv"] = st(L.compressor_overlap_kv_offset, L.ratio, g.head_dim)
            v["compressor_overlap_gate"] = st(L.compressor_overlap_gate_offset, L.ratio, g.head_dim)
            v["indexer_overlap_kv"] = st(L.indexer_overlap_kv_offset, L.ratio, g.index_head_dim)
            v["indexer_overlap_gate"] = st(L.indexer_overlap_gate_offset, L.ratio, g.index_head_dim)
        return v
