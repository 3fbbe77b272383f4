"""DeepSeek-V4 KV cache plan (C++) and its arena views: layer classes from the
published compress ratios, region sizes and offsets worked out by hand for one
configuration, alignment of every region, worst-class totals, bounds, and views
that tile the arenas without overlap.

Layer classes and record fields follow
crates/spark-abi/vendor/sparkpipe/model-families/dsv4/include/sparkpipe/spark_dsv4_cache_plan.h."""
import pytest
import torch

from sparkpipe_rs_b200.core import core
from sparkpipe_rs_b200.models.dsv4_cache import Dsv4CacheArena, build_plan, plan_config

D = core().dsv4_cache_plan


def test_layer_classes():
    F, P = D.Variant.FLASH, D.Variant.PRO
    assert [D.compression_ratio(F, i) for i in range(6)] == [0, 0, 4, 128, 4, 128]
    assert [D.compression_ratio(P, i) for i in range(6)] == [128, 128, 4, 128, 4, 128]
    assert D.compression_ratio(F, 42) == 4 and D.compression_ratio(P, 60) == 4
    assert D.compression_ratio(F, 0, True) == 0 and D.compression_ratio(P, 0, True) == 0
    with pytest.raises(Exception):
        D.compression_ratio(F, 43)
    p = build_plan(plan_config("flash", mtp=True, sequences=4, max_context=4096))
    assert (p.sliding_layers, p.compressed_sparse_layers, p.heavily_compressed_layers) == (3, 21, 20)
    assert len(p.layers) == 44 and p.layers[-1].mtp_layer and p.layers[-1].absolute_layer == 43
    p = build_plan(plan_config("pro", mtp=True, sequences=4, max_context=4096))
    assert (p.sliding_layers, p.compressed_sparse_layers, p.heavily_compressed_layers) == (1, 30, 31)


def test_sizes_by_hand():
    # Flash layer 2 (ratio 4) and 3 (ratio 128); 8-bit content, 16-bit RoPE, 8-bit indexer, 32-bit state
    cfg = plan_config("flash", first_layer=2, layers=2, sequences=2, max_context=50000, aggregate_context=100000)
    p = build_plan(cfg)
    csa, hca = p.layers
    assert csa.attn_class == D.AttnClass.COMPRESSED_SPARSE and hca.attn_class == D.AttnClass.HEAVILY_COMPRESSED
    # sliding: 127 entries x 448 content bytes, then 127 x 64 x 2 RoPE bytes at the next 256 B
    assert csa.sliding_entries_per_sequence == 127
    assert (csa.sliding_content_offset, csa.sliding_rope_offset, csa.sliding_sequence_stride) == (0, 57088, 73472)
    # history: ceil(100000 / 4) = 25000 entries -> 49 pages of 512 = 25088
    assert csa.compressed_entries == 25088
    assert (csa.compressed_content_offset, csa.compressed_rope_offset, csa.indexer_history_offset) == (
        0, 11239424, 14450688)
    assert csa.history_arena_bytes == 17661952
    # ratio 128: ceil(100000 / 128) = 782 -> 2 pages = 1024 entries, no indexer
    assert hca.compressed_entries == 1024 and hca.indexer_history_offset == 0
    assert hca.history_arena_bytes == 1024 * 448 + 1024 * 64 * 2
    # compressor state of one ratio-4 sequence (fp32): 3 x 1024 kv, 3 x 1024 gate, 3 x 256 x 2,
    # then 4 x 512 x 2 and 4 x 128 x 2 overlap
    assert (csa.compressor_kv_offset, csa.compressor_gate_offset, csa.indexer_kv_offset, csa.indexer_gate_offset) == (
        0, 12288, 24576, 27648)
    assert (csa.compressor_overlap_kv_offset, csa.compressor_overlap_gate_offset) == (30720, 38912)
    assert (csa.indexer_overlap_kv_offset, csa.indexer_overlap_gate_offset, csa.state_sequence_stride) == (
        47104, 49152, 51200)
    # ratio 128: 127 tokens x 512 x 4 B for kv and gate
    assert hca.compressor_buffer_tokens == 127 and hca.state_sequence_stride == 2 * 127 * 512 * 4
    # arenas: layers one after the other, aligned
    assert hca.sliding_arena_offset == csa.sliding_arena_bytes == 2 * 73472
    assert hca.history_arena_offset == csa.history_arena_bytes
    assert p.total_arena_bytes == p.sliding_arena_bytes + p.history_arena_bytes + p.state_arena_bytes
    # worst class: every layer ratio 4 for history, ratio 128 for state
    assert p.worst_history_bytes == 2 * csa.history_arena_bytes
    assert p.worst_state_bytes == 2 * 2 * hca.state_sequence_stride
    assert p.worst_total_bytes >= p.total_arena_bytes


def test_alignment_and_bounds():
    cfg = plan_config("pro", sequences=3, max_context=8192, alignment=1024, content_bits=4, state_bits=16)
    p = build_plan(cfg)
    for L in p.layers:
        for f in ("sliding_rope_offset", "sliding_sequence_stride", "sliding_arena_offset", "compressed_rope_offset",
                  "indexer_history_offset", "history_arena_offset", "history_arena_bytes", "compressor_gate_offset",
                  "state_sequence_stride", "state_arena_offset"):
            assert getattr(L, f) % 1024 == 0, f
    for bad in (dict(alignment=100), dict(page_entries=500), dict(content_bits=12)):
        with pytest.raises(Exception):
            build_plan(plan_config("flash", sequences=2, max_context=1024, **bad))
    with pytest.raises(Exception):
        build_plan(plan_config("flash", first_layer=40, layers=4, sequences=2, max_context=1024))
    with pytest.raises(Exception):
        build_plan(plan_config("flash", sequences=2, max_context=(1 << 20) + 1))
    with pytest.raises(Exception):
        build_plan(plan_config("flash", sequences=4, max_context=16, aggregate_context=2))


def test_arena_views_tile_without_overlap():
    p = build_plan(plan_config("flash", first_layer=0, layers=5, mtp=True, sequences=3, max_context=2048))
    a = Dsv4CacheArena(p, "cpu")
    assert a.nbytes == p.total_arena_bytes
    owner = {name: torch.zeros(t.numel(), dtype=torch.int32) for name, t in
             (("sliding", a.sliding), ("history", a.history), ("state", a.state))}
    base = {name: t.data_ptr() for name, t in (("sliding", a.sliding), ("history", a.history), ("state", a.state))}
    for i in range(len(p.layers)):
        v = a.layer_view(i)
        for k, t in v.items():
            if not isinstance(t, torch.Tensor):
                continue
            arena = "sliding" if k.startswith("sliding") else (
                "history" if k in ("compressed_content", "compressed_rope", "indexer_history") else "state")
            assert (t.data_ptr() - base[arena]) % 256 == 0
            t.fill_(1)
            off = t.data_ptr() - base[arena]
            if t.dim() == 2:
                for s in range(t.shape[0]):
                    seg = owner[arena][off + s * t.stride(0): off + s * t.stride(0) + t.shape[1]]
                    assert int(seg.sum()) == 0, (i, k)
                    seg += 1
            else:
                seg = owner[arena][off: off + t.numel()]
                assert int(seg.sum()) == 0, (i, k)
                seg += 1
        if v["ratio"] == 0:
            assert "compressed_content" not in v
        elif v["ratio"] == 4:
            assert "indexer_history" in v and v["indexer_overlap_gate"].shape[0] == 3
