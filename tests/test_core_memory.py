"""KvArena / Arena / StatePool / BatchSequenceTable / row allocator of the C++ runtime.

Scenarios follow the reference's spark-core tests (crates/spark-core/tests/kv_arena.rs,
arena.rs, state_pool.rs, batch_sequence_table.rs, row_allocator.rs).
"""
import pytest

from sparkpipe_rs_b200.core import core, StatusError


def arena(blocks=8, resident=0):
    c = core().KvArenaConfig()
    c.physical_block_count = blocks
    c.block_token_count = 16
    c.resident_block_capacity = resident
    c.layer_count = 2
    c.kv_head_count = 1
    c.head_dim = 576
    c.bytes_per_scalar = 2
    c.key_device_base = 0x1000
    return core().KvArena(c)


def test_kv_arena_acquire_lowest_free_and_generation():
    a = arena(4)
    assert [a.acquire_block() for _ in range(4)] == [0, 1, 2, 3]
    with pytest.raises(StatusError) as e:
        a.acquire_block()
    assert e.value.status == "capacity_exceeded"
    g = a.generation(2)
    a.free_block(2)
    assert a.generation(2) == g + 1
    assert a.acquire_block() == 2
    assert a.allocated_block_count == 5


def test_kv_arena_refcount_rules():
    a = arena(4)
    b = a.acquire_block()
    assert a.reference_count(b) == 0
    with pytest.raises(StatusError):
        a.release_block_reference(b)  # releasing at zero is rejected
    a.retain_block(b)
    a.retain_block(b)
    with pytest.raises(StatusError) as e:
        a.free_block(b)
    assert e.value.status == "busy"
    a.release_block_reference(b)
    a.release_block_reference(b)
    a.free_block(b)
    a.free_block(b)  # freeing a free block is a no-op
    assert not a.is_allocated(b)
    assert a.retained_block_count == 2 and a.released_reference_count == 2


def test_kv_arena_device_addresses_follow_stride():
    a = arena(4)
    b = a.acquire_block()
    stride = 16 * 2 * 1 * 576 * 2
    assert a.key_block_stride_bytes == stride
    a.acquire_block()
    v = a.resolve_block(1)
    assert v.key_device_address == 0x1000 + stride
    assert a.value_device_address(b) == 0  # no value payload configured


def test_kv_arena_resident_capacity_evicts_lru_lowest_refcount():
    a = arena(6, resident=2)
    blocks = [a.acquire_block() for _ in range(3)]
    a.mark_block_resident(blocks[0])
    a.mark_block_resident(blocks[1])
    a.retain_block(blocks[0])  # referenced blocks are evicted last
    a.mark_block_resident(blocks[2])
    assert a.is_resident(blocks[0]) and not a.is_resident(blocks[1]) and a.is_resident(blocks[2])
    assert a.resident_evicted_block_count == 1
    assert a.resident_block_count == 2


def test_kv_arena_trim_stalls_when_everything_protected():
    a = arena(4, resident=4)
    bs = [a.acquire_block() for _ in range(2)]
    for b in bs:
        a.mark_block_resident(b)
    with pytest.raises(StatusError):
        a.trim_resident_blocks(bs, 0)
    assert a.resident_capacity_stall_count == 1
    assert a.evict_resident_blocks_to_limit(0, bs) == 0  # quiet variant
    assert a.evict_resident_blocks_to_limit(0, []) == 2


def test_kv_arena_reset_keeps_cumulative_counters():
    a = arena(4, resident=1)
    x, y = a.acquire_block(), a.acquire_block()
    a.mark_block_resident(x)
    a.mark_block_resident(y)
    ev = a.resident_evicted_block_count
    a.reset()
    assert a.resident_evicted_block_count == ev and a.epoch == 0 and a.allocated_block_count == 0
    assert a.generation(0) == 0


def test_arena_size_classes_and_stale_handles():
    ar = core().Arena([(24, 2), (100, 1)])
    h1 = ar.acquire(10)
    assert h1.class_index == 0 and ar.class_slot_bytes(0) == 32  # rounded to 16 bytes
    h2 = ar.acquire(50)
    assert h2.class_index == 1
    ar.write(h1, b"hello")
    assert ar.read(h1, 5) == b"hello"
    ar.release(h1)
    with pytest.raises(StatusError):
        ar.release(h1)  # stale handle
    h3 = ar.acquire(10)
    assert h3.slot_index == h1.slot_index and h3.generation == h1.generation + 1
    with pytest.raises(StatusError):
        ar.acquire(1000)
    with pytest.raises(StatusError):
        core().Arena([(64, 1), (32, 1)])  # sizes must strictly increase


def test_state_pool():
    p = core().StatePool(2, 64)
    a, b = p.acquire(), p.acquire()
    assert {a, b} == {0, 1} and p.acquire() == -1
    p.release(a)
    with pytest.raises(StatusError):
        p.release(a)
    assert p.free_count == 1 and p.acquire() == a


def test_batch_sequence_table_lifecycle_and_threshold():
    t = core().BatchSequenceTable(4, 2)
    h = t.admit(77, 100, 0, 3)
    assert t.sequence(h).sequence_id == 77 and t.active_count == 1
    t.pause_for_tool(h)
    assert t.awaiting_tool_count == 1
    t.begin_exchange(h, 25)
    assert t.sequence(h).context_tokens == 125 and t.sequence(h).exchange_number == 1
    for i in range(3):
        t.admit(i, 1, 0, 1)
    # firing threshold = active * lanes * topk / experts, clamped
    assert t.firing_threshold(8, 256, 1024) == max(1, 4 * 2 * 8 // 256)
    assert t.firing_threshold(8, 4, 10) == 10
    t.complete(h)
    with pytest.raises(StatusError):
        t.sequence(h)  # generation bumped: stale
    h2 = t.admit(5, 1, 0, 1)
    assert (h2 & ((1 << 14) - 1)) == (h & ((1 << 14) - 1)) and h2 != h


# row allocator: ported scenarios (milli fixed point traces)
def ra(slots, cap, cost=1000):
    return core().row_allocator_assign(slots, cap, cost)


def test_row_allocator_saturated_wave_is_all_real():
    assert ra([(2900, 5, 0)] * 8, 8) == (8, [0] * 8)


def test_row_allocator_undersubscribed_fills_by_alpha():
    total, b = ra([(2900, 5, 0), (1300, 5, 0)], 8)
    assert total == 8 and b == [5, 1]


def test_row_allocator_suppressed_and_probe():
    assert ra([(900, 0, 0), (2900, 5, 0)], 16) == (7, [0, 5])
    total, b = ra([(1000, 5, 1), (2900, 5, 0)], 4)
    assert b[0] == 2  # the probe grant comes first


def test_row_allocator_cost_weighting_and_zero_cap():
    assert ra([(2900, 5, 0), (1300, 5, 0)], 8, 600) == (8, [5, 1])
    assert ra([(2900, 5, 0), (1300, 5, 0)], 2, 600) == (2, [0, 0])
    assert ra([(2900, 5, 0)] * 2, 0)[0] == 0
    assert ra([(2900, 5, 0)] * 4, 2) == (2, [0, 0, 0, 0])


def test_row_allocator_deterministic_ties_prefer_lower_index():
    total, b = ra([(2000, 3, 0), (2000, 3, 0)], 3)
    assert b == [1, 0]
