"""Prefix cache: hash parity with the reference's pinned values and reuse scenarios
(crates/spark-core/tests/prefix_cache.rs)."""
import pytest

from sparkpipe_rs_b200.core import core, StatusError


def tokens(start, n):
    return list(range(start, start + n))


def test_hash_block_matches_reference_values():
    C = core()
    assert C.prefix_hash_block(tokens(1000, 4), C.EMPTY_PARENT_HASH) == 17187592518832544614
    h = (C.EMPTY_PARENT_HASH ^ 1099511628211) * 1099511628211 % (1 << 64)
    h ^= h >> 32
    assert C.prefix_hash_block([], C.EMPTY_PARENT_HASH) == h


def test_hash_prompt_matches_reference_values():
    C = core()
    r = C.prefix_hash_prompt(4, C.EMPTY_PARENT_HASH, tokens(1000, 16))
    assert r.prompt_hash == 11250298247205927079
    assert (r.block_count, r.last_block_token_count, r.hashed_token_count) == (4, 4, 16)
    ids = [100000 + i * 37 for i in range(80)]
    assert C.prefix_hash_prompt(16, C.EMPTY_PARENT_HASH, ids).prompt_hash == 14918569915938236142
    assert C.prefix_hash_prompt(16, C.EMPTY_PARENT_HASH, ids[:48]).prompt_hash == 1825709821990993003
    e = C.prefix_hash_prompt(4, C.EMPTY_PARENT_HASH, [])
    assert e.prompt_hash == C.EMPTY_PARENT_HASH and e.block_count == 0
    for bad in (0, 257):
        with pytest.raises(StatusError):
            C.prefix_hash_prompt(bad, C.EMPTY_PARENT_HASH, ids)


def test_chained_block_hash_matches_full_hash():
    C = core()
    ids = [100000 + i * 37 for i in range(80)]
    chained = C.EMPTY_PARENT_HASH
    for end in range(16, 81, 16):
        full = C.prefix_hash_prompt(16, C.EMPTY_PARENT_HASH, ids[:end]).prompt_hash
        chained = C.prefix_hash_prompt(16, chained, ids[end - 16:end]).prompt_hash
        assert chained == full


def test_second_sequence_reuses_committed_blocks():
    c = core().PrefixCache(4, 16, 8)
    p = tokens(1000, 16)
    r1 = c.reserve_prompt(1, p)
    assert r1.reusable_token_count == 0 and len(r1.physical_blocks) == 4
    c.commit(1, 16)
    lk = c.probe_prompt(p)
    # reuse stops one token short of the prompt (the last token is recomputed)
    assert lk.matched_token_count == 12 and lk.matched_block_count == 3
    r2 = c.reserve_prompt(2, p)
    assert r2.reusable_token_count == 12
    assert r2.physical_blocks[:3] == r1.physical_blocks[:3]
    assert r2.physical_blocks[3] != r1.physical_blocks[3]
    assert c.reference_count(r1.physical_blocks[0]) == 2
    assert c.stats.hits == 1 and c.stats.hit_tokens == 12


def test_released_blocks_stay_warm_and_evict_lru():
    c = core().PrefixCache(4, 4, 8)
    p = tokens(1, 9)  # 3 blocks, two full
    c.reserve_prompt(1, p)
    c.commit(1, 9)
    c.release_sequence(1)
    assert c.warm_blocks == 2 and c.free_blocks == 2  # the partial block was freed
    assert c.probe_prompt(p).matched_block_count == 2
    # a different prompt needing 4 blocks evicts the warm ones (oldest first)
    r = c.reserve_prompt(2, tokens(500, 16))
    assert len(r.physical_blocks) == 4 and c.stats.evicted_blocks == 2
    assert c.probe_prompt(p).matched_block_count == 0


def test_reservation_is_all_or_nothing():
    c = core().PrefixCache(4, 3, 8)
    c.reserve_prompt(1, tokens(0, 8))
    with pytest.raises(StatusError) as e:
        c.reserve_prompt(2, tokens(100, 8))
    assert e.value.status == "capacity_exceeded"
    assert not c.has_sequence(2) and c.free_blocks == 1


def test_capacity_growth_and_cancel():
    c = core().PrefixCache(4, 8, 4)
    c.reserve_prompt(7, tokens(0, 5))
    c.ensure_sequence_token_capacity(7, 13)
    assert len(c.block_table(7)) == 4
    c.cancel_reservation(7)
    assert c.free_blocks == 8 and c.stats.cancellations == 1
    with pytest.raises(StatusError):
        c.release_sequence(7)
    with pytest.raises(StatusError):
        c.reserve_prompt(1, [])


def test_decode_blocks_commit_after_append():
    c = core().PrefixCache(4, 8, 4)
    c.reserve_prompt(1, tokens(0, 3))
    c.append_tokens(1, [50, 51, 52, 53, 54])
    c.ensure_sequence_token_capacity(1, 8)
    c.commit(1, 8)
    lk = c.probe_prompt(tokens(0, 3) + [50, 51, 52, 53, 54, 99])
    assert lk.matched_token_count == 8


def test_bind_committed_prefix_from_sequence():
    c = core().PrefixCache(4, 8, 4)
    c.reserve_prompt(1, tokens(0, 10))
    c.commit(1, 10)
    assert c.bind_committed_prefix_from_sequence(1, 2, 10) == 8
    assert c.block_table(2) == c.block_table(1)[:2]
    with pytest.raises(StatusError):
        c.bind_committed_prefix_from_sequence(1, 2, 4)
