"""Work packets, identity, MTP draft tree and the KV directory (C++)."""
import numpy as np
import pytest

from sparkpipe_rs_b200.core import core, StatusError


def W():
    return core().work_control


def ident(phase=2):
    i = W().Identity()
    i.control_generation = i.transaction_id = i.dispatch_generation = i.request_generation = i.step_generation = 1
    i.step_chunk_count = 1
    i.transaction_phase = phase
    return i


def test_fingerprint_is_fnv1a_with_zero_remap():
    assert W().fingerprint_bytes(b"") == 0
    h = 14695981039346656037
    for b in b"abc":
        h = ((h ^ b) * 1099511628211) % (1 << 64)
    assert W().fingerprint_bytes(b"abc") == h


def test_identity_validation():
    W().validate_identity(ident())
    bad = ident()
    bad.step_chunk_index = 1
    with pytest.raises(StatusError):
        W().validate_identity(bad)
    with pytest.raises(StatusError):
        W().validate_identity(ident(phase=9))


def test_mtp_tree_topology_and_resolution():
    mt = W().mtp_tree
    assert mt.topology_is_valid()
    assert [mt.accepted_token_count(p) for p in range(6)] == [0, 1, 2, 2, 3, 3]
    cand = [10, 11, 12, 13, 14]
    # verifier rows: row0 predicts cand0 -> row1 predicts cand1 -> row2 predicts cand4
    assert mt.resolve(cand, [10, 11, 14, 0, 0, 0], 100) == (5, 3, 4, 5)
    assert mt.resolve(cand, [10, 12, 0, 0, 0, 0], 100) == (3, 2, 3, 3)
    assert mt.resolve(cand, [99, 0, 0, 0, 0, 0], 100) == (0, 0, 1, 0)
    with pytest.raises(StatusError):
        mt.resolve(cand, [100, 0, 0, 0, 0, 0], 100)
    assert mt.resolution_is_valid(5, 3, 5) and not mt.resolution_is_valid(5, 2, 5)
    assert mt.resolution_is_valid(0, 0, 0) and not mt.resolution_is_valid(3, 1, 1)


def test_queue_depth_buckets_and_chunks():
    assert W().queue_depth(1023) == 1024
    assert W().select_batch_bucket(17) == 32 and W().select_batch_bucket(1024) == 1024
    with pytest.raises(StatusError):
        W().select_batch_bucket(1025)
    assert W().execution_chunk_shape(100, 6, 256, 1024) == (42, 3)


def test_packet_from_scheduler_plan_roundtrips_and_validates():
    C = core()
    sc = C.SchedulerConfig()
    sc.max_batch, sc.block_tokens, sc.num_blocks, sc.max_model_len = 4, 64, 64, 1024
    s = C.Scheduler(sc)
    s.add_request(C.RequestSpec(1, list(range(30)), 4))
    s.add_request(C.RequestSpec(2, list(range(50, 70)), 4))
    plan = s.schedule()
    cfg = W().Config()
    cfg.output_vocab_count = 1000
    p = W().build_step_packet(plan, ident(1), cfg, 0)
    W().validate_packet(p, cfg)
    assert p.new_token_count == 50 and len(p.lanes) == 2
    raw = p.serialize()
    q = W().deserialize(raw)
    assert q.fingerprint() == p.fingerprint() and q.serialize() == raw
    s.complete(plan, np.array([3, 4], np.int32))
    dp = W().build_step_packet(s.schedule(), ident(2), cfg, 1)
    W().validate_packet(dp, cfg)
    assert [l.input_token_id for l in dp.lanes] == [3, 4]
    assert [l.context_token_count for l in dp.lanes] == [31, 21]
    tampered = bytearray(raw)
    tampered[0] ^= 1
    with pytest.raises(StatusError):
        W().deserialize(bytes(tampered))
    with pytest.raises(StatusError):
        W().deserialize(raw[:-1])


def test_kv_directory_sharing_pins_and_sweep():
    d = W().KvDirectory(16, 4)
    b0, hit = d.acquire(1, 0, 0)
    assert not hit
    d.mark_resident(1, 0)
    b1, hit = d.acquire(2, 0, 0)
    assert b1 != b0
    # identical content shares the resident block
    d.acquire(3, 0, 777)
    d.mark_resident(3, 0)
    b3, hit = d.acquire(4, 0, 777)
    assert hit and d.shared_hits == 1
    d.pin(1, 0)
    d.acquire(5, 0, 0)  # takes the last free block
    assert d.free_blocks == 0 and d.sweeps == 0
    # pool exhausted: the clock sweep evicts unpinned entries (second chance)
    d.acquire(6, 0, 0)
    assert d.sweeps >= 1
    assert d.find(1, 0) is not None  # pinned survives
    d.release_sequence(5)
    assert d.find(5, 0) is None
    g = d.generation
    d.reset()
    assert d.generation == g + 1 and d.live_entries == 0 and d.free_blocks == 4
