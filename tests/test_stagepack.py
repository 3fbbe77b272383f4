"""Checkpoint layout (stage packs), on CPU: writer / index / reader round trip of a
model's weights, fail-closed resolve, expert-parallel row ranges and
tensor-parallel shards read from the file, fingerprint checks, index atomicity, and
a model forward from loaded weights equal to the in-memory one. Behaviour follows
the stage-pack resolve contract and the shard read of the reference
(spark_glm52_stagepack.h:11-52, spark_tp_shard.h:132-148)."""
import json
import os

import pytest
import torch

from sparkpipe_rs_b200.core import StatusError, core
from sparkpipe_rs_b200.models import checkpoint as ckpt
from sparkpipe_rs_b200.models.config import tiny
from sparkpipe_rs_b200.models.weights import init_weights

S = core().stagepack
NOT_FOUND, SCHEMA, HASH, INVALID = 3, 6, 7, 1


@pytest.fixture(scope="module")
def packed(tmp_path_factory):
    cfg = tiny()
    w = init_weights(cfg, seed=3, dtype=torch.float32)
    root = tmp_path_factory.mktemp("pack") / "tiny"
    n = ckpt.save_pack(root, cfg, w)
    assert n == sum(t.numel() * t.element_size() for t in w.values())
    return cfg, w, root


def test_round_trip_is_bit_exact_and_regions_are_aligned(packed):
    cfg, w, root = packed
    got = ckpt.load_pack(root, cfg, verify=True)
    assert set(got) == set(w)
    for k in w:
        assert torch.equal(got[k], w[k]), k
    pk = S.Pack.open(str(root))
    assert pk.model_id == cfg.name and json.loads(pk.metadata)["config"]["hidden_size"] == cfg.hidden_size
    for name in pk.names():
        assert pk.entry(name)["offset"] % S.ALIGN == 0


def test_resolve_fails_closed(packed):
    cfg, w, root = packed
    pk = S.Pack.open(str(root))
    shape = list(w["l0.w_o"].shape)
    r = pk.resolve("l0.w_o", "F32", shape, 4)
    assert r.tensor_bytes == w["l0.w_o"].numel() * 4 and r.file_path.endswith(".bin")
    for args, code in [(("nope", "F32", shape, 4), NOT_FOUND), (("l0.w_o", "BF16", shape, 2), SCHEMA),
                       (("l0.w_o", "F32", shape[::-1], 4), SCHEMA), (("l0.w_o", "F32", shape + [1], 4), SCHEMA)]:
        with pytest.raises(StatusError) as e:
            pk.resolve(*args)
        assert e.value.code == code
    out = torch.empty(3)
    with pytest.raises(StatusError) as e:
        pk.read("l0.w_o", out.data_ptr(), 12)  # destination must be exactly the tensor
    assert e.value.code == INVALID


def test_expert_rows_and_tensor_parallel_shards(packed):
    from sparkpipe_rs_b200.parallel.tensor_parallel import shard_weights

    cfg, w, root = packed
    ep = ckpt.load_pack(root, cfg, experts=(2, 5))
    ref = init_weights(cfg, seed=3, dtype=torch.float32, experts=(2, 5))
    for k in ref:
        assert torch.equal(ep[k], ref[k]), k
    for deg, rank in ((2, 1), (4, 2)):
        shard = ckpt.load_pack(root, cfg, tp=(deg, rank))
        want = shard_weights(cfg, w, deg, rank)
        for k in want:
            assert torch.equal(shard[k], want[k]), (deg, rank, k)


def test_fingerprint_detects_corruption_and_index_is_atomic(packed, tmp_path):
    cfg, w, root = packed
    pk = S.Pack.open(str(root))
    e = pk.entry("lm_head")
    data = bytearray((root / e["file"]).read_bytes())
    bad = tmp_path / "bad"
    bad.mkdir()
    for f in os.listdir(root):
        (bad / f).write_bytes((root / f).read_bytes())
    data[e["offset"] + 100] ^= 0x40
    (bad / e["file"]).write_bytes(bytes(data))
    with pytest.raises(StatusError) as x:
        ckpt.load_pack(bad, cfg, verify=True)
    assert x.value.code == HASH
    half = S.Writer(str(tmp_path / "half"), "m")          # never finished: no index
    t = torch.ones(4)
    half.add("x", "F32", [4], 4, t.data_ptr(), 16)
    with pytest.raises(StatusError) as x:
        S.Pack.open(str(tmp_path / "half"))
    assert x.value.code == NOT_FOUND
    with pytest.raises(ValueError):
        ckpt.load_pack(root, cfg.replace(hidden_size=cfg.hidden_size * 2))  # another model shape


def test_cpu_model_from_pack_matches_in_memory_weights(packed):
    from sparkpipe_rs_b200.models import oracle

    cfg, w, root = packed
    loaded = ckpt.load_pack(root, cfg)
    prompt = torch.randint(0, cfg.vocab_size, (12,), generator=torch.Generator().manual_seed(1))
    a, la = oracle.greedy_generate(cfg, w, prompt, 4)
    b, lb = oracle.greedy_generate(cfg, loaded, prompt, 4)
    assert torch.equal(a, b) and torch.equal(la, lb)
