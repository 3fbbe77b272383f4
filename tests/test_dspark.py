"""dSpark drafter and speculator on CPU: contract validation, hidden-tap plan over
pipeline stages, drafting shapes and determinism, confidence truncation, the
sequence state machine and verification accounting.

Constants and flags follow
crates/spark-abi/vendor/sparkpipe/model-families/glm52/include/sparkpipe/spark_glm52_dspark.h."""
import pytest
import torch

from sparkpipe_rs_b200.models.dspark import (FLAG_DRAFT_READY, FLAG_TAPS_READY, FLAG_VALID, FLAG_VERIFY_INFLIGHT,
                                             RESULT_CONFIDENCE_TRUNCATED, VERIFY_ACCEPTED_ALL, VERIFY_REJECTED,
                                             DsparkContract, DsparkDrafter, DsparkSpeculator, hidden_tap_plan)


def contract(**kw):
    base = dict(target_layers=78, hidden=64, vocab=300, heads=4, head_dim=16, draft_layers=2, markov_rank=16)
    base.update(kw)
    return DsparkContract(**base)


def test_contract_and_tap_plan():
    c = contract(aux_layer_ids=[8, 23, 39, 55, 70])
    assert c.capture_layers == [7, 22, 38, 54, 69]
    plan = hidden_tap_plan(c, [20, 20, 19, 19])
    assert [(p["stage_index"], p["layer_offset_in_stage"]) for p in plan] == [(0, 7), (1, 2), (1, 18), (2, 14), (3, 10)]
    assert len(contract().aux_layer_ids) == 5  # spread over the depth by default
    for bad in (dict(aux_layer_ids=[0, 5]), dict(aux_layer_ids=[9, 8]), dict(max_speculative_tokens=8),
                dict(min_confidence_milli=0)):
        with pytest.raises(ValueError):
            contract(**bad)
    with pytest.raises(ValueError):
        hidden_tap_plan(c, [20, 20])


def test_drafter_shapes_and_determinism():
    torch.manual_seed(0)
    c = contract()
    d = DsparkDrafter(c).eval()
    taps = torch.randn(3, 5, 64)
    t1, p1 = d(taps, torch.tensor([1, 2, 3]))
    t2, p2 = d(taps, torch.tensor([1, 2, 3]))
    assert t1.shape == (3, 7) and p1.shape == (3, 7)
    assert torch.equal(t1, t2) and torch.equal(p1, p2)
    assert ((p1 >= 0) & (p1 <= 1)).all() and (t1 < c.vocab).all()
    # the Markov head makes each token depend on the one before it
    t3, _ = d(taps, torch.tensor([4, 2, 3]))
    assert torch.equal(t3[1:], t1[1:])


def test_speculator_states_truncation_and_verify():
    torch.manual_seed(0)
    c = contract(min_confidence_milli=1)  # keep everything
    d = DsparkDrafter(c).eval()
    spec = DsparkSpeculator(d, sequences=2)
    spec.begin(0, request_id=5, sequence_id=9, position=100)
    with pytest.raises(RuntimeError):
        spec.draft([0])  # no taps yet
    spec.taps_ready(0, torch.randn(5, 64), last_token=7)
    assert spec.state[0]["flags"] == FLAG_VALID | FLAG_TAPS_READY
    (toks, flags), = spec.draft([0]).values()
    assert len(toks) == 7 and flags == 0 and spec.state[0]["flags"] == FLAG_VALID | FLAG_DRAFT_READY
    sent = spec.dispatch_verify(0)
    assert spec.state[0]["flags"] & FLAG_VERIFY_INFLIGHT and sent == toks
    verifier = toks[:3] + [(toks[3] + 1) % c.vocab] + [1, 2, 3, 4]
    acc, com, vflags = spec.verify_result(0, verifier)
    assert (acc, com, vflags) == (3, 4, VERIFY_REJECTED) and spec.state[0]["position"] == 104
    assert spec.counters["accepted"] == 3 and spec.counters["rejected"] == 4 and spec.state[0]["flags"] == FLAG_VALID
    # all accepted
    spec.taps_ready(0, torch.randn(5, 64), last_token=1)
    toks = spec.draft([0], requested=2)[0][0]
    spec.dispatch_verify(0)
    assert spec.verify_result(0, toks + [9]) == (2, 3, VERIFY_ACCEPTED_ALL)
    # a threshold above every confidence: nothing survives
    strict = DsparkSpeculator(DsparkDrafter(contract(min_confidence_milli=1000)).eval(), sequences=1)
    strict.begin(0, 1, 1, 0)
    strict.taps_ready(0, torch.randn(5, 64), last_token=3)
    (toks, flags), = strict.draft([0]).values()
    assert toks == [] and flags == RESULT_CONFIDENCE_TRUNCATED and strict.counters["rejected_by_confidence"] == 1
