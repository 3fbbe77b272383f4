"""Routing semantics of the fp32 oracle (CPU): plain top-k and group-limited routing
(DeepSeek-V2 group_limited_greedy: a group scores its best expert; DeepSeek-V3
noaux_tc: the sum of its best two) against a per-token restatement."""
import pytest
import torch

from sparkpipe_rs_b200.models import oracle
from sparkpipe_rs_b200.models.config import MLAMoEConfig, get_config


@pytest.mark.parametrize("method,scoring", [("noaux_tc", "sigmoid"), ("group_limited_greedy", "softmax"),
                                            ("greedy", "softmax")])
def test_group_limited_routing_matches_per_token_rule(method, scoring):
    E, G, keep_g, k = 32, 4, 2, 4
    ng = G if method != "greedy" else 1
    cfg = MLAMoEConfig(n_routed_experts=E, num_experts_per_tok=k, scoring_func=scoring, n_group=ng,
                       topk_group=keep_g if ng > 1 else 1, topk_method=method, norm_topk_prob=True,
                       routed_scaling_factor=2.0)
    g = torch.Generator().manual_seed(3)
    x = torch.randn(12, E, generator=g)
    b = torch.randn(E, generator=g) * 0.1 if scoring == "sigmoid" else None
    ids, w, _ = oracle.route(cfg, x, torch.eye(E), b)
    sc = x.sigmoid() if scoring == "sigmoid" else x.softmax(-1)
    sel = sc + b if b is not None else sc
    gs = E // ng
    for t in range(x.shape[0]):
        if ng > 1:
            groups = [sorted(sel[t, i * gs:(i + 1) * gs].tolist(), reverse=True) for i in range(ng)]
            score = [v[0] + v[1] if method == "noaux_tc" else v[0] for v in groups]
            kept = sorted(range(ng), key=lambda i: -score[i])[:keep_g]
            cand = [e for e in range(E) if e // gs in kept]
        else:
            cand = list(range(E))
        best = sorted(cand, key=lambda e: -float(sel[t, e]))[:k]
        assert sorted(best) == sorted(ids[t].tolist())
        ref = sc[t, best] / sc[t, best].sum() * 2.0
        got = {int(e): float(v) for e, v in zip(ids[t], w[t])}
        for e, r in zip(best, ref.tolist()):
            assert abs(got[e] - r) < 1e-6


def test_v3_preset_is_group_limited():
    c = get_config("v3")
    assert c.group_limited and c.n_group == 8 and c.topk_group == 4 and c.topk_method == "noaux_tc"
    assert abs(c.param_count() / 1e9 - 671.0) < 1.0
    assert not get_config("k2").group_limited and not get_config("v2_lite").group_limited
