"""Hardware probes: the statistics and request checks on CPU, every probe kind on
the GPU (small shapes)."""
import pytest
import torch

from sparkpipe_rs_b200.utils import probes


def test_percentiles_and_summary():
    xs = list(range(1, 101))
    assert probes.percentile(xs, 50) == 50 and probes.percentile(xs, 95) == 95 and probes.percentile(xs, 99) == 99
    assert probes.percentile([7], 99) == 7
    with pytest.raises(ValueError):
        probes.percentile([], 50)
    s = probes.latency_summary([5, 1, 3])
    assert (s["sample_count"], s["latency_min_ns"], s["latency_p50_ns"], s["latency_max_ns"]) == (3, 1, 3, 5)


def test_requests_validate_and_fake_timer(tmp_path):
    with pytest.raises(ValueError):
        probes.KernelRequest("conv2d").validate()
    with pytest.raises(ValueError):
        probes.KernelRequest("gemm_bf16", iters=0).validate()
    with pytest.raises(ValueError):
        probes.TransportRequest("device_copy", nbytes=6).validate()
    calls = []
    ns = probes.time_samples(lambda: calls.append(1), 4, warmup=2, timer=lambda fn: (fn(), 1000 + len(calls))[1])
    assert len(calls) == 6 and ns == [1003.0, 1004.0, 1005.0, 1006.0]
    f = tmp_path / "a.bin"
    f.write_bytes(b"abc")
    assert probes.file_sha256(f) == "ba7816bf8f01cfea414140de5dae2223b00361a396177a9cb410ff61f20015ad"


@pytest.mark.gpu
@pytest.mark.parametrize("kind,kw", [("gemm_bf16", dict(m=1024, n=64, k=512)),
                                     ("mla_decode", dict(batch=8, heads=16, ctx=300)),
                                     ("prefill_attention", dict(q_tokens=256, ctx=700, heads=4)),
                                     ("moe_topk", dict(batch=33, experts=64, top_k=6))])
def test_kernel_probes(kind, kw):
    r = probes.kernel_probe(probes.KernelRequest(kind, iters=5, **kw))
    assert r["status"] == "ok" and r["numerical"] == "pass", r
    assert r["sample_count"] == 5 and 0 < r["latency_p50_ns"] <= r["latency_p99_ns"]
    assert r["resources"] and not r["spills"] and len(r["kernel_artifact_sha256"]) == 64


@pytest.mark.gpu
def test_transport_and_topology_probes():
    for kind in ("device_copy", "h2d", "d2h"):
        r = probes.transport_probe(probes.TransportRequest(kind, nbytes=8 << 20, iters=3))
        assert r["status"] == "ok" and r["integrity"] == "pass" and r["gbs"] > 0, r
    t = probes.topology_probe(iters=3)
    assert t["status"] == "ok" and len(t["devices"]) == torch.cuda.device_count()
    assert t["devices"][0]["sms"] > 0 and t["peer_access"][0][0]
