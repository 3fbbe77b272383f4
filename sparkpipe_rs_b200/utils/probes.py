"""Hardware probes: kernel, transport and topology providers.

Each probe takes a request, runs on the GPU and returns one result record:

  kernel     one hot kernel of this package at a requested shape: per-sample device
             latency (CUDA events around each launch; p50 / p95 / p99 / min / max ns),
             achieved TFLOP/s and GB/s from the algorithmic FLOPs and bytes and their
             fraction of the measured peaks, a numerical pass against a plain fp32
             PyTorch reference, resource receipts of the kernels that ran (registers,
             local-memory (spill) bytes, static shared memory: cudaFuncGetAttributes)
             and the SHA-256 of the kernel library that was loaded.
  transport  a byte path (device copy, host<->device from pinned memory, peer copy
             between two GPUs, NCCL all-reduce / all-gather across the process group)
             at a payload size: the same latency percentiles, GB/s (bus bandwidth for
             collectives) and an integrity pass (the received bytes are checked).
  topology   the box: devices, SMs, memory, compute capability, peer-access matrix,
             active NVLink links per device (NVML, read only), and the measured small
             peer-copy latency of every device pair.

    python -m sparkpipe_rs_b200.utils.probes kernel --kind gemm_bf16 --m 4096 --n 64 --k 2048
    python -m sparkpipe_rs_b200.utils.probes kernel --kind mla_decode --batch 64 --heads 16 --ctx 1024
    python -m sparkpipe_rs_b200.utils.probes transport --kind device_copy --bytes 268435456
    python -m sparkpipe_rs_b200.utils.probes topology

Reference behaviour: the provider interfaces of
crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_hardware_kernel_probe.h,
spark_hardware_transport_probe.h and spark_hardware_topology_probe.h (request /
result records: latency percentiles, throughput, resource metrics, numerical and
integrity flags, artifact hashes). The providers here are this framework's own.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import math
import os
from dataclasses import dataclass
from pathlib import Path

import torch

KERNEL_KINDS = ("gemm_bf16", "mla_decode", "prefill_attention", "moe_topk")
TRANSPORT_KINDS = ("device_copy", "h2d", "d2h", "peer_copy", "nccl_all_reduce", "nccl_all_gather")
KERNEL_PREFIX = {"gemm_bf16": "gemm_bf16_kernel", "mla_decode": "mla_", "prefill_attention": "prefill_attn",
                 "moe_topk": "moe_topk_kernel"}


def percentile(samples, q: float) -> float:
    """Nearest-rank percentile (q in [0, 100]) of a non-empty sample list."""
    if not samples:
        raise ValueError("no samples")
    s = sorted(samples)
    rank = max(1, math.ceil(q / 100.0 * len(s)))
    return float(s[min(rank, len(s)) - 1])


def latency_summary(ns) -> dict:
    return {"sample_count": len(ns), "latency_min_ns": int(min(ns)), "latency_p50_ns": int(percentile(ns, 50)),
            "latency_p95_ns": int(percentile(ns, 95)), "latency_p99_ns": int(percentile(ns, 99)),
            "latency_max_ns": int(max(ns))}


def file_sha256(path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def measured_peaks() -> dict:
    p = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    try:
        return json.loads(p.read_text())
    except (OSError, ValueError):
        return {}


def time_samples(fn, iters: int, warmup: int = 3, timer=None) -> list:
    """Per-sample device latency in ns: CUDA events around each call (or `timer(fn)`)."""
    if iters < 1:
        raise ValueError("iters must be >= 1")
    for _ in range(warmup):
        fn()
    if timer is not None:
        return [float(timer(fn)) for _ in range(iters)]
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
    for a, b in ev:
        a.record()
        fn()
        b.record()
    torch.cuda.synchronize()
    return [a.elapsed_time(b) * 1e6 for a, b in ev]


@dataclass
class KernelRequest:
    kind: str
    iters: int = 50
    m: int = 4096
    n: int = 64
    k: int = 2048
    batch: int = 64
    heads: int = 16
    ctx: int = 1024
    q_tokens: int = 1024
    experts: int = 64
    top_k: int = 6
    check: bool = True

    def validate(self):
        if self.kind not in KERNEL_KINDS:
            raise ValueError(f"unknown kernel kind {self.kind!r}; one of {KERNEL_KINDS}")
        if self.iters < 1 or min(self.m, self.n, self.k, self.batch, self.heads, self.ctx, self.q_tokens) < 1:
            raise ValueError("sizes and iterations must be positive")


def _rel_err(out, ref) -> float:
    ref = ref.float()
    return float((out.float() - ref).abs().max() / ref.abs().max().clamp_min(1e-6))


def _kernel_case(r: KernelRequest, dev):
    """(callable, flops, bytes, numerical check -> relative error or None)."""
    from sparkpipe_rs_b200 import ops
    g = torch.Generator(device=dev).manual_seed(0)
    if r.kind == "gemm_bf16":
        x = torch.randn(r.n, r.k, device=dev, generator=g).bfloat16()
        w = (torch.randn(r.m, r.k, device=dev, generator=g) * 0.05).bfloat16()
        out = torch.empty(r.n, r.m, device=dev, dtype=torch.bfloat16)
        fn = lambda: ops.linear(x, w, out=out)  # noqa: E731
        check = lambda: _rel_err(out, x.float() @ w.float().t())  # noqa: E731
        return fn, 2.0 * r.m * r.n * r.k, 2.0 * (r.m * r.k + r.n * r.k + r.m * r.n), check
    if r.kind == "mla_decode":
        B, H, L = r.batch, r.heads, r.ctx
        nb = math.ceil(L / 64)
        cache = torch.randn(B * nb * 64, 576, device=dev, generator=g).bfloat16()
        bt = torch.randperm(B * nb, device=dev, generator=g).int().view(B, nb)
        ctx = torch.full((B,), L, device=dev, dtype=torch.int32)
        q = torch.randn(B, H, 576, device=dev, generator=g).bfloat16()
        out = torch.empty(B, H, 512, device=dev, dtype=torch.bfloat16)
        splits = ops.mla_decode_splits(B, H, L, ops.kernels().num_sms())
        scale = 1 / math.sqrt(192)
        o_part = torch.empty(B, splits, H, 512, device=dev) if splits > 1 else None
        lse = torch.empty(B, splits, H, device=dev) if splits > 1 else None
        fn = lambda: ops.mla_decode(q, cache, bt, ctx, out, splits, scale, o_part, lse)  # noqa: E731

        def check():
            errs = []
            for b in range(min(B, 4)):
                rows = (bt[b].long()[:, None] * 64 + torch.arange(64, device=dev)).flatten()[:L]
                kv = cache[rows].float()
                ref = ((q[b].float() @ kv.t()) * scale).softmax(-1) @ kv[:, :512]
                errs.append(_rel_err(out[b], ref))
            return max(errs)
        return fn, 2.0 * B * H * L * (576 + 512), 2.0 * B * L * 576, check
    if r.kind == "prefill_attention":
        Tq, Tk, H = r.q_tokens, max(r.ctx, r.q_tokens), r.heads
        q = torch.randn(Tq, H, 192, device=dev, generator=g).bfloat16()
        kv = torch.randn(Tk, H, 256, device=dev, generator=g).bfloat16()
        kpe = torch.randn(Tk, 576, device=dev, generator=g).bfloat16()[:, 512:]
        o = torch.empty(Tq, H, 128, device=dev, dtype=torch.bfloat16)
        cu_q = torch.tensor([0, Tq], device=dev, dtype=torch.int32)
        cu_k = torch.tensor([0, Tk], device=dev, dtype=torch.int32)
        scale = 1 / math.sqrt(192)
        fn = lambda: ops.prefill_attention(q, kv[:, :, :128], kpe, kv[:, :, 128:], o, cu_q, cu_k, Tq, scale)  # noqa: E731
        pairs = Tq * Tk - Tq * (Tq - 1) / 2

        def check():
            if Tq * Tk * H > (1 << 28):
                return None  # too large for the fp32 reference
            kk = torch.cat([kv[:, :, :128].float(), kpe.float()[:, None, :].expand(Tk, H, 64)], -1)
            s = torch.einsum("qhd,khd->hqk", q.float(), kk) * scale
            lim = (Tk - Tq + torch.arange(Tq, device=dev))[:, None]
            s = s.masked_fill(~(torch.arange(Tk, device=dev)[None, :] <= lim)[None], float("-inf"))
            return _rel_err(o, torch.einsum("hqk,khd->qhd", s.softmax(-1), kv[:, :, 128:].float()))
        return fn, pairs * H * 640.0, 2.0 * (Tq * H * 320 + Tk * (H * 256 + 64)), check
    # moe_topk
    T, E, k = r.batch, r.experts, r.top_k
    logits = torch.randn(T, E, device=dev, generator=g)
    res = {}

    def fn():
        res["ids"], res["w"] = ops.moe_topk(logits, None, k, 0, False, 1.0)

    def check():
        ref = logits.softmax(-1).topk(k, -1).indices.sort(-1).values
        return 0.0 if torch.equal(res["ids"][:, :k].long().sort(-1).values, ref) else 1.0
    return fn, 0.0, 4.0 * T * (E + 2 * k), check


def kernel_probe(req: KernelRequest, timer=None) -> dict:
    """Runs one kernel probe; returns the result record (status "ok" or "failed: ...")."""
    req.validate()
    from sparkpipe_rs_b200 import _ext, ops
    dev = torch.device("cuda", torch.cuda.current_device())
    fn, flops, nbytes, check = _kernel_case(req, dev)
    ns = time_samples(fn, req.iters, timer=timer)
    res = {"probe": "kernel", "kind": req.kind, "request": req.__dict__, **latency_summary(ns)}
    t = percentile(ns, 50) * 1e-9
    peaks = measured_peaks()
    res["tflops"] = flops / t / 1e12 if flops else 0.0
    res["gbs"] = nbytes / t / 1e9
    if peaks.get("bf16_tflops") and flops:
        res["frac_of_measured_bf16"] = res["tflops"] / float(peaks["bf16_tflops"])
    if peaks.get("hbm_gbs"):
        res["frac_of_measured_hbm"] = res["gbs"] / float(peaks["hbm_gbs"])
    err = check() if req.check else None
    res["numerical"] = "not_checked" if err is None else ("pass" if err < 3e-2 else f"fail (rel err {err:.3g})")
    res["status_word"] = int(ops.status_word())
    pref = KERNEL_PREFIX[req.kind]
    res["resources"] = [a for a in _ext.kernels().kernel_attributes() if a["name"].startswith(pref)]
    res["spills"] = any(a["local_bytes"] > 0 for a in res["resources"])
    so = Path(_ext.kernels().__file__)
    res["kernel_artifact_sha256"] = file_sha256(so)
    res["native_tensor_core"] = req.kind != "moe_topk"
    ok = not res["numerical"].startswith("fail") and res["status_word"] == 0
    res["status"] = "ok" if ok else "failed"
    return res


@dataclass
class TransportRequest:
    kind: str
    nbytes: int = 64 << 20
    iters: int = 20
    peer: int = 1

    def validate(self):
        if self.kind not in TRANSPORT_KINDS:
            raise ValueError(f"unknown transport {self.kind!r}; one of {TRANSPORT_KINDS}")
        if self.nbytes < 4 or self.nbytes % 4 or self.iters < 1:
            raise ValueError("payload must be a positive multiple of 4 bytes, iters >= 1")


def transport_probe(req: TransportRequest, timer=None) -> dict:
    req.validate()
    dev = torch.device("cuda", torch.cuda.current_device())
    n = req.nbytes // 4
    pattern = torch.arange(n, device=dev, dtype=torch.int32) * 2654435761
    bus = 1.0
    if req.kind == "device_copy":
        dst = torch.empty_like(pattern)
        fn = lambda: dst.copy_(pattern)  # noqa: E731
        verify = lambda: torch.equal(dst, pattern)  # noqa: E731
    elif req.kind in ("h2d", "d2h"):
        host = torch.empty(n, dtype=torch.int32, pin_memory=True)
        if req.kind == "h2d":
            host.copy_(pattern.cpu())
            dst = torch.empty_like(pattern)
            fn = lambda: dst.copy_(host, non_blocking=True)  # noqa: E731
            verify = lambda: torch.equal(dst, pattern)  # noqa: E731
        else:
            fn = lambda: host.copy_(pattern, non_blocking=True)  # noqa: E731
            verify = lambda: torch.equal(host, pattern.cpu())  # noqa: E731
    elif req.kind == "peer_copy":
        if torch.cuda.device_count() < 2:
            return {"probe": "transport", "kind": req.kind, "status": "unavailable: needs two GPUs"}
        other = torch.device("cuda", req.peer if req.peer != dev.index else (dev.index + 1) % torch.cuda.device_count())
        dst = torch.empty(n, dtype=torch.int32, device=other)
        fn = lambda: dst.copy_(pattern)  # noqa: E731
        verify = lambda: torch.equal(dst.to(dev), pattern)  # noqa: E731
    else:
        import torch.distributed as dist
        if not (dist.is_available() and dist.is_initialized()):
            return {"probe": "transport", "kind": req.kind, "status": "unavailable: no process group"}
        W, rank = dist.get_world_size(), dist.get_rank()
        if req.kind == "nccl_all_reduce":
            buf = torch.ones(n, device=dev, dtype=torch.float32)
            fn = lambda: dist.all_reduce(buf)  # noqa: E731
            bus = 2.0 * (W - 1) / W

            def verify():
                buf.fill_(rank + 1)
                dist.all_reduce(buf)
                return bool((buf == W * (W + 1) / 2).all())
        else:
            part = torch.full((n // W,), float(rank), device=dev)
            full = torch.empty(n // W * W, device=dev)
            fn = lambda: dist.all_gather_into_tensor(full, part)  # noqa: E731
            bus = (W - 1) / W

            def verify():
                dist.all_gather_into_tensor(full, part)
                return bool(torch.equal(full.view(W, -1)[:, 0].cpu(), torch.arange(W, dtype=torch.float32)))
    ns = time_samples(fn, req.iters, timer=timer)
    res = {"probe": "transport", "kind": req.kind, "request": req.__dict__, **latency_summary(ns)}
    t = percentile(ns, 50) * 1e-9
    res["gbs"] = req.nbytes / t / 1e9
    res["bus_gbs"] = res["gbs"] * bus
    res["integrity"] = "pass" if verify() else "fail"
    res["status"] = "ok" if res["integrity"] == "pass" else "failed"
    return res


def topology_probe(latency_bytes: int = 4096, iters: int = 20) -> dict:
    n = torch.cuda.device_count()
    devs = []
    for i in range(n):
        p = torch.cuda.get_device_properties(i)
        devs.append({"index": i, "name": p.name, "sms": p.multi_processor_count,
                     "memory_bytes": p.total_memory, "capability": f"{p.major}.{p.minor}"})
    peer = [[(i == j) or torch.cuda.can_device_access_peer(i, j) for j in range(n)] for i in range(n)]
    links = []
    try:
        import pynvml
        pynvml.nvmlInit()
        for i in range(n):
            h = pynvml.nvmlDeviceGetHandleByIndex(i)
            up = 0
            for link in range(18):
                try:
                    up += int(pynvml.nvmlDeviceGetNvLinkState(h, link) == pynvml.NVML_FEATURE_ENABLED)
                except pynvml.NVMLError:
                    break
            links.append(up)
        pynvml.nvmlShutdown()
    except Exception as e:  # NVML missing: report, do not guess
        links = f"unavailable: {type(e).__name__}"
    lat = [[None] * n for _ in range(n)]
    for i in range(n):
        for j in range(n):
            if i == j or not peer[i][j]:
                continue
            src = torch.zeros(latency_bytes // 4, dtype=torch.int32, device=f"cuda:{i}")
            dst = torch.empty_like(src, device=f"cuda:{j}")
            with torch.cuda.device(i):
                lat[i][j] = int(percentile(time_samples(lambda: dst.copy_(src), iters), 50))
    return {"probe": "topology", "devices": devs, "peer_access": peer, "nvlink_links_up": links,
            "peer_copy_latency_p50_ns": lat, "status": "ok"}


def main():
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="probe", required=True)
    k = sub.add_parser("kernel")
    k.add_argument("--kind", required=True, choices=KERNEL_KINDS)
    for name, default in (("iters", 50), ("m", 4096), ("n", 64), ("k", 2048), ("batch", 64), ("heads", 16),
                          ("ctx", 1024), ("q_tokens", 1024), ("experts", 64), ("top_k", 6)):
        k.add_argument(f"--{name.replace('_', '-')}", type=int, default=default, dest=name)
    k.add_argument("--no-check", action="store_true")
    t = sub.add_parser("transport")
    t.add_argument("--kind", required=True, choices=TRANSPORT_KINDS)
    t.add_argument("--bytes", type=int, default=64 << 20)
    t.add_argument("--iters", type=int, default=20)
    t.add_argument("--peer", type=int, default=1)
    sub.add_parser("topology")
    a = ap.parse_args()
    if "LOCAL_RANK" in os.environ:
        torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    if a.probe == "kernel":
        req = KernelRequest(a.kind, a.iters, a.m, a.n, a.k, a.batch, a.heads, a.ctx, a.q_tokens, a.experts, a.top_k,
                            not a.no_check)
        out = kernel_probe(req)
    elif a.probe == "transport":
        if a.kind.startswith("nccl") and "WORLD_SIZE" in os.environ:
            import datetime
            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
        out = transport_probe(TransportRequest(a.kind, a.bytes, a.iters, a.peer))
    else:
        out = topology_probe()
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
