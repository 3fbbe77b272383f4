"""Multi-node host fabric: memlink planning, a multi-lane loopback transfer, and the
fabric topology model."""
import os
import socket
import threading

import pytest

from sparkpipe_rs_b200 import _ext


def _f():
    return _ext.core().fabric


def _free_base(lanes):
    for _ in range(50):
        s = socket.socket()
        s.bind(("127.0.0.1", 0))
        base = s.getsockname()[1]
        s.close()
        if base + lanes < 65000:
            return base
    raise RuntimeError("no port")


def test_partition_covers_chunk_aligned():
    f = _f()
    total = 37 * f.CHUNK_BYTES + 12345
    parts = [f.partition(total, 8, i) for i in range(8)]
    assert parts[0].offset == 0 and sum(p.bytes for p in parts) == total
    for a, b in zip(parts, parts[1:]):
        assert a.offset + a.bytes == b.offset and b.offset % f.CHUNK_BYTES == 0
    assert max(p.bytes for p in parts) - min(p.bytes for p in parts) <= 2 * f.CHUNK_BYTES
    assert f.partition(10, 4, 3).bytes in (0, 10)
    with pytest.raises(Exception):
        f.partition(10, 65, 0)
    with pytest.raises(Exception):
        f.partition(10, 4, 4)


def test_neighbors_and_endpoints():
    f = _f()
    assert f.neighbor_rank(0, 13, f.Direction.PREVIOUS) == 12 and f.neighbor_rank(12, 13, f.Direction.NEXT) == 0
    assert f.host_from_template("spark-{rank}.local", 7) == "spark-7.local"
    e = f.neighbor_endpoint(3, 4, f.Direction.NEXT, "node{rank}", 56000, 8)
    assert (e.host, e.base_port, e.lanes) == ("node0", 56000, 8)
    with pytest.raises(Exception):
        f.neighbor_endpoint(0, 4, f.Direction.NEXT, "n{rank}", 65530, 8)


def test_multi_lane_loopback_transfer():
    f = _f()
    lanes = 8
    base = _free_base(lanes)
    src = os.urandom(9 * f.CHUNK_BYTES + 777)
    dst = bytearray(len(src))
    got = {}
    t = threading.Thread(target=lambda: got.setdefault("n", f.receive(base, lanes, dst, 20000)))
    t.start()
    sent = f.send("127.0.0.1", base, lanes, src, 20000)
    t.join()
    assert sent == len(src) and got["n"] == len(src) and bytes(dst) == src


def test_receive_times_out_without_sender():
    f = _f()
    base = _free_base(2)
    with pytest.raises(Exception):
        f.receive(base, 2, bytearray(16), 200)


def test_topology_validation_and_routes():
    f = _f()
    ring = f.default_topology(f.Mode.RING_DEBUG_SINGLE_RAIL, 13, 2)
    f.validate(ring)
    r = f.resolve_route(ring, 4)
    assert (r.first_hop, r.hops, r.port, r.switched) == (3, 2, 0, False)
    r = f.resolve_route(ring, 11)  # 4 back vs 9 forward
    assert (r.first_hop, r.hops, r.port) == (1, 4, 1)
    sw = f.default_topology(f.Mode.SINGLE_SWITCH_SINGLE_RAIL, 8, 0)
    r = f.resolve_route(sw, 5)
    assert r.switched and r.first_hop == f.NO_NODE and r.hops == 2
    dual = f.default_topology(f.Mode.DUAL_SWITCH_DUAL_RAIL, 8, 0)
    f.validate(dual)
    with pytest.raises(Exception):
        f.resolve_route(dual, 1)
    bad = f.default_topology(f.Mode.SINGLE_SWITCH_SINGLE_RAIL, 8, 0, 9601)
    with pytest.raises(Exception):
        f.validate(bad)
    ring.ports = 1
    with pytest.raises(Exception):
        f.validate(ring)
    with pytest.raises(Exception):
        f.resolve_route(sw, 0)
    assert f.mode_name(f.Mode.RING_DEBUG_SINGLE_RAIL) == "ring-debug-single-rail"
