"""Stage-module services: the device-allocation ledger (cap, rollback, release),
pack-region loads, atomic slot claims and the destroy quiesce, typed environment
settings. Host memory stands in for the device here; the CUDA allocator is covered
by the GPU test at the end."""
import ctypes
import os
import threading

import pytest
import torch

from sparkpipe_rs_b200 import _ext


def _sm():
    return _ext.core().stage_module


def test_ledger_rollback_release_and_cap():
    sm = _sm()
    led = sm.DeviceLedger("t", sm.HostAllocator())
    a = led.allocate(100)
    z = led.allocate(64, zeroed=True)
    assert ctypes.string_at(z, 64) == b"\0" * 64
    assert led.count == 2 and led.bytes_resident == 164
    mark = led.count
    for _ in range(10):
        led.allocate(8)
    led.rollback(mark)
    assert led.count == 2 and led.bytes_resident == 164
    led.release_all()
    assert led.count == 0 and led.bytes_resident == 0
    for _ in range(sm.MAX_DEVICE_ALLOCATIONS):
        led.allocate(1)
    with pytest.raises(Exception):
        led.allocate(1)
    assert a


def test_python_allocator_and_pack_regions(tmp_path):
    sm = _sm()
    live = {}

    class Bufs(sm.Allocator):  # a Python allocator through the native ledger
        def allocate(self, n):
            b = ctypes.create_string_buffer(int(n))
            live[ctypes.addressof(b)] = b
            return ctypes.addressof(b)

        def release(self, p):
            live.pop(p)

        def zero(self, p, n):
            ctypes.memset(p, 0, n)
            return _ext.core().Status.OK

        def copy_from_host(self, d, s, n):
            ctypes.memmove(d, s, n)
            return _ext.core().Status.OK

    pack = tmp_path / "w.pack"
    data = os.urandom(3 << 20)
    pack.write_bytes(data)
    assert sm.pack_read(str(pack), 1000, 5000) == data[1000:6000]
    led = sm.DeviceLedger("loader", Bufs())
    p = sm.load_device_region(led, str(pack), 4096, 2 << 20)
    assert ctypes.string_at(p, 2 << 20) == data[4096:4096 + (2 << 20)]
    # a region past the end of the pack fails and leaves nothing allocated
    with pytest.raises(Exception):
        sm.load_device_region(led, str(pack), len(data) - 10, 100)
    assert led.count == 1 and len(live) == 1
    led.release_all()
    assert not live


def test_slot_claims_and_quiesce():
    sm = _sm()
    t = sm.SlotTable(4)
    got = [t.claim() for _ in range(5)]
    assert got[:4] == [0, 1, 2, 3] and got[4] is None and t.free_count == 0
    t.release(2)
    assert t.admit(3) == 1 and t.claim() == 2
    t.release_set([0, 1, 2, 3])
    assert t.claim_set([1, 3]) == _ext.core().Status.OK
    assert t.claim_set([0, 3]) == _ext.core().Status.BUSY  # all or nothing: 0 stays free
    assert not t.claimed(0) and t.claimed(1) and t.claimed(3)
    assert t.wait_all_free(2_000_000) == _ext.core().Status.BUSY
    threading.Timer(0.05, lambda: t.release_set([1, 3])).start()
    assert t.wait_all_free(5_000_000_000) == _ext.core().Status.OK


def test_environment_settings(monkeypatch):
    sm = _sm()
    monkeypatch.setenv("SPB_TEST_N", "12")
    assert sm.env_unsigned("t", "SPB_TEST_N", 1, 64, 7) == 12
    assert sm.env_unsigned("t", "SPB_TEST_MISSING", 1, 64, 7) == 7
    monkeypatch.setenv("SPB_TEST_N", "99")
    with pytest.raises(Exception):
        sm.env_unsigned("t", "SPB_TEST_N", 1, 64, 7)
    monkeypatch.setenv("SPB_TEST_N", "x1")
    with pytest.raises(Exception):
        sm.env_unsigned("t", "SPB_TEST_N", 1, 64, 7)
    monkeypatch.setenv("SPB_TEST_S", "abc")
    assert sm.env_text("t", "SPB_TEST_S", "d") == "abc"


@pytest.mark.gpu
def test_cuda_ledger_loads_pack_region(tmp_path):
    from sparkpipe_rs_b200.core.stage_module import cuda_allocator

    sm = _sm()
    k = _ext.kernels()
    pack = tmp_path / "w.pack"
    data = os.urandom(1 << 20)
    pack.write_bytes(data)
    led = sm.DeviceLedger("gpu", cuda_allocator(0))
    p = sm.load_device_region(led, str(pack), 8192, 512 << 10)
    back = torch.empty(512 << 10, dtype=torch.uint8)
    assert k.raw_copy(back.data_ptr(), p, 512 << 10) == 0
    assert bytes(back.numpy()) == data[8192:8192 + (512 << 10)]
    z = led.allocate(4096, zeroed=True)
    assert k.raw_copy(back.data_ptr(), z, 4096) == 0 and not back[:4096].any()
    led.release_all()
    assert led.bytes_resident == 0
