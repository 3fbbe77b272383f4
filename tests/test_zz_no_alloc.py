"""The allocation-free MLA decode entry point, called through its exported C symbol.

For callers that cannot allocate device memory (see mla_decode_noalloc.h): the
symbol is loaded with ctypes from the compiled kernel library, run twice in a
row on different inputs, and each output is checked against the regular
mla_decode op on the same inputs. This file is collected last on purpose.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _lib():
    from sparkpipe_rs_b200 import _ext

    _ext.kernels()  # builds / loads the library the symbol lives in
    lib = ctypes.CDLL(str(_ext._so_path("_sp_kernels")))
    fn = lib.sp_mla_decode_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p, ctypes.c_int,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                   ctypes.c_void_p]
    st = lib.sp_mla_decode_noalloc_status
    st.restype = ctypes.c_int
    st.argtypes = [ctypes.c_void_p]
    return fn, st


def _call(fn, q, cache, bt, ctx, out, splits, scale):
    stream = torch.cuda.current_stream().cuda_stream
    return fn(q.data_ptr(), cache.data_ptr(), cache.shape[0], bt.data_ptr(), bt.shape[1], ctx.data_ptr(),
              out.data_ptr(), q.shape[0], q.shape[1], splits, scale, stream)


def test_noalloc_matches_regular_entry_point_twice():
    from sparkpipe_rs_b200 import ops

    fn, status = _lib()
    g = torch.Generator(device=DEV).manual_seed(42)
    B, H, nblocks, maxb, splits = 8, 16, 64, 12, 3
    scale = 1.0 / math.sqrt(192)
    cache = torch.randn(nblocks * 64, 576, device=DEV, generator=g).bfloat16()
    for call in range(2):
        ctx = torch.randint(1, maxb * 64, (B,), device=DEV, generator=g).int()
        bt = torch.stack([torch.randperm(nblocks, device=DEV, generator=g)[:maxb] for _ in range(B)]).int()
        q = torch.randn(B, H, 576, device=DEV, generator=g).bfloat16()
        got = torch.empty(B, H, 512, device=DEV, dtype=torch.bfloat16)
        rc = _call(fn, q, cache, bt, ctx, got, splits, scale)
        assert rc == 0, f"call {call}: return code {rc}"
        want = torch.empty_like(got)
        ops.mla_decode(q, cache, bt, ctx, want, splits, scale)
        torch.cuda.synchronize()
        torch.testing.assert_close(got.float(), want.float(), atol=2e-2, rtol=2e-2)
        assert status(torch.cuda.current_stream().cuda_stream) == 0


def _case(B, H, maxb, seed, device=DEV):
    g = torch.Generator(device=device).manual_seed(seed)
    nblocks = B * maxb
    cache = torch.randn(nblocks * 64, 576, device=device, generator=g).bfloat16()
    ctx = torch.randint(1, maxb * 64, (B,), device=device, generator=g).int()
    bt = torch.randperm(nblocks, device=device, generator=g).int().view(B, maxb)
    q = torch.randn(B, H, 576, device=device, generator=g).bfloat16()
    return q, cache, bt, ctx


@pytest.mark.parametrize("B,H,maxb,splits", [(5, 16, 6, 1),      # no split: no scratch is used
                                             (73, 16, 8, 7)])    # the largest request the scratch accepts
def test_noalloc_no_split_and_largest_accepted_request(B, H, maxb, splits):
    from sparkpipe_rs_b200 import ops

    fn, status = _lib()
    # batch * splits * heads * 513 floats: 73 * 7 * 16 * 513 = 4,194,288 of 4,194,304
    assert splits == 1 or B * splits * H * 513 <= (16 << 20) // 4 < B * (splits + 1) * H * 513
    q, cache, bt, ctx = _case(B, H, maxb, seed=B + splits)
    scale = 1.0 / math.sqrt(192)
    for _ in range(2):
        got = torch.empty(B, H, 512, device=DEV, dtype=torch.bfloat16)
        assert _call(fn, q, cache, bt, ctx, got, splits, scale) == 0
        want = torch.empty_like(got)
        ops.mla_decode(q, cache, bt, ctx, want, splits, scale)
        torch.cuda.synchronize()
        torch.testing.assert_close(got.float(), want.float(), atol=2e-2, rtol=2e-2)
    assert status(torch.cuda.current_stream().cuda_stream) == 0
    # one more split no longer fits: refused before any launch
    out = torch.empty(B, H, 512, device=DEV, dtype=torch.bfloat16)
    if splits > 1:
        assert _call(fn, q, cache, bt, ctx, out, splits + 1, scale) == -2


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs a second GPU")
def test_noalloc_on_a_second_device():
    from sparkpipe_rs_b200 import ops

    fn, status = _lib()
    dev = torch.device("cuda", 1)
    with torch.cuda.device(dev):
        q, cache, bt, ctx = _case(8, 16, 10, seed=7, device=dev)
        got = torch.empty(8, 16, 512, device=dev, dtype=torch.bfloat16)
        assert _call(fn, q, cache, bt, ctx, got, 3, 0.07) == 0   # first call on this device resolves its symbols
        want = torch.empty_like(got)
        ops.mla_decode(q, cache, bt, ctx, want, 3, 0.07)
        torch.cuda.synchronize(dev)
        torch.testing.assert_close(got.float(), want.float(), atol=2e-2, rtol=2e-2)
        assert status(torch.cuda.current_stream(dev).cuda_stream) == 0


def test_noalloc_rejects_oversized_scratch():
    fn, _ = _lib()
    B, H = 512, 128
    q = torch.zeros(1, 16, 576, device=DEV, dtype=torch.bfloat16)
    cache = torch.zeros(64, 576, device=DEV, dtype=torch.bfloat16)
    bt = torch.zeros(1, 1, device=DEV, dtype=torch.int32)
    ctx = torch.ones(1, device=DEV, dtype=torch.int32)
    out = torch.zeros(1, 16, 512, device=DEV, dtype=torch.bfloat16)
    stream = torch.cuda.current_stream().cuda_stream
    # claims a batch whose partials do not fit the 16 MiB scratch: refused before any launch
    rc = fn(q.data_ptr(), cache.data_ptr(), 64, bt.data_ptr(), 1, ctx.data_ptr(), out.data_ptr(), B, H, 16,
            0.1, stream)
    assert rc == -2
