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
    st.argtypes = []
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
        assert status() == 0


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
