"""The CUDA allocator of the stage-module device ledger (``core().stage_module``):
raw ``cudaMalloc`` / ``cudaFree`` / ``cudaMemset`` / ``cudaMemcpy`` from the kernels
extension, so a stage module's device memory is tracked and released by the native
ledger (at most 4096 allocations, rollback on a failed load).

    ledger = core().stage_module.DeviceLedger("stage0", cuda_allocator(0))
    ptr = core().stage_module.load_device_region(ledger, "weights.pack", offset, nbytes)
"""
from __future__ import annotations

from .. import _ext

_CLS = None


def cuda_allocator(device: int = 0):
    global _CLS
    if _CLS is None:
        core = _ext.core()
        k = _ext.kernels()

        class CudaAllocator(core.stage_module.Allocator):
            def __init__(self, dev):
                super().__init__()
                self.dev = int(dev)

            def allocate(self, nbytes):
                return int(k.raw_alloc(int(nbytes), self.dev))

            def release(self, ptr):
                k.raw_free(int(ptr))

            def zero(self, ptr, nbytes):
                return core.Status(int(k.raw_zero(int(ptr), int(nbytes))))

            def copy_from_host(self, dst, src, nbytes):
                return core.Status(int(k.raw_copy(int(dst), int(src), int(nbytes))))

        _CLS = CudaAllocator
    return _CLS(device)
