// Allocation-free variant of the MLA decode entry point (declared in
// mla_decode_noalloc.h, which explains who needs it). It runs the same kernels
// as sp::mla_decode; only the split-KV scratch comes from a file-scope device
// array instead of caller- or allocator-provided memory.
#include <cuda_runtime.h>

#include <mutex>

#include "launch.h"
#include "mla_decode_noalloc.h"

namespace {

constexpr unsigned kScratchFloats = SP_MLA_NOALLOC_SCRATCH_BYTES / sizeof(float);
constexpr int kMaxDevices = 64;
constexpr int kLatent = 512;

// The shared scratch: split partial outputs followed by their log-sum-exps.
static __device__ __align__(256) float g_mla_scratch[kScratchFloats];
// Status word of the bounded waits inside the kernel.
static __device__ __align__(256) int g_mla_status;

// Device addresses of the two symbols, resolved once per device. In host code
// the symbol names are host-side stand-ins, never device addresses.
struct DeviceSymbols {
  float* scratch = nullptr;
  int* status = nullptr;
  bool ready = false;
};
DeviceSymbols g_dev[kMaxDevices];
std::mutex g_mu;

int resolve_symbols(int dev, DeviceSymbols** out) {
  if (dev < 0 || dev >= kMaxDevices) return SP_NOALLOC_SETUP_FAILED;
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceSymbols& s = g_dev[dev];
  if (!s.ready) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_mla_scratch);  // the current device is `dev`
    if (e != cudaSuccess || p == nullptr) return e != cudaSuccess ? int(e) : SP_NOALLOC_SETUP_FAILED;
    s.scratch = static_cast<float*>(p);
    p = nullptr;
    e = cudaGetSymbolAddress(&p, g_mla_status);
    if (e != cudaSuccess || p == nullptr) return e != cudaSuccess ? int(e) : SP_NOALLOC_SETUP_FAILED;
    s.status = static_cast<int*>(p);
    s.ready = true;
  }
  *out = &s;
  return SP_NOALLOC_OK;
}

}  // namespace

extern "C" int sp_mla_decode_noalloc(const void* q, const void* cache, long long num_slots, const int* block_table,
                                     int max_blocks, const int* context_lens, void* out, int batch, int heads,
                                     int splits, float scale, void* stream) {
  if (!q || !cache || !block_table || !context_lens || !out) return SP_NOALLOC_BAD_ARGUMENT;
  if (batch <= 0 || heads <= 0 || heads % 16 != 0 || splits <= 0 || max_blocks <= 0 || num_slots <= 0)
    return SP_NOALLOC_BAD_ARGUMENT;
  const unsigned long long need =
      splits > 1 ? (unsigned long long)batch * splits * heads * (kLatent + 1) : 0ull;
  if (need > kScratchFloats) return SP_NOALLOC_SCRATCH_TOO_SMALL;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return int(e);
  DeviceSymbols* sym = nullptr;
  int rc = resolve_symbols(dev, &sym);
  if (rc != SP_NOALLOC_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the status word must start at zero for this call; the partials are fully
  // written by the kernel and need no clearing
  e = cudaMemsetAsync(sym->status, 0, sizeof(int), s);
  if (e != cudaSuccess) return int(e);
  sp::MlaDecodeLaunch l;
  l.q = q;
  l.cache = cache;
  l.num_slots = num_slots;
  l.block_table = block_table;
  l.max_blocks = max_blocks;
  l.context_lens = context_lens;
  l.out = out;
  l.o_part = splits > 1 ? sym->scratch : nullptr;
  l.lse_part = splits > 1 ? sym->scratch + (size_t)batch * splits * heads * kLatent : nullptr;
  l.B = batch;
  l.H = heads;
  l.splits = splits;
  l.scale = scale;
  l.err = sym->status;
  l.stream = s;
  try {
    sp::mla_decode(l);
  } catch (...) {
    return SP_NOALLOC_BAD_ARGUMENT;
  }
  e = cudaGetLastError();
  return e == cudaSuccess ? SP_NOALLOC_OK : int(e);
}

extern "C" int sp_mla_decode_noalloc_status(void* stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  DeviceSymbols* sym = nullptr;
  if (resolve_symbols(dev, &sym) != SP_NOALLOC_OK) return -1;
  // the kernels of the caller's stream must have finished before the word is read
  if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) return -1;
  int v = 0;
  if (cudaMemcpy(&v, sym->status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
  if (cudaMemset(sym->status, 0, sizeof(int)) != cudaSuccess) return -1;
  return v;
}
