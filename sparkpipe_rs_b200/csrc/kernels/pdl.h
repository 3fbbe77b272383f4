// Host-side launch helper: every kernel of this package is launched through
// launch_k(), which attaches the programmatic-stream-serialization attribute
// (PDL) unless it is disabled with SPARKPIPE_PDL=0. Kernels launched this way
// call griddep_wait() before their first dependent memory access.
#pragma once
#include <cuda_runtime.h>

#include <cstdlib>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_set>

namespace sp {

inline bool pdl_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = std::getenv("SPARKPIPE_PDL");
    on = (e && e[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

// Every kernel asks for the maximum shared-memory carveout, so consecutive
// kernels of a decode step never force an SM to reconfigure L1 / shared memory.
inline void prefer_max_smem_carveout(const void* kern) {
  static std::mutex mu;
  static std::unordered_set<const void*> done;
  std::lock_guard<std::mutex> lk(mu);
  if (done.insert(kern).second) cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
}

template <typename... KArgs, typename... Args>
inline void launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
  prefer_max_smem_carveout(reinterpret_cast<const void*>(kern));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  if (pdl_enabled()) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e != cudaSuccess) throw std::runtime_error(std::string("kernel launch failed: ") + cudaGetErrorString(e));
}

}  // namespace sp
