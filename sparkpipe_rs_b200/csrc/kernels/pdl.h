// Host-side launch helper: every kernel of this package is launched through
// launch_k(), which attaches the programmatic-stream-serialization attribute
// (PDL) unless it is disabled with SPARKPIPE_PDL=0. Kernels launched this way
// call griddep_wait() before their first dependent memory access.
#pragma once
#include <cuda_runtime.h>

#include <cstdlib>
#include <mutex>
#include <set>
#include <stdexcept>
#include <string>
#include <tuple>

namespace sp {

inline bool pdl_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = std::getenv("SPARKPIPE_PDL");
    on = (e && e[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

// Function attributes belong to each device's instance of a kernel, so every
// (attribute, value) is applied once per (kernel, device), under a lock, with the
// return code checked: a second GPU driven by the same process gets its own opt-in.
inline void set_func_attr_once(const void* kern, cudaFuncAttribute attr, int value) {
  static std::mutex mu;
  static std::set<std::tuple<const void*, int, int, int>> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) throw std::runtime_error(std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  std::lock_guard<std::mutex> lk(mu);
  if (!done.insert({kern, dev, int(attr), value}).second) return;
  e = cudaFuncSetAttribute(kern, attr, value);
  if (e != cudaSuccess) {
    done.erase({kern, dev, int(attr), value});
    throw std::runtime_error(std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  }
}

// Opt-in to `bytes` of dynamic shared memory (kernels above 48 KB need it).
template <typename K>
inline void set_smem_bytes(K kern, int bytes) {
  set_func_attr_once(reinterpret_cast<const void*>(kern), cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

// Every kernel asks for the maximum shared-memory carveout, so consecutive
// kernels of a decode step never force an SM to reconfigure L1 / shared memory.
inline void prefer_max_smem_carveout(const void* kern) {
  set_func_attr_once(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
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
