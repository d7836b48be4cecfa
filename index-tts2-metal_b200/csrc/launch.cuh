// Kernel launch with programmatic dependent launch (PDL): the next kernel in
// the stream may start its prologue while this one drains. Every kernel
// launched through here calls griddep_wait() before it touches memory written
// by its predecessor, so ordering is preserved. ITTS_PDL=0 in the environment
// turns the attribute off (plain stream order).
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdlib>
#include <utility>

namespace itts {

inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("ITTS_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

// Runs a set-up call (e.g. a kernel's shared-memory opt-in) once per device
// ordinal: keep one instance per kernel as a function-local static. Ordinals
// beyond the table (never seen on one node) simply repeat the call.
class PerDeviceOnce {
 public:
  template <typename F>
  cudaError_t run(F&& setup) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const bool tracked = dev >= 0 && dev < kMaxOrdinals;
    if (tracked && done_[dev].load(std::memory_order_acquire)) return cudaSuccess;
    e = setup();
    if (e == cudaSuccess && tracked) done_[dev].store(true, std::memory_order_release);
    return e;
  }

 private:
  static constexpr int kMaxOrdinals = 1024;
  std::atomic<bool> done_[kMaxOrdinals] = {};
};

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// As launch_pdl, for a kernel launched in thread-block clusters of
// `cluster_x` CTAs along x.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                               unsigned cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster_x;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace itts
