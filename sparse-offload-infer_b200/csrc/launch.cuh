// cudaLaunchKernelEx wrapper: optional thread-block cluster along y and
// optional programmatic dependent launch (PDL).
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <utility>

namespace soinfer {

template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                      int cluster_y, bool pdl, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  unsigned n = 0;
  if (cluster_y > 1) {
    attrs[n].id = cudaLaunchAttributeClusterDimension;
    attrs[n].val.clusterDim.x = 1;
    attrs[n].val.clusterDim.y = cluster_y;
    attrs[n].val.clusterDim.z = 1;
    ++n;
  }
  if (pdl) {
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Raises Kernel's dynamic shared-memory limit to at least `bytes` on the
// current device.  The attribute belongs to the device, so the value already
// set is remembered per device (a process that drives several GPUs sets it on
// each); the call is a no-op once the device's limit is high enough.
template <auto Kernel>
cudaError_t ensure_smem_attr(int bytes) {
  constexpr int kMaxDev = 64;
  static std::atomic<int> set_bytes[kMaxDev];  // static storage: zero-initialised
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDev) return cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (set_bytes[dev].load(std::memory_order_acquire) >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  int cur = set_bytes[dev].load(std::memory_order_relaxed);
  while (cur < bytes && !set_bytes[dev].compare_exchange_weak(cur, bytes, std::memory_order_release)) {
  }
  return cudaSuccess;
}

}  // namespace soinfer
