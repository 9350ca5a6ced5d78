// ks_launch.cuh -- per-device launch attributes.
//
// A kernel that needs more than 48 KB of dynamic shared memory must have
// cudaFuncAttributeMaxDynamicSharedMemorySize raised on every device it runs
// on.  One process may drive several GPUs (ks_ctx_create_all), so the
// attribute is set once per (kernel, device), tracked in a bit mask.
#pragma once
#include <cuda_runtime.h>

#include <atomic>

namespace ksb {

template <class Kernel>
cudaError_t ensure_dynamic_smem(Kernel kernel, size_t bytes, std::atomic<unsigned> &done_mask) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned bit = dev < 32 ? 1u << dev : 0u;
  if (bit && (done_mask.load() & bit)) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess && bit) done_mask.fetch_or(bit);
  return e;
}

}  // namespace ksb
