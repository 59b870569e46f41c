// pdl.cuh — programmatic dependent launch helpers.
//
// Every kernel of a window chain is launched with programmatic stream serialisation.  A kernel may read
// immutable data (weights) before griddep_wait(); it reads its predecessor's outputs, and writes any
// buffer, only after griddep_wait().  griddep_launch() lets the next kernel's CTAs start their prologue
// (weight prefetch) while this grid finishes.
#pragma once
#include "common.cuh"

namespace clm {

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Raises a kernel's dynamic shared memory limit once per (kernel, device); never inside stream capture.
template <typename... KArgs>
int ensure_smem(void (*kernel)(KArgs...), size_t bytes) {
  if (bytes <= 48 * 1024) return CLM_OK;
  int dev = 0;
  CLM_CUDA(cudaGetDevice(&dev));
  static thread_local const void* last_kernel[64];
  static thread_local size_t last_bytes[64];
  const size_t slot = (reinterpret_cast<uintptr_t>(reinterpret_cast<const void*>(kernel)) / 16 + dev) % 64;
  if (last_kernel[slot] == reinterpret_cast<const void*>(kernel) && last_bytes[slot] >= bytes) return CLM_OK;
  const size_t want = bytes > 200 * 1024 ? bytes : 200 * 1024;
  CLM_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)want));
  last_kernel[slot] = reinterpret_cast<const void*>(kernel);
  last_bytes[slot] = want;
  return CLM_OK;
}

// Kernel launches issued through launch_pdl on this thread (engines record per-graph launch counts).
inline thread_local unsigned long long t_kernel_launches = 0;

template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  // The implicit default streams keep plain serialisation (griddepcontrol.wait then returns at once).
  cfg.numAttrs = (st == nullptr || st == cudaStreamLegacy || st == cudaStreamPerThread) ? 0 : 1;
  CLM_CUDA(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
  ++t_kernel_launches;
  return CLM_OK;
}

}  // namespace clm
