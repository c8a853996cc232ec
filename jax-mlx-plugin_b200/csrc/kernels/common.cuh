// Shared helpers for the sm_100a kernels: error plumbing, dtype conversion,
// warp reductions.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <atomic>
#include <string>
#include <utility>

#include "b200_kernels.h"

namespace b200 {

// Records `msg` as the calling thread's last error and returns `code`.
int set_error(int code, const std::string& msg);

#define B200_CHECK_ARG(cond, msg)                                  \
  do {                                                             \
    if (!(cond)) return ::b200::set_error(B200_ERR_INVALID, msg);  \
  } while (0)

#define B200_CUDA_TRY(expr)                                                          \
  do {                                                                               \
    cudaError_t e_ = (expr);                                                         \
    if (e_ != cudaSuccess)                                                           \
      return ::b200::set_error(B200_ERR_CUDA, std::string(#expr) + ": " +            \
                                                  cudaGetErrorString(e_));           \
  } while (0)

// Launch-error check after a <<<>>> launch.
#define B200_LAUNCH_CHECK() B200_CUDA_TRY(cudaGetLastError())

template <typename T> struct Io;
template <> struct Io<float> {
  __device__ static __forceinline__ float to_f(float v) { return v; }
  __device__ static __forceinline__ float from_f(float v) { return v; }
};
template <> struct Io<__nv_bfloat16> {
  __device__ static __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ static __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Programmatic dependent launch.  Kernels started through launch_k() may be
// launched while the previous kernel on the stream is still finishing.  Every
// such kernel calls pdl_wait() before its first global memory access:
// griddepcontrol.wait returns once the previous grid has completed and its
// writes are visible, so reads after it see the producer's results and writes
// after it cannot race the producer's reads.  No kernel triggers its dependents
// early (griddepcontrol.launch_dependents): the trigger is the implicit one at
// block exit, so the next grid's launch overlaps only this grid's drain.  The
// wait is a no-op for a kernel launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// False when the environment sets B200_PDL=0 (every launch then waits for the
// previous kernel to finish before it starts, as a plain <<<>>> launch does).
bool pdl_enabled();

// Kernels this library has launched in this process (b200_kernel_launches()).
extern std::atomic<unsigned long long> g_kernel_launches;

// cudaLaunchKernelEx with the programmatic-serialization attribute; the kernel
// must begin with pdl_wait().
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                     cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (e == cudaSuccess) g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
  return e;
}

// launch_k + the launch-error check, returning from the calling function.
#define B200_LAUNCH(...) B200_CUDA_TRY(::b200::launch_k(__VA_ARGS__))

inline int num_sms() {
  static int n = [] {
    int dev = 0, v = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
      cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v;
  }();
  return n;
}

}  // namespace b200
