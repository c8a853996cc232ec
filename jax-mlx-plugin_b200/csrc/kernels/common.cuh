// Shared helpers for the sm_100a kernels: error plumbing, dtype conversion,
// warp reductions.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <string>

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
