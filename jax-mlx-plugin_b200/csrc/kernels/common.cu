// Error state and version of the kernel library.
#include "common.cuh"

#include <stdlib.h>

namespace b200 {
namespace {
thread_local std::string g_last_error;
}
int set_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}
bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("B200_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}
}  // namespace b200

extern "C" const char* b200_last_error(void) { return b200::g_last_error.c_str(); }
extern "C" const char* b200_kernels_version(void) { return "b200-kernels 0.1.0 sm_100a"; }

namespace b200 {
std::atomic<unsigned long long> g_kernel_launches{0};
}  // namespace b200
extern "C" uint64_t b200_kernel_launches(void) {
  return (uint64_t)b200::g_kernel_launches.load(std::memory_order_relaxed);
}

// ------------------------------------------------------------ TMA + errors --
#include <cudaTypedefs.h>

#include <mutex>
#include <map>
#include <set>
#include <string>

#include "tc.cuh"

namespace b200 {

int make_tmap(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
              const uint64_t* strides_bytes, const uint32_t* box, int elem_bytes, bool atom32) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      fn = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }();
  if (!encode) return set_error(B200_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if ((uintptr_t)base % 16) return set_error(B200_ERR_INVALID, "TMA base address not 16-byte aligned");
  cuuint64_t gdim[5];
  cuuint64_t gstr[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
    if (i > 0) {
      if (strides_bytes[i - 1] % 16) return set_error(B200_ERR_INVALID, "TMA stride not a multiple of 16 bytes");
      gstr[i - 1] = strides_bytes[i - 1];
    }
  }
  const CUtensorMapDataType dt = elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                                 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUresult r = encode(map, dt, (cuuint32_t)rank, const_cast<void*>(base), gdim, gstr, bx, es,
                      CU_TENSOR_MAP_INTERLEAVE_NONE,
                      atom32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(B200_ERR_INVALID, "cuTensorMapEncodeTiled failed with code " + std::to_string((int)r));
  return B200_OK;
}

int allow_dynamic_smem(const void* fn, int bytes, const char* what) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> done;  // (kernel, device) -> bytes allowed
  int dev = 0;
  B200_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(mu);
  auto it = done.find({fn, dev});
  if (it != done.end() && it->second >= bytes) return B200_OK;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
    return set_error(B200_ERR_CUDA, std::string("cudaFuncSetAttribute(") + what + ") failed");
  done[{fn, dev}] = bytes;
  return B200_OK;
}

namespace {
std::mutex g_word_mu;
int* g_words[64] = {nullptr};
}  // namespace

int* device_error_word() {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_word_mu);
  if (dev < 0 || dev >= 64) return nullptr;
  if (!g_words[dev]) {
    if (cudaMalloc(&g_words[dev], sizeof(int)) != cudaSuccess) return nullptr;
    cudaMemset(g_words[dev], 0, sizeof(int));
    cudaDeviceSynchronize();
  }
  return g_words[dev];
}

// The current device's error word if some kernel has already been given it;
// never allocates (nullptr when no launch on this device took the word yet).
static int* device_error_word_if_made() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lk(g_word_mu);
  if (dev < 0 || dev >= 64) return nullptr;
  return g_words[dev];
}

}  // namespace b200

// The allocation-free GEMM's word is read first and without allocating; the
// shared word is read only if a launch on this device already made it, so a
// process that only calls b200_gemm_noalloc never allocates here either.
extern "C" int b200_device_error(int clear) {
  const int v2 = b200::noalloc_error_take(clear);
  int v = 0;
  if (int* w = b200::device_error_word_if_made()) {
    if (cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    if (clear && v) cudaMemset(w, 0, sizeof(int));
  }
  if (v) return v;
  return v2;
}
