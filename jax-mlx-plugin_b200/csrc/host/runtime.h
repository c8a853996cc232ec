// Device runtime: one CUDA stream per device, a caching allocator, NVRTC
// compilation of the generated kernels, and NCCL (loaded at first use).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "plan.h"

namespace b200 {

[[noreturn]] void cuda_fail(cudaError_t e, const char* what);
#define B200_CUDA(expr)                                      \
  do {                                                       \
    cudaError_t e_ = (expr);                                 \
    if (e_ != cudaSuccess) ::b200::cuda_fail(e_, #expr);     \
  } while (0)

// Size-class caching allocator for one device.  All users of the memory run on
// the device's single stream, so a block freed after its last use was enqueued
// can be handed out again immediately (stream order protects it).
class Allocator {
 public:
  explicit Allocator(int ordinal) : ordinal_(ordinal) {}
  ~Allocator();
  void* alloc(size_t bytes);
  void free(void* p, size_t bytes);
  void release_cache();
  int64_t in_use() const { return in_use_; }
  int64_t peak() const { return peak_; }
  int64_t reserved() const { return reserved_; }
  int64_t num_allocs() const { return num_allocs_; }
  static size_t round(size_t bytes);

 private:
  int ordinal_;
  std::mutex mu_;
  std::map<size_t, std::vector<void*>> cache_;
  int64_t in_use_ = 0, peak_ = 0, reserved_ = 0, num_allocs_ = 0;
};

struct Device {
  int ordinal = 0;  // CUDA device ordinal in this process
  cudaStream_t stream = nullptr;
  // Data-parallel collectives run here, ordered after the compute stream by
  // events, so that a gradient bucket's all-reduce overlaps the rest of the
  // backward pass (created with the first collective).
  cudaStream_t comm_stream = nullptr;
  std::unique_ptr<Allocator> alloc;
  std::recursive_mutex mu;  // serializes submission to the stream
  std::string name;
  int sms = 0;
  int64_t total_mem = 0;
  void activate() const;
};

// Shared ownership of a device allocation; returns it to the allocator.
struct DeviceMem {
  Device* dev = nullptr;
  void* ptr = nullptr;
  size_t bytes = 0;
  bool owned = true;
  std::function<void(void*)> on_release;  // for views of foreign memory
  DeviceMem(Device* d, size_t b);
  DeviceMem(Device* d, void* foreign, size_t b) : dev(d), ptr(foreign), bytes(b), owned(false) {}
  ~DeviceMem();
  DeviceMem(const DeviceMem&) = delete;
  DeviceMem& operator=(const DeviceMem&) = delete;
};

// NVRTC: CUDA C source -> sm_100a cubin, cached in the process by source hash
// and, when B200_CACHE_DIR names a directory, on disk across processes.
// B200_NO_JIT=1: refuse to compile (an executable must arrive with its
// cubins, e.g. through PJRT_Executable_DeserializeAndLoad).
std::string nvrtc_compile(const std::string& source, const std::string& name);
// The key nvrtc_compile files a source's cubin under: it names the source and
// the NVRTC options, so a cubin stored under it (e.g. in a serialized
// executable) is valid for exactly that source.
std::string nvrtc_key(const std::string& source);
// Several sources compiled on parallel threads (one cubin each, same order).
std::vector<std::string> nvrtc_compile_all(const std::vector<std::string>& sources,
                                           const std::string& name);

// Loaded generated kernels of one executable on one device.
struct LoadedModule {
  std::vector<CUmodule> mods;
  std::map<std::string, CUfunction> fns;
  std::vector<std::shared_ptr<DeviceMem>> consts;
  ~LoadedModule();
};
// One module per cubin, names[i] defined by cubins[i]; `alias` entries map a
// name to the function of another.
std::unique_ptr<LoadedModule> load_module(Device& d, const std::vector<std::string>& cubins,
                                          const std::vector<std::vector<std::string>>& names,
                                          const std::map<std::string, std::string>& alias);

// Host-side fault injection.  B200_FAULT (read once per process) lists
// failure points, comma-separated: alloc, compile, execute, nccl_init.  At a
// listed point the plugin throws the error that the real failure there
// raises (alloc: RESOURCE_EXHAUSTED, compile and execute: INTERNAL,
// nccl_init: UNAVAILABLE), so a caller's error handling can be tested with no
// GPU failing.  Unset: nothing happens.
void fault_point(const char* where);

// B200_OVERLAP_COLLECTIVES (default 1): gradient all-reduces are cut into
// buckets placed where their gradients are ready, and run on each device's
// communication stream; 0 runs them after the backward pass on the compute
// stream.
bool overlap_collectives();

// Generated kernels launched by launch() in this process.
extern std::atomic<unsigned long long> g_generated_launches;
// Launch a generated kernel.
void launch(Device& d, CUfunction f, const int64_t grid[3], const int64_t block[3], int smem,
            std::vector<void*>& args);

// ------------------------------------------------------------------ NCCL --
struct Nccl;
// Communicator over a set of devices.  Single process: every device local.
// Multi-process: `unique_id` (128 bytes) exchanged by the caller.
struct NcclComms {
  std::vector<void*> comms;  // ncclComm_t per local device
  // Set (once) when the communicator was aborted: every later collective on
  // it fails with this reason instead of waiting for peers that may be gone.
  std::mutex mu;
  bool aborted = false;
  std::string abort_reason;
  ~NcclComms();
};
// The first asynchronous NCCL error of any of the communicator's ranks here
// (ncclCommGetAsyncError), or "" while all are healthy.
std::string nccl_async_error(NcclComms& c);
// ncclCommAbort on every local rank (its kernels stop waiting for peers and
// exit); the communicator is unusable afterwards.  Safe to call from a thread
// other than the one issuing collectives; a second call does nothing.
void nccl_abort(NcclComms& c, const std::string& reason);
bool nccl_available(std::string* why);
std::vector<char> nccl_unique_id();
std::unique_ptr<NcclComms> nccl_init_all(const std::vector<Device*>& devs);
std::unique_ptr<NcclComms> nccl_init_rank(Device* dev, int nranks, int rank,
                                          const std::vector<char>& uid);
// On each device's `streams[i]` (its compute stream when empty).
void nccl_all_reduce(const std::vector<Device*>& devs, NcclComms& c,
                     const std::vector<const void*>& in, const std::vector<void*>& out,
                     int64_t count, DType dt, int op,
                     const std::vector<cudaStream_t>& streams = {});

}  // namespace b200
