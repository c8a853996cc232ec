// Device runtime implementation.  The CUDA driver is reached through
// cudaGetDriverEntryPoint and NCCL through dlopen, so the plugin library loads
// on a machine without a GPU driver (where every device call fails cleanly).
#include "runtime.h"

#include <dlfcn.h>
#include <nccl.h>
#include <nvrtc.h>

#include <algorithm>
#include <cstdlib>
#include <cstdio>
#include <unistd.h>
#include <atomic>
#include <thread>
#include <cstring>
#include <functional>

namespace b200 {

void cuda_fail(cudaError_t e, const char* what) {
  throw PjrtErr(e == cudaErrorMemoryAllocation ? 8 : 13,
                std::string(what) + ": " + cudaGetErrorString(e));
}

// ------------------------------------------------------- fault injection --
void fault_point(const char* where) {
  static const std::vector<std::string> points = [] {
    std::vector<std::string> v;
    const char* e = getenv("B200_FAULT");
    std::string cur;
    for (const char* q = e ? e : ""; ; ++q) {
      if (*q == ',' || *q == '\0') {
        if (!cur.empty()) v.push_back(cur);
        cur.clear();
        if (*q == '\0') break;
      } else if (*q != ' ') {
        cur += *q;
      }
    }
    return v;
  }();
  if (points.empty()) return;
  const std::string w(where);
  if (std::find(points.begin(), points.end(), w) == points.end()) return;
  const int code = w == "alloc" ? 8 : w == "nccl_init" ? 14 : 13;
  throw PjrtErr(code, "injected fault at " + w + " (B200_FAULT)");
}

// ------------------------------------------------------------ allocator --
size_t Allocator::round(size_t b) {
  if (b == 0) b = 1;
  if (b < (1u << 20)) return (b + 511) & ~size_t(511);
  return (b + (2u << 20) - 1) & ~size_t((2u << 20) - 1);
}
void* Allocator::alloc(size_t bytes) {
  fault_point("alloc");
  const size_t sz = round(bytes);
  std::lock_guard<std::mutex> lk(mu_);
  auto it = cache_.find(sz);
  void* p = nullptr;
  if (it != cache_.end() && !it->second.empty()) {
    p = it->second.back();
    it->second.pop_back();
  } else {
    int cur = 0;
    cudaGetDevice(&cur);
    if (cur != ordinal_) cudaSetDevice(ordinal_);
    cudaError_t e = cudaMalloc(&p, sz);
    if (e != cudaSuccess) {
      cudaGetLastError();
      // give cached blocks back and retry once
      for (auto& kv : cache_)
        for (void* q : kv.second) { cudaFree(q); reserved_ -= (int64_t)kv.first; }
      cache_.clear();
      e = cudaMalloc(&p, sz);
    }
    if (cur != ordinal_) cudaSetDevice(cur);
    if (e != cudaSuccess) {
      cudaGetLastError();
      throw PjrtErr(8, "device " + std::to_string(ordinal_) + ": out of memory allocating " +
                           std::to_string(sz) + " bytes");
    }
    reserved_ += (int64_t)sz;
  }
  in_use_ += (int64_t)sz;
  peak_ = std::max(peak_, in_use_);
  ++num_allocs_;
  return p;
}
void Allocator::free(void* p, size_t bytes) {
  if (!p) return;
  const size_t sz = round(bytes);
  std::lock_guard<std::mutex> lk(mu_);
  cache_[sz].push_back(p);
  in_use_ -= (int64_t)sz;
}
void Allocator::release_cache() {
  std::lock_guard<std::mutex> lk(mu_);
  for (auto& kv : cache_)
    for (void* q : kv.second) { cudaFree(q); reserved_ -= (int64_t)kv.first; }
  cache_.clear();
}
Allocator::~Allocator() { release_cache(); }

void Device::activate() const {
  int cur = -1;
  cudaGetDevice(&cur);
  if (cur != ordinal) B200_CUDA(cudaSetDevice(ordinal));
}

DeviceMem::DeviceMem(Device* d, size_t b) : dev(d), bytes(b) { ptr = d->alloc->alloc(b); }
DeviceMem::~DeviceMem() {
  if (owned && dev && ptr) dev->alloc->free(ptr, bytes);
  if (!owned && on_release) on_release(ptr);
}

// --------------------------------------------------------- driver entry --
namespace {
template <typename F>
F driver_fn(const char* name) {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &fn, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || !fn)
    throw PjrtErr(13, std::string("CUDA driver entry point not found: ") + name);
  return reinterpret_cast<F>(fn);
}
struct Driver {
  CUresult (*ModuleLoadData)(CUmodule*, const void*);
  CUresult (*ModuleGetFunction)(CUfunction*, CUmodule, const char*);
  CUresult (*ModuleUnload)(CUmodule);
  CUresult (*GetErrorString)(CUresult, const char**);
  CUresult (*LaunchKernelEx)(const CUlaunchConfig*, CUfunction, void**, void**);
  static Driver& get() {
    static Driver d = [] {
      Driver x;
      x.ModuleLoadData = driver_fn<decltype(x.ModuleLoadData)>("cuModuleLoadData");
      x.ModuleGetFunction = driver_fn<decltype(x.ModuleGetFunction)>("cuModuleGetFunction");
      x.ModuleUnload = driver_fn<decltype(x.ModuleUnload)>("cuModuleUnload");
      x.GetErrorString = driver_fn<decltype(x.GetErrorString)>("cuGetErrorString");
      x.LaunchKernelEx = driver_fn<decltype(x.LaunchKernelEx)>("cuLaunchKernelEx");
      return x;
    }();
    return d;
  }
};
void cu_check(CUresult r, const char* what) {
  if (r == CUDA_SUCCESS) return;
  const char* s = "unknown";
  Driver::get().GetErrorString(r, &s);
  throw PjrtErr(13, std::string(what) + ": " + s);
}
}  // namespace

// ----------------------------------------------------------------- NVRTC --
namespace {
const char* const kNvrtcOpts[] = {"--gpu-architecture=sm_100a", "--std=c++17", "-lineinfo",
                                  "--fmad=true", "--diag-suppress=177,550"};
// 128-bit name for a source: FNV-1a and std::hash, plus the length.
std::string source_key(const std::string& source) {
  uint64_t f = 1469598103934665603ull;
  for (unsigned char ch : source) f = (f ^ ch) * 1099511628211ull;
  char buf[64];
  snprintf(buf, sizeof buf, "%016llx%016llx-%zu", (unsigned long long)f,
           (unsigned long long)std::hash<std::string>()(source), source.size());
  return buf;
}
std::string cache_path(const std::string& key) {
  const char* dir = getenv("B200_CACHE_DIR");
  if (!dir || !*dir) return "";
  int ver[2] = {0, 0};
  nvrtcVersion(&ver[0], &ver[1]);
  return std::string(dir) + "/b200-nvrtc" + std::to_string(ver[0]) + "." + std::to_string(ver[1]) +
         "-" + key + ".cubin";
}
}  // namespace

// The key names the source and the options, not the NVRTC build: an sm_100a
// cubin from any NVRTC release loads on any driver that runs this plugin, and
// one process may resolve libnvrtc to another release than the next (a
// framework imported first can bring its own).  The on-disk cache file name
// adds the NVRTC version on top.
std::string nvrtc_key(const std::string& source) {
  static const std::string opt_text = [] {
    std::string t;
    for (const char* o : kNvrtcOpts) t += std::string(o) + " ";
    return t;
  }();
  return source_key(opt_text + source);
}

std::string nvrtc_compile(const std::string& source, const std::string& name) {
  static std::mutex mu;
  static std::map<std::string, std::string> cache;
  const std::string key = nvrtc_key(source);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  const std::string path = cache_path(key);
  if (!path.empty()) {
    if (FILE* f = fopen(path.c_str(), "rb")) {
      std::string cubin;
      char buf[1 << 16];
      size_t n;
      while ((n = fread(buf, 1, sizeof buf, f)) > 0) cubin.append(buf, n);
      fclose(f);
      if (!cubin.empty()) {
        std::lock_guard<std::mutex> lk(mu);
        cache[key] = cubin;
        return cubin;
      }
    }
  }
  static const bool no_jit = [] {
    const char* v = getenv("B200_NO_JIT");
    return v && v[0] == '1';
  }();
  if (no_jit)
    throw PjrtErr(9, "generated kernels need compiling but B200_NO_JIT=1 forbids NVRTC here (load "
                     "a serialized executable that carries its cubins)");
  nvrtcProgram prog;
  if (nvrtcCreateProgram(&prog, source.c_str(), (name + ".cu").c_str(), 0, nullptr, nullptr) !=
      NVRTC_SUCCESS)
    throw PjrtErr(13, "nvrtcCreateProgram failed");
  nvrtcResult r = nvrtcCompileProgram(prog, (int)(sizeof kNvrtcOpts / sizeof kNvrtcOpts[0]),
                                      kNvrtcOpts);
  if (r != NVRTC_SUCCESS) {
    size_t n = 0;
    nvrtcGetProgramLogSize(prog, &n);
    std::string log(n, '\0');
    nvrtcGetProgramLog(prog, &log[0]);
    nvrtcDestroyProgram(&prog);
    throw PjrtErr(13, "NVRTC compile of generated kernels failed: " + log.substr(0, 4000));
  }
  size_t n = 0;
  nvrtcGetCUBINSize(prog, &n);
  std::string cubin(n, '\0');
  nvrtcGetCUBIN(prog, &cubin[0]);
  nvrtcDestroyProgram(&prog);
  if (!path.empty()) {  // write-then-rename: readers never see a partial file
    const std::string tmp = path + ".tmp" + std::to_string((unsigned long long)getpid());
    if (FILE* f = fopen(tmp.c_str(), "wb")) {
      const bool ok = fwrite(cubin.data(), 1, cubin.size(), f) == cubin.size();
      if (fclose(f) == 0 && ok) rename(tmp.c_str(), path.c_str());
      else remove(tmp.c_str());
    }
  }
  std::lock_guard<std::mutex> lk(mu);
  cache[key] = cubin;
  return cubin;
}

std::vector<std::string> nvrtc_compile_all(const std::vector<std::string>& sources,
                                           const std::string& name) {
  std::vector<std::string> out(sources.size());
  if (sources.size() <= 1) {
    for (size_t i = 0; i < sources.size(); ++i) out[i] = nvrtc_compile(sources[i], name);
    return out;
  }
  std::vector<std::string> errs(sources.size());
  std::vector<std::thread> th;
  std::atomic<size_t> next{0};
  const size_t nt = std::min<size_t>(sources.size(),
                                     std::max<unsigned>(1, std::thread::hardware_concurrency()));
  for (size_t t = 0; t < nt; ++t)
    th.emplace_back([&] {
      for (size_t i; (i = next++) < sources.size();) {
        try {
          out[i] = nvrtc_compile(sources[i], name + "_" + std::to_string(i));
        } catch (const std::exception& e) {
          errs[i] = e.what();
        }
      }
    });
  for (auto& t : th) t.join();
  for (auto& e : errs)
    if (!e.empty()) throw PjrtErr(13, e);
  return out;
}

LoadedModule::~LoadedModule() {
  for (CUmodule m : mods)
    if (m) Driver::get().ModuleUnload(m);
}

std::unique_ptr<LoadedModule> load_module(Device& d, const std::vector<std::string>& cubins,
                                          const std::vector<std::vector<std::string>>& names,
                                          const std::map<std::string, std::string>& alias) {
  auto m = std::make_unique<LoadedModule>();
  if (cubins.empty()) return m;
  d.activate();
  cudaFree(nullptr);  // make the primary context current
  auto& drv = Driver::get();
  for (size_t u = 0; u < cubins.size(); ++u) {
    CUmodule mod = nullptr;
    cu_check(drv.ModuleLoadData(&mod, cubins[u].data()), "cuModuleLoadData");
    m->mods.push_back(mod);
    for (auto& n : names.at(u)) {
      CUfunction f;
      cu_check(drv.ModuleGetFunction(&f, mod, n.c_str()), "cuModuleGetFunction");
      m->fns[n] = f;
    }
  }
  for (auto& kv : alias) m->fns[kv.first] = m->fns.at(kv.second);
  return m;
}

// Generated kernels begin with griddepcontrol.wait, so they are launched with
// programmatic stream serialization (B200_PDL=0 turns it off): a kernel's
// blocks may be scheduled while the previous kernel on the stream finishes.
void launch(Device& d, CUfunction f, const int64_t grid[3], const int64_t block[3], int smem,
            std::vector<void*>& args) {
  static const bool pdl = [] {
    const char* e = getenv("B200_PDL");
    return !(e && e[0] == '0');
  }();
  // A kernel over an empty index space (a reduction with no outputs) has
  // nothing to do; the driver would reject its zero-sized grid.
  if (grid[0] <= 0 || grid[1] <= 0 || grid[2] <= 0) return;
  CUlaunchAttribute attr[1];
  attr[0].id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
  attr[0].value.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  CUlaunchConfig cfg = {};
  cfg.gridDimX = (unsigned)grid[0];
  cfg.gridDimY = (unsigned)grid[1];
  cfg.gridDimZ = (unsigned)grid[2];
  cfg.blockDimX = (unsigned)block[0];
  cfg.blockDimY = (unsigned)block[1];
  cfg.blockDimZ = (unsigned)block[2];
  cfg.sharedMemBytes = (unsigned)smem;
  cfg.hStream = (CUstream)d.stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cu_check(Driver::get().LaunchKernelEx(&cfg, f, args.data(), nullptr), "cuLaunchKernelEx");
  g_generated_launches.fetch_add(1, std::memory_order_relaxed);
}

std::atomic<unsigned long long> g_generated_launches{0};

// ------------------------------------------------------------------ NCCL --
struct Nccl {
  void* h = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommInitAll)(ncclComm_t*, int, const int*) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  std::string why;
  static Nccl& get() {
    static Nccl n = [] {
      Nccl x;
      const char* env = std::getenv("B200_NCCL_LIBRARY");
      const char* cands[] = {env, "libnccl.so.2", "/usr/lib/x86_64-linux-gnu/libnccl.so.2"};
      for (const char* c : cands) {
        if (!c) continue;
        x.h = dlopen(c, RTLD_NOW | RTLD_NOLOAD);
        if (!x.h) x.h = dlopen(c, RTLD_NOW | RTLD_LOCAL);
        if (x.h) break;
      }
      if (!x.h) { x.why = "libnccl.so.2 not found"; return x; }
      auto sym = [&](const char* s) { return dlsym(x.h, s); };
      x.GetUniqueId = (decltype(x.GetUniqueId))sym("ncclGetUniqueId");
      x.CommInitRank = (decltype(x.CommInitRank))sym("ncclCommInitRank");
      x.CommInitAll = (decltype(x.CommInitAll))sym("ncclCommInitAll");
      x.CommDestroy = (decltype(x.CommDestroy))sym("ncclCommDestroy");
      x.AllReduce = (decltype(x.AllReduce))sym("ncclAllReduce");
      x.GroupStart = (decltype(x.GroupStart))sym("ncclGroupStart");
      x.GroupEnd = (decltype(x.GroupEnd))sym("ncclGroupEnd");
      x.GetErrorString = (decltype(x.GetErrorString))sym("ncclGetErrorString");
      x.CommGetAsyncError = (decltype(x.CommGetAsyncError))sym("ncclCommGetAsyncError");
      x.CommAbort = (decltype(x.CommAbort))sym("ncclCommAbort");
      if (!x.AllReduce || !x.CommInitAll || !x.CommInitRank) x.why = "libnccl lacks symbols";
      return x;
    }();
    return n;
  }
};
static void nccl_check(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return;
  auto& n = Nccl::get();
  throw PjrtErr(13, std::string(what) + ": " + (n.GetErrorString ? n.GetErrorString(r) : "error"));
}
bool nccl_available(std::string* why) {
  auto& n = Nccl::get();
  if (why) *why = n.why;
  return n.why.empty();
}
// Teardown is local: ncclCommAbort frees this process's ranks without the
// synchronization with peers that ncclCommDestroy's implicit finalize does, so
// a process whose peers already left (or are leaving at the same time) does
// not wait on them.  The owner has drained its streams before this runs.
NcclComms::~NcclComms() {
  auto& n = Nccl::get();
  std::lock_guard<std::mutex> lk(mu);
  if (aborted) return;  // ncclCommAbort already released them
  for (void* c : comms) {
    if (!c) continue;
    if (n.CommAbort) n.CommAbort((ncclComm_t)c);
    else if (n.CommDestroy) n.CommDestroy((ncclComm_t)c);
  }
}
std::string nccl_async_error(NcclComms& c) {
  auto& n = Nccl::get();
  if (!n.CommGetAsyncError) return "";
  std::lock_guard<std::mutex> lk(c.mu);
  if (c.aborted) return "";
  for (void* x : c.comms) {
    ncclResult_t st = ncclSuccess;
    if (x && n.CommGetAsyncError((ncclComm_t)x, &st) == ncclSuccess && st != ncclSuccess &&
        st != ncclInProgress)
      return std::string("NCCL asynchronous error: ") + (n.GetErrorString ? n.GetErrorString(st) : "?");
  }
  return "";
}
void nccl_abort(NcclComms& c, const std::string& reason) {
  auto& n = Nccl::get();
  std::lock_guard<std::mutex> lk(c.mu);
  if (c.aborted) return;
  c.aborted = true;
  c.abort_reason = reason;
  for (void* x : c.comms)
    if (x && n.CommAbort) n.CommAbort((ncclComm_t)x);
}
std::vector<char> nccl_unique_id() {
  auto& n = Nccl::get();
  if (!n.why.empty()) throw PjrtErr(9, "NCCL unavailable: " + n.why);
  ncclUniqueId id;
  nccl_check(n.GetUniqueId(&id), "ncclGetUniqueId");
  return std::vector<char>(id.internal, id.internal + sizeof(id.internal));
}
std::unique_ptr<NcclComms> nccl_init_all(const std::vector<Device*>& devs) {
  auto& n = Nccl::get();
  if (!n.why.empty()) throw PjrtErr(9, "NCCL unavailable: " + n.why);
  auto c = std::make_unique<NcclComms>();
  std::vector<int> ords;
  for (auto* d : devs) ords.push_back(d->ordinal);
  std::vector<ncclComm_t> cs(devs.size());
  nccl_check(n.CommInitAll(cs.data(), (int)devs.size(), ords.data()), "ncclCommInitAll");
  for (auto x : cs) c->comms.push_back(x);
  return c;
}
std::unique_ptr<NcclComms> nccl_init_rank(Device* dev, int nranks, int rank,
                                          const std::vector<char>& uid) {
  auto& n = Nccl::get();
  if (!n.why.empty()) throw PjrtErr(9, "NCCL unavailable: " + n.why);
  ncclUniqueId id;
  if (uid.size() != sizeof(id.internal)) throw PjrtErr(3, "bad NCCL unique id size");
  std::memcpy(id.internal, uid.data(), uid.size());
  dev->activate();
  ncclComm_t comm;
  nccl_check(n.CommInitRank(&comm, nranks, id, rank), "ncclCommInitRank");
  auto c = std::make_unique<NcclComms>();
  c->comms.push_back(comm);
  return c;
}
bool overlap_collectives() {
  static const bool on = [] {
    const char* v = getenv("B200_OVERLAP_COLLECTIVES");
    return !(v && v[0] == '0');
  }();
  return on;
}

void nccl_all_reduce(const std::vector<Device*>& devs, NcclComms& c,
                     const std::vector<const void*>& in, const std::vector<void*>& out,
                     int64_t count, DType dt, int op, const std::vector<cudaStream_t>& streams) {
  auto& n = Nccl::get();
  ncclDataType_t t;
  switch (dt) {
    case DType::F32: t = ncclFloat32; break;
    case DType::BF16: t = ncclBfloat16; break;
    case DType::F64: t = ncclFloat64; break;
    case DType::S32: t = ncclInt32; break;
    case DType::U32: t = ncclUint32; break;
    case DType::S64: t = ncclInt64; break;
    case DType::U64: t = ncclUint64; break;
    default: throw PjrtErr(12, "all_reduce element type not supported by NCCL");
  }
  const ncclRedOp_t ops[] = {ncclSum, ncclProd, ncclMax, ncclMin};
  nccl_check(n.GroupStart(), "ncclGroupStart");
  for (size_t i = 0; i < devs.size(); ++i) {
    devs[i]->activate();
    nccl_check(n.AllReduce(in[i], out[i], (size_t)count, t, ops[op], (ncclComm_t)c.comms.at(i),
                           streams.empty() ? devs[i]->stream : streams.at(i)),
               "ncclAllReduce");
  }
  nccl_check(n.GroupEnd(), "ncclGroupEnd");
}

}  // namespace b200
