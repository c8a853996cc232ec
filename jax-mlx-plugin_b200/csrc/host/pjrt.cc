// PJRT C API implementation (GetPjrtApi) for N CUDA devices.
//
// Replaces the reference's PJRT surface (src/jax_mlx_pjrt.cpp:535-1650 and
// the API table at :9481-9670).  Differences that matter to callers:
//   - every entry point catches C++ exceptions and returns a PJRT_Error;
//   - events are real (cudaEvent-backed), not always-ready (ref :559-587);
//   - OutputElementTypes/OutputDimensions report the compiled program's real
//     types and shapes (ref :1466-1527 always said F32 / left data unset);
//   - Buffer_IsOnCpu is false (ref :1254-1257 said true);
//   - DefaultDeviceAssignment is implemented (ref :935 was a stub);
//   - executables run replicated over several devices with NCCL all_reduce.
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdio>
#include <cstring>
#include <functional>
#include <set>
#include <thread>

#include "b200_kernels.h"
#include "gemm_ws.h"
#include "b200_pjrt.h"
#include "b200_pjrt_inspect.h"
#include "passes.h"
#include "plan.h"
#include "runtime.h"

using namespace b200;

// ------------------------------------------------------------ objects ---
struct PJRT_Error {
  PJRT_Error_Code code;
  std::string msg;
};

// The outcome of an Execute's collectives as the NCCL watchdog saw it: set
// when it aborted a communicator the Execute used, before the abort lets the
// stuck kernels (and so the Execute's events) finish.
struct CollectiveStatus {
  std::mutex mu;
  PJRT_Error_Code code = PJRT_Error_Code_OK;
  std::string msg;
  void fail(PJRT_Error_Code c, const std::string& m) {
    std::lock_guard<std::mutex> lk(mu);
    if (code == PJRT_Error_Code_OK) code = c, msg = m;
  }
  bool failed(PJRT_Error_Code* c, std::string* m) {
    std::lock_guard<std::mutex> lk(mu);
    if (code == PJRT_Error_Code_OK) return false;
    *c = code;
    *m = msg;
    return true;
  }
};

struct PJRT_Event {
  std::mutex mu;
  std::condition_variable cv;
  cudaEvent_t ev = nullptr;
  std::shared_ptr<CollectiveStatus> status;  // the producing Execute's collectives
  int ordinal = -1;
  bool host_set = false;  // for host-completed events
  bool host_done = false;
  PJRT_Error_Code code = PJRT_Error_Code_OK;
  std::string msg;
  virtual ~PJRT_Event() {
    if (ev) cudaEventDestroy(ev);
  }
};

struct PJRT_DeviceDescription {
  int id = 0;
  int process_index = 0;
  std::string kind, debug, tostr;
  std::vector<PJRT_NamedValue> attrs;
  std::string cc;
  int64_t cores = 0;
};

struct PJRT_Memory {
  int id = 0;
  std::string kind = "device";
  std::string debug, tostr;
  PJRT_Device* device = nullptr;
};

struct PJRT_Device {
  PJRT_DeviceDescription desc;
  Device* dev = nullptr;  // null when not addressable from this process
  PJRT_Memory* memory = nullptr;
  int local_hardware_id = -1;
};

struct PJRT_TopologyDescription {
  std::vector<PJRT_DeviceDescription*> descs;
  std::string name = "b200", version;
};

struct PJRT_Client {
  std::vector<std::unique_ptr<Device>> local;
  std::vector<std::unique_ptr<PJRT_Device>> devices;  // global order
  std::vector<PJRT_Device*> device_ptrs, addressable;
  std::vector<std::unique_ptr<PJRT_Memory>> memories;
  std::vector<PJRT_Memory*> memory_ptrs;
  int process_index = 0, num_nodes = 1;
  std::string version;
  PJRT_KeyValueGetCallback kv_get = nullptr;
  void* kv_get_arg = nullptr;
  PJRT_KeyValuePutCallback kv_put = nullptr;
  void* kv_put_arg = nullptr;
  std::mutex exec_mu;
  std::map<std::vector<int>, std::unique_ptr<NcclComms>> comms;  // keyed by global device ids
  std::atomic<int64_t> comm_counter{0};
  PJRT_TopologyDescription topo;
  std::unique_ptr<struct NcclWatchdog> watchdog;  // started with the first collective
};

// Host watchdog over the client's collectives (NCCL's own kernels wait for
// peers without bound).  Each collective an Execute enqueues is followed by a
// CUDA event; a thread polls the pending events every 2 ms and, while one is
// not reached, the communicator's asynchronous error state.  On an NCCL error,
// or when the event is still pending B200_NCCL_TIMEOUT_MS (default 600000)
// after the collective was enqueued (a peer rank that left or stalled), it
// marks the Execute failed (INTERNAL or DEADLINE_EXCEEDED) and aborts the
// communicator (ncclCommAbort): the waiting kernels exit, the Execute's events
// complete with that error, and every later collective on the communicator is
// refused (ABORTED) instead of hanging.
struct NcclWatchdog {
  struct Item {
    cudaEvent_t ev;
    NcclComms* comms;
    std::shared_ptr<CollectiveStatus> status;
    std::chrono::steady_clock::time_point deadline;
    std::string what;
  };
  std::mutex mu;
  std::condition_variable cv;
  std::vector<Item> items;
  bool stop = false;
  int64_t timeout_ms;
  std::thread th;
  NcclWatchdog() {
    const char* v = std::getenv("B200_NCCL_TIMEOUT_MS");
    timeout_ms = v && std::atoll(v) > 0 ? std::atoll(v) : 600000;
    th = std::thread([this] { loop(); });
  }
  ~NcclWatchdog() {
    {
      std::lock_guard<std::mutex> lk(mu);
      stop = true;
    }
    cv.notify_all();
    th.join();
    for (auto& it : items) cudaEventDestroy(it.ev);
  }
  void watch(Device& d, cudaStream_t stream, NcclComms* comms, std::shared_ptr<CollectiveStatus> status,
             const std::string& what) {
    cudaEvent_t ev = nullptr;
    d.activate();
    B200_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    B200_CUDA(cudaEventRecord(ev, stream));
    {
      std::lock_guard<std::mutex> lk(mu);
      items.push_back({ev, comms, std::move(status),
                       std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms), what});
    }
    cv.notify_all();
  }
  void loop() {
    std::unique_lock<std::mutex> lk(mu);
    while (!stop) {
      if (items.empty()) {
        cv.wait(lk, [&] { return stop || !items.empty(); });
        continue;
      }
      cv.wait_for(lk, std::chrono::milliseconds(2));
      const auto now = std::chrono::steady_clock::now();
      for (size_t i = 0; i < items.size();) {
        Item& it = items[i];
        const cudaError_t r = cudaEventQuery(it.ev);
        std::string why;
        PJRT_Error_Code code = PJRT_Error_Code_INTERNAL;
        if (r == cudaSuccess) {
        } else if (r != cudaErrorNotReady) {
          why = std::string("CUDA error while waiting for ") + it.what + ": " + cudaGetErrorString(r);
        } else if (!(why = nccl_async_error(*it.comms)).empty()) {
          why = it.what + ": " + why;
        } else if (now >= it.deadline) {
          code = PJRT_Error_Code_DEADLINE_EXCEEDED;
          why = it.what + " did not complete within B200_NCCL_TIMEOUT_MS=" + std::to_string(timeout_ms) +
                " ms (a peer rank left or stalled); the communicator was aborted";
        } else {
          ++i;
          continue;
        }
        if (!why.empty()) {
          it.status->fail(code, why);
          nccl_abort(*it.comms, why);
        }
        cudaEventDestroy(it.ev);
        items.erase(items.begin() + (long)i);
      }
    }
  }
};

struct PJRT_Buffer {
  PJRT_Client* client = nullptr;
  PJRT_Device* device = nullptr;
  TensorType type;
  std::shared_ptr<DeviceMem> mem;
  std::shared_ptr<PJRT_Event> ready;  // definition event
  std::atomic<int> ext_refs{0};
  bool deleted = false;
  std::vector<int64_t> dims;  // for Dimensions()
};

namespace {

struct Exe {
  PJRT_Client* client = nullptr;
  Plan plan;
  std::vector<std::string> cubins;  // one per compilation unit of the plan
  std::string name, fingerprint, text, compile_options;
  std::vector<int64_t> out_dims_flat;
  std::vector<size_t> out_dim_sizes;
  std::vector<PJRT_Buffer_Type> out_types;
  std::vector<const char*> out_kinds;
  std::vector<size_t> out_kind_sizes;
  std::mutex mu;
  std::map<int, std::unique_ptr<LoadedModule>> modules;  // by device ordinal
  std::vector<PJRT_Device*> addressable;                 // replica order, this process
  std::vector<int> replica_of;                           // per addressable device
  int64_t num_replicas = 1;
  std::vector<PJRT_NamedValue> cost;
  // B200_TIMING=1: device time of each Execute's launch sequence (device 0)
  std::mutex timing_mu;
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> timings;
  // CUDA-graph replay (one device per Execute), by device ordinal
  std::map<int, std::unique_ptr<struct GraphState>> graphs;
  int graph_ok = -1;  // -1 undecided, 0 no, 1 yes
};

// CUDA-graph replay of a plan on one device.  The plan's slots get fixed
// buffers; the launch sequence between collectives is captured once (after an
// eager warm-up run) and replayed: an Execute then costs one copy per argument
// into the fixed parameter buffers, one graph launch per segment, and one copy
// per output into a fresh buffer, instead of a host launch per kernel.
struct GraphState {
  int eager_runs = 0;
  bool disabled = false;
  std::vector<std::vector<void*>> ptr;  // [1][slot] fixed pointers
  std::vector<std::shared_ptr<DeviceMem>> mem;
  std::shared_ptr<DeviceMem> gemm_ws;   // workspace shared by the captured GEMMs
  std::vector<std::pair<int, int>> items;  // (0, graph index) or (1, step index)
  std::vector<cudaGraphExec_t> execs;
  ~GraphState() {
    for (auto g : execs) cudaGraphExecDestroy(g);
  }
};

}  // namespace

struct PJRT_Executable {
  std::shared_ptr<Exe> exe;
};
struct PJRT_LoadedExecutable {
  std::shared_ptr<Exe> exe;
  bool deleted = false;
};

namespace {

PJRT_Error* make_err(int code, const std::string& msg) {
  return new PJRT_Error{(PJRT_Error_Code)code, msg};
}

#define PJRT_TRY try {
#define PJRT_CATCH                                                     \
  }                                                                    \
  catch (const PjrtErr& e) { return make_err(e.code, e.what()); }      \
  catch (const std::exception& e) { return make_err(13, e.what()); }   \
  catch (...) { return make_err(2, "unknown exception"); }             \
  return nullptr;

bool env_flag(const char* n) {
  const char* v = std::getenv(n);
  return v && *v && std::strcmp(v, "0") != 0;
}

std::shared_ptr<PJRT_Event> record_event(Device& d) {
  auto e = std::make_shared<PJRT_Event>();
  d.activate();
  B200_CUDA(cudaEventCreateWithFlags(&e->ev, cudaEventDisableTiming));
  B200_CUDA(cudaEventRecord(e->ev, d.stream));
  e->ordinal = d.ordinal;
  return e;
}
PJRT_Event* ready_event() {
  auto* e = new PJRT_Event;
  e->host_set = true;
  e->host_done = true;
  return e;
}
// Event objects handed to PJRT keep a shared_ptr to the underlying state.
struct EventHandle : PJRT_Event {
  std::shared_ptr<PJRT_Event> inner;
};

PJRT_Event* handle_of(const std::shared_ptr<PJRT_Event>& inner) {
  auto* h = new EventHandle;
  h->inner = inner;
  return h;
}

bool event_ready(PJRT_Event* e, PJRT_Error_Code* code, std::string* msg) {
  if (auto* h = dynamic_cast<EventHandle*>(e)) return event_ready(h->inner.get(), code, msg);
  std::lock_guard<std::mutex> lk(e->mu);
  if (e->host_set) {
    *code = e->code;
    *msg = e->msg;
    return e->host_done;
  }
  if (!e->ev) return true;
  cudaError_t r = cudaEventQuery(e->ev);
  if (r == cudaErrorNotReady) return false;
  if (r != cudaSuccess) {
    *code = PJRT_Error_Code_INTERNAL;
    *msg = cudaGetErrorString(r);
  } else if (e->status) {
    e->status->failed(code, msg);
  }
  return true;
}
void event_wait(PJRT_Event* e, PJRT_Error_Code* code, std::string* msg) {
  if (auto* h = dynamic_cast<EventHandle*>(e)) return event_wait(h->inner.get(), code, msg);
  if (e->host_set) {
    std::unique_lock<std::mutex> lk(e->mu);
    e->cv.wait(lk, [&] { return e->host_done; });
    *code = e->code;
    *msg = e->msg;
    return;
  }
  if (!e->ev) return;
  cudaError_t r = cudaEventSynchronize(e->ev);
  if (r != cudaSuccess) {
    *code = PJRT_Error_Code_INTERNAL;
    *msg = cudaGetErrorString(r);
  } else if (e->status) {
    e->status->failed(code, msg);
  }
}

DType to_dtype(PJRT_Buffer_Type t) {
  switch (t) {
    case PJRT_Buffer_Type_PRED: return DType::PRED;
    case PJRT_Buffer_Type_S8: return DType::S8;
    case PJRT_Buffer_Type_S16: return DType::S16;
    case PJRT_Buffer_Type_S32: return DType::S32;
    case PJRT_Buffer_Type_S64: return DType::S64;
    case PJRT_Buffer_Type_U8: return DType::U8;
    case PJRT_Buffer_Type_U16: return DType::U16;
    case PJRT_Buffer_Type_U32: return DType::U32;
    case PJRT_Buffer_Type_U64: return DType::U64;
    case PJRT_Buffer_Type_F32: return DType::F32;
    case PJRT_Buffer_Type_F64: return DType::F64;
    case PJRT_Buffer_Type_BF16: return DType::BF16;
    default: throw PjrtErr(12, "buffer element type " + std::to_string((int)t) + " is not supported");
  }
}

int64_t kv_timeout_ms() {
  const char* v = std::getenv("B200_KV_TIMEOUT_MS");
  return v ? std::atoll(v) : 120000;
}

// The error constructor handed to KV-store callbacks: jaxlib's C++ wrappers
// report a failed or timed-out store operation by calling
// (*args->callback_error)(code, message, size) and returning the result.
PJRT_Error* kv_callback_error(PJRT_Error_Code code, const char* msg, size_t n) {
  return new PJRT_Error{code, std::string(msg ? msg : "", msg ? n : 0)};
}
PJRT_CallbackError g_kv_callback_error = &kv_callback_error;

std::string kv_get(PJRT_KeyValueGetCallback cb, void* user_arg, const std::string& key) {
  if (!cb) throw PjrtErr(9, "multi-process execution needs the client's KV-store callbacks");
  PJRT_KeyValueGetCallback_Args a{};
  a.struct_size = sizeof(a);
  a.key = key.data();
  a.key_size = key.size();
  a.timeout_in_ms = (int)kv_timeout_ms();
  a.callback_error = &g_kv_callback_error;
  a.user_arg = user_arg;
  PJRT_Error* e = cb(&a);
  if (e) {
    const int code = e->code ? (int)e->code : 4;
    std::string m = e->msg;
    delete e;  // made by kv_callback_error above
    throw PjrtErr(code, "KV get '" + key + "' failed: " + m);
  }
  // A callback that could not produce the value (a Python one whose store
  // raised or timed out returns no error object) leaves it unset.
  if (!a.value)
    throw PjrtErr(4, "KV get '" + key + "' returned no value (the key-value store's get failed "
                     "or timed out; did rank 0 reach its first collective?)");
  std::string v(a.value, a.value_size);
  if (a.value_deleter_callback) a.value_deleter_callback(a.value);
  return v;
}
void kv_put(PJRT_KeyValuePutCallback cb, void* user_arg, const std::string& key,
            const std::string& val) {
  if (!cb) throw PjrtErr(9, "multi-process execution needs the client's KV-store callbacks");
  PJRT_KeyValuePutCallback_Args a{};
  a.struct_size = sizeof(a);
  a.key = key.data();
  a.key_size = key.size();
  a.value = val.data();
  a.value_size = val.size();
  a.callback_error = &g_kv_callback_error;
  a.user_arg = user_arg;
  PJRT_Error* e = cb(&a);
  if (e) {
    const int code = e->code ? (int)e->code : 13;
    std::string m = e->msg;
    delete e;
    throw PjrtErr(code, "KV put '" + key + "' failed: " + m);
  }
}
std::string kv_get(PJRT_Client* c, const std::string& key) { return kv_get(c->kv_get, c->kv_get_arg, key); }
void kv_put(PJRT_Client* c, const std::string& key, const std::string& val) {
  kv_put(c->kv_put, c->kv_put_arg, key, val);
}

// ---------------------------------------------- bytecode -> text (jaxlib) --
// JAX hands the plugin a StableHLO portable artifact (MLIR bytecode).  As in
// the reference (src/jax_mlx_pjrt.cpp:671-830) it is turned into text through
// the MLIR/StableHLO C API that jaxlib has loaded in this process.
// Path 1: the MLIR / StableHLO C API, when some library in the process exports
// it (Reactant.jl does; reference src/jax_mlx_pjrt.cpp:671-745).  Returns false
// when the API is not loaded.
bool bytecode_via_c_api(const std::string& code, std::string* out) {
  struct StrRef { const char* data; size_t length; };
  struct Handle { void* ptr; };
  using CtxCreate = Handle (*)();
  using CtxDestroy = void (*)(Handle);
  using Deser = Handle (*)(StrRef, Handle);
  using GetOp = Handle (*)(Handle);
  using Print = void (*)(Handle, void (*)(StrRef, void*), void*);
  using ModDestroy = void (*)(Handle);
  using Register = void (*)(Handle);
  void* self = RTLD_DEFAULT;
  auto deser = (Deser)dlsym(self, "stablehloDeserializePortableArtifactNoError");
  auto ctxc = (CtxCreate)dlsym(self, "mlirContextCreate");
  auto ctxd = (CtxDestroy)dlsym(self, "mlirContextDestroy");
  auto getop = (GetOp)dlsym(self, "mlirModuleGetOperation");
  auto print = (Print)dlsym(self, "mlirOperationPrint");
  auto moddel = (ModDestroy)dlsym(self, "mlirModuleDestroy");
  auto reg = (Register)dlsym(self, "stablehloRegisterAllDialects");
  if (!deser || !ctxc || !getop || !print) return false;
  Handle ctx = ctxc();
  if (reg) reg(ctx);
  Handle mod = deser(StrRef{code.data(), code.size()}, ctx);
  if (!mod.ptr) {
    if (ctxd) ctxd(ctx);
    throw PjrtErr(3, "failed to deserialize the StableHLO portable artifact");
  }
  print(getop(mod), [](StrRef s, void* u) { static_cast<std::string*>(u)->append(s.data, s.length); },
        out);
  if (moddel) moddel(mod);
  if (ctxd) ctxd(ctx);
  return true;
}

// Path 2: jaxlib's Python bindings, when the plugin lives in a Python process
// (the `jax.jit` case; reference src/jax_mlx_pjrt.cpp:747-822).  The CPython
// entry points are looked up in the process (a Python executable exports
// them), so the plugin does not link against libpython.  Under the GIL:
//   ctx = jax._src.interpreters.mlir.make_ir_context()
//   module = jaxlib.mlir._mlir_libs._stablehlo.deserialize_portable_artifact(ctx, code)
//   text = str(module)
// Returns false when Python is not running or either module cannot be
// imported; a deserializer that raises is an INVALID_ARGUMENT error.
bool bytecode_via_python(const std::string& code, std::string* out) {
  using Obj = void*;
  struct Py {
    int (*IsInitialized)();
    int (*GILEnsure)();
    void (*GILRelease)(int);
    Obj (*Import)(const char*);
    Obj (*GetAttr)(Obj, const char*);
    Obj (*CallObject)(Obj, Obj);
    Obj (*Bytes)(const char*, ssize_t);
    Obj (*Tuple)(ssize_t, ...);
    Obj (*Str)(Obj);
    const char* (*Utf8)(Obj, ssize_t*);
    void (*DecRef)(Obj);
    void (*Fetch)(Obj*, Obj*, Obj*);
    void (*Clear)();
  };
  static const Py py = [] {
    Py p{};
    auto sym = [](const char* n) { return dlsym(RTLD_DEFAULT, n); };
    p.IsInitialized = (int (*)())sym("Py_IsInitialized");
    p.GILEnsure = (int (*)())sym("PyGILState_Ensure");
    p.GILRelease = (void (*)(int))sym("PyGILState_Release");
    p.Import = (Obj(*)(const char*))sym("PyImport_ImportModule");
    p.GetAttr = (Obj(*)(Obj, const char*))sym("PyObject_GetAttrString");
    p.CallObject = (Obj(*)(Obj, Obj))sym("PyObject_CallObject");
    p.Bytes = (Obj(*)(const char*, ssize_t))sym("PyBytes_FromStringAndSize");
    p.Tuple = (Obj(*)(ssize_t, ...))sym("PyTuple_Pack");
    p.Str = (Obj(*)(Obj))sym("PyObject_Str");
    p.Utf8 = (const char* (*)(Obj, ssize_t*))sym("PyUnicode_AsUTF8AndSize");
    p.DecRef = (void (*)(Obj))sym("Py_DecRef");
    p.Fetch = (void (*)(Obj*, Obj*, Obj*))sym("PyErr_Fetch");
    p.Clear = (void (*)())sym("PyErr_Clear");
    return p;
  }();
  if (!py.IsInitialized || !py.GILEnsure || !py.GILRelease || !py.Import || !py.GetAttr ||
      !py.CallObject || !py.Bytes || !py.Tuple || !py.Str || !py.Utf8 || !py.DecRef ||
      !py.Fetch || !py.Clear || !py.IsInitialized())
    return false;
  const int gil = py.GILEnsure();
  std::vector<Obj> held;  // released (in reverse) before the GIL
  auto keep = [&](Obj o) { if (o) held.push_back(o); return o; };
  auto py_error = [&]() {
    Obj t = nullptr, v = nullptr, tb = nullptr;
    py.Fetch(&t, &v, &tb);
    std::string msg = "unknown Python error";
    if (v) {
      if (Obj s = py.Str(v)) {
        ssize_t n = 0;
        if (const char* c = py.Utf8(s, &n)) msg.assign(c, (size_t)n);
        py.DecRef(s);
      }
    }
    for (Obj o : {t, v, tb}) if (o) py.DecRef(o);
    py.Clear();
    return msg;
  };
  bool ok = false;
  std::string failure;
  do {
    Obj mlir = keep(py.Import("jax._src.interpreters.mlir"));
    Obj shlo = mlir ? keep(py.Import("jaxlib.mlir._mlir_libs._stablehlo")) : nullptr;
    if (!mlir || !shlo) { py.Clear(); break; }  // no jax in this process
    Obj make_ctx = keep(py.GetAttr(mlir, "make_ir_context"));
    Obj deser = keep(py.GetAttr(shlo, "deserialize_portable_artifact"));
    if (!make_ctx || !deser) { py.Clear(); break; }
    Obj ctx = keep(py.CallObject(make_ctx, nullptr));
    if (!ctx) { failure = "make_ir_context() raised: " + py_error(); break; }
    Obj bytes = keep(py.Bytes(code.data(), (ssize_t)code.size()));
    Obj args = bytes ? keep(py.Tuple(2, ctx, bytes)) : nullptr;
    Obj module = args ? keep(py.CallObject(deser, args)) : nullptr;
    if (!module) { failure = "deserialize_portable_artifact raised: " + py_error(); break; }
    Obj text = keep(py.Str(module));
    ssize_t n = 0;
    const char* c = text ? py.Utf8(text, &n) : nullptr;
    if (!c) { failure = "str(module) failed: " + py_error(); break; }
    out->assign(c, (size_t)n);
    ok = true;
  } while (false);
  for (auto it = held.rbegin(); it != held.rend(); ++it) py.DecRef(*it);
  py.GILRelease(gil);
  if (!failure.empty()) throw PjrtErr(3, "StableHLO portable artifact: " + failure);
  return ok;
}

// JAX hands the plugin a StableHLO portable artifact (MLIR bytecode); it is
// turned into text by whichever MLIR front end the process has loaded.
std::string bytecode_to_text(const std::string& code) {
  std::string out;
  if (bytecode_via_c_api(code, &out)) return out;
  if (bytecode_via_python(code, &out)) return out;
  throw PjrtErr(12,
                "program is MLIR bytecode but neither the StableHLO C API nor jaxlib's Python "
                "bindings are loaded in this process; pass StableHLO text (format \"mlir\") instead");
}

// Minimal protobuf walk: CompileOptionsProto.executable_build_options (3)
// .num_replicas (4) / .num_partitions (5).
bool pb_varint(const uint8_t*& p, const uint8_t* e, uint64_t* v) {
  *v = 0;
  for (int s = 0; p < e && s < 64; s += 7) {
    uint8_t b = *p++;
    *v |= (uint64_t)(b & 0x7f) << s;
    if (!(b & 0x80)) return true;
  }
  return false;
}
void pb_fields(const std::string& buf, const std::function<void(int, int, uint64_t, const std::string&)>& f) {
  const uint8_t* p = (const uint8_t*)buf.data();
  const uint8_t* e = p + buf.size();
  while (p < e) {
    uint64_t key;
    if (!pb_varint(p, e, &key)) return;
    int field = (int)(key >> 3), wt = (int)(key & 7);
    if (wt == 0) {
      uint64_t v;
      if (!pb_varint(p, e, &v)) return;
      f(field, wt, v, "");
    } else if (wt == 2) {
      uint64_t n;
      if (!pb_varint(p, e, &n) || p + n > e) return;
      f(field, wt, 0, std::string((const char*)p, n));
      p += n;
    } else if (wt == 1) {
      p += 8;
    } else if (wt == 5) {
      p += 4;
    } else {
      return;
    }
  }
}
void replicas_from_options(const std::string& opts, int64_t* reps, int64_t* parts) {
  pb_fields(opts, [&](int f, int wt, uint64_t, const std::string& sub) {
    if (f == 3 && wt == 2)
      pb_fields(sub, [&](int g, int wt2, uint64_t v, const std::string&) {
        if (wt2 != 0) return;
        if (g == 4 && v > 0) *reps = (int64_t)v;
        if (g == 5 && v > 0) *parts = (int64_t)v;
      });
  });
}

// StableHLO text as given, or a portable artifact (MLIR bytecode, magic
// "ML\xefR") converted to text.
std::string program_text(const std::string& code) {
  if (code.size() >= 4 && code.compare(0, 4, "ML\xefR") == 0) return bytecode_to_text(code);
  return code;
}

// prebuilt: cubins by nvrtc_key of their source (from a serialized
// executable); a unit whose key is there is not compiled again.
std::shared_ptr<Exe> compile(PJRT_Client* c, const std::string& code, const std::string& opts,
                             const std::map<std::string, std::string>* prebuilt = nullptr) {
  fault_point("compile");
  const std::string text = program_text(code);
  Module m = parse_module(text);
  int64_t reps = 1, parts = 1;
  replicas_from_options(opts, &reps, &parts);
  if (m.num_replicas > 1) reps = m.num_replicas;
  if (m.num_partitions > 1) parts = m.num_partitions;
  if (parts > 1)
    throw PjrtErr(12, "num_partitions > 1 (SPMD partitioning) is not supported; use pmap or "
                      "shard_map style replication");
  m.num_replicas = reps;
  auto e = std::make_shared<Exe>();
  e->client = c;
  e->plan = build_plan(m);
  e->plan.num_replicas = reps;
  e->num_replicas = reps;
  e->text = text;
  e->compile_options = opts;
  e->name = m.name.empty() ? "main" : m.name;
  e->fingerprint = std::to_string(std::hash<std::string>()(text));
  if (!e->plan.kernel_names.empty()) {
    std::vector<std::string> todo;
    std::vector<size_t> todo_at;
    e->cubins.assign(e->plan.units.size(), std::string());
    for (size_t u = 0; u < e->plan.units.size(); ++u) {
      auto it = prebuilt ? prebuilt->find(nvrtc_key(e->plan.units[u])) : decltype(prebuilt->end()){};
      if (prebuilt && it != prebuilt->end()) {
        e->cubins[u] = it->second;
      } else {
        todo.push_back(e->plan.units[u]);
        todo_at.push_back(u);
      }
    }
    if (!todo.empty()) {
      if (prebuilt && env_flag("B200_NO_JIT")) {
        std::string carried;
        for (auto& kv : *prebuilt) carried += " [" + kv.first + "]";
        throw PjrtErr(9, "serialized executable: " + std::to_string(todo.size()) + " of " +
                             std::to_string(e->plan.units.size()) +
                             " kernel units of the re-planned program have no cubin in it (first "
                             "missing key [" + nvrtc_key(todo[0]) + "]; carried:" + carried +
                             ") and B200_NO_JIT=1 forbids compiling them");
      }
      auto built = nvrtc_compile_all(todo, "b200_" + e->fingerprint);
      for (size_t i = 0; i < built.size(); ++i) e->cubins[todo_at[i]] = std::move(built[i]);
    }
  }
  for (auto& t : e->plan.output_types) {
    e->out_dim_sizes.push_back(t.dims.size());
    e->out_dims_flat.insert(e->out_dims_flat.end(), t.dims.begin(), t.dims.end());
    e->out_types.push_back((PJRT_Buffer_Type)t.dtype);
    e->out_kinds.push_back("device");
    e->out_kind_sizes.push_back(6);
  }
  // replica r runs on global device r
  if ((int64_t)c->device_ptrs.size() < reps)
    throw PjrtErr(3, "program needs " + std::to_string(reps) + " replicas but the client has " +
                         std::to_string(c->device_ptrs.size()) + " devices");
  for (int64_t r = 0; r < reps; ++r) {
    PJRT_Device* d = c->device_ptrs[r];
    if (d->dev) {
      e->addressable.push_back(d);
      e->replica_of.push_back((int)r);
    }
  }
  if (env_flag("B200_DUMP")) {
    std::fprintf(stderr, "[b200] graph:\n%s\n[b200] plan:\n%s\n", e->plan.graph_dump.c_str(),
                 dump_plan(e->plan).c_str());
  }
  return e;
}

void kcheck(int rc, const char* what) {
  if (rc != 0) throw PjrtErr(rc == B200_ERR_INVALID ? 3 : 13, std::string(what) + ": " + b200_last_error());
}

NcclComms& comms_for(PJRT_Client* c, Exe& e) {
  std::vector<int> ids;
  for (int64_t r = 0; r < e.num_replicas; ++r) ids.push_back((int)r);
  auto it = c->comms.find(ids);
  if (it != c->comms.end()) {
    std::lock_guard<std::mutex> lk(it->second->mu);
    if (it->second->aborted)
      throw PjrtErr(10, "the NCCL communicator of these replicas was aborted earlier (" +
                            it->second->abort_reason + "); no further collectives run on it");
    return *it->second;
  }
  fault_point("nccl_init");
  std::unique_ptr<NcclComms> comm;
  if (c->num_nodes == 1) {
    std::vector<Device*> devs;
    for (auto* d : e.addressable) devs.push_back(d->dev);
    comm = nccl_init_all(devs);
  } else {
    if (e.addressable.size() != 1)
      throw PjrtErr(12, "multi-process execution supports one device per process");
    const int rank = e.replica_of[0];
    const std::string key = "b200/nccl_uid/" + std::to_string(e.num_replicas);
    std::vector<char> uid;
    if (rank == 0) {
      uid = nccl_unique_id();
      kv_put(c, key, std::string(uid.begin(), uid.end()));
    } else {
      std::string v = kv_get(c, key);
      uid.assign(v.begin(), v.end());
    }
    comm = nccl_init_rank(e.addressable[0]->dev, (int)e.num_replicas, rank, uid);
  }
  auto& ref = *comm;
  c->comms[ids] = std::move(comm);
  return ref;
}

// A GEMM step's call.  st.in = {A, B[, bias]}; the bias is read only by the
// bias epilogues (ip[11] 1 or 2).  st.args, when present, name the bf16 lo
// planes of an A / B that a producer wrote split (slot -1: not split).
template <typename PtrOf>
static int64_t gemm_step_ws_bytes(const Step& st, PtrOf P, void* stream) {
  const void* bias = (st.ip[11] == 1 || st.ip[11] == 2) ? P(st.in[2]) : nullptr;
  const void* a_lo = st.args.size() >= 2 && st.args[0].slot >= 0 ? P(st.args[0].slot) : nullptr;
  const void* b_lo = st.args.size() >= 2 && st.args[1].slot >= 0 ? P(st.args[1].slot) : nullptr;
  if (a_lo || b_lo)
    return b200_gemm_planes_workspace_bytes(P(st.in[0]), a_lo, P(st.in[1]), b_lo, P(st.out[0]), bias,
                                            st.ip[0], st.ip[1], st.ip[2], st.ip[3], st.ip[4], st.ip[5],
                                            st.ip[6], st.ip[7], st.ip[8], st.ip[9], st.ip[10], st.fp[0],
                                            st.dtype, st.dtype2, (int)st.ip[11], stream);
  return b200_gemm_workspace_bytes(P(st.in[0]), P(st.in[1]), P(st.out[0]), bias, st.ip[0], st.ip[1],
                                   st.ip[2], st.ip[3], st.ip[4], st.ip[5], st.ip[6], st.ip[7], st.ip[8],
                                   st.ip[9], st.ip[10], st.fp[0], st.dtype, st.dtype2, (int)st.ip[11],
                                   stream);
}
template <typename PtrOf>
static int gemm_step_run(const Step& st, PtrOf P, void* stream, void* ws, size_t ws_bytes) {
  const void* bias = (st.ip[11] == 1 || st.ip[11] == 2) ? P(st.in[2]) : nullptr;
  const void* a_lo = st.args.size() >= 2 && st.args[0].slot >= 0 ? P(st.args[0].slot) : nullptr;
  const void* b_lo = st.args.size() >= 2 && st.args[1].slot >= 0 ? P(st.args[1].slot) : nullptr;
  if (a_lo || b_lo)
    return b200_gemm_planes_ws(P(st.in[0]), a_lo, P(st.in[1]), b_lo, P(st.out[0]), bias, st.ip[0],
                               st.ip[1], st.ip[2], st.ip[3], st.ip[4], st.ip[5], st.ip[6], st.ip[7],
                               st.ip[8], st.ip[9], st.ip[10], st.fp[0], st.dtype, st.dtype2,
                               (int)st.ip[11], stream, ws, ws_bytes);
  return b200_gemm_ws(P(st.in[0]), P(st.in[1]), P(st.out[0]), bias, st.ip[0], st.ip[1], st.ip[2],
                      st.ip[3], st.ip[4], st.ip[5], st.ip[6], st.ip[7], st.ip[8], st.ip[9], st.ip[10],
                      st.fp[0], st.dtype, st.dtype2, (int)st.ip[11], stream, ws, ws_bytes);
}

// Graph replay applies to single-device Executes of plans whose slots fit a
// fixed budget (each slot gets its own buffer, no reuse): B200_GRAPH_MAX_GB
// (default 1), B200_GRAPHS=0 turns it off.
GraphState* graph_state(Exe& e, const std::vector<PJRT_Device*>& devs) {
  if (devs.size() != 1) return nullptr;
  static const bool off = [] {
    const char* v = std::getenv("B200_GRAPHS");
    return v && std::strcmp(v, "0") == 0;
  }();
  if (off) return nullptr;
  const Plan& p = e.plan;
  if (e.graph_ok < 0) {
    int64_t bytes = 0;
    for (auto& sl : p.slots)
      if (sl.kind != Slot::CONST) bytes += sl.bytes;
    static const int64_t limit = [] {
      const char* v = std::getenv("B200_GRAPH_MAX_GB");
      const double gb = v ? std::atof(v) : 1.0;
      return (int64_t)(gb * (double)(1ll << 30));
    }();
    e.graph_ok = (bytes <= limit && p.steps.size() >= 4) ? 1 : 0;
  }
  if (!e.graph_ok) return nullptr;
  auto& g = e.graphs[devs[0]->dev->ordinal];
  if (!g) g = std::make_unique<GraphState>();
  return g->disabled ? nullptr : g.get();
}

template <typename StepFn>
void build_graphs(Exe& e, GraphState& gs, PJRT_Device* pd, StepFn& exec_step,
                  std::shared_ptr<DeviceMem>*& gemm_ws_override) {
  const Plan& p = e.plan;
  Device& dev = *pd->dev;
  dev.activate();
  auto& mod = *e.modules.at(dev.ordinal);
  gs.ptr.assign(1, std::vector<void*>(p.slots.size(), nullptr));
  gs.mem.assign(p.slots.size(), nullptr);
  for (size_t s = 0; s < p.slots.size(); ++s) {
    const Slot& sl = p.slots[s];
    if (sl.kind == Slot::CONST) {
      gs.ptr[0][s] = mod.consts.at(sl.index)->ptr;
    } else if (sl.parent < 0) {
      gs.mem[s] = std::make_shared<DeviceMem>(&dev, (size_t)std::max<int64_t>(sl.bytes, 1));
      gs.ptr[0][s] = gs.mem[s]->ptr;
    }
  }
  for (size_t s = 0; s < p.slots.size(); ++s)  // views into all-reduce buckets
    if (p.slots[s].parent >= 0)
      gs.ptr[0][s] = static_cast<uint8_t*>(gs.ptr[0][p.slots[s].parent]) + p.slots[s].offset;
  int64_t ws = 0;
  auto P = [&](int s) -> void* { return s < 0 ? nullptr : gs.ptr[0][s]; };
  for (const Step& st : p.steps)
    if (st.kind == StepKind::Gemm)
      ws = std::max<int64_t>(ws, gemm_step_ws_bytes(st, P, dev.stream));
  if (ws > 0) gs.gemm_ws = std::make_shared<DeviceMem>(&dev, (size_t)ws);
  gemm_ws_override = &gs.gemm_ws;
  try {
    size_t si = 0;
    while (si < p.steps.size()) {
      if (p.steps[si].kind == StepKind::AllReduce) {
        gs.items.push_back({1, (int)si});
        ++si;
        continue;
      }
      cudaGraph_t graph = nullptr;
      B200_CUDA(cudaStreamBeginCapture(dev.stream, cudaStreamCaptureModeRelaxed));
      try {
        for (; si < p.steps.size() && p.steps[si].kind != StepKind::AllReduce; ++si) exec_step(si, gs.ptr);
      } catch (...) {
        cudaStreamEndCapture(dev.stream, &graph);
        if (graph) cudaGraphDestroy(graph);
        throw;
      }
      B200_CUDA(cudaStreamEndCapture(dev.stream, &graph));
      cudaGraphExec_t exec = nullptr;
      const cudaError_t r = cudaGraphInstantiate(&exec, graph, 0);
      cudaGraphDestroy(graph);
      B200_CUDA(r);
      gs.items.push_back({0, (int)gs.execs.size()});
      gs.execs.push_back(exec);
    }
  } catch (...) {
    // capture did not work for this plan: stay eager
    for (auto g : gs.execs) cudaGraphExecDestroy(g);
    gs.execs.clear();
    gs.items.clear();
    gs.disabled = true;
    cudaGetLastError();
  }
  gemm_ws_override = nullptr;
}

template <typename StepFn>
void run_graphs(Exe& e, GraphState& gs, PJRT_Device* pd, const std::vector<void*>& args,
                StepFn& exec_step, std::shared_ptr<DeviceMem>*& gemm_ws_override) {
  const Plan& p = e.plan;
  Device& dev = *pd->dev;
  dev.activate();
  for (int s : p.param_slots)
    if (p.slots[s].bytes > 0)
      B200_CUDA(cudaMemcpyAsync(gs.ptr[0][s], args[s], (size_t)p.slots[s].bytes,
                                cudaMemcpyDeviceToDevice, dev.stream));
  gemm_ws_override = &gs.gemm_ws;
  for (auto& it : gs.items) {
    if (it.first == 0) B200_CUDA(cudaGraphLaunch(gs.execs[it.second], dev.stream));
    else exec_step((size_t)it.second, gs.ptr);
  }
  gemm_ws_override = nullptr;
}

void execute(PJRT_LoadedExecutable* le, PJRT_LoadedExecutable_Execute_Args* a) {
  fault_point("execute");
  Exe& e = *le->exe;
  PJRT_Client* c = e.client;
  const Plan& p = e.plan;
  if (le->deleted) throw PjrtErr(9, "executable was deleted");
  std::vector<PJRT_Device*> devs;
  if (a->execute_device) {
    if (a->num_devices != 1) throw PjrtErr(3, "execute_device requires num_devices == 1");
    devs.push_back(a->execute_device);
  } else {
    if (a->num_devices != e.addressable.size())
      throw PjrtErr(3, "Execute got " + std::to_string(a->num_devices) + " argument lists for " +
                           std::to_string(e.addressable.size()) + " addressable replicas");
    devs = e.addressable;
  }
  const size_t nd = devs.size();
  if (a->num_args != p.param_slots.size())
    throw PjrtErr(3, "Execute got " + std::to_string(a->num_args) + " arguments, program takes " +
                         std::to_string(p.param_slots.size()));
  std::lock_guard<std::mutex> xl(c->exec_mu);
  // modules + constants per device
  for (auto* pd : devs) {
    if (!pd->dev) throw PjrtErr(3, "device is not addressable from this process");
    std::lock_guard<std::mutex> lk(e.mu);
    auto& slot = e.modules[pd->dev->ordinal];
    if (!slot) {
      auto m = load_module(*pd->dev, e.cubins, p.unit_names, p.kernel_alias);
      for (auto& cd : p.consts) {
        (void)cd;
      }
      for (size_t s = 0; s < p.slots.size(); ++s) {
        const Slot& sl = p.slots[s];
        if (sl.kind != Slot::CONST) continue;
        auto mem = std::make_shared<DeviceMem>(pd->dev, (size_t)sl.bytes);
        const ConstData& cd = p.consts.at(sl.index);
        pd->dev->activate();
        B200_CUDA(cudaMemcpy(mem->ptr, cd.bytes.data(), (size_t)sl.bytes, cudaMemcpyHostToDevice));
        if ((int)m->consts.size() <= sl.index) m->consts.resize(sl.index + 1);
        m->consts[sl.index] = mem;
      }
      slot = std::move(m);
    }
  }
  // bind slots
  std::vector<std::vector<void*>> ptr(nd, std::vector<void*>(p.slots.size(), nullptr));
  std::vector<std::vector<std::shared_ptr<DeviceMem>>> owned(nd, std::vector<std::shared_ptr<DeviceMem>>(p.slots.size()));
  for (size_t d = 0; d < nd; ++d) {
    for (size_t i = 0; i < a->num_args; ++i) {
      PJRT_Buffer* b = a->argument_lists[d][i];
      if (!b || b->deleted || !b->mem) throw PjrtErr(3, "argument " + std::to_string(i) + " is deleted or null");
      const TensorType& want = p.param_types[i];
      if (b->type != want)
        throw PjrtErr(3, "argument " + std::to_string(i) + " has type " + b->type.str() +
                             ", program expects " + want.str());
      if (b->device != devs[d]) throw PjrtErr(3, "argument " + std::to_string(i) + " lives on another device");
      ptr[d][p.param_slots[i]] = b->mem->ptr;
      owned[d][p.param_slots[i]] = b->mem;
    }
    auto& mod = *e.modules.at(devs[d]->dev->ordinal);
    for (size_t s = 0; s < p.slots.size(); ++s)
      if (p.slots[s].kind == Slot::CONST) ptr[d][s] = mod.consts.at(p.slots[s].index)->ptr;
  }
  static const bool timing = env_flag("B200_TIMING");
  cudaEvent_t t_start = nullptr, t_stop = nullptr;
  if (timing) {
    devs[0]->dev->activate();
    B200_CUDA(cudaEventCreate(&t_start));
    B200_CUDA(cudaEventCreate(&t_stop));
    B200_CUDA(cudaEventRecord(t_start, devs[0]->dev->stream));
  }
  std::function<void(size_t, int)> ensure = [&](size_t d, int s) {
    if (s < 0 || ptr[d][s]) return;
    const Slot& sl = p.slots[s];
    if (sl.parent >= 0) {  // a view into its parent (an all-reduce bucket piece)
      ensure(d, sl.parent);
      owned[d][s] = owned[d][sl.parent];
      ptr[d][s] = static_cast<uint8_t*>(ptr[d][sl.parent]) + sl.offset;
      return;
    }
    owned[d][s] = std::make_shared<DeviceMem>(devs[d]->dev, (size_t)std::max<int64_t>(sl.bytes, 1));
    ptr[d][s] = owned[d][s]->ptr;
  };
  std::shared_ptr<DeviceMem>* gemm_ws_override = nullptr;
  // one step of the plan on every device, with slot pointers `ptr`
  // collectives of this Execute: followed by events the client's NCCL
  // watchdog polls (its verdict reaches the Execute's events through cst)
  std::shared_ptr<CollectiveStatus> cst;
  auto watch_collectives = [&](const std::vector<Device*>& dd, const std::vector<cudaStream_t>& ss,
                               NcclComms& comm, const char* what) {
    if (!cst) cst = std::make_shared<CollectiveStatus>();
    if (!c->watchdog) c->watchdog = std::make_unique<NcclWatchdog>();
    for (size_t i = 0; i < dd.size(); ++i)
      c->watchdog->watch(*dd[i], ss[i], &comm, cst, std::string(what) + " of " + e.name);
  };
  // Collectives in flight on the communication streams (eager execution with
  // B200_OVERLAP_COLLECTIVES): the slots they read or write, the event each
  // device's communication stream records when it is done, and the temps whose
  // release waits for it.  A later step touching one of those slots first makes
  // its compute stream wait for the event; so does the end of the Execute.
  struct InFlight {
    std::set<int> slots;
    std::vector<cudaEvent_t> done;
    std::vector<int> release;
  };
  std::vector<InFlight> inflight;
  bool async_coll = false;
  auto root_of = [&](int sl) { return sl >= 0 && p.slots[sl].parent >= 0 ? p.slots[sl].parent : sl; };
  auto retire = [&](InFlight& f) {
    for (size_t d = 0; d < nd; ++d) {
      Device& dev = *devs[d]->dev;
      dev.activate();
      B200_CUDA(cudaStreamWaitEvent(dev.stream, f.done[d], 0));
      cudaEventDestroy(f.done[d]);
      for (int sl : f.release) {
        owned[d][sl].reset();
        ptr[d][sl] = nullptr;
      }
    }
  };
  auto wait_for_slots = [&](const Step& st) {
    if (inflight.empty()) return;
    std::set<int> touched;
    for (auto* v : {&st.in, &st.out})
      for (int sl : *v)
        if (sl >= 0) touched.insert(root_of(sl));
    for (auto& a : st.args)
      if (a.slot >= 0) touched.insert(root_of(a.slot));
    for (size_t i = 0; i < inflight.size();) {
      bool hit = false;
      for (int sl : touched) hit = hit || inflight[i].slots.count(sl);
      if (!hit) {
        ++i;
        continue;
      }
      retire(inflight[i]);
      inflight.erase(inflight.begin() + (long)i);
    }
  };
  // Order a collective on each device's communication stream after the
  // compute stream's work so far; returns those streams.
  auto comm_streams = [&](const std::vector<Device*>& dd) {
    std::vector<cudaStream_t> ss;
    for (Device* d : dd) {
      d->activate();
      if (!d->comm_stream) B200_CUDA(cudaStreamCreateWithFlags(&d->comm_stream, cudaStreamNonBlocking));
      cudaEvent_t ev;
      B200_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
      B200_CUDA(cudaEventRecord(ev, d->stream));
      B200_CUDA(cudaStreamWaitEvent(d->comm_stream, ev, 0));
      cudaEventDestroy(ev);
      ss.push_back(d->comm_stream);
    }
    return ss;
  };
  auto track = [&](const Step& st, const std::vector<Device*>& dd, const std::vector<cudaStream_t>& ss,
                   size_t si) {
    InFlight f;
    for (auto* v : {&st.in, &st.out})
      for (int sl : *v)
        if (sl >= 0) f.slots.insert(root_of(sl));
    for (size_t d = 0; d < dd.size(); ++d) {
      dd[d]->activate();
      cudaEvent_t ev;
      B200_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
      B200_CUDA(cudaEventRecord(ev, ss[d]));
      f.done.push_back(ev);
    }
    for (auto* v : {&st.in, &st.out})
      for (int sl : *v)
        if (sl >= 0 && p.slots[sl].kind == Slot::TEMP && p.temp_last[sl] == (int)si) f.release.push_back(sl);
    inflight.push_back(std::move(f));
  };
  auto exec_step = [&](size_t si, std::vector<std::vector<void*>>& ptr) {
    const Step& st = p.steps[si];
    if (st.kind == StepKind::AllReduce && !st.args.empty()) {
      // bucketed: copy the pieces into one flat buffer, one collective, copy back
      const size_t es = (size_t)dtype_size((DType)st.dtype);
      const int bucket = st.out.back();
      std::vector<Device*> dd;
      std::vector<const void*> in;
      std::vector<void*> out;
      for (size_t d = 0; d < nd; ++d) {
        Device& dev = *devs[d]->dev;
        dev.activate();
        uint8_t* bk = static_cast<uint8_t*>(ptr[d][bucket]);
        for (size_t k = 0; k < st.args.size(); k += 2) {
          if (st.args[k].f == 1.f) continue;  // computed in the bucket already
          if (e.num_replicas == 1) {
            B200_CUDA(cudaMemcpyAsync(ptr[d][st.args[k + 1].slot], ptr[d][st.args[k].slot],
                                      (size_t)st.args[k + 1].i * es, cudaMemcpyDeviceToDevice, dev.stream));
          } else {
            B200_CUDA(cudaMemcpyAsync(bk + (size_t)st.args[k].i * es, ptr[d][st.args[k].slot],
                                      (size_t)st.args[k + 1].i * es, cudaMemcpyDeviceToDevice, dev.stream));
          }
        }
        dd.push_back(devs[d]->dev);
        in.push_back(bk);
        out.push_back(bk);
      }
      if (e.num_replicas != 1) {
        NcclComms& comm = comms_for(c, e);
        std::vector<cudaStream_t> ss;
        if (async_coll) ss = comm_streams(dd);
        else for (Device* d : dd) ss.push_back(d->stream);
        nccl_all_reduce(dd, comm, in, out, st.ip[0], (DType)st.dtype, (int)st.ip[1], ss);
        watch_collectives(dd, ss, comm, "all_reduce bucket");
        for (size_t d = 0; d < nd; ++d) {
          Device& dev = *devs[d]->dev;
          dev.activate();
          const uint8_t* bk = static_cast<const uint8_t*>(ptr[d][bucket]);
          for (size_t k = 0; k < st.args.size(); k += 2)
            if (st.args[k].f != 1.f)  // (aliased pieces are read in place)
              B200_CUDA(cudaMemcpyAsync(ptr[d][st.args[k + 1].slot], bk + (size_t)st.args[k].i * es,
                                        (size_t)st.args[k + 1].i * es, cudaMemcpyDeviceToDevice,
                                        ss[d]));
        }
        if (async_coll) track(st, dd, ss, si);
      }
    } else if (st.kind == StepKind::AllReduce) {
      std::vector<Device*> dd;
      std::vector<const void*> in;
      std::vector<void*> out;
      for (size_t d = 0; d < nd; ++d) {
        dd.push_back(devs[d]->dev);
        in.push_back(ptr[d][st.in[0]]);
        out.push_back(ptr[d][st.out[0]]);
      }
      if (e.num_replicas == 1) {
        for (size_t d = 0; d < nd; ++d) {
          dd[d]->activate();
          B200_CUDA(cudaMemcpyAsync(out[d], in[d], (size_t)p.slots[st.out[0]].bytes,
                                    cudaMemcpyDeviceToDevice, dd[d]->stream));
        }
      } else {
        NcclComms& comm = comms_for(c, e);
        std::vector<cudaStream_t> ss;
        if (async_coll) ss = comm_streams(dd);
        else for (Device* d : dd) ss.push_back(d->stream);
        nccl_all_reduce(dd, comm, in, out, st.ip[0], (DType)st.dtype, (int)st.ip[1], ss);
        watch_collectives(dd, ss, comm, "all_reduce");
        if (async_coll) track(st, dd, ss, si);
      }
    } else {
      for (size_t d = 0; d < nd; ++d) {
        Device& dev = *devs[d]->dev;
        dev.activate();
        void* const* P = ptr[d].data();
        auto slotp = [&](int s) -> void* { return s < 0 ? nullptr : P[s]; };
        switch (st.kind) {
          case StepKind::Kernel: {
            auto& mod = *e.modules.at(dev.ordinal);
            std::vector<void*> vals;
            vals.reserve(st.args.size());
            for (auto& arg : st.args) vals.push_back(slotp(arg.slot));
            std::vector<void*> args;
            if (st.table) args.push_back(vals.data());  // one parameter: the pointer table
            else
              for (auto& v : vals) args.push_back(&v);
            launch(dev, mod.fns.at(st.name), st.grid, st.block, st.smem, args);
            break;
          }
          case StepKind::LayerNorm:
            kcheck(b200_ln_residual_fwd(slotp(st.in[0]), slotp(st.in[1]), slotp(st.in[2]),
                                        slotp(st.in[3]), slotp(st.out[0]), slotp(st.out[1]), nullptr,
                                        nullptr, st.ip[0], st.ip[1], st.fp[0], st.dtype,
                                        (int)st.ip[2], dev.stream),
                   "layer_norm");
            break;
          case StepKind::Sdpa:
            if (st.out.size() > 1)
              kcheck(b200_sdpa_fwd_lse(slotp(st.in[0]), slotp(st.in[1]), slotp(st.in[2]),
                                       slotp(st.out[0]), (float*)slotp(st.out[1]), st.ip[0], st.ip[1],
                                       st.ip[2], st.ip[3], st.ip[4], st.ip.data() + 5, st.fp[0],
                                       (int)st.ip[17], st.dtype, dev.stream),
                     "sdpa");
            else
              kcheck(b200_sdpa_fwd_strided(slotp(st.in[0]), slotp(st.in[1]), slotp(st.in[2]),
                                           slotp(st.out[0]), st.ip[0], st.ip[1], st.ip[2], st.ip[3],
                                           st.ip[4], st.ip.data() + 5, st.fp[0], (int)st.ip[17],
                                           st.dtype, dev.stream),
                     "sdpa");
            break;
          case StepKind::SdpaBwd:
            kcheck(b200_sdpa_bwd(slotp(st.in[0]), slotp(st.in[1]), slotp(st.in[2]), slotp(st.in[3]),
                                 slotp(st.in[4]), (const float*)slotp(st.in[5]), slotp(st.out[0]),
                                 slotp(st.out[1]), slotp(st.out[2]), st.ip[0], st.ip[1], st.ip[2],
                                 st.ip[3], st.ip.data() + 4, st.fp[0], (int)st.ip[28], st.dtype,
                                 dev.stream),
                   "sdpa_bwd");
            break;
          case StepKind::Gemm: {
            // split-K partials / bf16 planes come from the caching allocator
            // (released after the launch: stream order protects the reuse)
            auto SP = [&](int s) -> void* { return s < 0 ? nullptr : slotp(s); };
            const int64_t wsb = gemm_step_ws_bytes(st, SP, dev.stream);
            std::shared_ptr<DeviceMem> ws;
            if (wsb > 0) {
              // graph capture / replay: the graph's fixed workspace
              if (gemm_ws_override && *gemm_ws_override) ws = *gemm_ws_override;
              else ws = std::make_shared<DeviceMem>(&dev, (size_t)wsb);
            }
            kcheck(gemm_step_run(st, SP, dev.stream, ws ? ws->ptr : nullptr,
                                 wsb > 0 ? (size_t)wsb : 0),
                   "gemm");
            break;
          }
          case StepKind::Copy:
            B200_CUDA(cudaMemcpyAsync(slotp(st.out[0]), slotp(st.in[0]),
                                      (size_t)p.slots[st.out[0]].bytes, cudaMemcpyDeviceToDevice,
                                      dev.stream));
            break;
          default:
            break;
        }
      }
    }
  };
  GraphState* gs = graph_state(e, devs);
  if (gs && gs->execs.empty() && gs->eager_runs >= 1) build_graphs(e, *gs, devs[0], exec_step, gemm_ws_override);
  if (gs && !gs->execs.empty()) {
    run_graphs(e, *gs, devs[0], ptr[0], exec_step, gemm_ws_override);
    for (size_t o = 0; o < p.output_slots.size(); ++o) {
      const int sl = p.output_slots[o];
      owned[0][sl] = std::make_shared<DeviceMem>(devs[0]->dev, (size_t)std::max<int64_t>(p.slots[sl].bytes, 1));
      B200_CUDA(cudaMemcpyAsync(owned[0][sl]->ptr, gs->ptr[0][sl], (size_t)p.slots[sl].bytes,
                                cudaMemcpyDeviceToDevice, devs[0]->dev->stream));
    }
  } else {
  if (gs) gs->eager_runs++;
  async_coll = overlap_collectives() && e.num_replicas > 1;
  for (size_t si = 0; si < p.steps.size(); ++si) {
    const Step& st = p.steps[si];
    for (size_t d = 0; d < nd; ++d) {
      for (int s : st.out) ensure(d, s);
      for (int s : st.in) ensure(d, s);
    }
    wait_for_slots(st);
    exec_step(si, ptr);
    if (env_flag("B200_SYNC_STEPS")) {
      for (size_t d = 0; d < nd; ++d) {
        devs[d]->dev->activate();
        cudaError_t r = cudaStreamSynchronize(devs[d]->dev->stream);
        if (r != cudaSuccess) throw PjrtErr(13, "step " + st.name + " failed: " + cudaGetErrorString(r));
      }
    }
    // release temps whose last use was this step (stream order makes reuse
    // safe; a collective in flight releases its own when it is waited for)
    if (!(async_coll && st.kind == StepKind::AllReduce && e.num_replicas != 1))
      for (size_t d = 0; d < nd; ++d)
        for (auto* v : {&st.in, &st.out})
          for (int s : *v)
            if (s >= 0 && p.slots[s].kind == Slot::TEMP && p.temp_last[s] == (int)si) {
              owned[d][s].reset();
              ptr[d][s] = nullptr;
            }
  }
  for (auto& f : inflight) retire(f);  // outputs are complete only after every collective
  inflight.clear();
  }
  if (timing) {
    devs[0]->dev->activate();
    B200_CUDA(cudaEventRecord(t_stop, devs[0]->dev->stream));
    std::lock_guard<std::mutex> lk(e.timing_mu);
    e.timings.emplace_back(t_start, t_stop);
  }
  for (size_t d = 0; d < nd; ++d) {
    auto ev = record_event(*devs[d]->dev);
    ev->status = cst;
    if (a->device_complete_events) a->device_complete_events[d] = handle_of(ev);
    for (size_t o = 0; o < p.output_slots.size(); ++o) {
      int s = p.output_slots[o];
      auto* b = new PJRT_Buffer;
      b->client = c;
      b->device = devs[d];
      b->type = p.slots[s].type;
      b->dims = b->type.dims;
      b->mem = owned[d][s];
      if (!b->mem) {  // zero-size output never touched by a step
        b->mem = std::make_shared<DeviceMem>(devs[d]->dev, 1);
      }
      b->ready = ev;
      a->output_lists[d][o] = b;
    }
  }
}

// ------------------------------------------------------ client creation --
std::string device_kind() { return "NVIDIA B200"; }

// Clients still alive when the process exits (a caller that never destroyed
// its client): their collective watchdogs are stopped and communicators
// released by an exit hook, before the CUDA runtime's own teardown, so no
// helper thread or NCCL resource outlives the runtime under it.
std::mutex g_clients_mu;
std::set<PJRT_Client*> g_clients;
void teardown_live_clients() {
  std::lock_guard<std::mutex> lk(g_clients_mu);
  for (PJRT_Client* c : g_clients) {
    c->watchdog.reset();
    c->comms.clear();
  }
}

PJRT_Client* create_client(const PJRT_Client_Create_Args* args) {
  auto c = std::make_unique<PJRT_Client>();
  std::vector<int> visible;
  int64_t node_id = 0, num_nodes = 1;
  for (size_t i = 0; i < args->num_options; ++i) {
    const PJRT_NamedValue& v = args->create_options[i];
    std::string name(v.name, v.name_size);
    if (name == "visible_devices" && v.type == PJRT_NamedValue_kInt64List)
      for (size_t k = 0; k < v.value_size; ++k) visible.push_back((int)v.int64_array_value[k]);
    if (name == "node_id" && v.type == PJRT_NamedValue_kInt64) node_id = v.int64_value;
    if (name == "num_nodes" && v.type == PJRT_NamedValue_kInt64) num_nodes = v.int64_value;
  }
  int count = 0;
  cudaError_t r = cudaGetDeviceCount(&count);
  if (r != cudaSuccess || count == 0) {
    cudaGetLastError();
    throw PjrtErr(14, std::string("no CUDA device available: ") + cudaGetErrorString(r));
  }
  if (visible.empty())
    for (int i = 0; i < count; ++i) visible.push_back(i);
  c->process_index = (int)node_id;
  c->num_nodes = (int)num_nodes;
  c->kv_get = args->kv_get_callback;
  c->kv_get_arg = args->kv_get_user_arg;
  c->kv_put = args->kv_put_callback;
  c->kv_put_arg = args->kv_put_user_arg;
  int rt = 0, drv = 0;
  cudaRuntimeGetVersion(&rt);
  cudaDriverGetVersion(&drv);
  c->version = "b200-pjrt 0.1.0; cuda runtime " + std::to_string(rt) + ", driver " + std::to_string(drv);
  const int local_n = (int)visible.size();
  for (int li = 0; li < local_n; ++li) {
    auto d = std::make_unique<Device>();
    d->ordinal = visible[li];
    B200_CUDA(cudaSetDevice(d->ordinal));
    B200_CUDA(cudaFree(nullptr));
    B200_CUDA(cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking));
    cudaDeviceProp prop;
    B200_CUDA(cudaGetDeviceProperties(&prop, d->ordinal));
    d->name = prop.name;
    d->sms = prop.multiProcessorCount;
    d->total_mem = (int64_t)prop.totalGlobalMem;
    d->alloc = std::make_unique<Allocator>(d->ordinal);
    c->local.push_back(std::move(d));
  }
  // global devices: node-major, local_n per node (homogeneous nodes assumed)
  for (int64_t nidx = 0; nidx < num_nodes; ++nidx)
    for (int li = 0; li < local_n; ++li) {
      auto pd = std::make_unique<PJRT_Device>();
      const int gid = (int)(nidx * local_n + li);
      pd->desc.id = gid;
      pd->desc.process_index = (int)nidx;
      pd->desc.kind = device_kind();
      pd->desc.debug = "b200:" + std::to_string(gid);
      pd->desc.tostr = "B200Device(id=" + std::to_string(gid) + ", process=" + std::to_string(nidx) + ")";
      pd->desc.cc = "10.0";
      if (nidx == node_id) {
        pd->dev = c->local[li].get();
        pd->local_hardware_id = pd->dev->ordinal;
        pd->desc.cores = pd->dev->sms;
      }
      PJRT_NamedValue cc{};
      cc.struct_size = sizeof(cc);
      cc.name = "compute_capability";
      cc.name_size = std::strlen(cc.name);
      cc.type = PJRT_NamedValue_kString;
      cc.string_value = pd->desc.cc.c_str();
      cc.value_size = pd->desc.cc.size();
      PJRT_NamedValue cores{};
      cores.struct_size = sizeof(cores);
      cores.name = "core_count";
      cores.name_size = std::strlen(cores.name);
      cores.type = PJRT_NamedValue_kInt64;
      cores.int64_value = pd->desc.cores;
      cores.value_size = 1;
      pd->desc.attrs = {cc, cores};
      auto mem = std::make_unique<PJRT_Memory>();
      mem->id = gid;
      mem->device = pd.get();
      mem->debug = "b200_hbm:" + std::to_string(gid);
      mem->tostr = "MEMORY_SPACE(device, id=" + std::to_string(gid) + ")";
      pd->memory = mem.get();
      if (pd->dev) {
        c->addressable.push_back(pd.get());
        c->memory_ptrs.push_back(mem.get());
      }
      c->device_ptrs.push_back(pd.get());
      c->memories.push_back(std::move(mem));
      c->devices.push_back(std::move(pd));
    }
  for (auto* d : c->device_ptrs) c->topo.descs.push_back(&d->desc);
  c->topo.version = c->version;
  {
    std::lock_guard<std::mutex> lk(g_clients_mu);
    static const bool hooked = (std::atexit(teardown_live_clients), true);
    (void)hooked;
    g_clients.insert(c.get());
  }
  return c.release();
}

// --------------------------------------------------------------- buffers --
PJRT_Buffer* buffer_from_host(PJRT_Client* c, const PJRT_Client_BufferFromHostBuffer_Args* a,
                              PJRT_Event** done) {
  PJRT_Device* pd = a->device;
  if (!pd && a->memory) pd = a->memory->device;
  if (!pd) pd = c->addressable.at(0);
  if (!pd->dev) throw PjrtErr(3, "BufferFromHostBuffer: device is not addressable");
  TensorType t;
  t.dtype = to_dtype(a->type);
  t.dims.assign(a->dims, a->dims + a->num_dims);
  const int es = dtype_size(t.dtype);
  if (a->byte_strides && a->num_byte_strides) {
    int64_t expect = es;
    for (int i = (int)a->num_dims - 1; i >= 0; --i) {
      if (t.dims[i] != 1 && a->byte_strides[i] != expect)
        throw PjrtErr(12, "BufferFromHostBuffer: only dense row-major host layouts are supported");
      expect *= t.dims[i];
    }
  }
  auto b = std::make_unique<PJRT_Buffer>();
  b->client = c;
  b->device = pd;
  b->type = t;
  b->dims = t.dims;
  Device& d = *pd->dev;
  std::lock_guard<std::recursive_mutex> lk(d.mu);
  b->mem = std::make_shared<DeviceMem>(&d, (size_t)std::max<int64_t>(t.bytes(), 1));
  d.activate();
  if (t.bytes() > 0)
    B200_CUDA(cudaMemcpyAsync(b->mem->ptr, a->data, (size_t)t.bytes(), cudaMemcpyHostToDevice, d.stream));
  b->ready = record_event(d);
  cudaPointerAttributes attr{};
  const bool pinned = cudaPointerGetAttributes(&attr, a->data) == cudaSuccess &&
                      (attr.type == cudaMemoryTypeHost);
  cudaGetLastError();
  if (pinned && a->host_buffer_semantics == PJRT_HostBufferSemantics_kImmutableOnlyDuringCall) {
    B200_CUDA(cudaEventSynchronize(b->ready->ev));
    *done = ready_event();
  } else if (pinned) {
    *done = handle_of(b->ready);
  } else {
    *done = ready_event();  // pageable source: cudaMemcpyAsync staged it before returning
  }
  return b.release();
}

}  // namespace

// =================================================================== API ===
extern "C" {

static PJRT_Error* Error_Destroy(PJRT_Error_Destroy_Args* a) {
  delete a->error;
  return nullptr;
}
static PJRT_Error* Error_Message(PJRT_Error_Message_Args* a) {
  a->message = a->error->msg.c_str();
  a->message_size = a->error->msg.size();
  return nullptr;
}
static PJRT_Error* Error_GetCode(PJRT_Error_GetCode_Args* a) {
  a->code = a->error->code;
  return nullptr;
}
static PJRT_Error* Plugin_Initialize(PJRT_Plugin_Initialize_Args*) { return nullptr; }

static int64_t kStablehloCur[3] = {1, 9, 0};
static int64_t kStablehloMin[3] = {0, 9, 0};
static PJRT_NamedValue kPluginAttrs[3];
static PJRT_Error* Plugin_Attributes(PJRT_Plugin_Attributes_Args* a) {
  static bool init = [] {
    auto set_list = [](PJRT_NamedValue& v, const char* n, int64_t* arr) {
      v = PJRT_NamedValue{};
      v.struct_size = sizeof(v);
      v.name = n;
      v.name_size = std::strlen(n);
      v.type = PJRT_NamedValue_kInt64List;
      v.int64_array_value = arr;
      v.value_size = 3;
    };
    set_list(kPluginAttrs[0], "stablehlo_current_version", kStablehloCur);
    set_list(kPluginAttrs[1], "stablehlo_minimum_version", kStablehloMin);
    kPluginAttrs[2] = PJRT_NamedValue{};
    kPluginAttrs[2].struct_size = sizeof(PJRT_NamedValue);
    kPluginAttrs[2].name = "xla_version";
    kPluginAttrs[2].name_size = 11;
    kPluginAttrs[2].type = PJRT_NamedValue_kInt64;
    kPluginAttrs[2].int64_value = 2;
    kPluginAttrs[2].value_size = 1;
    return true;
  }();
  (void)init;
  a->attributes = kPluginAttrs;
  a->num_attributes = 3;
  return nullptr;
}

// ---- events
static PJRT_Error* Event_Destroy(PJRT_Event_Destroy_Args* a) {
  delete a->event;
  return nullptr;
}
static PJRT_Error* Event_IsReady(PJRT_Event_IsReady_Args* a) {
  PJRT_Error_Code code = PJRT_Error_Code_OK;
  std::string msg;
  a->is_ready = event_ready(a->event, &code, &msg);
  return nullptr;
}
static PJRT_Error* Event_Error(PJRT_Event_Error_Args* a) {
  PJRT_Error_Code code = PJRT_Error_Code_OK;
  std::string msg;
  event_wait(a->event, &code, &msg);
  return code == PJRT_Error_Code_OK ? nullptr : make_err(code, msg);
}
static PJRT_Error* Event_Await(PJRT_Event_Await_Args* a) {
  PJRT_Error_Code code = PJRT_Error_Code_OK;
  std::string msg;
  event_wait(a->event, &code, &msg);
  return code == PJRT_Error_Code_OK ? nullptr : make_err(code, msg);
}
static PJRT_Error* Event_OnReady(PJRT_Event_OnReady_Args* a) {
  PJRT_Event* ev = a->event;
  auto cb = a->callback;
  void* ua = a->user_arg;
  PJRT_Error_Code code = PJRT_Error_Code_OK;
  std::string msg;
  if (event_ready(ev, &code, &msg)) {
    cb(code == PJRT_Error_Code_OK ? nullptr : make_err(code, msg), ua);
    return nullptr;
  }
  // wait on a helper thread; the event must outlive the callback (PJRT contract)
  std::thread([ev, cb, ua] {
    PJRT_Error_Code c2 = PJRT_Error_Code_OK;
    std::string m2;
    event_wait(ev, &c2, &m2);
    cb(c2 == PJRT_Error_Code_OK ? nullptr : make_err(c2, m2), ua);
  }).detach();
  return nullptr;
}
static PJRT_Error* Event_Create(PJRT_Event_Create_Args* a) {
  auto* e = new PJRT_Event;
  e->host_set = true;
  a->event = e;
  return nullptr;
}
static PJRT_Error* Event_Set(PJRT_Event_Set_Args* a) {
  PJRT_Event* e = a->event;
  {
    std::lock_guard<std::mutex> lk(e->mu);
    e->host_done = true;
    e->code = a->error_code;
    if (a->error_message) e->msg.assign(a->error_message, a->error_message_size);
  }
  e->cv.notify_all();
  return nullptr;
}

// ---- client
static PJRT_Error* Client_Create(PJRT_Client_Create_Args* a) {
  PJRT_TRY
  a->client = create_client(a);
  PJRT_CATCH
}
static PJRT_Error* Client_Destroy(PJRT_Client_Destroy_Args* a) {
  PJRT_TRY
  PJRT_Client* c = a->client;
  for (auto& d : c->local) {
    d->activate();
    cudaStreamSynchronize(d->stream);  // the watchdog still guards collectives here
  }
  {
    std::lock_guard<std::mutex> lk(g_clients_mu);
    g_clients.erase(c);
  }
  c->watchdog.reset();
  c->comms.clear();
  for (auto& d : c->local) {
    d->activate();
    d->alloc->release_cache();
    cudaStreamDestroy(d->stream);
  }
  delete c;
  PJRT_CATCH
}
static PJRT_Error* Client_PlatformName(PJRT_Client_PlatformName_Args* a) {
  static const char kName[] = "b200";
  a->platform_name = kName;
  a->platform_name_size = 4;
  return nullptr;
}
static PJRT_Error* Client_ProcessIndex(PJRT_Client_ProcessIndex_Args* a) {
  a->process_index = a->client->process_index;
  return nullptr;
}
static PJRT_Error* Client_PlatformVersion(PJRT_Client_PlatformVersion_Args* a) {
  a->platform_version = a->client->version.c_str();
  a->platform_version_size = a->client->version.size();
  return nullptr;
}
static PJRT_Error* Client_Devices(PJRT_Client_Devices_Args* a) {
  a->devices = a->client->device_ptrs.data();
  a->num_devices = a->client->device_ptrs.size();
  return nullptr;
}
static PJRT_Error* Client_AddressableDevices(PJRT_Client_AddressableDevices_Args* a) {
  a->addressable_devices = a->client->addressable.data();
  a->num_addressable_devices = a->client->addressable.size();
  return nullptr;
}
static PJRT_Error* Client_LookupDevice(PJRT_Client_LookupDevice_Args* a) {
  for (auto* d : a->client->device_ptrs)
    if (d->desc.id == a->id) { a->device = d; return nullptr; }
  return make_err(5, "no device with id " + std::to_string(a->id));
}
static PJRT_Error* Client_LookupAddressableDevice(PJRT_Client_LookupAddressableDevice_Args* a) {
  for (auto* d : a->client->addressable)
    if (d->local_hardware_id == a->local_hardware_id) { a->addressable_device = d; return nullptr; }
  return make_err(5, "no addressable device with local id " + std::to_string(a->local_hardware_id));
}
static PJRT_Error* Client_AddressableMemories(PJRT_Client_AddressableMemories_Args* a) {
  a->addressable_memories = a->client->memory_ptrs.data();
  a->num_addressable_memories = a->client->memory_ptrs.size();
  return nullptr;
}
static PJRT_Error* Client_Compile(PJRT_Client_Compile_Args* a) {
  PJRT_TRY
  std::string fmt(a->program->format, a->program->format_size);
  if (fmt != "mlir") throw PjrtErr(3, "program format '" + fmt + "' is not supported (want mlir)");
  std::string code(a->program->code, a->program->code_size);
  std::string opts(a->compile_options ? a->compile_options : "", a->compile_options_size);
  auto* le = new PJRT_LoadedExecutable;
  le->exe = compile(a->client, code, opts);
  a->executable = le;
  PJRT_CATCH
}
static PJRT_Error* Client_DefaultDeviceAssignment(PJRT_Client_DefaultDeviceAssignment_Args* a) {
  const int64_t need = (int64_t)a->num_replicas * a->num_partitions;
  if ((int64_t)a->client->device_ptrs.size() < need)
    return make_err(3, "not enough devices for " + std::to_string(need) + " replicas x partitions");
  if ((int64_t)a->default_assignment_size < need) return make_err(3, "assignment buffer too small");
  for (int64_t i = 0; i < need; ++i) a->default_assignment[i] = a->client->device_ptrs[i]->desc.id;
  return nullptr;
}
static PJRT_Error* Client_BufferFromHostBuffer(PJRT_Client_BufferFromHostBuffer_Args* a) {
  PJRT_TRY
  PJRT_Event* done = nullptr;
  a->buffer = buffer_from_host(a->client, a, &done);
  a->done_with_host_buffer = done;
  PJRT_CATCH
}
static PJRT_Error* Client_CreateViewOfDeviceBuffer(PJRT_Client_CreateViewOfDeviceBuffer_Args* a) {
  PJRT_TRY
  PJRT_Device* pd = a->device ? a->device : (a->memory ? a->memory->device : nullptr);
  if (!pd || !pd->dev) throw PjrtErr(3, "CreateViewOfDeviceBuffer: device required");
  auto* b = new PJRT_Buffer;
  b->client = a->client;
  b->device = pd;
  b->type.dtype = to_dtype(a->element_type);
  b->type.dims.assign(a->dims, a->dims + a->num_dims);
  b->dims = b->type.dims;
  // a view does not own the memory; the caller's callback runs when it is released
  auto mem = std::make_shared<DeviceMem>(pd->dev, a->device_buffer_ptr, (size_t)b->type.bytes());
  auto cb = a->on_delete_callback;
  void* arg = a->on_delete_callback_arg;
  if (cb) mem->on_release = [cb, arg](void* p) { cb(p, arg); };
  b->mem = mem;
  b->ready = nullptr;
  a->buffer = b;
  PJRT_CATCH
}
static PJRT_Error* Client_TopologyDescription(PJRT_Client_TopologyDescription_Args* a) {
  a->topology = &a->client->topo;
  return nullptr;
}

// ---- device descriptions / devices / memories
static PJRT_Error* DeviceDescription_Id(PJRT_DeviceDescription_Id_Args* a) {
  a->id = a->device_description->id;
  return nullptr;
}
static PJRT_Error* DeviceDescription_ProcessIndex(PJRT_DeviceDescription_ProcessIndex_Args* a) {
  a->process_index = a->device_description->process_index;
  return nullptr;
}
static PJRT_Error* DeviceDescription_Attributes(PJRT_DeviceDescription_Attributes_Args* a) {
  a->attributes = a->device_description->attrs.data();
  a->num_attributes = a->device_description->attrs.size();
  return nullptr;
}
static PJRT_Error* DeviceDescription_Kind(PJRT_DeviceDescription_Kind_Args* a) {
  a->device_kind = a->device_description->kind.c_str();
  a->device_kind_size = a->device_description->kind.size();
  return nullptr;
}
static PJRT_Error* DeviceDescription_DebugString(PJRT_DeviceDescription_DebugString_Args* a) {
  a->debug_string = a->device_description->debug.c_str();
  a->debug_string_size = a->device_description->debug.size();
  return nullptr;
}
static PJRT_Error* DeviceDescription_ToString(PJRT_DeviceDescription_ToString_Args* a) {
  a->to_string = a->device_description->tostr.c_str();
  a->to_string_size = a->device_description->tostr.size();
  return nullptr;
}
static PJRT_Error* Device_GetDescription(PJRT_Device_GetDescription_Args* a) {
  a->device_description = &a->device->desc;
  return nullptr;
}
static PJRT_Error* Device_IsAddressable(PJRT_Device_IsAddressable_Args* a) {
  a->is_addressable = a->device->dev != nullptr;
  return nullptr;
}
static PJRT_Error* Device_LocalHardwareId(PJRT_Device_LocalHardwareId_Args* a) {
  a->local_hardware_id = a->device->local_hardware_id;
  return nullptr;
}
static PJRT_Error* Device_AddressableMemories(PJRT_Device_AddressableMemories_Args* a) {
  a->memories = &a->device->memory;
  a->num_memories = a->device->dev ? 1 : 0;
  return nullptr;
}
static PJRT_Error* Device_DefaultMemory(PJRT_Device_DefaultMemory_Args* a) {
  a->memory = a->device->memory;
  return nullptr;
}
static PJRT_Error* Device_MemoryStats(PJRT_Device_MemoryStats_Args* a) {
  if (!a->device->dev) return make_err(3, "device is not addressable");
  Allocator& al = *a->device->dev->alloc;
  a->bytes_in_use = al.in_use();
  a->peak_bytes_in_use = al.peak();
  a->peak_bytes_in_use_is_set = true;
  a->num_allocs = al.num_allocs();
  a->num_allocs_is_set = true;
  a->bytes_reserved = al.reserved();
  a->bytes_reserved_is_set = true;
  a->bytes_limit = a->device->dev->total_mem;
  a->bytes_limit_is_set = true;
  return nullptr;
}
static PJRT_Error* Memory_Id(PJRT_Memory_Id_Args* a) {
  a->id = a->memory->id;
  return nullptr;
}
static PJRT_Error* Memory_Kind(PJRT_Memory_Kind_Args* a) {
  a->kind = a->memory->kind.c_str();
  a->kind_size = a->memory->kind.size();
  return nullptr;
}
static PJRT_Error* Memory_Kind_Id(PJRT_Memory_Kind_Id_Args* a) {
  a->kind_id = 0;
  return nullptr;
}
static PJRT_Error* Memory_DebugString(PJRT_Memory_DebugString_Args* a) {
  a->debug_string = a->memory->debug.c_str();
  a->debug_string_size = a->memory->debug.size();
  return nullptr;
}
static PJRT_Error* Memory_ToString(PJRT_Memory_ToString_Args* a) {
  a->to_string = a->memory->tostr.c_str();
  a->to_string_size = a->memory->tostr.size();
  return nullptr;
}
static PJRT_Error* Memory_AddressableByDevices(PJRT_Memory_AddressableByDevices_Args* a) {
  a->devices = &a->memory->device;
  a->num_devices = 1;
  return nullptr;
}

// ---- executables
static PJRT_Error* Executable_Destroy(PJRT_Executable_Destroy_Args* a) {
  delete a->executable;
  return nullptr;
}
static PJRT_Error* Executable_Name(PJRT_Executable_Name_Args* a) {
  a->executable_name = a->executable->exe->name.c_str();
  a->executable_name_size = a->executable->exe->name.size();
  return nullptr;
}
static PJRT_Error* Executable_NumReplicas(PJRT_Executable_NumReplicas_Args* a) {
  a->num_replicas = (size_t)a->executable->exe->num_replicas;
  return nullptr;
}
static PJRT_Error* Executable_NumPartitions(PJRT_Executable_NumPartitions_Args* a) {
  a->num_partitions = 1;
  return nullptr;
}
static PJRT_Error* Executable_NumOutputs(PJRT_Executable_NumOutputs_Args* a) {
  a->num_outputs = a->executable->exe->plan.output_types.size();
  return nullptr;
}
static PJRT_Error* Executable_SizeOfGeneratedCodeInBytes(PJRT_Executable_SizeOfGeneratedCodeInBytes_Args* a) {
  int64_t n = 0;
  for (auto& c : a->executable->exe->cubins) n += (int64_t)c.size();
  a->size_in_bytes = n;
  return nullptr;
}
static PJRT_Error* Executable_GetCostAnalysis(PJRT_Executable_GetCostAnalysis_Args* a) {
  a->num_properties = 0;
  a->properties = nullptr;
  return nullptr;
}
static PJRT_Error* Executable_OutputMemoryKinds(PJRT_Executable_OutputMemoryKinds_Args* a) {
  Exe& e = *a->executable->exe;
  a->num_outputs = e.out_kinds.size();
  a->memory_kinds = e.out_kinds.data();
  a->memory_kind_sizes = e.out_kind_sizes.data();
  return nullptr;
}
static PJRT_Error* Executable_OutputElementTypes(PJRT_Executable_OutputElementTypes_Args* a) {
  Exe& e = *a->executable->exe;
  a->output_types = e.out_types.data();
  a->num_output_types = e.out_types.size();
  return nullptr;
}
static PJRT_Error* Executable_OutputDimensions(PJRT_Executable_OutputDimensions_Args* a) {
  Exe& e = *a->executable->exe;
  a->num_outputs = e.out_dim_sizes.size();
  a->dims = e.out_dims_flat.data();
  a->dim_sizes = e.out_dim_sizes.data();
  return nullptr;
}
static PJRT_Error* Executable_Fingerprint(PJRT_Executable_Fingerprint_Args* a) {
  a->executable_fingerprint = a->executable->exe->fingerprint.c_str();
  a->executable_fingerprint_size = a->executable->exe->fingerprint.size();
  return nullptr;
}
static PJRT_Error* Executable_OptimizedProgram(PJRT_Executable_OptimizedProgram_Args* a) {
  Exe& e = *a->executable->exe;
  PJRT_Program* p = a->program;
  static const char kFmt[] = "mlir";
  if (!p->code) {
    p->code_size = e.text.size();
  } else {
    std::memcpy(p->code, e.text.data(), std::min(p->code_size, e.text.size()));
    p->code_size = e.text.size();
  }
  p->format = kFmt;
  p->format_size = 4;
  return nullptr;
}
struct SerializedBlob {
  std::string bytes;
};
static void delete_blob(PJRT_SerializedExecutable* b) { delete reinterpret_cast<SerializedBlob*>(b); }
static void delete_opts(PJRT_SerializedCompileOptions* b) { delete reinterpret_cast<SerializedBlob*>(b); }
static PJRT_Error* Executable_Serialize(PJRT_Executable_Serialize_Args* a) {
  // Serialized form "B200EXE2": the program text, the compile options, and the
  // generated kernels' cubins, each under the nvrtc_key of its source.  Loading
  // re-plans the program (host work, milliseconds) and takes every kernel
  // whose source still has the same key from the blob instead of compiling it.
  const Exe& e = *a->executable->exe;
  auto* blob = new SerializedBlob;
  auto put = [&](const std::string& s) {
    uint64_t n = s.size();
    blob->bytes.append((const char*)&n, 8);
    blob->bytes += s;
  };
  blob->bytes = "B200EXE2";
  put(e.text);
  put(e.compile_options);
  put(std::to_string(e.cubins.size()));
  for (size_t u = 0; u < e.cubins.size(); ++u) {
    put(nvrtc_key(e.plan.units.at(u)));
    put(e.cubins[u]);
  }
  a->serialized_bytes = blob->bytes.data();
  a->serialized_bytes_size = blob->bytes.size();
  a->serialized_executable = reinterpret_cast<PJRT_SerializedExecutable*>(blob);
  a->serialized_executable_deleter = delete_blob;
  return nullptr;
}
static PJRT_Error* Executable_GetCompileOptions(PJRT_Executable_GetCompileOptions_Args* a) {
  auto* blob = new SerializedBlob{a->executable->exe->compile_options};
  a->serialized_bytes = blob->bytes.data();
  a->serialized_bytes_size = blob->bytes.size();
  a->serialized_compile_options = reinterpret_cast<PJRT_SerializedCompileOptions*>(blob);
  a->serialized_compile_options_deleter = delete_opts;
  return nullptr;
}
static PJRT_Error* Executable_DeserializeAndLoad(PJRT_Executable_DeserializeAndLoad_Args* a) {
  PJRT_TRY
  std::string s(a->serialized_executable, a->serialized_executable_size);
  const bool v2 = s.size() >= 16 && s.compare(0, 8, "B200EXE2") == 0;
  if (!v2 && (s.size() < 16 || s.compare(0, 8, "B200EXE1") != 0))
    throw PjrtErr(3, "not a B200 serialized executable");
  size_t off = 8;
  auto get = [&]() {
    if (off + 8 > s.size()) throw PjrtErr(3, "truncated serialized executable");
    uint64_t n;
    std::memcpy(&n, s.data() + off, 8);
    off += 8;
    if (off + n > s.size()) throw PjrtErr(3, "truncated serialized executable");
    std::string r = s.substr(off, n);
    off += n;
    return r;
  };
  std::string text = get();
  std::string opts = get();
  std::map<std::string, std::string> prebuilt;
  if (v2) {
    const std::string count = get();
    const long n = std::strtol(count.c_str(), nullptr, 10);
    if (n < 0 || n > (1 << 20)) throw PjrtErr(3, "corrupt serialized executable");
    for (long u = 0; u < n; ++u) {
      std::string key = get();
      prebuilt[key] = get();
    }
  }
  if (a->overridden_serialized_compile_options && a->overridden_serialized_compile_options_size)
    opts.assign(a->overridden_serialized_compile_options, a->overridden_serialized_compile_options_size);
  auto* le = new PJRT_LoadedExecutable;
  le->exe = compile(a->client, text, opts, v2 ? &prebuilt : nullptr);
  a->loaded_executable = le;
  PJRT_CATCH
}
static PJRT_Error* LoadedExecutable_Destroy(PJRT_LoadedExecutable_Destroy_Args* a) {
  delete a->executable;
  return nullptr;
}
static PJRT_Error* LoadedExecutable_GetExecutable(PJRT_LoadedExecutable_GetExecutable_Args* a) {
  a->executable = new PJRT_Executable{a->loaded_executable->exe};
  return nullptr;
}
static PJRT_Error* LoadedExecutable_AddressableDevices(PJRT_LoadedExecutable_AddressableDevices_Args* a) {
  a->addressable_devices = a->executable->exe->addressable.data();
  a->num_addressable_devices = a->executable->exe->addressable.size();
  return nullptr;
}
static PJRT_Error* LoadedExecutable_Delete(PJRT_LoadedExecutable_Delete_Args* a) {
  a->executable->deleted = true;
  return nullptr;
}
static PJRT_Error* LoadedExecutable_IsDeleted(PJRT_LoadedExecutable_IsDeleted_Args* a) {
  a->is_deleted = a->executable->deleted;
  return nullptr;
}
static PJRT_Error* LoadedExecutable_Execute(PJRT_LoadedExecutable_Execute_Args* a) {
  PJRT_TRY
  execute(a->executable, a);
  PJRT_CATCH
}
static PJRT_Error* LoadedExecutable_Fingerprint(PJRT_LoadedExecutable_Fingerprint_Args* a) {
  a->executable_fingerprint = a->executable->exe->fingerprint.c_str();
  a->executable_fingerprint_size = a->executable->exe->fingerprint.size();
  return nullptr;
}

// ---- buffers
static PJRT_Error* Buffer_Destroy(PJRT_Buffer_Destroy_Args* a) {
  delete a->buffer;
  return nullptr;
}
static PJRT_Error* Buffer_ElementType(PJRT_Buffer_ElementType_Args* a) {
  a->type = (PJRT_Buffer_Type)a->buffer->type.dtype;
  return nullptr;
}
static PJRT_Error* Buffer_Dimensions(PJRT_Buffer_Dimensions_Args* a) {
  a->dims = a->buffer->dims.data();
  a->num_dims = a->buffer->dims.size();
  return nullptr;
}
static PJRT_Error* Buffer_UnpaddedDimensions(PJRT_Buffer_UnpaddedDimensions_Args* a) {
  a->unpadded_dims = a->buffer->dims.data();
  a->num_dims = a->buffer->dims.size();
  return nullptr;
}
static PJRT_Error* Buffer_DynamicDimensionIndices(PJRT_Buffer_DynamicDimensionIndices_Args* a) {
  a->dynamic_dim_indices = nullptr;
  a->num_dynamic_dims = 0;
  return nullptr;
}
static PJRT_Error* Buffer_OnDeviceSizeInBytes(PJRT_Buffer_OnDeviceSizeInBytes_Args* a) {
  a->on_device_size_in_bytes = (size_t)a->buffer->type.bytes();
  return nullptr;
}
static PJRT_Error* Buffer_Device(PJRT_Buffer_Device_Args* a) {
  a->device = a->buffer->device;
  return nullptr;
}
static PJRT_Error* Buffer_Memory(PJRT_Buffer_Memory_Args* a) {
  a->memory = a->buffer->device->memory;
  return nullptr;
}
static PJRT_Error* Buffer_Delete(PJRT_Buffer_Delete_Args* a) {
  a->buffer->deleted = true;
  a->buffer->mem.reset();
  return nullptr;
}
static PJRT_Error* Buffer_IsDeleted(PJRT_Buffer_IsDeleted_Args* a) {
  a->is_deleted = a->buffer->deleted;
  return nullptr;
}
static PJRT_Error* Buffer_IsOnCpu(PJRT_Buffer_IsOnCpu_Args* a) {
  a->is_on_cpu = false;
  return nullptr;
}
static PJRT_Error* Buffer_ReadyEvent(PJRT_Buffer_ReadyEvent_Args* a) {
  a->event = a->buffer->ready ? handle_of(a->buffer->ready) : ready_event();
  return nullptr;
}
static PJRT_Error* Buffer_UnsafePointer(PJRT_Buffer_UnsafePointer_Args* a) {
  a->buffer_pointer = a->buffer->mem ? (uintptr_t)a->buffer->mem->ptr : 0;
  return nullptr;
}
static PJRT_Error* Buffer_OpaqueDeviceMemoryDataPointer(PJRT_Buffer_OpaqueDeviceMemoryDataPointer_Args* a) {
  a->device_memory_ptr = a->buffer->mem ? a->buffer->mem->ptr : nullptr;
  return nullptr;
}
static PJRT_Error* Buffer_IncreaseExternalReferenceCount(PJRT_Buffer_IncreaseExternalReferenceCount_Args* a) {
  a->buffer->ext_refs++;
  return nullptr;
}
static PJRT_Error* Buffer_DecreaseExternalReferenceCount(PJRT_Buffer_DecreaseExternalReferenceCount_Args* a) {
  if (a->buffer->ext_refs.load() <= 0) return make_err(9, "external reference count is already zero");
  a->buffer->ext_refs--;
  return nullptr;
}
static PJRT_Error* Buffer_ToHostBuffer(PJRT_Buffer_ToHostBuffer_Args* a) {
  PJRT_TRY
  PJRT_Buffer* b = a->src;
  const size_t need = (size_t)b->type.bytes();
  if (!a->dst) {
    a->dst_size = need;
    return nullptr;
  }
  if (b->deleted || !b->mem) throw PjrtErr(9, "ToHostBuffer on a deleted buffer");
  if (a->dst_size < need) throw PjrtErr(3, "ToHostBuffer: destination too small");
  Device& d = *b->device->dev;
  std::lock_guard<std::recursive_mutex> lk(d.mu);
  d.activate();
  if (need) B200_CUDA(cudaMemcpyAsync(a->dst, b->mem->ptr, need, cudaMemcpyDeviceToHost, d.stream));
  auto ev = record_event(d);
  if (b->ready) ev->status = b->ready->status;  // a failed collective upstream fails the copy
  a->event = handle_of(ev);
  PJRT_CATCH
}
static PJRT_Error* Buffer_CopyRawToHost(PJRT_Buffer_CopyRawToHost_Args* a) {
  PJRT_TRY
  PJRT_Buffer* b = a->buffer;
  if (b->deleted || !b->mem) throw PjrtErr(9, "CopyRawToHost on a deleted buffer");
  if (a->offset < 0 || a->offset + a->transfer_size > b->type.bytes()) throw PjrtErr(11, "CopyRawToHost out of range");
  Device& d = *b->device->dev;
  d.activate();
  B200_CUDA(cudaMemcpyAsync(a->dst, (char*)b->mem->ptr + a->offset, (size_t)a->transfer_size,
                            cudaMemcpyDeviceToHost, d.stream));
  auto ev = record_event(d);
  if (b->ready) ev->status = b->ready->status;
  a->event = handle_of(ev);
  PJRT_CATCH
}
static PJRT_Error* Buffer_CopyToDevice(PJRT_Buffer_CopyToDevice_Args* a) {
  PJRT_TRY
  PJRT_Buffer* b = a->buffer;
  PJRT_Device* dst = a->dst_device;
  if (!dst->dev || !b->device->dev) throw PjrtErr(3, "CopyToDevice needs addressable devices");
  auto* nb = new PJRT_Buffer;
  nb->client = b->client;
  nb->device = dst;
  nb->type = b->type;
  nb->dims = b->dims;
  nb->mem = std::make_shared<DeviceMem>(dst->dev, (size_t)std::max<int64_t>(b->type.bytes(), 1));
  // order after the source's producer, then copy on the destination stream
  b->device->dev->activate();
  auto src_ev = record_event(*b->device->dev);
  dst->dev->activate();
  B200_CUDA(cudaStreamWaitEvent(dst->dev->stream, src_ev->ev, 0));
  B200_CUDA(cudaMemcpyPeerAsync(nb->mem->ptr, dst->dev->ordinal, b->mem->ptr, b->device->dev->ordinal,
                                (size_t)b->type.bytes(), dst->dev->stream));
  nb->ready = record_event(*dst->dev);
  // keep the source alive until the copy is done
  B200_CUDA(cudaStreamWaitEvent(b->device->dev->stream, nb->ready->ev, 0));
  a->dst_buffer = nb;
  PJRT_CATCH
}
static PJRT_Error* Buffer_CopyToMemory(PJRT_Buffer_CopyToMemory_Args* a) {
  PJRT_Buffer_CopyToDevice_Args c{};
  c.struct_size = sizeof(c);
  c.buffer = a->buffer;
  c.dst_device = a->dst_memory->device;
  PJRT_Error* e = Buffer_CopyToDevice(&c);
  a->dst_buffer = c.dst_buffer;
  return e;
}

// ---- topology
static PJRT_Error* TopologyDescription_Destroy(PJRT_TopologyDescription_Destroy_Args*) { return nullptr; }
static PJRT_Error* TopologyDescription_PlatformName(PJRT_TopologyDescription_PlatformName_Args* a) {
  a->platform_name = "b200";
  a->platform_name_size = 4;
  return nullptr;
}
static PJRT_Error* TopologyDescription_PlatformVersion(PJRT_TopologyDescription_PlatformVersion_Args* a) {
  a->platform_version = a->topology->version.c_str();
  a->platform_version_size = a->topology->version.size();
  return nullptr;
}
static PJRT_Error* TopologyDescription_GetDeviceDescriptions(PJRT_TopologyDescription_GetDeviceDescriptions_Args* a) {
  a->descriptions = a->topology->descs.data();
  a->num_descriptions = a->topology->descs.size();
  return nullptr;
}
static PJRT_Error* TopologyDescription_Attributes(PJRT_TopologyDescription_Attributes_Args* a) {
  a->attributes = nullptr;
  a->num_attributes = 0;
  return nullptr;
}

static PJRT_Error* Unimplemented(void*) { return make_err(12, "this PJRT entry point is not implemented by the B200 plugin"); }

static PJRT_Api g_api;

__attribute__((visibility("default"))) const PJRT_Api* GetPjrtApi(void) {
  static bool init = [] {
    std::memset(&g_api, 0, sizeof(g_api));
    g_api.struct_size = sizeof(PJRT_Api);
    g_api.pjrt_api_version.struct_size = sizeof(PJRT_Api_Version);
    g_api.pjrt_api_version.major_version = B200_PJRT_API_MAJOR;
    g_api.pjrt_api_version.minor_version = B200_PJRT_API_MINOR;
    // every slot starts as Unimplemented, then the implemented ones are set
#define B200_FILL(name) g_api.PJRT_##name = reinterpret_cast<decltype(g_api.PJRT_##name)>(&Unimplemented);
    B200_PJRT_API_SLOTS(B200_FILL)
#undef B200_FILL
#define SET(name) g_api.PJRT_##name = reinterpret_cast<decltype(g_api.PJRT_##name)>(&name);
    SET(Error_Destroy) SET(Error_Message) SET(Error_GetCode)
    SET(Plugin_Initialize) SET(Plugin_Attributes)
    SET(Event_Destroy) SET(Event_IsReady) SET(Event_Error) SET(Event_Await) SET(Event_OnReady)
    SET(Event_Create) SET(Event_Set)
    SET(Client_Create) SET(Client_Destroy) SET(Client_PlatformName) SET(Client_ProcessIndex)
    SET(Client_PlatformVersion) SET(Client_Devices) SET(Client_AddressableDevices)
    SET(Client_LookupDevice) SET(Client_LookupAddressableDevice) SET(Client_AddressableMemories)
    SET(Client_Compile) SET(Client_DefaultDeviceAssignment) SET(Client_BufferFromHostBuffer)
    SET(Client_CreateViewOfDeviceBuffer) SET(Client_TopologyDescription)
    SET(DeviceDescription_Id) SET(DeviceDescription_ProcessIndex) SET(DeviceDescription_Attributes)
    SET(DeviceDescription_Kind) SET(DeviceDescription_DebugString) SET(DeviceDescription_ToString)
    SET(Device_GetDescription) SET(Device_IsAddressable) SET(Device_LocalHardwareId)
    SET(Device_AddressableMemories) SET(Device_DefaultMemory) SET(Device_MemoryStats)
    SET(Memory_Id) SET(Memory_Kind) SET(Memory_Kind_Id) SET(Memory_DebugString) SET(Memory_ToString)
    SET(Memory_AddressableByDevices)
    SET(Executable_Destroy) SET(Executable_Name) SET(Executable_NumReplicas)
    SET(Executable_NumPartitions) SET(Executable_NumOutputs)
    SET(Executable_SizeOfGeneratedCodeInBytes) SET(Executable_GetCostAnalysis)
    SET(Executable_OutputMemoryKinds) SET(Executable_OptimizedProgram) SET(Executable_Serialize)
    SET(Executable_OutputElementTypes) SET(Executable_OutputDimensions) SET(Executable_Fingerprint)
    SET(Executable_GetCompileOptions) SET(Executable_DeserializeAndLoad)
    SET(LoadedExecutable_Destroy) SET(LoadedExecutable_GetExecutable)
    SET(LoadedExecutable_AddressableDevices) SET(LoadedExecutable_Delete)
    SET(LoadedExecutable_IsDeleted) SET(LoadedExecutable_Execute) SET(LoadedExecutable_Fingerprint)
    SET(Buffer_Destroy) SET(Buffer_ElementType) SET(Buffer_Dimensions) SET(Buffer_UnpaddedDimensions)
    SET(Buffer_DynamicDimensionIndices) SET(Buffer_OnDeviceSizeInBytes) SET(Buffer_Device)
    SET(Buffer_Memory) SET(Buffer_Delete) SET(Buffer_IsDeleted) SET(Buffer_CopyToDevice)
    SET(Buffer_ToHostBuffer) SET(Buffer_IsOnCpu) SET(Buffer_ReadyEvent) SET(Buffer_UnsafePointer)
    SET(Buffer_IncreaseExternalReferenceCount) SET(Buffer_DecreaseExternalReferenceCount)
    SET(Buffer_OpaqueDeviceMemoryDataPointer) SET(Buffer_CopyToMemory) SET(Buffer_CopyRawToHost)
    SET(TopologyDescription_Destroy) SET(TopologyDescription_PlatformName)
    SET(TopologyDescription_PlatformVersion) SET(TopologyDescription_GetDeviceDescriptions)
    SET(TopologyDescription_Attributes)
#undef SET
    return true;
  }();
  (void)init;
  return &g_api;
}

// ---- diagnostics (no GPU needed)
__attribute__((visibility("default"))) int b200_pjrt_inspect(const char* mlir, size_t len, int what,
                                                             char** out) {
  std::string res;
  int code = 0;
  try {
    fault_point("compile");
    Module m = parse_module(program_text(std::string(mlir, len)));
    Plan p = build_plan(m);
    if (what == 0) res = p.graph_dump;
    else if (what == 1) res = dump_plan(p);
    else if (what == 2) res = p.source;
    else if (what == 4) {
      for (auto& u : p.units) res += nvrtc_key(u) + "\n";
    }
    else if (what == 3) {
      size_t n = 0;
      if (!p.kernel_names.empty())
        for (auto& c : nvrtc_compile_all(p.units, "inspect")) n += c.size();
      res = "ok " + std::to_string(n);
    } else res = "bad 'what'";
  } catch (const PjrtErr& e) {
    code = e.code;
    res = e.what();
  } catch (const std::exception& e) {
    code = 13;
    res = e.what();
  }
  *out = (char*)std::malloc(res.size() + 1);
  std::memcpy(*out, res.c_str(), res.size() + 1);
  return code;
}
__attribute__((visibility("default"))) void b200_pjrt_free(char* p) { std::free(p); }

__attribute__((visibility("default"))) uint64_t b200_pjrt_kernel_launches(void) {
  return (uint64_t)b200::g_generated_launches.load(std::memory_order_relaxed);
}

__attribute__((visibility("default"))) int b200_pjrt_execute_times(void* loaded_executable,
                                                                  double* ms, int max) {
  auto* le = static_cast<PJRT_LoadedExecutable*>(loaded_executable);
  if (!le) return -1;
  Exe& e = *le->exe;
  std::lock_guard<std::mutex> lk(e.timing_mu);
  int n = 0;
  for (auto& pr : e.timings) {
    float t = 0.f;
    cudaEventSynchronize(pr.second);
    if (cudaEventElapsedTime(&t, pr.first, pr.second) != cudaSuccess) t = -1.f;
    if (n < max && ms) ms[n] = t;
    ++n;
    cudaEventDestroy(pr.first);
    cudaEventDestroy(pr.second);
  }
  e.timings.clear();
  return n;
}

__attribute__((visibility("default"))) int b200_pjrt_kv_exchange(
    void* get_callback, void* get_user_arg, void* put_callback, void* put_user_arg, int rank,
    const char* key, size_t key_len, const char* value, size_t value_len, char** out,
    size_t* out_len) {
  std::string res;
  int code = 0;
  try {
    const std::string k(key ? key : "", key ? key_len : 0);
    if (rank == 0) {
      res.assign(value ? value : "", value ? value_len : 0);
      kv_put(reinterpret_cast<PJRT_KeyValuePutCallback>(put_callback), put_user_arg, k, res);
    } else {
      res = kv_get(reinterpret_cast<PJRT_KeyValueGetCallback>(get_callback), get_user_arg, k);
    }
  } catch (const PjrtErr& e) {
    code = e.code;
    res = e.what();
  } catch (const std::exception& e) {
    code = 13;
    res = e.what();
  }
  *out = (char*)std::malloc(res.size() + 1);
  std::memcpy(*out, res.data(), res.size());
  (*out)[res.size()] = 0;
  if (out_len) *out_len = res.size();
  return code;
}

__attribute__((visibility("default"))) void* b200_pjrt_device_stream(void* device) {
  auto* d = static_cast<PJRT_Device*>(device);
  return d && d->dev ? (void*)d->dev->stream : nullptr;
}

}  // extern "C"
