"""ctypes client for the B200 PJRT plugin (``libb200_pjrt.so``).

This is the binding jaxlib performs in C++ when ``xla_bridge.register_plugin``
loads a plugin (reference ``src/jax_mlx/plugin.py:24-47``): dlopen the library,
call ``GetPjrtApi()``, then drive ``PJRT_Client_Create`` / ``Compile`` /
``BufferFromHostBuffer`` / ``LoadedExecutable_Execute`` / ``ToHostBuffer``
through the function-pointer table.  JAX is not installed in this build's
environment, so tests and ``bench.py`` talk to the plugin through this module
exactly as jaxlib would.
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Callable, Dict, List, Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
# In-tree builds put the libraries in ../lib (csrc/Makefile); a wheel built with
# `make -C csrc LIB=../jax_b200/lib` carries them inside the package.
LIB_DIR = (os.path.join(_HERE, "lib") if os.path.exists(os.path.join(_HERE, "lib", "libb200_pjrt.so"))
           else os.path.join(os.path.dirname(_HERE), "lib"))
PJRT_LIB = os.path.join(LIB_DIR, "libb200_pjrt.so")

# PJRT_Api function-pointer slots, in ABI (v0.90) order.  Must match
# B200_PJRT_API_SLOTS in include/b200_pjrt.h (checked by the CPU tests).
API_SLOTS = """
Error_Destroy Error_Message Error_GetCode Plugin_Initialize Plugin_Attributes Event_Destroy
Event_IsReady Event_Error Event_Await Event_OnReady Client_Create Client_Destroy
Client_PlatformName Client_ProcessIndex Client_PlatformVersion Client_Devices
Client_AddressableDevices Client_LookupDevice Client_LookupAddressableDevice
Client_AddressableMemories Client_Compile Client_DefaultDeviceAssignment
Client_BufferFromHostBuffer DeviceDescription_Id DeviceDescription_ProcessIndex
DeviceDescription_Attributes DeviceDescription_Kind DeviceDescription_DebugString
DeviceDescription_ToString Device_GetDescription Device_IsAddressable Device_LocalHardwareId
Device_AddressableMemories Device_DefaultMemory Device_MemoryStats Memory_Id Memory_Kind
Memory_DebugString Memory_ToString Memory_AddressableByDevices Executable_Destroy
Executable_Name Executable_NumReplicas Executable_NumPartitions Executable_NumOutputs
Executable_SizeOfGeneratedCodeInBytes Executable_GetCostAnalysis Executable_OutputMemoryKinds
Executable_OptimizedProgram Executable_Serialize LoadedExecutable_Destroy
LoadedExecutable_GetExecutable LoadedExecutable_AddressableDevices LoadedExecutable_Delete
LoadedExecutable_IsDeleted LoadedExecutable_Execute Executable_DeserializeAndLoad
LoadedExecutable_Fingerprint Buffer_Destroy Buffer_ElementType Buffer_Dimensions
Buffer_UnpaddedDimensions Buffer_DynamicDimensionIndices Buffer_GetMemoryLayout
Buffer_OnDeviceSizeInBytes Buffer_Device Buffer_Memory Buffer_Delete Buffer_IsDeleted
Buffer_CopyToDevice Buffer_ToHostBuffer Buffer_IsOnCpu Buffer_ReadyEvent Buffer_UnsafePointer
Buffer_IncreaseExternalReferenceCount Buffer_DecreaseExternalReferenceCount
Buffer_OpaqueDeviceMemoryDataPointer CopyToDeviceStream_Destroy CopyToDeviceStream_AddChunk
CopyToDeviceStream_TotalBytes CopyToDeviceStream_GranuleSize CopyToDeviceStream_CurrentBytes
TopologyDescription_Create TopologyDescription_Destroy TopologyDescription_PlatformName
TopologyDescription_PlatformVersion TopologyDescription_GetDeviceDescriptions
TopologyDescription_Serialize TopologyDescription_Attributes Compile
Executable_OutputElementTypes Executable_OutputDimensions Buffer_CopyToMemory
Client_CreateViewOfDeviceBuffer Executable_Fingerprint Client_TopologyDescription
Executable_GetCompiledMemoryStats Memory_Kind_Id ExecuteContext_Create ExecuteContext_Destroy
Buffer_CopyRawToHost AsyncHostToDeviceTransferManager_Destroy
AsyncHostToDeviceTransferManager_TransferData Client_CreateBuffersForAsyncHostToDevice
AsyncHostToDeviceTransferManager_RetrieveBuffer AsyncHostToDeviceTransferManager_Device
AsyncHostToDeviceTransferManager_BufferCount AsyncHostToDeviceTransferManager_BufferSize
AsyncHostToDeviceTransferManager_SetBufferError AsyncHostToDeviceTransferManager_AddMetadata
Client_DmaMap Client_DmaUnmap Client_CreateUninitializedBuffer Client_UpdateGlobalProcessInfo
TopologyDescription_Deserialize Client_CreateAliasBuffer Client_FulfillAliasBuffer
LoadedExecutable_GetDeviceAssignment Client_CreateErrorBuffer
AsyncHostToDeviceTransferManager_TransferLiteral Buffer_CopyRawToHostFuture
Device_PoisonExecution Device_CreateAsyncTrackingEvent AsyncTrackingEvent_Destroy
Executable_GetCompileOptions Buffer_DonateWithControlDependency Event_Create Event_Set
""".split()

# PJRT_Buffer_Type numbering
PRED, S8, S16, S32, S64, U8, U16, U32, U64, F16, F32, F64, BF16 = range(1, 14)
_NP2PJRT = {np.dtype(np.bool_): PRED, np.dtype(np.int8): S8, np.dtype(np.int16): S16,
            np.dtype(np.int32): S32, np.dtype(np.int64): S64, np.dtype(np.uint8): U8,
            np.dtype(np.uint16): U16, np.dtype(np.uint32): U32, np.dtype(np.uint64): U64,
            np.dtype(np.float32): F32, np.dtype(np.float64): F64}
_PJRT2NP = {v: k for k, v in _NP2PJRT.items()}
_PJRT2NP[BF16] = np.dtype(np.uint16)  # bf16 bits travel as uint16 on the host


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """f32 values -> bf16 bit patterns (uint16), round to nearest even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    return np.where(nan, 0x7FC0, r).astype(np.uint16)


def from_bf16_bits(b: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> f32 values."""
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)

ERROR_CODES = {0: "OK", 1: "CANCELLED", 2: "UNKNOWN", 3: "INVALID_ARGUMENT",
               4: "DEADLINE_EXCEEDED", 5: "NOT_FOUND", 6: "ALREADY_EXISTS",
               7: "PERMISSION_DENIED", 8: "RESOURCE_EXHAUSTED", 9: "FAILED_PRECONDITION",
               10: "ABORTED", 11: "OUT_OF_RANGE", 12: "UNIMPLEMENTED", 13: "INTERNAL",
               14: "UNAVAILABLE", 15: "DATA_LOSS", 16: "UNAUTHENTICATED"}


class PjrtError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERROR_CODES.get(code, code)}: {msg}")
        self.code = code


def _struct(name, fields):
    return type(name, (C.Structure,), {"_fields_": [("struct_size", C.c_size_t),
                                                     ("extension_start", C.c_void_p)] + fields})


class NamedValue(C.Structure):
    class _U(C.Union):
        _fields_ = [("string_value", C.c_char_p), ("int64_value", C.c_int64),
                    ("int64_array_value", C.POINTER(C.c_int64)), ("float_value", C.c_float),
                    ("bool_value", C.c_bool)]
    _anonymous_ = ("u",)
    _fields_ = [("struct_size", C.c_size_t), ("extension_start", C.c_void_p),
                ("name", C.c_char_p), ("name_size", C.c_size_t), ("type", C.c_int),
                ("u", _U), ("value_size", C.c_size_t)]


KVGetArgs = _struct("KVGetArgs", [("key", C.c_char_p), ("key_size", C.c_size_t),
                                  ("timeout_in_ms", C.c_int), ("callback_error", C.c_void_p),
                                  ("user_arg", C.c_void_p), ("value", C.c_void_p),
                                  ("value_size", C.c_size_t), ("value_deleter_callback", C.c_void_p)])
KVPutArgs = _struct("KVPutArgs", [("key", C.c_char_p), ("key_size", C.c_size_t),
                                  ("value", C.c_void_p), ("value_size", C.c_size_t),
                                  ("callback_error", C.c_void_p), ("user_arg", C.c_void_p)])
# PJRT_CallbackError: the error constructor the plugin passes in each KV call
CALLBACK_ERROR = C.CFUNCTYPE(C.c_void_p, C.c_int, C.c_char_p, C.c_size_t)
KV_GET_CB = C.CFUNCTYPE(C.c_void_p, C.POINTER(KVGetArgs))
KV_PUT_CB = C.CFUNCTYPE(C.c_void_p, C.POINTER(KVPutArgs))
VALUE_DELETER = C.CFUNCTYPE(None, C.c_void_p)

A = {
    "Error_Destroy": [("error", C.c_void_p)],
    "Error_Message": [("error", C.c_void_p), ("message", C.c_char_p), ("message_size", C.c_size_t)],
    "Error_GetCode": [("error", C.c_void_p), ("code", C.c_int)],
    "Plugin_Initialize": [],
    "Plugin_Attributes": [("attributes", C.POINTER(NamedValue)), ("num_attributes", C.c_size_t)],
    "Event_Destroy": [("event", C.c_void_p)],
    "Event_IsReady": [("event", C.c_void_p), ("is_ready", C.c_bool)],
    "Event_Await": [("event", C.c_void_p)],
    "Client_Create": [("create_options", C.POINTER(NamedValue)), ("num_options", C.c_size_t),
                      ("kv_get_callback", C.c_void_p), ("kv_get_user_arg", C.c_void_p),
                      ("kv_put_callback", C.c_void_p), ("kv_put_user_arg", C.c_void_p),
                      ("client", C.c_void_p), ("kv_try_get_callback", C.c_void_p),
                      ("kv_try_get_user_arg", C.c_void_p)],
    "Client_Destroy": [("client", C.c_void_p)],
    "Client_PlatformName": [("client", C.c_void_p), ("platform_name", C.c_char_p),
                            ("platform_name_size", C.c_size_t)],
    "Client_PlatformVersion": [("client", C.c_void_p), ("platform_version", C.c_char_p),
                               ("platform_version_size", C.c_size_t)],
    "Client_ProcessIndex": [("client", C.c_void_p), ("process_index", C.c_int)],
    "Client_Devices": [("client", C.c_void_p), ("devices", C.POINTER(C.c_void_p)),
                       ("num_devices", C.c_size_t)],
    "Client_AddressableDevices": [("client", C.c_void_p), ("addressable_devices", C.POINTER(C.c_void_p)),
                                  ("num_addressable_devices", C.c_size_t)],
    "Client_DefaultDeviceAssignment": [("client", C.c_void_p), ("num_replicas", C.c_int),
                                       ("num_partitions", C.c_int), ("default_assignment_size", C.c_size_t),
                                       ("default_assignment", C.POINTER(C.c_int))],
    "Client_Compile": [("client", C.c_void_p), ("program", C.c_void_p), ("compile_options", C.c_char_p),
                       ("compile_options_size", C.c_size_t), ("executable", C.c_void_p)],
    "Client_BufferFromHostBuffer": [("client", C.c_void_p), ("data", C.c_void_p), ("type", C.c_int),
                                    ("dims", C.POINTER(C.c_int64)), ("num_dims", C.c_size_t),
                                    ("byte_strides", C.POINTER(C.c_int64)), ("num_byte_strides", C.c_size_t),
                                    ("host_buffer_semantics", C.c_int), ("device", C.c_void_p),
                                    ("memory", C.c_void_p), ("device_layout", C.c_void_p),
                                    ("done_with_host_buffer", C.c_void_p), ("buffer", C.c_void_p)],
    "Device_GetDescription": [("device", C.c_void_p), ("device_description", C.c_void_p)],
    "Device_LocalHardwareId": [("device", C.c_void_p), ("local_hardware_id", C.c_int)],
    "Device_MemoryStats": [("device", C.c_void_p), ("bytes_in_use", C.c_int64),
                           ("peak_bytes_in_use", C.c_int64), ("peak_set", C.c_bool),
                           ("num_allocs", C.c_int64), ("num_allocs_set", C.c_bool),
                           ("largest_alloc_size", C.c_int64), ("largest_set", C.c_bool),
                           ("bytes_limit", C.c_int64), ("bytes_limit_set", C.c_bool),
                           ("bytes_reserved", C.c_int64), ("bytes_reserved_set", C.c_bool),
                           ("peak_bytes_reserved", C.c_int64), ("peak_reserved_set", C.c_bool),
                           ("bytes_reservable_limit", C.c_int64), ("reservable_set", C.c_bool),
                           ("largest_free_block_bytes", C.c_int64), ("largest_free_set", C.c_bool),
                           ("pool_bytes", C.c_int64), ("pool_set", C.c_bool),
                           ("peak_pool_bytes", C.c_int64), ("peak_pool_set", C.c_bool)],
    "DeviceDescription_Id": [("device_description", C.c_void_p), ("id", C.c_int)],
    "DeviceDescription_Kind": [("device_description", C.c_void_p), ("device_kind", C.c_char_p),
                               ("device_kind_size", C.c_size_t)],
    "LoadedExecutable_Destroy": [("executable", C.c_void_p)],
    "LoadedExecutable_GetExecutable": [("loaded_executable", C.c_void_p), ("executable", C.c_void_p)],
    "LoadedExecutable_AddressableDevices": [("executable", C.c_void_p),
                                            ("addressable_devices", C.POINTER(C.c_void_p)),
                                            ("num_addressable_devices", C.c_size_t)],
    "LoadedExecutable_Execute": [("executable", C.c_void_p), ("options", C.c_void_p),
                                 ("argument_lists", C.c_void_p), ("num_devices", C.c_size_t),
                                 ("num_args", C.c_size_t), ("output_lists", C.c_void_p),
                                 ("device_complete_events", C.c_void_p), ("execute_device", C.c_void_p)],
    "Executable_Destroy": [("executable", C.c_void_p)],
    "Executable_NumOutputs": [("executable", C.c_void_p), ("num_outputs", C.c_size_t)],
    "Executable_NumReplicas": [("executable", C.c_void_p), ("num_replicas", C.c_size_t)],
    "Executable_OutputElementTypes": [("executable", C.c_void_p), ("output_types", C.POINTER(C.c_int)),
                                      ("num_output_types", C.c_size_t)],
    "Executable_OutputDimensions": [("executable", C.c_void_p), ("num_outputs", C.c_size_t),
                                    ("dims", C.POINTER(C.c_int64)), ("dim_sizes", C.POINTER(C.c_size_t))],
    "Executable_Serialize": [("executable", C.c_void_p), ("serialized_bytes", C.c_void_p),
                             ("serialized_bytes_size", C.c_size_t), ("serialized_executable", C.c_void_p),
                             ("serialized_executable_deleter", C.c_void_p)],
    "Executable_DeserializeAndLoad": [("client", C.c_void_p), ("serialized_executable", C.c_void_p),
                                      ("serialized_executable_size", C.c_size_t),
                                      ("loaded_executable", C.c_void_p),
                                      ("overridden_serialized_compile_options", C.c_void_p),
                                      ("overridden_serialized_compile_options_size", C.c_size_t)],
    "Buffer_Destroy": [("buffer", C.c_void_p)],
    "Buffer_Delete": [("buffer", C.c_void_p)],
    "Buffer_IsDeleted": [("buffer", C.c_void_p), ("is_deleted", C.c_bool)],
    "Buffer_IsOnCpu": [("buffer", C.c_void_p), ("is_on_cpu", C.c_bool)],
    "Buffer_ElementType": [("buffer", C.c_void_p), ("type", C.c_int)],
    "Buffer_Dimensions": [("buffer", C.c_void_p), ("dims", C.POINTER(C.c_int64)), ("num_dims", C.c_size_t)],
    "Buffer_OnDeviceSizeInBytes": [("buffer", C.c_void_p), ("on_device_size_in_bytes", C.c_size_t)],
    "Buffer_Device": [("buffer", C.c_void_p), ("device", C.c_void_p)],
    "Buffer_ReadyEvent": [("buffer", C.c_void_p), ("event", C.c_void_p)],
    "Buffer_UnsafePointer": [("buffer", C.c_void_p), ("buffer_pointer", C.c_size_t)],
    "Buffer_IncreaseExternalReferenceCount": [("buffer", C.c_void_p)],
    "Buffer_DecreaseExternalReferenceCount": [("buffer", C.c_void_p)],
    "Buffer_ToHostBuffer": [("src", C.c_void_p), ("host_layout", C.c_void_p), ("dst", C.c_void_p),
                            ("dst_size", C.c_size_t), ("event", C.c_void_p)],
    "Buffer_CopyToDevice": [("buffer", C.c_void_p), ("dst_device", C.c_void_p), ("dst_buffer", C.c_void_p)],
}
ARGS = {k: _struct(k + "_Args", v) for k, v in A.items()}
ProgramStruct = _struct("PJRT_Program", [("code", C.c_char_p), ("code_size", C.c_size_t),
                                         ("format", C.c_char_p), ("format_size", C.c_size_t)])


class ApiVersion(C.Structure):
    _fields_ = [("struct_size", C.c_size_t), ("extension_start", C.c_void_p),
                ("major_version", C.c_int), ("minor_version", C.c_int)]


class Api:
    """The plugin's PJRT_Api table, callable by slot name."""

    def __init__(self, path: str = PJRT_LIB):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} not built (run __graft_entry__.build())")
        self.lib = C.CDLL(path)
        self.lib.GetPjrtApi.restype = C.c_void_p
        self.ptr = self.lib.GetPjrtApi()
        hdr = ApiVersion.from_address(self.ptr + 16)
        self.version = (hdr.major_version, hdr.minor_version)
        self.struct_size = C.c_size_t.from_address(self.ptr).value
        base = self.ptr + 16 + C.sizeof(ApiVersion)
        self._fn: Dict[str, C._CFuncPtr] = {}
        proto = C.CFUNCTYPE(C.c_void_p, C.c_void_p)
        for i, name in enumerate(API_SLOTS):
            addr = C.c_void_p.from_address(base + 8 * i).value
            self._fn[name] = proto(addr) if addr else None

    def raw(self, name: str, args) -> Optional[int]:
        args.struct_size = C.sizeof(args)
        return self._fn[name](C.addressof(args))

    def call(self, name: str, **kw):
        a = ARGS[name]()
        for k, v in kw.items():
            setattr(a, k, v)
        self.check(self.raw(name, a))
        return a

    def check(self, err: Optional[int]):
        if not err:
            return
        m = ARGS["Error_Message"](error=err)
        self.raw("Error_Message", m)
        msg = C.string_at(m.message, m.message_size).decode(errors="replace")
        g = ARGS["Error_GetCode"](error=err)
        self.raw("Error_GetCode", g)
        self.raw("Error_Destroy", ARGS["Error_Destroy"](error=err))
        raise PjrtError(g.code, msg)

    def await_event(self, ev: Optional[int]):
        if not ev:
            return
        try:
            self.call("Event_Await", event=ev)
        finally:
            self.raw("Event_Destroy", ARGS["Event_Destroy"](event=ev))


_API: Optional[Api] = None


def api() -> Api:
    global _API
    if _API is None:
        _API = Api()
    return _API


class Buffer:
    def __init__(self, client: "Client", handle: int):
        self.client, self.handle = client, handle

    @property
    def dtype(self) -> int:
        return api().call("Buffer_ElementType", buffer=self.handle).type

    @property
    def shape(self):
        a = api().call("Buffer_Dimensions", buffer=self.handle)
        return tuple(a.dims[i] for i in range(a.num_dims))

    def device_pointer(self) -> int:
        return api().call("Buffer_UnsafePointer", buffer=self.handle).buffer_pointer

    def ready(self):
        ev = api().call("Buffer_ReadyEvent", buffer=self.handle).event
        api().await_event(ev)

    def to_host_async(self, out: np.ndarray) -> int:
        """Start a device->host copy into `out`; returns the PJRT event."""
        a = api().call("Buffer_ToHostBuffer", src=self.handle, dst=out.ctypes.data,
                       dst_size=out.nbytes)
        return a.event

    def to_numpy(self, out: Optional[np.ndarray] = None) -> np.ndarray:
        if out is None:
            out = np.empty(self.shape, dtype=_PJRT2NP[self.dtype])
        api().await_event(self.to_host_async(out))
        return out

    def delete(self):
        api().call("Buffer_Delete", buffer=self.handle)

    def destroy(self):
        if self.handle:
            api().call("Buffer_Destroy", buffer=self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


class Executable:
    def __init__(self, client: "Client", handle: int):
        self.client, self.handle = client, handle
        exe = api().call("LoadedExecutable_GetExecutable", loaded_executable=handle).executable
        try:
            self.num_outputs = api().call("Executable_NumOutputs", executable=exe).num_outputs
            self.num_replicas = api().call("Executable_NumReplicas", executable=exe).num_replicas
            t = api().call("Executable_OutputElementTypes", executable=exe)
            self.output_types = [t.output_types[i] for i in range(t.num_output_types)]
            d = api().call("Executable_OutputDimensions", executable=exe)
            dims, off = [], 0
            for i in range(d.num_outputs):
                n = d.dim_sizes[i]
                dims.append(tuple(d.dims[off + k] for k in range(n)))
                off += n
            self.output_shapes = dims
        finally:
            api().call("Executable_Destroy", executable=exe)
        a = api().call("LoadedExecutable_AddressableDevices", executable=handle)
        self.devices = [a.addressable_devices[i] for i in range(a.num_addressable_devices)]

    def execute(self, args: Sequence[Sequence[Buffer]], wait: bool = False) -> List[List[Buffer]]:
        """args[d][i]: argument i on addressable device d.  Returns outputs[d][o]."""
        nd = len(args)
        na = len(args[0]) if nd else 0
        rows = [(C.c_void_p * max(na, 1))(*[b.handle for b in a]) for a in args]
        arg_lists = (C.c_void_p * nd)(*[C.addressof(r) for r in rows])
        outs = [(C.c_void_p * max(self.num_outputs, 1))() for _ in range(nd)]
        out_lists = (C.c_void_p * nd)(*[C.addressof(o) for o in outs])
        events = (C.c_void_p * nd)()
        api().call("LoadedExecutable_Execute", executable=self.handle, options=None,
                   argument_lists=C.addressof(arg_lists), num_devices=nd, num_args=na,
                   output_lists=C.addressof(out_lists), device_complete_events=C.addressof(events),
                   execute_device=None)
        for e in events:
            if wait:
                api().await_event(e)
            elif e:
                api().raw("Event_Destroy", ARGS["Event_Destroy"](event=e))
        return [[Buffer(self.client, outs[d][o]) for o in range(self.num_outputs)] for d in range(nd)]

    def device_times_ms(self) -> List[float]:
        """Device time of each Execute since the last call (needs B200_TIMING=1)."""
        f = api().lib.b200_pjrt_execute_times
        f.restype, f.argtypes = C.c_int, [C.c_void_p, C.POINTER(C.c_double), C.c_int]
        buf = (C.c_double * 4096)()
        n = f(self.handle, buf, 4096)
        return [buf[i] for i in range(min(n, 4096))]

    def serialize(self) -> bytes:
        exe = api().call("LoadedExecutable_GetExecutable", loaded_executable=self.handle).executable
        try:
            a = api().call("Executable_Serialize", executable=exe)
            data = C.string_at(a.serialized_bytes, a.serialized_bytes_size)
            C.CFUNCTYPE(None, C.c_void_p)(a.serialized_executable_deleter)(a.serialized_executable)
            return data
        finally:
            api().call("Executable_Destroy", executable=exe)

    def destroy(self):
        if self.handle:
            api().call("LoadedExecutable_Destroy", executable=self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


def kv_callbacks(store):
    """The PJRT key-value callbacks over `store` (``set(key: str, value: bytes)``,
    ``get(key: str) -> bytes``).  In a multi-process job the plugin's rank 0
    publishes the NCCL unique id through the put callback and every other rank
    reads it back through the get callback (values are raw bytes, zeros
    included).  A value handed out by get stays alive until the plugin calls
    its deleter.  Returns (get_cb, put_cb, keep): keep holds every ctypes
    object that must outlive the client."""
    values = {}

    def deleter(p):
        values.pop(p, None)

    del_cb = VALUE_DELETER(deleter)

    def fail(a, exc):
        """A store failure as a PJRT error made by the plugin's callback_error
        (DEADLINE_EXCEEDED for a timeout, UNKNOWN otherwise); without one the
        value stays unset, which the plugin also reports as a failed get."""
        if not a.callback_error:
            return None
        make = C.cast(a.callback_error, C.POINTER(CALLBACK_ERROR))[0]
        msg = f"{type(exc).__name__}: {exc}".encode()
        return make(4 if isinstance(exc, TimeoutError) else 2, msg, len(msg))

    def kv_get(args):
        a = args.contents
        key = C.string_at(a.key, a.key_size).decode()
        try:
            val = store.get(key)
        except Exception as exc:  # noqa: BLE001 -- reported to the plugin
            return fail(a, exc)
        buf = C.create_string_buffer(val, len(val))
        addr = C.addressof(buf)
        values[addr] = buf
        a.value, a.value_size = addr, len(val)
        a.value_deleter_callback = C.cast(del_cb, C.c_void_p)
        return None

    def kv_put(args):
        a = args.contents
        key = C.string_at(a.key, a.key_size).decode()
        try:
            store.set(key, C.string_at(a.value, a.value_size))
        except Exception as exc:  # noqa: BLE001
            return fail(a, exc)
        return None

    get_cb, put_cb = KV_GET_CB(kv_get), KV_PUT_CB(kv_put)
    return get_cb, put_cb, [get_cb, put_cb, del_cb, values]


class Client:
    """A PJRT client of the B200 plugin.

    options: create options forwarded as PJRT_NamedValues ("node_id",
    "num_nodes": ints; "visible_devices": list of ints).  kv: an object with
    ``set(key: str, value: bytes)`` and ``get(key: str) -> bytes`` (e.g. a
    torch.distributed store) used for multi-process NCCL bootstrap.
    """

    def __init__(self, options: Optional[dict] = None, kv=None):
        self._keep = []
        opts = []
        for k, v in (options or {}).items():
            nv = NamedValue()
            nv.struct_size = C.sizeof(NamedValue)
            kb = k.encode()
            self._keep.append(kb)
            nv.name, nv.name_size = kb, len(kb)
            if isinstance(v, (list, tuple)):
                arr = (C.c_int64 * len(v))(*v)
                self._keep.append(arr)
                nv.type, nv.int64_array_value, nv.value_size = 2, C.cast(arr, C.POINTER(C.c_int64)), len(v)
            else:
                nv.type, nv.int64_value, nv.value_size = 1, int(v), 1
            opts.append(nv)
        arr = (NamedValue * max(len(opts), 1))(*opts)
        get_cb = put_cb = None
        if kv is not None:
            get_cb, put_cb, keep = kv_callbacks(kv)
            self._keep += keep
        a = api().call("Client_Create", create_options=C.cast(arr, C.POINTER(NamedValue)),
                       num_options=len(opts),
                       kv_get_callback=C.cast(get_cb, C.c_void_p) if get_cb else None,
                       kv_put_callback=C.cast(put_cb, C.c_void_p) if put_cb else None)
        self.handle = a.client
        d = api().call("Client_Devices", client=self.handle)
        self.devices = [d.devices[i] for i in range(d.num_devices)]
        ad = api().call("Client_AddressableDevices", client=self.handle)
        self.addressable_devices = [ad.addressable_devices[i] for i in range(ad.num_addressable_devices)]

    @property
    def platform_name(self) -> str:
        a = api().call("Client_PlatformName", client=self.handle)
        return C.string_at(a.platform_name, a.platform_name_size).decode()

    @property
    def platform_version(self) -> str:
        a = api().call("Client_PlatformVersion", client=self.handle)
        return C.string_at(a.platform_version, a.platform_version_size).decode()

    def device_id(self, dev: int) -> int:
        desc = api().call("Device_GetDescription", device=dev).device_description
        return api().call("DeviceDescription_Id", device_description=desc).id

    def device_kind(self, dev: int) -> str:
        desc = api().call("Device_GetDescription", device=dev).device_description
        a = api().call("DeviceDescription_Kind", device_description=desc)
        return C.string_at(a.device_kind, a.device_kind_size).decode()

    def device_stream(self, dev: Optional[int] = None) -> int:
        """cudaStream_t the plugin uses for `dev` (event timing, profiling)."""
        f = api().lib.b200_pjrt_device_stream
        f.restype, f.argtypes = C.c_void_p, [C.c_void_p]
        return f(dev if dev is not None else self.addressable_devices[0]) or 0

    def memory_stats(self, dev: int) -> dict:
        a = api().call("Device_MemoryStats", device=dev)
        return {"bytes_in_use": a.bytes_in_use, "peak_bytes_in_use": a.peak_bytes_in_use,
                "bytes_reserved": a.bytes_reserved, "num_allocs": a.num_allocs}

    def compile(self, mlir_text: str, compile_options: bytes = b"") -> Executable:
        code = mlir_text.encode() if isinstance(mlir_text, str) else mlir_text
        prog = ProgramStruct()
        prog.struct_size = C.sizeof(ProgramStruct)
        cbuf = C.create_string_buffer(code, len(code))
        prog.code = C.cast(cbuf, C.c_char_p)
        prog.code_size = len(code)
        prog.format, prog.format_size = b"mlir", 4
        a = api().call("Client_Compile", client=self.handle, program=C.addressof(prog),
                       compile_options=compile_options, compile_options_size=len(compile_options))
        return Executable(self, a.executable)

    def deserialize(self, data: bytes) -> Executable:
        buf = C.create_string_buffer(data, len(data))
        a = api().call("Executable_DeserializeAndLoad", client=self.handle,
                       serialized_executable=C.addressof(buf), serialized_executable_size=len(data))
        return Executable(self, a.loaded_executable)

    def buffer_from_host_ptr(self, ptr: int, pjrt_type: int, shape: Sequence[int],
                             device: Optional[int] = None, semantics: int = 1):
        """Copy host memory at `ptr` (dense row-major) to a new device buffer.
        Returns (Buffer, done_event); the host memory must stay valid until
        done_event completes (semantics 1 = kImmutableUntilTransferCompletes)."""
        dims = (C.c_int64 * max(len(shape), 1))(*shape)
        a = api().call("Client_BufferFromHostBuffer", client=self.handle, data=ptr, type=pjrt_type,
                       dims=C.cast(dims, C.POINTER(C.c_int64)), num_dims=len(shape),
                       host_buffer_semantics=semantics,
                       device=device if device is not None else self.addressable_devices[0])
        return Buffer(self, a.buffer), a.done_with_host_buffer

    def buffer_from_numpy(self, x: np.ndarray, device: Optional[int] = None, bf16: bool = False) -> Buffer:
        x = np.require(x, requirements="C")  # keeps 0-d arrays 0-d
        t = BF16 if bf16 else _NP2PJRT[x.dtype]
        b, ev = self.buffer_from_host_ptr(x.ctypes.data, t, x.shape, device, semantics=0)
        api().await_event(ev)
        return b

    def destroy(self):
        if self.handle:
            api().call("Client_Destroy", client=self.handle)
            self.handle = None


def kv_exchange(store, rank: int, key: str, value: bytes = b"") -> bytes:
    """The plugin's NCCL-id exchange over `store` without a device
    (b200_pjrt_kv_exchange): rank 0 puts `value` under `key`, any other rank
    gets it.  Raises PjrtError with the plugin's code when the store fails."""
    lib = api().lib
    fn = lib.b200_pjrt_kv_exchange
    fn.argtypes = [C.c_void_p] * 4 + [C.c_int, C.c_char_p, C.c_size_t, C.c_char_p, C.c_size_t,
                                      C.POINTER(C.c_void_p), C.POINTER(C.c_size_t)]
    fn.restype = C.c_int
    lib.b200_pjrt_free.argtypes = [C.c_void_p]
    get_cb, put_cb, keep = kv_callbacks(store)
    out, n = C.c_void_p(), C.c_size_t(0)
    k = key.encode()
    rc = fn(C.cast(get_cb, C.c_void_p), None, C.cast(put_cb, C.c_void_p), None, rank, k, len(k),
            value, len(value), C.byref(out), C.byref(n))
    res = C.string_at(out.value, n.value)
    lib.b200_pjrt_free(out)
    del keep
    if rc:
        raise PjrtError(rc, res.decode(errors="replace"))
    return res


def kernel_launches() -> int:
    """Kernels started so far in this process: the plugin's generated kernels
    (b200_pjrt_kernel_launches) plus the hand-written ones of the kernel library
    it calls (b200_kernel_launches).  Read before and after a region to count
    its launches."""
    from . import kernels
    f = api().lib.b200_pjrt_kernel_launches
    f.restype, f.argtypes = C.c_uint64, []
    return int(f()) + int(kernels.lib().b200_kernel_launches())


def inspect(mlir_text, what: int = 1) -> str:
    """Run the compile pipeline without a device (see include/b200_pjrt_inspect.h).
    mlir_text: StableHLO text (str) or the program's bytes (text, or a portable
    artifact that needs jaxlib's MLIR C API in the process)."""
    lib = api().lib
    lib.b200_pjrt_inspect.argtypes = [C.c_char_p, C.c_size_t, C.c_int, C.POINTER(C.c_void_p)]
    lib.b200_pjrt_inspect.restype = C.c_int
    lib.b200_pjrt_free.argtypes = [C.c_void_p]
    out = C.c_void_p()
    b = mlir_text if isinstance(mlir_text, bytes) else mlir_text.encode()
    rc = lib.b200_pjrt_inspect(b, len(b), what, C.byref(out))
    s = C.string_at(out.value).decode()
    lib.b200_pjrt_free(out)
    if rc:
        raise PjrtError(rc, s)
    return s
