/*
 * b200_pjrt.h — the PJRT C ABI (version 0.90) as implemented by the B200 plugin.
 *
 * This header is this project's own statement of the PJRT plugin ABI that jaxlib
 * binds when it dlopen()s a plugin and calls GetPjrtApi().  It replaces the
 * reference's vendored XLA header (third_party/xla/pjrt/c/pjrt_c_api.h, API
 * version 0.90 at :92/:107, PJRT_Api table at :2758-2918).  Only the argument
 * structs that the plugin reads or writes are spelled out; every other slot of
 * the PJRT_Api table keeps its position through an opaque argument pointer.
 *
 * ABI rules that this file must keep (a mismatch is a silent memory corruption
 * in the caller):
 *   - every *_Args struct starts with {size_t struct_size; PJRT_Extension_Base*},
 *   - field order and types of each struct are those of the 0.90 ABI,
 *   - the PJRT_Api function-pointer slots appear in exactly the 0.90 order.
 *
 * Entry point (replaces reference src/jax_mlx_pjrt.cpp:9481-9483):
 *   const PJRT_Api* GetPjrtApi(void);
 */
#ifndef B200_PJRT_H_
#define B200_PJRT_H_

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200_PJRT_API_MAJOR 0
#define B200_PJRT_API_MINOR 90

/* Size of a struct up to and including `last`: the value callers put in
 * struct_size, so that older callers can pass shorter structs. */
#define B200_PJRT_SIZE_UPTO(T, last) (offsetof(T, last) + sizeof(((T*)0)->last))

typedef struct PJRT_Error PJRT_Error;
typedef struct PJRT_Event PJRT_Event;
typedef struct PJRT_Client PJRT_Client;
typedef struct PJRT_Device PJRT_Device;
typedef struct PJRT_DeviceDescription PJRT_DeviceDescription;
typedef struct PJRT_Memory PJRT_Memory;
typedef struct PJRT_Executable PJRT_Executable;
typedef struct PJRT_LoadedExecutable PJRT_LoadedExecutable;
typedef struct PJRT_Buffer PJRT_Buffer;
typedef struct PJRT_TopologyDescription PJRT_TopologyDescription;
typedef struct PJRT_ExecuteContext PJRT_ExecuteContext;
typedef struct PJRT_SerializedExecutable PJRT_SerializedExecutable;
typedef struct PJRT_SerializedCompileOptions PJRT_SerializedCompileOptions;
typedef struct PJRT_SerializedTopology PJRT_SerializedTopology;
typedef struct PJRT_DeviceAssignmentSerialized PJRT_DeviceAssignmentSerialized;
typedef struct PJRT_SendCallbackInfo PJRT_SendCallbackInfo;
typedef struct PJRT_RecvCallbackInfo PJRT_RecvCallbackInfo;

typedef struct PJRT_Extension_Base {
  size_t struct_size;
  int type; /* PJRT_Extension_Type */
  struct PJRT_Extension_Base* next;
} PJRT_Extension_Base;

typedef struct PJRT_Api_Version {
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  int major_version;
  int minor_version;
} PJRT_Api_Version;

/* ------------------------------------------------------------- enums ---- */
typedef enum {
  PJRT_Error_Code_OK = 0,
  PJRT_Error_Code_CANCELLED = 1,
  PJRT_Error_Code_UNKNOWN = 2,
  PJRT_Error_Code_INVALID_ARGUMENT = 3,
  PJRT_Error_Code_DEADLINE_EXCEEDED = 4,
  PJRT_Error_Code_NOT_FOUND = 5,
  PJRT_Error_Code_ALREADY_EXISTS = 6,
  PJRT_Error_Code_PERMISSION_DENIED = 7,
  PJRT_Error_Code_RESOURCE_EXHAUSTED = 8,
  PJRT_Error_Code_FAILED_PRECONDITION = 9,
  PJRT_Error_Code_ABORTED = 10,
  PJRT_Error_Code_OUT_OF_RANGE = 11,
  PJRT_Error_Code_UNIMPLEMENTED = 12,
  PJRT_Error_Code_INTERNAL = 13,
  PJRT_Error_Code_UNAVAILABLE = 14,
  PJRT_Error_Code_DATA_LOSS = 15,
  PJRT_Error_Code_UNAUTHENTICATED = 16
} PJRT_Error_Code;

typedef enum {
  PJRT_NamedValue_kString = 0,
  PJRT_NamedValue_kInt64,
  PJRT_NamedValue_kInt64List,
  PJRT_NamedValue_kFloat,
  PJRT_NamedValue_kBool
} PJRT_NamedValue_Type;

/* Element types, numbered as in the 0.90 ABI. */
typedef enum {
  PJRT_Buffer_Type_INVALID = 0,
  PJRT_Buffer_Type_PRED,
  PJRT_Buffer_Type_S8,
  PJRT_Buffer_Type_S16,
  PJRT_Buffer_Type_S32,
  PJRT_Buffer_Type_S64,
  PJRT_Buffer_Type_U8,
  PJRT_Buffer_Type_U16,
  PJRT_Buffer_Type_U32,
  PJRT_Buffer_Type_U64,
  PJRT_Buffer_Type_F16,
  PJRT_Buffer_Type_F32,
  PJRT_Buffer_Type_F64,
  PJRT_Buffer_Type_BF16,
  PJRT_Buffer_Type_C64,
  PJRT_Buffer_Type_C128
  /* fp8/fp4/int4 follow in the ABI; the plugin rejects them. */
} PJRT_Buffer_Type;

typedef enum {
  PJRT_HostBufferSemantics_kImmutableOnlyDuringCall = 0,
  PJRT_HostBufferSemantics_kImmutableUntilTransferCompletes,
  PJRT_HostBufferSemantics_kImmutableZeroCopy,
  PJRT_HostBufferSemantics_kMutableZeroCopy
} PJRT_HostBufferSemantics;

typedef enum {
  PJRT_Buffer_MemoryLayout_Type_Tiled = 0,
  PJRT_Buffer_MemoryLayout_Type_Strides
} PJRT_Buffer_MemoryLayout_Type;

/* ------------------------------------------------------ named values ---- */
typedef struct PJRT_NamedValue {
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  const char* name;
  size_t name_size;
  PJRT_NamedValue_Type type;
  union {
    const char* string_value;
    int64_t int64_value;
    const int64_t* int64_array_value;
    float float_value;
    bool bool_value;
  };
  size_t value_size; /* elements for lists/strings, 1 for scalars */
} PJRT_NamedValue;

/* Callback types carried by PJRT_Client_Create. */
typedef PJRT_Error* (*PJRT_CallbackError)(PJRT_Error_Code code, const char* message,
                                          size_t message_size);
typedef void (*PJRT_KeyValueGetCallback_ValueDeleter)(char* value);
typedef struct PJRT_KeyValueGetCallback_Args {
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  const char* key;
  size_t key_size;
  int timeout_in_ms;
  PJRT_CallbackError* callback_error;
  void* user_arg;
  char* value; /* out */
  size_t value_size;
  PJRT_KeyValueGetCallback_ValueDeleter value_deleter_callback;
} PJRT_KeyValueGetCallback_Args;
typedef PJRT_Error* (*PJRT_KeyValueGetCallback)(PJRT_KeyValueGetCallback_Args* args);

typedef struct PJRT_KeyValuePutCallback_Args {
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  const char* key;
  size_t key_size;
  const char* value;
  size_t value_size;
  PJRT_CallbackError* callback_error;
  void* user_arg;
} PJRT_KeyValuePutCallback_Args;
typedef PJRT_Error* (*PJRT_KeyValuePutCallback)(PJRT_KeyValuePutCallback_Args* args);
typedef void* PJRT_KeyValueTryGetCallback; /* slot only; not used */

typedef void (*PJRT_Event_OnReadyCallback)(PJRT_Error* error, void* user_arg);

/* Shorthand for the common header of every argument struct. */
#define B200_ARGS_HEAD            \
  size_t struct_size;             \
  PJRT_Extension_Base* extension_start

/* -------------------------------------------------------------- errors -- */
typedef struct { B200_ARGS_HEAD; PJRT_Error* error; } PJRT_Error_Destroy_Args;
typedef struct { B200_ARGS_HEAD; const PJRT_Error* error; const char* message; size_t message_size; } PJRT_Error_Message_Args;
typedef struct { B200_ARGS_HEAD; const PJRT_Error* error; PJRT_Error_Code code; } PJRT_Error_GetCode_Args;

/* -------------------------------------------------------------- plugin -- */
typedef struct { B200_ARGS_HEAD; } PJRT_Plugin_Initialize_Args;
typedef struct { B200_ARGS_HEAD; const PJRT_NamedValue* attributes; size_t num_attributes; } PJRT_Plugin_Attributes_Args;

/* -------------------------------------------------------------- events -- */
typedef struct { B200_ARGS_HEAD; PJRT_Event* event; } PJRT_Event_Destroy_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Event* event; bool is_ready; } PJRT_Event_IsReady_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Event* event; } PJRT_Event_Error_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Event* event; } PJRT_Event_Await_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Event* event; PJRT_Event_OnReadyCallback callback; void* user_arg; } PJRT_Event_OnReady_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Event* event; } PJRT_Event_Create_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Event* event; PJRT_Error_Code error_code; const char* error_message; size_t error_message_size; } PJRT_Event_Set_Args;

/* -------------------------------------------------------------- client -- */
typedef struct {
  B200_ARGS_HEAD;
  const PJRT_NamedValue* create_options;
  size_t num_options;
  PJRT_KeyValueGetCallback kv_get_callback;
  void* kv_get_user_arg;
  PJRT_KeyValuePutCallback kv_put_callback;
  void* kv_put_user_arg;
  PJRT_Client* client; /* out */
  PJRT_KeyValueTryGetCallback kv_try_get_callback;
  void* kv_try_get_user_arg;
} PJRT_Client_Create_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Client* client; } PJRT_Client_Destroy_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Client* client; const char* platform_name; size_t platform_name_size; } PJRT_Client_PlatformName_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Client* client; int process_index; } PJRT_Client_ProcessIndex_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Client* client; const char* platform_version; size_t platform_version_size; } PJRT_Client_PlatformVersion_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Client* client; PJRT_TopologyDescription* topology; } PJRT_Client_TopologyDescription_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Client* client; PJRT_Device* const* devices; size_t num_devices; } PJRT_Client_Devices_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Client* client; PJRT_Device* const* addressable_devices; size_t num_addressable_devices; } PJRT_Client_AddressableDevices_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Client* client; int id; PJRT_Device* device; } PJRT_Client_LookupDevice_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Client* client; int local_hardware_id; PJRT_Device* addressable_device; } PJRT_Client_LookupAddressableDevice_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Client* client; PJRT_Memory* const* addressable_memories; size_t num_addressable_memories; } PJRT_Client_AddressableMemories_Args;

typedef struct PJRT_Program {
  B200_ARGS_HEAD;
  char* code;
  size_t code_size;
  const char* format; /* "mlir" (text or portable-artifact bytecode) */
  size_t format_size;
} PJRT_Program;

typedef struct { B200_ARGS_HEAD; PJRT_Client* client; const PJRT_Program* program; const char* compile_options; size_t compile_options_size; PJRT_LoadedExecutable* executable; } PJRT_Client_Compile_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Client* client; int num_replicas; int num_partitions; size_t default_assignment_size; int* default_assignment; } PJRT_Client_DefaultDeviceAssignment_Args;

typedef struct {
  B200_ARGS_HEAD;
  const int64_t* minor_to_major;
  size_t minor_to_major_size;
  const int64_t* tile_dims;
  const size_t* tile_dim_sizes;
  size_t num_tiles;
} PJRT_Buffer_MemoryLayout_Tiled;
typedef struct { B200_ARGS_HEAD; const int64_t* byte_strides; size_t num_byte_strides; } PJRT_Buffer_MemoryLayout_Strides;
typedef struct PJRT_Buffer_MemoryLayout {
  B200_ARGS_HEAD;
  union {
    PJRT_Buffer_MemoryLayout_Tiled tiled;
    PJRT_Buffer_MemoryLayout_Strides strides;
  };
  PJRT_Buffer_MemoryLayout_Type type;
} PJRT_Buffer_MemoryLayout;

typedef struct {
  B200_ARGS_HEAD;
  PJRT_Client* client;
  const void* data;
  PJRT_Buffer_Type type;
  const int64_t* dims;
  size_t num_dims;
  const int64_t* byte_strides;
  size_t num_byte_strides;
  PJRT_HostBufferSemantics host_buffer_semantics;
  PJRT_Device* device;
  PJRT_Memory* memory;
  PJRT_Buffer_MemoryLayout* device_layout;
  PJRT_Event* done_with_host_buffer; /* out */
  PJRT_Buffer* buffer;               /* out */
} PJRT_Client_BufferFromHostBuffer_Args;

typedef struct {
  B200_ARGS_HEAD;
  PJRT_Client* client;
  void* device_buffer_ptr;
  const int64_t* dims;
  size_t num_dims;
  PJRT_Buffer_Type element_type;
  PJRT_Buffer_MemoryLayout* layout;
  PJRT_Device* device;
  void (*on_delete_callback)(void* device_buffer_ptr, void* user_arg);
  void* on_delete_callback_arg;
  intptr_t stream;
  PJRT_Buffer* buffer; /* out */
  PJRT_Memory* memory;
} PJRT_Client_CreateViewOfDeviceBuffer_Args;

typedef struct {
  B200_ARGS_HEAD;
  PJRT_Client* client;
  const int64_t* shape_dims;
  size_t shape_num_dims;
  PJRT_Buffer_Type shape_element_type;
  PJRT_Buffer_MemoryLayout* shape_layout;
  PJRT_Device* device;
  PJRT_Memory* memory;
  PJRT_Buffer* buffer; /* out */
} PJRT_Client_CreateUninitializedBuffer_Args;

/* -------------------------------------------------- device description -- */
typedef struct { B200_ARGS_HEAD; PJRT_DeviceDescription* device_description; int id; } PJRT_DeviceDescription_Id_Args;
typedef struct { B200_ARGS_HEAD; PJRT_DeviceDescription* device_description; int process_index; } PJRT_DeviceDescription_ProcessIndex_Args;
typedef struct { B200_ARGS_HEAD; PJRT_DeviceDescription* device_description; size_t num_attributes; const PJRT_NamedValue* attributes; } PJRT_DeviceDescription_Attributes_Args;
typedef struct { B200_ARGS_HEAD; PJRT_DeviceDescription* device_description; const char* device_kind; size_t device_kind_size; } PJRT_DeviceDescription_Kind_Args;
typedef struct { B200_ARGS_HEAD; PJRT_DeviceDescription* device_description; const char* debug_string; size_t debug_string_size; } PJRT_DeviceDescription_DebugString_Args;
typedef struct { B200_ARGS_HEAD; PJRT_DeviceDescription* device_description; const char* to_string; size_t to_string_size; } PJRT_DeviceDescription_ToString_Args;

/* -------------------------------------------------------------- device -- */
typedef struct { B200_ARGS_HEAD; PJRT_Device* device; PJRT_DeviceDescription* device_description; } PJRT_Device_GetDescription_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Device* device; bool is_addressable; } PJRT_Device_IsAddressable_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Device* device; int local_hardware_id; } PJRT_Device_LocalHardwareId_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Device* device; PJRT_Memory* const* memories; size_t num_memories; } PJRT_Device_AddressableMemories_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Device* device; PJRT_Memory* memory; } PJRT_Device_DefaultMemory_Args;
typedef struct {
  B200_ARGS_HEAD;
  PJRT_Device* device;
  int64_t bytes_in_use;
  int64_t peak_bytes_in_use;
  bool peak_bytes_in_use_is_set;
  int64_t num_allocs;
  bool num_allocs_is_set;
  int64_t largest_alloc_size;
  bool largest_alloc_size_is_set;
  int64_t bytes_limit;
  bool bytes_limit_is_set;
  int64_t bytes_reserved;
  bool bytes_reserved_is_set;
  int64_t peak_bytes_reserved;
  bool peak_bytes_reserved_is_set;
  int64_t bytes_reservable_limit;
  bool bytes_reservable_limit_is_set;
  int64_t largest_free_block_bytes;
  bool largest_free_block_bytes_is_set;
  int64_t pool_bytes;
  bool pool_bytes_is_set;
  int64_t peak_pool_bytes;
  bool peak_pool_bytes_is_set;
} PJRT_Device_MemoryStats_Args;

/* -------------------------------------------------------------- memory -- */
typedef struct { B200_ARGS_HEAD; PJRT_Memory* memory; int id; } PJRT_Memory_Id_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Memory* memory; const char* kind; size_t kind_size; } PJRT_Memory_Kind_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Memory* memory; int kind_id; } PJRT_Memory_Kind_Id_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Memory* memory; const char* debug_string; size_t debug_string_size; } PJRT_Memory_DebugString_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Memory* memory; const char* to_string; size_t to_string_size; } PJRT_Memory_ToString_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Memory* memory; PJRT_Device* const* devices; size_t num_devices; } PJRT_Memory_AddressableByDevices_Args;

/* ---------------------------------------------------------- executable -- */
typedef struct { B200_ARGS_HEAD; PJRT_Executable* executable; } PJRT_Executable_Destroy_Args;
typedef struct { B200_ARGS_HEAD; PJRT_LoadedExecutable* executable; } PJRT_LoadedExecutable_Destroy_Args;
typedef struct { B200_ARGS_HEAD; PJRT_LoadedExecutable* loaded_executable; PJRT_Executable* executable; } PJRT_LoadedExecutable_GetExecutable_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Executable* executable; const char* executable_name; size_t executable_name_size; } PJRT_Executable_Name_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Executable* executable; size_t num_replicas; } PJRT_Executable_NumReplicas_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Executable* executable; size_t num_partitions; } PJRT_Executable_NumPartitions_Args;
typedef struct { B200_ARGS_HEAD; PJRT_LoadedExecutable* executable; PJRT_Device* const* addressable_devices; size_t num_addressable_devices; } PJRT_LoadedExecutable_AddressableDevices_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Executable* executable; PJRT_Program* program; } PJRT_Executable_OptimizedProgram_Args;
typedef struct { B200_ARGS_HEAD; PJRT_LoadedExecutable* executable; } PJRT_LoadedExecutable_Delete_Args;
typedef struct { B200_ARGS_HEAD; PJRT_LoadedExecutable* executable; bool is_deleted; } PJRT_LoadedExecutable_IsDeleted_Args;

typedef struct PJRT_ExecuteOptions {
  B200_ARGS_HEAD;
  PJRT_SendCallbackInfo** send_callbacks;
  PJRT_RecvCallbackInfo** recv_callbacks;
  size_t num_send_ops;
  size_t num_recv_ops;
  int launch_id;
  const int64_t* non_donatable_input_indices;
  size_t num_non_donatable_input_indices;
  PJRT_ExecuteContext* context;
  const char* call_location;
  size_t num_tasks;
  int* task_ids;
  int64_t* incarnation_ids;
} PJRT_ExecuteOptions;

typedef struct {
  B200_ARGS_HEAD;
  PJRT_LoadedExecutable* executable;
  PJRT_ExecuteOptions* options;
  PJRT_Buffer* const* const* argument_lists; /* [num_devices][num_args] */
  size_t num_devices;
  size_t num_args;
  PJRT_Buffer** const* output_lists; /* [num_devices][num_outputs], caller-allocated */
  PJRT_Event** device_complete_events; /* [num_devices] or NULL */
  PJRT_Device* execute_device;
} PJRT_LoadedExecutable_Execute_Args;

typedef struct { B200_ARGS_HEAD; PJRT_Executable* executable; size_t num_outputs; } PJRT_Executable_NumOutputs_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Executable* executable; int64_t size_in_bytes; } PJRT_Executable_SizeOfGeneratedCodeInBytes_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Executable* executable; const char* executable_fingerprint; size_t executable_fingerprint_size; } PJRT_Executable_Fingerprint_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Executable* executable; size_t num_properties; const PJRT_NamedValue* properties; } PJRT_Executable_GetCostAnalysis_Args;
typedef struct {
  B200_ARGS_HEAD;
  PJRT_Executable* executable;
  int64_t generated_code_size_in_bytes;
  int64_t argument_size_in_bytes;
  int64_t output_size_in_bytes;
  int64_t alias_size_in_bytes;
  int64_t temp_size_in_bytes;
  int64_t host_generated_code_size_in_bytes;
  int64_t host_argument_size_in_bytes;
  int64_t host_output_size_in_bytes;
  int64_t host_alias_size_in_bytes;
  int64_t host_temp_size_in_bytes;
  int64_t peak_memory_in_bytes;
  int64_t total_size_in_bytes;
} PJRT_Executable_GetCompiledMemoryStats_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Executable* executable; PJRT_Buffer_Type* output_types; size_t num_output_types; } PJRT_Executable_OutputElementTypes_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Executable* executable; size_t num_outputs; const int64_t* dims; const size_t* dim_sizes; } PJRT_Executable_OutputDimensions_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Executable* executable; size_t num_outputs; const char* const* memory_kinds; const size_t* memory_kind_sizes; } PJRT_Executable_OutputMemoryKinds_Args;
typedef struct {
  B200_ARGS_HEAD;
  const PJRT_Executable* executable;
  const char* serialized_bytes;
  size_t serialized_bytes_size;
  PJRT_SerializedExecutable* serialized_executable;
  void (*serialized_executable_deleter)(PJRT_SerializedExecutable* exec);
} PJRT_Executable_Serialize_Args;
typedef struct {
  B200_ARGS_HEAD;
  PJRT_Executable* executable;
  const char* serialized_bytes;
  size_t serialized_bytes_size;
  PJRT_SerializedCompileOptions* serialized_compile_options;
  void (*serialized_compile_options_deleter)(PJRT_SerializedCompileOptions* options);
} PJRT_Executable_GetCompileOptions_Args;
typedef struct {
  B200_ARGS_HEAD;
  PJRT_Client* client;
  const char* serialized_executable;
  size_t serialized_executable_size;
  PJRT_LoadedExecutable* loaded_executable;
  const char* overridden_serialized_compile_options;
  size_t overridden_serialized_compile_options_size;
} PJRT_Executable_DeserializeAndLoad_Args;
typedef struct { B200_ARGS_HEAD; PJRT_LoadedExecutable* executable; const char* executable_fingerprint; size_t executable_fingerprint_size; } PJRT_LoadedExecutable_Fingerprint_Args;
typedef struct {
  B200_ARGS_HEAD;
  PJRT_LoadedExecutable* executable;
  const char* serialized_bytes;
  size_t serialized_bytes_size;
  PJRT_DeviceAssignmentSerialized* serialized_device_assignment;
  void (*serialized_device_assignment_deleter)(PJRT_DeviceAssignmentSerialized* da);
} PJRT_LoadedExecutable_GetDeviceAssignment_Args;

/* -------------------------------------------------------------- buffer -- */
typedef struct { B200_ARGS_HEAD; PJRT_Buffer* buffer; } PJRT_Buffer_Destroy_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Buffer* buffer; PJRT_Buffer_Type type; } PJRT_Buffer_ElementType_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Buffer* buffer; const int64_t* dims; size_t num_dims; } PJRT_Buffer_Dimensions_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Buffer* buffer; const int64_t* unpadded_dims; size_t num_dims; } PJRT_Buffer_UnpaddedDimensions_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Buffer* buffer; const size_t* dynamic_dim_indices; size_t num_dynamic_dims; } PJRT_Buffer_DynamicDimensionIndices_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Buffer* buffer; PJRT_Buffer_MemoryLayout layout; } PJRT_Buffer_GetMemoryLayout_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Buffer* src; PJRT_Buffer_MemoryLayout* host_layout; void* dst; size_t dst_size; PJRT_Event* event; } PJRT_Buffer_ToHostBuffer_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Buffer* buffer; size_t on_device_size_in_bytes; } PJRT_Buffer_OnDeviceSizeInBytes_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Buffer* buffer; } PJRT_Buffer_Delete_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Buffer* buffer; bool is_deleted; } PJRT_Buffer_IsDeleted_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Buffer* buffer; void* dst; int64_t offset; int64_t transfer_size; PJRT_Event* event; } PJRT_Buffer_CopyRawToHost_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Buffer* buffer; PJRT_Device* dst_device; PJRT_Buffer* dst_buffer; } PJRT_Buffer_CopyToDevice_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Buffer* buffer; PJRT_Memory* dst_memory; PJRT_Buffer* dst_buffer; } PJRT_Buffer_CopyToMemory_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Buffer* buffer; bool is_on_cpu; } PJRT_Buffer_IsOnCpu_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Buffer* buffer; PJRT_Device* device; } PJRT_Buffer_Device_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Buffer* buffer; PJRT_Memory* memory; } PJRT_Buffer_Memory_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Buffer* buffer; PJRT_Event* event; } PJRT_Buffer_ReadyEvent_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Buffer* buffer; uintptr_t buffer_pointer; } PJRT_Buffer_UnsafePointer_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Buffer* buffer; } PJRT_Buffer_IncreaseExternalReferenceCount_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Buffer* buffer; } PJRT_Buffer_DecreaseExternalReferenceCount_Args;
typedef struct { B200_ARGS_HEAD; PJRT_Buffer* buffer; void* device_memory_ptr; } PJRT_Buffer_OpaqueDeviceMemoryDataPointer_Args;

/* ------------------------------------------------------------ topology -- */
typedef struct { B200_ARGS_HEAD; const char* topology_name; size_t topology_name_size; const PJRT_NamedValue* create_options; size_t num_options; PJRT_TopologyDescription* topology; } PJRT_TopologyDescription_Create_Args;
typedef struct { B200_ARGS_HEAD; PJRT_TopologyDescription* topology; } PJRT_TopologyDescription_Destroy_Args;
typedef struct { B200_ARGS_HEAD; PJRT_TopologyDescription* topology; const char* platform_version; size_t platform_version_size; } PJRT_TopologyDescription_PlatformVersion_Args;
typedef struct { B200_ARGS_HEAD; const PJRT_TopologyDescription* topology; const char* platform_name; size_t platform_name_size; } PJRT_TopologyDescription_PlatformName_Args;
typedef struct { B200_ARGS_HEAD; const PJRT_TopologyDescription* topology; PJRT_DeviceDescription* const* descriptions; size_t num_descriptions; } PJRT_TopologyDescription_GetDeviceDescriptions_Args;
typedef struct { B200_ARGS_HEAD; PJRT_TopologyDescription* topology; const PJRT_NamedValue* attributes; size_t num_attributes; } PJRT_TopologyDescription_Attributes_Args;
typedef struct { B200_ARGS_HEAD; const PJRT_TopologyDescription* topology; const PJRT_Program* program; const char* compile_options; size_t compile_options_size; PJRT_Client* client; PJRT_Executable* executable; } PJRT_Compile_Args;

/* ---------------------------------------------------------- API table -- */
/* Every slot of the 0.90 PJRT_Api table, in ABI order.  X(Name) expands to a
 * pointer `PJRT_Error* (*PJRT_Name)(PJRT_Name_Args*)`. */
#define B200_PJRT_API_SLOTS(X)                                                       \
  X(Error_Destroy) X(Error_Message) X(Error_GetCode)                                 \
  X(Plugin_Initialize) X(Plugin_Attributes)                                          \
  X(Event_Destroy) X(Event_IsReady) X(Event_Error) X(Event_Await) X(Event_OnReady)   \
  X(Client_Create) X(Client_Destroy) X(Client_PlatformName) X(Client_ProcessIndex)   \
  X(Client_PlatformVersion) X(Client_Devices) X(Client_AddressableDevices)           \
  X(Client_LookupDevice) X(Client_LookupAddressableDevice)                           \
  X(Client_AddressableMemories) X(Client_Compile) X(Client_DefaultDeviceAssignment)  \
  X(Client_BufferFromHostBuffer)                                                     \
  X(DeviceDescription_Id) X(DeviceDescription_ProcessIndex)                          \
  X(DeviceDescription_Attributes) X(DeviceDescription_Kind)                          \
  X(DeviceDescription_DebugString) X(DeviceDescription_ToString)                     \
  X(Device_GetDescription) X(Device_IsAddressable) X(Device_LocalHardwareId)         \
  X(Device_AddressableMemories) X(Device_DefaultMemory) X(Device_MemoryStats)        \
  X(Memory_Id) X(Memory_Kind) X(Memory_DebugString) X(Memory_ToString)               \
  X(Memory_AddressableByDevices)                                                     \
  X(Executable_Destroy) X(Executable_Name) X(Executable_NumReplicas)                 \
  X(Executable_NumPartitions) X(Executable_NumOutputs)                               \
  X(Executable_SizeOfGeneratedCodeInBytes) X(Executable_GetCostAnalysis)             \
  X(Executable_OutputMemoryKinds) X(Executable_OptimizedProgram)                     \
  X(Executable_Serialize)                                                            \
  X(LoadedExecutable_Destroy) X(LoadedExecutable_GetExecutable)                      \
  X(LoadedExecutable_AddressableDevices) X(LoadedExecutable_Delete)                  \
  X(LoadedExecutable_IsDeleted) X(LoadedExecutable_Execute)                          \
  X(Executable_DeserializeAndLoad) X(LoadedExecutable_Fingerprint)                   \
  X(Buffer_Destroy) X(Buffer_ElementType) X(Buffer_Dimensions)                       \
  X(Buffer_UnpaddedDimensions) X(Buffer_DynamicDimensionIndices)                     \
  X(Buffer_GetMemoryLayout) X(Buffer_OnDeviceSizeInBytes) X(Buffer_Device)           \
  X(Buffer_Memory) X(Buffer_Delete) X(Buffer_IsDeleted) X(Buffer_CopyToDevice)       \
  X(Buffer_ToHostBuffer) X(Buffer_IsOnCpu) X(Buffer_ReadyEvent)                      \
  X(Buffer_UnsafePointer) X(Buffer_IncreaseExternalReferenceCount)                   \
  X(Buffer_DecreaseExternalReferenceCount) X(Buffer_OpaqueDeviceMemoryDataPointer)   \
  X(CopyToDeviceStream_Destroy) X(CopyToDeviceStream_AddChunk)                       \
  X(CopyToDeviceStream_TotalBytes) X(CopyToDeviceStream_GranuleSize)                 \
  X(CopyToDeviceStream_CurrentBytes)                                                 \
  X(TopologyDescription_Create) X(TopologyDescription_Destroy)                       \
  X(TopologyDescription_PlatformName) X(TopologyDescription_PlatformVersion)         \
  X(TopologyDescription_GetDeviceDescriptions) X(TopologyDescription_Serialize)      \
  X(TopologyDescription_Attributes)                                                  \
  X(Compile)                                                                         \
  X(Executable_OutputElementTypes) X(Executable_OutputDimensions)                    \
  X(Buffer_CopyToMemory) X(Client_CreateViewOfDeviceBuffer)                          \
  X(Executable_Fingerprint) X(Client_TopologyDescription)                            \
  X(Executable_GetCompiledMemoryStats) X(Memory_Kind_Id)                             \
  X(ExecuteContext_Create) X(ExecuteContext_Destroy) X(Buffer_CopyRawToHost)         \
  X(AsyncHostToDeviceTransferManager_Destroy)                                        \
  X(AsyncHostToDeviceTransferManager_TransferData)                                   \
  X(Client_CreateBuffersForAsyncHostToDevice)                                        \
  X(AsyncHostToDeviceTransferManager_RetrieveBuffer)                                 \
  X(AsyncHostToDeviceTransferManager_Device)                                         \
  X(AsyncHostToDeviceTransferManager_BufferCount)                                    \
  X(AsyncHostToDeviceTransferManager_BufferSize)                                     \
  X(AsyncHostToDeviceTransferManager_SetBufferError)                                 \
  X(AsyncHostToDeviceTransferManager_AddMetadata)                                    \
  X(Client_DmaMap) X(Client_DmaUnmap)                                                \
  X(Client_CreateUninitializedBuffer) X(Client_UpdateGlobalProcessInfo)              \
  X(TopologyDescription_Deserialize) X(Client_CreateAliasBuffer)                     \
  X(Client_FulfillAliasBuffer) X(LoadedExecutable_GetDeviceAssignment)               \
  X(Client_CreateErrorBuffer) X(AsyncHostToDeviceTransferManager_TransferLiteral)    \
  X(Buffer_CopyRawToHostFuture) X(Device_PoisonExecution)                            \
  X(Device_CreateAsyncTrackingEvent) X(AsyncTrackingEvent_Destroy)                   \
  X(Executable_GetCompileOptions) X(Buffer_DonateWithControlDependency)              \
  X(Event_Create) X(Event_Set)

#define B200_PJRT_SLOT_FIELD(name) PJRT_Error* (*PJRT_##name)(struct PJRT_##name##_Args_* args);

/* Argument structs of slots the plugin does not implement stay incomplete. */
typedef struct PJRT_Api {
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  PJRT_Api_Version pjrt_api_version;
  B200_PJRT_API_SLOTS(B200_PJRT_SLOT_FIELD)
} PJRT_Api;

#define B200_PJRT_API_NUM_SLOTS 128

/* The one exported symbol of libb200_pjrt.so. */
__attribute__((visibility("default"))) const PJRT_Api* GetPjrtApi(void);

#ifdef __cplusplus
}
#endif
#endif /* B200_PJRT_H_ */
