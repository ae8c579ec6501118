/* pjrt_b200_abi.h — the PJRT C-API v0.55 binary interface, restated for the B200 plugin.
 *
 * A PJRT plugin is a shared library whose only export is `GetPjrtApi()`, returning a table of
 * function pointers; every entry takes one "Args" struct that begins with `struct_size` and
 * `extension_start`.  The layout (field order and types) must match the caller's copy of the
 * header exactly, so this file restates, field for field, the structs of openxla/xla
 * `xla/pjrt/c/pjrt_c_api.h` at commit 76da7301 (API major 0, minor 55) — the version the
 * reference plugin vendors at third_party/xla/pjrt/c/pjrt_c_api.h:67,82 (PROVENANCE.md:6-8).
 *
 * Only the Args structs of the entry points this plugin implements are defined in full; every
 * other table slot is declared with an incomplete Args type (a pointer to it has the same ABI).
 * tests/test_abi_layout.py checks every offset here against a fixture generated from the
 * upstream header (tests/golden/pjrt_abi_offsets.json).
 */
#ifndef PJRT_B200_ABI_H_
#define PJRT_B200_ABI_H_

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PJRT_API_MAJOR 0
#define PJRT_API_MINOR 55

typedef enum {
  PJRT_Extension_Type_Gpu_Custom_Call = 0,
  PJRT_Extension_Type_Profiler,
  PJRT_Extension_Type_Custom_Partitioner,
  PJRT_Extension_Type_Stream,
  PJRT_Extension_Type_Layouts,
  PJRT_Extension_Type_FFI,
} PJRT_Extension_Type;

typedef struct PJRT_Extension_Base {
  size_t struct_size;
  PJRT_Extension_Type type;
  struct PJRT_Extension_Base* next;
} PJRT_Extension_Base;

/* Every Args struct starts with these two fields. */
#define PJRT_B200_HEAD          \
  size_t struct_size;           \
  PJRT_Extension_Base* extension_start

typedef struct PJRT_Api_Version {
  PJRT_B200_HEAD;
  int major_version;
  int minor_version;
} PJRT_Api_Version;

/* ---- opaque handles (defined by the plugin) ---- */
typedef struct PJRT_Error PJRT_Error;
typedef struct PJRT_Event PJRT_Event;
typedef struct PJRT_Client PJRT_Client;
typedef struct PJRT_Device PJRT_Device;
typedef struct PJRT_Memory PJRT_Memory;
typedef struct PJRT_DeviceDescription PJRT_DeviceDescription;
typedef struct PJRT_TopologyDescription PJRT_TopologyDescription;
typedef struct PJRT_Executable PJRT_Executable;
typedef struct PJRT_LoadedExecutable PJRT_LoadedExecutable;
typedef struct PJRT_Buffer PJRT_Buffer;
typedef struct PJRT_ExecuteContext PJRT_ExecuteContext;
typedef struct PJRT_CopyToDeviceStream PJRT_CopyToDeviceStream;

typedef enum {
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

typedef PJRT_Error* (*PJRT_CallbackError)(PJRT_Error_Code code, const char* message,
                                          size_t message_size);

typedef enum {
  PJRT_NamedValue_kString = 0,
  PJRT_NamedValue_kInt64,
  PJRT_NamedValue_kInt64List,
  PJRT_NamedValue_kFloat,
  PJRT_NamedValue_kBool,
} PJRT_NamedValue_Type;

typedef struct PJRT_NamedValue {
  PJRT_B200_HEAD;
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
  size_t value_size;
} PJRT_NamedValue;

typedef enum {
  PJRT_Buffer_Type_INVALID,
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
  PJRT_Buffer_Type_C128,
  PJRT_Buffer_Type_F8E5M2,
  PJRT_Buffer_Type_F8E4M3FN,
  PJRT_Buffer_Type_F8E4M3B11FNUZ,
  PJRT_Buffer_Type_F8E5M2FNUZ,
  PJRT_Buffer_Type_F8E4M3FNUZ,
  PJRT_Buffer_Type_S4,
  PJRT_Buffer_Type_U4,
  PJRT_Buffer_Type_TOKEN,
  PJRT_Buffer_Type_S2,
  PJRT_Buffer_Type_U2,
  PJRT_Buffer_Type_F8E4M3,
  PJRT_Buffer_Type_F8E3M4,
} PJRT_Buffer_Type;

typedef enum {
  PJRT_HostBufferSemantics_kImmutableOnlyDuringCall,
  PJRT_HostBufferSemantics_kImmutableUntilTransferCompletes,
  PJRT_HostBufferSemantics_kImmutableZeroCopy,
  PJRT_HostBufferSemantics_kMutableZeroCopy,
} PJRT_HostBufferSemantics;

typedef enum {
  PJRT_Buffer_MemoryLayout_Type_Tiled = 0,
  PJRT_Buffer_MemoryLayout_Type_Strides,
} PJRT_Buffer_MemoryLayout_Type;

typedef struct PJRT_Buffer_MemoryLayout_Tiled {
  PJRT_B200_HEAD;
  const int64_t* minor_to_major;
  size_t minor_to_major_size;
  const int64_t* tile_dims;
  const size_t* tile_dim_sizes;
  size_t num_tiles;
} PJRT_Buffer_MemoryLayout_Tiled;

typedef struct PJRT_Buffer_MemoryLayout_Strides {
  PJRT_B200_HEAD;
  const int64_t* byte_strides;
  size_t num_byte_strides;
} PJRT_Buffer_MemoryLayout_Strides;

typedef struct PJRT_Buffer_MemoryLayout {
  PJRT_B200_HEAD;
  union {
    PJRT_Buffer_MemoryLayout_Tiled tiled;
    PJRT_Buffer_MemoryLayout_Strides strides;
  };
  PJRT_Buffer_MemoryLayout_Type type;
} PJRT_Buffer_MemoryLayout;

/* ---------------------------------------------------------------- errors */
typedef struct PJRT_Error_Destroy_Args { PJRT_B200_HEAD; PJRT_Error* error; } PJRT_Error_Destroy_Args;
typedef struct PJRT_Error_Message_Args {
  PJRT_B200_HEAD;
  const PJRT_Error* error;
  const char* message;
  size_t message_size;
} PJRT_Error_Message_Args;
typedef struct PJRT_Error_GetCode_Args {
  PJRT_B200_HEAD;
  const PJRT_Error* error;
  PJRT_Error_Code code;
} PJRT_Error_GetCode_Args;

/* ---------------------------------------------------------------- plugin */
typedef struct PJRT_Plugin_Initialize_Args { PJRT_B200_HEAD; } PJRT_Plugin_Initialize_Args;
typedef struct PJRT_Plugin_Attributes_Args {
  PJRT_B200_HEAD;
  const PJRT_NamedValue* attributes;
  size_t num_attributes;
} PJRT_Plugin_Attributes_Args;

/* ---------------------------------------------------------------- events */
typedef void (*PJRT_Event_OnReadyCallback)(PJRT_Error* error, void* user_arg);
typedef struct PJRT_Event_Destroy_Args { PJRT_B200_HEAD; PJRT_Event* event; } PJRT_Event_Destroy_Args;
typedef struct PJRT_Event_IsReady_Args { PJRT_B200_HEAD; PJRT_Event* event; bool is_ready; } PJRT_Event_IsReady_Args;
typedef struct PJRT_Event_Error_Args { PJRT_B200_HEAD; PJRT_Event* event; } PJRT_Event_Error_Args;
typedef struct PJRT_Event_Await_Args { PJRT_B200_HEAD; PJRT_Event* event; } PJRT_Event_Await_Args;
typedef struct PJRT_Event_OnReady_Args {
  PJRT_B200_HEAD;
  PJRT_Event* event;
  PJRT_Event_OnReadyCallback callback;
  void* user_arg;
} PJRT_Event_OnReady_Args;

/* ---------------------------------------------------------------- client */
typedef void (*PJRT_KeyValueGetCallback_ValueDeleter)(char* value);
typedef struct PJRT_KeyValueGetCallback_Args {
  PJRT_B200_HEAD;
  const char* key;
  size_t key_size;
  int timeout_in_ms;
  PJRT_CallbackError* callback_error;
  void* user_arg;
  char* value;
  size_t value_size;
  PJRT_KeyValueGetCallback_ValueDeleter value_deleter_callback;
} PJRT_KeyValueGetCallback_Args;
typedef PJRT_Error* (*PJRT_KeyValueGetCallback)(PJRT_KeyValueGetCallback_Args* args);
typedef struct PJRT_KeyValuePutCallback_Args {
  PJRT_B200_HEAD;
  const char* key;
  size_t key_size;
  const char* value;
  size_t value_size;
  PJRT_CallbackError* callback_error;
  void* user_arg;
} PJRT_KeyValuePutCallback_Args;
typedef PJRT_Error* (*PJRT_KeyValuePutCallback)(PJRT_KeyValuePutCallback_Args* args);

typedef struct PJRT_Client_Create_Args {
  PJRT_B200_HEAD;
  const PJRT_NamedValue* create_options;
  size_t num_options;
  PJRT_KeyValueGetCallback kv_get_callback;
  void* kv_get_user_arg;
  PJRT_KeyValuePutCallback kv_put_callback;
  void* kv_put_user_arg;
  PJRT_Client* client;
} PJRT_Client_Create_Args;
typedef struct PJRT_Client_Destroy_Args { PJRT_B200_HEAD; PJRT_Client* client; } PJRT_Client_Destroy_Args;
typedef struct PJRT_Client_PlatformName_Args {
  PJRT_B200_HEAD;
  PJRT_Client* client;
  const char* platform_name;
  size_t platform_name_size;
} PJRT_Client_PlatformName_Args;
typedef struct PJRT_Client_ProcessIndex_Args {
  PJRT_B200_HEAD;
  PJRT_Client* client;
  int process_index;
} PJRT_Client_ProcessIndex_Args;
typedef struct PJRT_Client_PlatformVersion_Args {
  PJRT_B200_HEAD;
  PJRT_Client* client;
  const char* platform_version;
  size_t platform_version_size;
} PJRT_Client_PlatformVersion_Args;
typedef struct PJRT_Client_TopologyDescription_Args {
  PJRT_B200_HEAD;
  PJRT_Client* client;
  PJRT_TopologyDescription* topology;
} PJRT_Client_TopologyDescription_Args;
typedef struct PJRT_Client_Devices_Args {
  PJRT_B200_HEAD;
  PJRT_Client* client;
  PJRT_Device* const* devices;
  size_t num_devices;
} PJRT_Client_Devices_Args;
typedef struct PJRT_Client_AddressableDevices_Args {
  PJRT_B200_HEAD;
  PJRT_Client* client;
  PJRT_Device* const* addressable_devices;
  size_t num_addressable_devices;
} PJRT_Client_AddressableDevices_Args;
typedef struct PJRT_Client_LookupDevice_Args {
  PJRT_B200_HEAD;
  PJRT_Client* client;
  int id;
  PJRT_Device* device;
} PJRT_Client_LookupDevice_Args;
typedef struct PJRT_Client_LookupAddressableDevice_Args {
  PJRT_B200_HEAD;
  PJRT_Client* client;
  int local_hardware_id;
  PJRT_Device* addressable_device;
} PJRT_Client_LookupAddressableDevice_Args;
typedef struct PJRT_Client_AddressableMemories_Args {
  PJRT_B200_HEAD;
  PJRT_Client* client;
  PJRT_Memory* const* addressable_memories;
  size_t num_addressable_memories;
} PJRT_Client_AddressableMemories_Args;

typedef struct PJRT_Program {
  PJRT_B200_HEAD;
  char* code;
  size_t code_size;
  const char* format;
  size_t format_size;
} PJRT_Program;

typedef struct PJRT_Client_Compile_Args {
  PJRT_B200_HEAD;
  PJRT_Client* client;
  const PJRT_Program* program;
  const char* compile_options;
  size_t compile_options_size;
  PJRT_LoadedExecutable* executable;
} PJRT_Client_Compile_Args;
typedef struct PJRT_Client_DefaultDeviceAssignment_Args {
  PJRT_B200_HEAD;
  PJRT_Client* client;
  int num_replicas;
  int num_partitions;
  size_t default_assignment_size;
  int* default_assignment;
} PJRT_Client_DefaultDeviceAssignment_Args;
typedef struct PJRT_Client_BufferFromHostBuffer_Args {
  PJRT_B200_HEAD;
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
  PJRT_Event* done_with_host_buffer;
  PJRT_Buffer* buffer;
} PJRT_Client_BufferFromHostBuffer_Args;

/* ---------------------------------------------------------------- device descriptions */
typedef struct PJRT_DeviceDescription_Id_Args {
  PJRT_B200_HEAD;
  PJRT_DeviceDescription* device_description;
  int id;
} PJRT_DeviceDescription_Id_Args;
typedef struct PJRT_DeviceDescription_ProcessIndex_Args {
  PJRT_B200_HEAD;
  PJRT_DeviceDescription* device_description;
  int process_index;
} PJRT_DeviceDescription_ProcessIndex_Args;
typedef struct PJRT_DeviceDescription_Attributes_Args {
  PJRT_B200_HEAD;
  PJRT_DeviceDescription* device_description;
  size_t num_attributes;
  const PJRT_NamedValue* attributes;
} PJRT_DeviceDescription_Attributes_Args;
typedef struct PJRT_DeviceDescription_Kind_Args {
  PJRT_B200_HEAD;
  PJRT_DeviceDescription* device_description;
  const char* device_kind;
  size_t device_kind_size;
} PJRT_DeviceDescription_Kind_Args;
typedef struct PJRT_DeviceDescription_DebugString_Args {
  PJRT_B200_HEAD;
  PJRT_DeviceDescription* device_description;
  const char* debug_string;
  size_t debug_string_size;
} PJRT_DeviceDescription_DebugString_Args;
typedef struct PJRT_DeviceDescription_ToString_Args {
  PJRT_B200_HEAD;
  PJRT_DeviceDescription* device_description;
  const char* to_string;
  size_t to_string_size;
} PJRT_DeviceDescription_ToString_Args;

/* ---------------------------------------------------------------- devices */
typedef struct PJRT_Device_GetDescription_Args {
  PJRT_B200_HEAD;
  PJRT_Device* device;
  PJRT_DeviceDescription* device_description;
} PJRT_Device_GetDescription_Args;
typedef struct PJRT_Device_IsAddressable_Args {
  PJRT_B200_HEAD;
  PJRT_Device* device;
  bool is_addressable;
} PJRT_Device_IsAddressable_Args;
typedef struct PJRT_Device_LocalHardwareId_Args {
  PJRT_B200_HEAD;
  PJRT_Device* device;
  int local_hardware_id;
} PJRT_Device_LocalHardwareId_Args;
typedef struct PJRT_Device_AddressableMemories_Args {
  PJRT_B200_HEAD;
  PJRT_Device* device;
  PJRT_Memory* const* memories;
  size_t num_memories;
} PJRT_Device_AddressableMemories_Args;
typedef struct PJRT_Device_DefaultMemory_Args {
  PJRT_B200_HEAD;
  PJRT_Device* device;
  PJRT_Memory* memory;
} PJRT_Device_DefaultMemory_Args;
typedef struct PJRT_Device_MemoryStats_Args {
  PJRT_B200_HEAD;
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

/* ---------------------------------------------------------------- memories */
typedef struct PJRT_Memory_Id_Args { PJRT_B200_HEAD; PJRT_Memory* memory; int id; } PJRT_Memory_Id_Args;
typedef struct PJRT_Memory_Kind_Args {
  PJRT_B200_HEAD;
  PJRT_Memory* memory;
  const char* kind;
  size_t kind_size;
} PJRT_Memory_Kind_Args;
typedef struct PJRT_Memory_Kind_Id_Args { PJRT_B200_HEAD; PJRT_Memory* memory; int kind_id; } PJRT_Memory_Kind_Id_Args;
typedef struct PJRT_Memory_DebugString_Args {
  PJRT_B200_HEAD;
  PJRT_Memory* memory;
  const char* debug_string;
  size_t debug_string_size;
} PJRT_Memory_DebugString_Args;
typedef struct PJRT_Memory_ToString_Args {
  PJRT_B200_HEAD;
  PJRT_Memory* memory;
  const char* to_string;
  size_t to_string_size;
} PJRT_Memory_ToString_Args;
typedef struct PJRT_Memory_AddressableByDevices_Args {
  PJRT_B200_HEAD;
  PJRT_Memory* memory;
  PJRT_Device* const* devices;
  size_t num_devices;
} PJRT_Memory_AddressableByDevices_Args;

/* ---------------------------------------------------------------- execute context */
typedef struct PJRT_ExecuteContext_Create_Args {
  PJRT_B200_HEAD;
  PJRT_ExecuteContext* context;
} PJRT_ExecuteContext_Create_Args;
typedef struct PJRT_ExecuteContext_Destroy_Args {
  PJRT_B200_HEAD;
  PJRT_ExecuteContext* context;
} PJRT_ExecuteContext_Destroy_Args;

/* ---------------------------------------------------------------- executables */
typedef struct PJRT_Executable_Destroy_Args { PJRT_B200_HEAD; PJRT_Executable* executable; } PJRT_Executable_Destroy_Args;
typedef struct PJRT_LoadedExecutable_Destroy_Args {
  PJRT_B200_HEAD;
  PJRT_LoadedExecutable* executable;
} PJRT_LoadedExecutable_Destroy_Args;
typedef struct PJRT_LoadedExecutable_GetExecutable_Args {
  PJRT_B200_HEAD;
  PJRT_LoadedExecutable* loaded_executable;
  PJRT_Executable* executable;
} PJRT_LoadedExecutable_GetExecutable_Args;
typedef struct PJRT_Executable_Name_Args {
  PJRT_B200_HEAD;
  PJRT_Executable* executable;
  const char* executable_name;
  size_t executable_name_size;
} PJRT_Executable_Name_Args;
typedef struct PJRT_Executable_NumReplicas_Args {
  PJRT_B200_HEAD;
  PJRT_Executable* executable;
  size_t num_replicas;
} PJRT_Executable_NumReplicas_Args;
typedef struct PJRT_Executable_NumPartitions_Args {
  PJRT_B200_HEAD;
  PJRT_Executable* executable;
  size_t num_partitions;
} PJRT_Executable_NumPartitions_Args;
typedef struct PJRT_LoadedExecutable_AddressableDevices_Args {
  PJRT_B200_HEAD;
  PJRT_LoadedExecutable* executable;
  PJRT_Device* const* addressable_devices;
  size_t num_addressable_devices;
} PJRT_LoadedExecutable_AddressableDevices_Args;
typedef struct PJRT_LoadedExecutable_Delete_Args {
  PJRT_B200_HEAD;
  PJRT_LoadedExecutable* executable;
} PJRT_LoadedExecutable_Delete_Args;
typedef struct PJRT_LoadedExecutable_IsDeleted_Args {
  PJRT_B200_HEAD;
  PJRT_LoadedExecutable* executable;
  bool is_deleted;
} PJRT_LoadedExecutable_IsDeleted_Args;

typedef struct PJRT_Chunk {
  void* data;
  size_t size;
  void (*deleter)(void* data, void* deleter_arg);
  void* deleter_arg;
} PJRT_Chunk;
typedef PJRT_Error* (*PJRT_SendCallback)(PJRT_Chunk* chunk, PJRT_CallbackError* callback_error,
                                         size_t total_size_in_bytes, bool done, void* user_arg);
typedef void (*PJRT_RecvCallback)(PJRT_CopyToDeviceStream* stream, void* user_arg);
typedef struct PJRT_SendCallbackInfo {
  int64_t channel_id;
  void* user_arg;
  PJRT_SendCallback send_callback;
} PJRT_SendCallbackInfo;
typedef struct PJRT_RecvCallbackInfo {
  int64_t channel_id;
  void* user_arg;
  PJRT_RecvCallback recv_callback;
} PJRT_RecvCallbackInfo;
typedef struct PJRT_ExecuteOptions {
  PJRT_B200_HEAD;
  PJRT_SendCallbackInfo** send_callbacks;
  PJRT_RecvCallbackInfo** recv_callbacks;
  size_t num_send_ops;
  size_t num_recv_ops;
  int launch_id;
  const int64_t* non_donatable_input_indices;
  size_t num_non_donatable_input_indices;
} PJRT_ExecuteOptions;
typedef struct PJRT_LoadedExecutable_Execute_Args {
  PJRT_B200_HEAD;
  PJRT_LoadedExecutable* executable;
  PJRT_ExecuteOptions* options;
  PJRT_Buffer* const* const* argument_lists;
  size_t num_devices;
  size_t num_args;
  PJRT_Buffer** const* output_lists;
  PJRT_Event** device_complete_events;
  PJRT_Device* execute_device;
} PJRT_LoadedExecutable_Execute_Args;
typedef struct PJRT_Executable_NumOutputs_Args {
  PJRT_B200_HEAD;
  PJRT_Executable* executable;
  size_t num_outputs;
} PJRT_Executable_NumOutputs_Args;
typedef struct PJRT_Executable_SizeOfGeneratedCodeInBytes_Args {
  PJRT_B200_HEAD;
  PJRT_Executable* executable;
  int64_t size_in_bytes;
} PJRT_Executable_SizeOfGeneratedCodeInBytes_Args;
typedef struct PJRT_Executable_Fingerprint_Args {
  PJRT_B200_HEAD;
  PJRT_Executable* executable;
  const char* executable_fingerprint;
  size_t executable_fingerprint_size;
} PJRT_Executable_Fingerprint_Args;
typedef struct PJRT_Executable_OutputElementTypes_Args {
  PJRT_B200_HEAD;
  PJRT_Executable* executable;
  PJRT_Buffer_Type* output_types;
  size_t num_output_types;
} PJRT_Executable_OutputElementTypes_Args;
typedef struct PJRT_Executable_OutputDimensions_Args {
  PJRT_B200_HEAD;
  PJRT_Executable* executable;
  size_t num_outputs;
  const int64_t* dims;
  const size_t* dim_sizes;
} PJRT_Executable_OutputDimensions_Args;
typedef struct PJRT_Executable_OutputMemoryKinds_Args {
  PJRT_B200_HEAD;
  PJRT_Executable* executable;
  size_t num_outputs;
  const char* const* memory_kinds;
  const size_t* memory_kind_sizes;
} PJRT_Executable_OutputMemoryKinds_Args;
typedef struct PJRT_LoadedExecutable_Fingerprint_Args {
  PJRT_B200_HEAD;
  PJRT_LoadedExecutable* executable;
  const char* executable_fingerprint;
  size_t executable_fingerprint_size;
} PJRT_LoadedExecutable_Fingerprint_Args;

/* ---------------------------------------------------------------- buffers */
typedef struct PJRT_Buffer_Destroy_Args { PJRT_B200_HEAD; PJRT_Buffer* buffer; } PJRT_Buffer_Destroy_Args;
typedef struct PJRT_Buffer_ElementType_Args {
  PJRT_B200_HEAD;
  PJRT_Buffer* buffer;
  PJRT_Buffer_Type type;
} PJRT_Buffer_ElementType_Args;
typedef struct PJRT_Buffer_Dimensions_Args {
  PJRT_B200_HEAD;
  PJRT_Buffer* buffer;
  const int64_t* dims;
  size_t num_dims;
} PJRT_Buffer_Dimensions_Args;
typedef struct PJRT_Buffer_UnpaddedDimensions_Args {
  PJRT_B200_HEAD;
  PJRT_Buffer* buffer;
  const int64_t* unpadded_dims;
  size_t num_dims;
} PJRT_Buffer_UnpaddedDimensions_Args;
typedef struct PJRT_Buffer_DynamicDimensionIndices_Args {
  PJRT_B200_HEAD;
  PJRT_Buffer* buffer;
  const size_t* dynamic_dim_indices;
  size_t num_dynamic_dims;
} PJRT_Buffer_DynamicDimensionIndices_Args;
typedef struct PJRT_Buffer_GetMemoryLayout_Args {
  PJRT_B200_HEAD;
  PJRT_Buffer* buffer;
  PJRT_Buffer_MemoryLayout layout;
} PJRT_Buffer_GetMemoryLayout_Args;
typedef struct PJRT_Buffer_ToHostBuffer_Args {
  PJRT_B200_HEAD;
  PJRT_Buffer* src;
  PJRT_Buffer_MemoryLayout* host_layout;
  void* dst;
  size_t dst_size;
  PJRT_Event* event;
} PJRT_Buffer_ToHostBuffer_Args;
typedef struct PJRT_Buffer_OnDeviceSizeInBytes_Args {
  PJRT_B200_HEAD;
  PJRT_Buffer* buffer;
  size_t on_device_size_in_bytes;
} PJRT_Buffer_OnDeviceSizeInBytes_Args;
typedef struct PJRT_Buffer_Delete_Args { PJRT_B200_HEAD; PJRT_Buffer* buffer; } PJRT_Buffer_Delete_Args;
typedef struct PJRT_Buffer_IsDeleted_Args {
  PJRT_B200_HEAD;
  PJRT_Buffer* buffer;
  bool is_deleted;
} PJRT_Buffer_IsDeleted_Args;
typedef struct PJRT_Buffer_CopyToDevice_Args {
  PJRT_B200_HEAD;
  PJRT_Buffer* buffer;
  PJRT_Device* dst_device;
  PJRT_Buffer* dst_buffer;
} PJRT_Buffer_CopyToDevice_Args;
typedef struct PJRT_Buffer_CopyToMemory_Args {
  PJRT_B200_HEAD;
  PJRT_Buffer* buffer;
  PJRT_Memory* dst_memory;
  PJRT_Buffer* dst_buffer;
} PJRT_Buffer_CopyToMemory_Args;
typedef struct PJRT_Buffer_IsOnCpu_Args {
  PJRT_B200_HEAD;
  PJRT_Buffer* buffer;
  bool is_on_cpu;
} PJRT_Buffer_IsOnCpu_Args;
typedef struct PJRT_Buffer_Device_Args {
  PJRT_B200_HEAD;
  PJRT_Buffer* buffer;
  PJRT_Device* device;
} PJRT_Buffer_Device_Args;
typedef struct PJRT_Buffer_Memory_Args {
  PJRT_B200_HEAD;
  PJRT_Buffer* buffer;
  PJRT_Memory* memory;
} PJRT_Buffer_Memory_Args;
typedef struct PJRT_Buffer_ReadyEvent_Args {
  PJRT_B200_HEAD;
  PJRT_Buffer* buffer;
  PJRT_Event* event;
} PJRT_Buffer_ReadyEvent_Args;
typedef struct PJRT_Buffer_UnsafePointer_Args {
  PJRT_B200_HEAD;
  PJRT_Buffer* buffer;
  uintptr_t buffer_pointer;
} PJRT_Buffer_UnsafePointer_Args;
typedef struct PJRT_Buffer_IncreaseExternalReferenceCount_Args {
  PJRT_B200_HEAD;
  PJRT_Buffer* buffer;
} PJRT_Buffer_IncreaseExternalReferenceCount_Args;
typedef struct PJRT_Buffer_DecreaseExternalReferenceCount_Args {
  PJRT_B200_HEAD;
  PJRT_Buffer* buffer;
} PJRT_Buffer_DecreaseExternalReferenceCount_Args;
typedef struct PJRT_Buffer_OpaqueDeviceMemoryDataPointer_Args {
  PJRT_B200_HEAD;
  PJRT_Buffer* buffer;
  void* device_memory_ptr;
} PJRT_Buffer_OpaqueDeviceMemoryDataPointer_Args;

/* ---------------------------------------------------------------- topology */
typedef struct PJRT_TopologyDescription_Create_Args {
  PJRT_B200_HEAD;
  const char* topology_name;
  size_t topology_name_size;
  const PJRT_NamedValue* create_options;
  size_t num_options;
  PJRT_TopologyDescription* topology;
} PJRT_TopologyDescription_Create_Args;
typedef struct PJRT_TopologyDescription_Destroy_Args {
  PJRT_B200_HEAD;
  PJRT_TopologyDescription* topology;
} PJRT_TopologyDescription_Destroy_Args;
typedef struct PJRT_TopologyDescription_PlatformVersion_Args {
  PJRT_B200_HEAD;
  PJRT_TopologyDescription* topology;
  const char* platform_version;
  size_t platform_version_size;
} PJRT_TopologyDescription_PlatformVersion_Args;
typedef struct PJRT_TopologyDescription_PlatformName_Args {
  PJRT_B200_HEAD;
  PJRT_TopologyDescription* topology;
  const char* platform_name;
  size_t platform_name_size;
} PJRT_TopologyDescription_PlatformName_Args;
typedef struct PJRT_TopologyDescription_GetDeviceDescriptions_Args {
  PJRT_B200_HEAD;
  PJRT_TopologyDescription* topology;
  PJRT_DeviceDescription* const* descriptions;
  size_t num_descriptions;
} PJRT_TopologyDescription_GetDeviceDescriptions_Args;
typedef struct PJRT_TopologyDescription_Attributes_Args {
  PJRT_B200_HEAD;
  PJRT_TopologyDescription* topology;
  const PJRT_NamedValue* attributes;
  size_t num_attributes;
} PJRT_TopologyDescription_Attributes_Args;

/* Args types of entry points this plugin reports as UNIMPLEMENTED: declared, not defined. */
typedef struct PJRT_Client_CreateViewOfDeviceBuffer_Args PJRT_Client_CreateViewOfDeviceBuffer_Args;
typedef struct PJRT_Executable_GetCostAnalysis_Args PJRT_Executable_GetCostAnalysis_Args;
typedef struct PJRT_Executable_OptimizedProgram_Args PJRT_Executable_OptimizedProgram_Args;
typedef struct PJRT_Executable_Serialize_Args PJRT_Executable_Serialize_Args;
typedef struct PJRT_Executable_DeserializeAndLoad_Args PJRT_Executable_DeserializeAndLoad_Args;
typedef struct PJRT_Executable_GetCompiledMemoryStats_Args PJRT_Executable_GetCompiledMemoryStats_Args;
typedef struct PJRT_CopyToDeviceStream_Destroy_Args PJRT_CopyToDeviceStream_Destroy_Args;
typedef struct PJRT_CopyToDeviceStream_AddChunk_Args PJRT_CopyToDeviceStream_AddChunk_Args;
typedef struct PJRT_CopyToDeviceStream_TotalBytes_Args PJRT_CopyToDeviceStream_TotalBytes_Args;
typedef struct PJRT_CopyToDeviceStream_GranuleSize_Args PJRT_CopyToDeviceStream_GranuleSize_Args;
typedef struct PJRT_CopyToDeviceStream_CurrentBytes_Args PJRT_CopyToDeviceStream_CurrentBytes_Args;
typedef struct PJRT_TopologyDescription_Serialize_Args PJRT_TopologyDescription_Serialize_Args;
typedef struct PJRT_Compile_Args PJRT_Compile_Args;

/* ---------------------------------------------------------------- the function table */
#define PJRT_B200_FN(ret, name) ret (*name)(name##_Args * args)

typedef struct PJRT_Api {
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  PJRT_Api_Version pjrt_api_version;

  PJRT_B200_FN(void, PJRT_Error_Destroy);
  PJRT_B200_FN(void, PJRT_Error_Message);
  PJRT_B200_FN(PJRT_Error*, PJRT_Error_GetCode);

  PJRT_B200_FN(PJRT_Error*, PJRT_Plugin_Initialize);
  PJRT_B200_FN(PJRT_Error*, PJRT_Plugin_Attributes);

  PJRT_B200_FN(PJRT_Error*, PJRT_Event_Destroy);
  PJRT_B200_FN(PJRT_Error*, PJRT_Event_IsReady);
  PJRT_B200_FN(PJRT_Error*, PJRT_Event_Error);
  PJRT_B200_FN(PJRT_Error*, PJRT_Event_Await);
  PJRT_B200_FN(PJRT_Error*, PJRT_Event_OnReady);

  PJRT_B200_FN(PJRT_Error*, PJRT_Client_Create);
  PJRT_B200_FN(PJRT_Error*, PJRT_Client_Destroy);
  PJRT_B200_FN(PJRT_Error*, PJRT_Client_PlatformName);
  PJRT_B200_FN(PJRT_Error*, PJRT_Client_ProcessIndex);
  PJRT_B200_FN(PJRT_Error*, PJRT_Client_PlatformVersion);
  PJRT_B200_FN(PJRT_Error*, PJRT_Client_Devices);
  PJRT_B200_FN(PJRT_Error*, PJRT_Client_AddressableDevices);
  PJRT_B200_FN(PJRT_Error*, PJRT_Client_LookupDevice);
  PJRT_B200_FN(PJRT_Error*, PJRT_Client_LookupAddressableDevice);
  PJRT_B200_FN(PJRT_Error*, PJRT_Client_AddressableMemories);
  PJRT_B200_FN(PJRT_Error*, PJRT_Client_Compile);
  PJRT_B200_FN(PJRT_Error*, PJRT_Client_DefaultDeviceAssignment);
  PJRT_B200_FN(PJRT_Error*, PJRT_Client_BufferFromHostBuffer);

  PJRT_B200_FN(PJRT_Error*, PJRT_DeviceDescription_Id);
  PJRT_B200_FN(PJRT_Error*, PJRT_DeviceDescription_ProcessIndex);
  PJRT_B200_FN(PJRT_Error*, PJRT_DeviceDescription_Attributes);
  PJRT_B200_FN(PJRT_Error*, PJRT_DeviceDescription_Kind);
  PJRT_B200_FN(PJRT_Error*, PJRT_DeviceDescription_DebugString);
  PJRT_B200_FN(PJRT_Error*, PJRT_DeviceDescription_ToString);

  PJRT_B200_FN(PJRT_Error*, PJRT_Device_GetDescription);
  PJRT_B200_FN(PJRT_Error*, PJRT_Device_IsAddressable);
  PJRT_B200_FN(PJRT_Error*, PJRT_Device_LocalHardwareId);
  PJRT_B200_FN(PJRT_Error*, PJRT_Device_AddressableMemories);
  PJRT_B200_FN(PJRT_Error*, PJRT_Device_DefaultMemory);
  PJRT_B200_FN(PJRT_Error*, PJRT_Device_MemoryStats);

  PJRT_B200_FN(PJRT_Error*, PJRT_Memory_Id);
  PJRT_B200_FN(PJRT_Error*, PJRT_Memory_Kind);
  PJRT_B200_FN(PJRT_Error*, PJRT_Memory_DebugString);
  PJRT_B200_FN(PJRT_Error*, PJRT_Memory_ToString);
  PJRT_B200_FN(PJRT_Error*, PJRT_Memory_AddressableByDevices);

  PJRT_B200_FN(PJRT_Error*, PJRT_Executable_Destroy);
  PJRT_B200_FN(PJRT_Error*, PJRT_Executable_Name);
  PJRT_B200_FN(PJRT_Error*, PJRT_Executable_NumReplicas);
  PJRT_B200_FN(PJRT_Error*, PJRT_Executable_NumPartitions);
  PJRT_B200_FN(PJRT_Error*, PJRT_Executable_NumOutputs);
  PJRT_B200_FN(PJRT_Error*, PJRT_Executable_SizeOfGeneratedCodeInBytes);
  PJRT_B200_FN(PJRT_Error*, PJRT_Executable_GetCostAnalysis);
  PJRT_B200_FN(PJRT_Error*, PJRT_Executable_OutputMemoryKinds);
  PJRT_B200_FN(PJRT_Error*, PJRT_Executable_OptimizedProgram);
  PJRT_B200_FN(PJRT_Error*, PJRT_Executable_Serialize);

  PJRT_B200_FN(PJRT_Error*, PJRT_LoadedExecutable_Destroy);
  PJRT_B200_FN(PJRT_Error*, PJRT_LoadedExecutable_GetExecutable);
  PJRT_B200_FN(PJRT_Error*, PJRT_LoadedExecutable_AddressableDevices);
  PJRT_B200_FN(PJRT_Error*, PJRT_LoadedExecutable_Delete);
  PJRT_B200_FN(PJRT_Error*, PJRT_LoadedExecutable_IsDeleted);
  PJRT_B200_FN(PJRT_Error*, PJRT_LoadedExecutable_Execute);
  PJRT_B200_FN(PJRT_Error*, PJRT_Executable_DeserializeAndLoad);
  PJRT_B200_FN(PJRT_Error*, PJRT_LoadedExecutable_Fingerprint);

  PJRT_B200_FN(PJRT_Error*, PJRT_Buffer_Destroy);
  PJRT_B200_FN(PJRT_Error*, PJRT_Buffer_ElementType);
  PJRT_B200_FN(PJRT_Error*, PJRT_Buffer_Dimensions);
  PJRT_B200_FN(PJRT_Error*, PJRT_Buffer_UnpaddedDimensions);
  PJRT_B200_FN(PJRT_Error*, PJRT_Buffer_DynamicDimensionIndices);
  PJRT_B200_FN(PJRT_Error*, PJRT_Buffer_GetMemoryLayout);
  PJRT_B200_FN(PJRT_Error*, PJRT_Buffer_OnDeviceSizeInBytes);
  PJRT_B200_FN(PJRT_Error*, PJRT_Buffer_Device);
  PJRT_B200_FN(PJRT_Error*, PJRT_Buffer_Memory);
  PJRT_B200_FN(PJRT_Error*, PJRT_Buffer_Delete);
  PJRT_B200_FN(PJRT_Error*, PJRT_Buffer_IsDeleted);
  PJRT_B200_FN(PJRT_Error*, PJRT_Buffer_CopyToDevice);
  PJRT_B200_FN(PJRT_Error*, PJRT_Buffer_ToHostBuffer);
  PJRT_B200_FN(PJRT_Error*, PJRT_Buffer_IsOnCpu);
  PJRT_B200_FN(PJRT_Error*, PJRT_Buffer_ReadyEvent);
  PJRT_B200_FN(PJRT_Error*, PJRT_Buffer_UnsafePointer);
  PJRT_B200_FN(PJRT_Error*, PJRT_Buffer_IncreaseExternalReferenceCount);
  PJRT_B200_FN(PJRT_Error*, PJRT_Buffer_DecreaseExternalReferenceCount);
  PJRT_B200_FN(PJRT_Error*, PJRT_Buffer_OpaqueDeviceMemoryDataPointer);

  PJRT_B200_FN(PJRT_Error*, PJRT_CopyToDeviceStream_Destroy);
  PJRT_B200_FN(PJRT_Error*, PJRT_CopyToDeviceStream_AddChunk);
  PJRT_B200_FN(PJRT_Error*, PJRT_CopyToDeviceStream_TotalBytes);
  PJRT_B200_FN(PJRT_Error*, PJRT_CopyToDeviceStream_GranuleSize);
  PJRT_B200_FN(PJRT_Error*, PJRT_CopyToDeviceStream_CurrentBytes);

  PJRT_B200_FN(PJRT_Error*, PJRT_TopologyDescription_Create);
  PJRT_B200_FN(PJRT_Error*, PJRT_TopologyDescription_Destroy);
  PJRT_B200_FN(PJRT_Error*, PJRT_TopologyDescription_PlatformName);
  PJRT_B200_FN(PJRT_Error*, PJRT_TopologyDescription_PlatformVersion);
  PJRT_B200_FN(PJRT_Error*, PJRT_TopologyDescription_GetDeviceDescriptions);
  PJRT_B200_FN(PJRT_Error*, PJRT_TopologyDescription_Serialize);
  PJRT_B200_FN(PJRT_Error*, PJRT_TopologyDescription_Attributes);

  PJRT_B200_FN(PJRT_Error*, PJRT_Compile);

  PJRT_B200_FN(PJRT_Error*, PJRT_Executable_OutputElementTypes);
  PJRT_B200_FN(PJRT_Error*, PJRT_Executable_OutputDimensions);

  PJRT_B200_FN(PJRT_Error*, PJRT_Buffer_CopyToMemory);

  PJRT_B200_FN(PJRT_Error*, PJRT_Client_CreateViewOfDeviceBuffer);

  PJRT_B200_FN(PJRT_Error*, PJRT_Executable_Fingerprint);

  PJRT_B200_FN(PJRT_Error*, PJRT_Client_TopologyDescription);

  PJRT_B200_FN(PJRT_Error*, PJRT_Executable_GetCompiledMemoryStats);

  PJRT_B200_FN(PJRT_Error*, PJRT_Memory_Kind_Id);

  PJRT_B200_FN(PJRT_Error*, PJRT_ExecuteContext_Create);
  PJRT_B200_FN(PJRT_Error*, PJRT_ExecuteContext_Destroy);
} PJRT_Api;

#undef PJRT_B200_FN

#ifdef __cplusplus
}
#endif

#endif /* PJRT_B200_ABI_H_ */
