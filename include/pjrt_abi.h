/*
 * pjrt_abi.h - the subset of the PJRT C API ABI that clj-xla's host binds.
 *
 * clj-xla (src/clj_xla/pjrt.clj) does not compile against a header: it reads
 * the PJRT_Api function table and every argument struct at hard-coded byte
 * offsets through Java Panama FFM.  This header restates exactly those
 * layouts (field order and types follow the PJRT C API v0.114 that the
 * reference vendors at vendor/include/pjrt_c_api.h) and pins every offset the
 * host uses with a static_assert, citing the pjrt.clj line that reads it.
 * Only the structs the host touches are declared; the remaining PJRT_Api slots
 * are filled with an UNIMPLEMENTED stub by the library.
 */
#ifndef CLJXLA_PJRT_ABI_H_
#define CLJXLA_PJRT_ABI_H_

#include <stddef.h>
#include <stdint.h>
#include <stdbool.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct PJRT_Error PJRT_Error;
typedef struct PJRT_Event PJRT_Event;
typedef struct PJRT_Client PJRT_Client;
typedef struct PJRT_Device PJRT_Device;
typedef struct PJRT_Memory PJRT_Memory;
typedef struct PJRT_Buffer PJRT_Buffer;
typedef struct PJRT_LoadedExecutable PJRT_LoadedExecutable;
typedef struct PJRT_Extension_Base PJRT_Extension_Base;

/* PJRT_Error_Code: absl::StatusCode numbering. */
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

/* PJRT_Buffer_Type numbering (pjrt.clj:400 uses 2=S8, 4=S32, 10=F16, 11=F32, 13=BF16). */
typedef enum {
  PJRT_Buffer_Type_INVALID = 0,
  PJRT_Buffer_Type_PRED = 1,
  PJRT_Buffer_Type_S8 = 2,
  PJRT_Buffer_Type_S16 = 3,
  PJRT_Buffer_Type_S32 = 4,
  PJRT_Buffer_Type_S64 = 5,
  PJRT_Buffer_Type_U8 = 6,
  PJRT_Buffer_Type_U16 = 7,
  PJRT_Buffer_Type_U32 = 8,
  PJRT_Buffer_Type_U64 = 9,
  PJRT_Buffer_Type_F16 = 10,
  PJRT_Buffer_Type_F32 = 11,
  PJRT_Buffer_Type_F64 = 12,
  PJRT_Buffer_Type_BF16 = 13
} PJRT_Buffer_Type;

typedef enum {
  PJRT_NamedValue_kString = 0,
  PJRT_NamedValue_kInt64 = 1,
  PJRT_NamedValue_kInt64List = 2,
  PJRT_NamedValue_kFloat = 3,
  PJRT_NamedValue_kBool = 4
} PJRT_NamedValue_Type;

typedef struct PJRT_Api_Version {
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  int major_version;
  int minor_version;
} PJRT_Api_Version;

/* Every PJRT entry point has this shape: one args struct in, error (or NULL) out. */
typedef PJRT_Error* (*PJRT_Fn)(void* args);
typedef void (*PJRT_Error_Destroy_Fn)(void* args);

#define CLJXLA_PJRT_API_BYTES 984 /* pjrt.clj:207 reinterprets this many bytes */
#define CLJXLA_PJRT_NUM_FNS ((CLJXLA_PJRT_API_BYTES - 40) / 8)

typedef struct PJRT_Api {
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  PJRT_Api_Version pjrt_api_version;
  /* Function slots in PJRT C API order; slot i lives at byte 40 + 8*i. */
  void* fns[CLJXLA_PJRT_NUM_FNS];
} PJRT_Api;

/* Slot byte offsets read by the host (pjrt.clj:8-27). */
enum {
  PJRT_OFF_ERROR_DESTROY = 40,
  PJRT_OFF_ERROR_MESSAGE = 48,
  PJRT_OFF_ERROR_GET_CODE = 56,
  PJRT_OFF_PLUGIN_INITIALIZE = 64,
  PJRT_OFF_PLUGIN_ATTRIBUTES = 72,
  PJRT_OFF_EVENT_DESTROY = 80,
  PJRT_OFF_EVENT_IS_READY = 88,
  PJRT_OFF_EVENT_ERROR = 96,
  PJRT_OFF_EVENT_AWAIT = 104,
  PJRT_OFF_EVENT_ON_READY = 112,
  PJRT_OFF_CLIENT_CREATE = 120,
  PJRT_OFF_CLIENT_DESTROY = 128,
  PJRT_OFF_CLIENT_PLATFORM_NAME = 136,
  PJRT_OFF_CLIENT_PROCESS_INDEX = 144,
  PJRT_OFF_CLIENT_PLATFORM_VERSION = 152,
  PJRT_OFF_CLIENT_DEVICES = 160,
  PJRT_OFF_CLIENT_ADDRESSABLE_DEVICES = 168,
  PJRT_OFF_CLIENT_COMPILE = 200,
  PJRT_OFF_CLIENT_BUFFER_FROM_HOST_BUFFER = 216,
  PJRT_OFF_EXECUTABLE_DESTROY = 360,
  PJRT_OFF_EXECUTABLE_NUM_OUTPUTS = 392,
  PJRT_OFF_LOADED_EXECUTABLE_DESTROY = 440,
  PJRT_OFF_LOADED_EXECUTABLE_EXECUTE = 480,
  PJRT_OFF_BUFFER_DESTROY = 504,
  PJRT_OFF_BUFFER_ELEMENT_TYPE = 512,
  PJRT_OFF_BUFFER_DIMENSIONS = 520,
  PJRT_OFF_BUFFER_ON_DEVICE_SIZE = 552,
  PJRT_OFF_BUFFER_TO_HOST_BUFFER = 600
};

typedef struct PJRT_Error_Destroy_Args {
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  PJRT_Error* error;
} PJRT_Error_Destroy_Args;

typedef struct PJRT_Error_Message_Args {   /* pjrt.clj:69-75 */
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  const PJRT_Error* error;
  const char* message;
  size_t message_size;
} PJRT_Error_Message_Args;

typedef struct PJRT_Error_GetCode_Args {
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  const PJRT_Error* error;
  PJRT_Error_Code code;
} PJRT_Error_GetCode_Args;

/* The PJRT header's layout is 56 bytes; clj-xla's host writes option arrays
 * (pjrt.clj:226-231) and reads attribute arrays (pjrt.clj:131) with a 64-byte
 * element stride and sets struct_size = 64 in each element, so the library
 * steps through option arrays by the struct_size found in element 0 and
 * returns a single plugin attribute. */
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
  size_t value_size;
} PJRT_NamedValue;

typedef struct PJRT_Plugin_Initialize_Args {
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
} PJRT_Plugin_Initialize_Args;

typedef struct PJRT_Plugin_Attributes_Args {  /* pjrt.clj:116-146 */
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  const PJRT_NamedValue* attributes;
  size_t num_attributes;
} PJRT_Plugin_Attributes_Args;

typedef struct PJRT_Event_Destroy_Args {
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  PJRT_Event* event;
} PJRT_Event_Destroy_Args;

typedef struct PJRT_Event_IsReady_Args {
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  PJRT_Event* event;
  bool is_ready;
} PJRT_Event_IsReady_Args;

typedef struct PJRT_Event_Await_Args {
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  PJRT_Event* event;
} PJRT_Event_Await_Args;

typedef struct PJRT_Client_Create_Args {   /* pjrt.clj:261-275 */
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  const PJRT_NamedValue* create_options;
  size_t num_options;
  void* kv_get_callback;
  void* kv_get_user_arg;
  void* kv_put_callback;
  void* kv_put_user_arg;
  PJRT_Client* client;
  void* kv_try_get_callback;
  void* kv_try_get_user_arg;
} PJRT_Client_Create_Args;

typedef struct PJRT_Client_Destroy_Args {
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  PJRT_Client* client;
} PJRT_Client_Destroy_Args;

typedef struct PJRT_Client_PlatformName_Args {  /* pjrt.clj:277-291 */
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  PJRT_Client* client;
  const char* platform_name;
  size_t platform_name_size;
} PJRT_Client_PlatformName_Args;

typedef struct PJRT_Client_AddressableDevices_Args {  /* pjrt.clj:293-308 */
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  PJRT_Client* client;
  PJRT_Device* const* addressable_devices;
  size_t num_addressable_devices;
} PJRT_Client_AddressableDevices_Args;

typedef struct PJRT_Program {               /* pjrt.clj:320-326 */
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  char* code;
  size_t code_size;
  const char* format;
  size_t format_size;
} PJRT_Program;

typedef struct PJRT_Client_Compile_Args {   /* pjrt.clj:328-340 */
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  PJRT_Client* client;
  const PJRT_Program* program;
  const char* compile_options;
  size_t compile_options_size;
  PJRT_LoadedExecutable* executable;
} PJRT_Client_Compile_Args;

typedef struct PJRT_Client_BufferFromHostBuffer_Args {  /* pjrt.clj:390-421 */
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  PJRT_Client* client;
  const void* data;
  PJRT_Buffer_Type type;
  const int64_t* dims;
  size_t num_dims;
  const int64_t* byte_strides;
  size_t num_byte_strides;
  int host_buffer_semantics;
  PJRT_Device* device;
  PJRT_Memory* memory;
  void* device_layout;
  PJRT_Event* done_with_host_buffer;
  PJRT_Buffer* buffer;
} PJRT_Client_BufferFromHostBuffer_Args;

typedef struct PJRT_ExecuteOptions {        /* pjrt.clj:481-489 (host passes struct_size 112) */
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  void** send_callbacks;
  void** recv_callbacks;
  size_t num_send_ops;
  size_t num_recv_ops;
  int launch_id;
  const int64_t* non_donatable_input_indices;
  size_t num_non_donatable_input_indices;
  void* context;
  const char* call_location;
  size_t num_tasks;
  int* task_ids;
  int64_t* incarnation_ids;
} PJRT_ExecuteOptions;

typedef struct PJRT_LoadedExecutable_Execute_Args {  /* pjrt.clj:490-501 */
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  PJRT_LoadedExecutable* executable;
  PJRT_ExecuteOptions* options;
  PJRT_Buffer* const* const* argument_lists;
  size_t num_devices;
  size_t num_args;
  PJRT_Buffer** const* output_lists;
  PJRT_Event** device_complete_events;
  PJRT_Device* execute_device;
} PJRT_LoadedExecutable_Execute_Args;

typedef struct PJRT_LoadedExecutable_Destroy_Args {
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  PJRT_LoadedExecutable* executable;
} PJRT_LoadedExecutable_Destroy_Args;

typedef struct PJRT_Buffer_Destroy_Args {   /* pjrt.clj:436-452 */
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  PJRT_Buffer* buffer;
} PJRT_Buffer_Destroy_Args;

typedef struct PJRT_Buffer_ElementType_Args {
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  PJRT_Buffer* buffer;
  PJRT_Buffer_Type type;
} PJRT_Buffer_ElementType_Args;

typedef struct PJRT_Buffer_Dimensions_Args {
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  PJRT_Buffer* buffer;
  const int64_t* dims;
  size_t num_dims;
} PJRT_Buffer_Dimensions_Args;

typedef struct PJRT_Buffer_OnDeviceSizeInBytes_Args {
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  PJRT_Buffer* buffer;
  size_t on_device_size_in_bytes;
} PJRT_Buffer_OnDeviceSizeInBytes_Args;

typedef struct PJRT_Buffer_ToHostBuffer_Args {  /* pjrt.clj:538-548 */
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  PJRT_Buffer* src;
  void* host_layout;
  void* dst;
  size_t dst_size;
  PJRT_Event* event;
} PJRT_Buffer_ToHostBuffer_Args;

typedef struct PJRT_Executable_NumOutputs_Args {
  size_t struct_size;
  PJRT_Extension_Base* extension_start;
  void* executable;
  size_t num_outputs;
} PJRT_Executable_NumOutputs_Args;

#ifdef __cplusplus
}  /* extern "C" */

/* Offsets the Clojure host hard-codes. */
static_assert(offsetof(PJRT_Api, pjrt_api_version) == 16, "pjrt.clj:10");
static_assert(offsetof(PJRT_Api, fns) == PJRT_OFF_ERROR_DESTROY, "pjrt.clj:11");
static_assert(sizeof(PJRT_Api) == CLJXLA_PJRT_API_BYTES, "pjrt.clj:207");
static_assert(offsetof(PJRT_Error_Message_Args, error) == 16, "pjrt.clj:71");
static_assert(offsetof(PJRT_Error_Message_Args, message) == 24, "pjrt.clj:73");
static_assert(offsetof(PJRT_Error_Message_Args, message_size) == 32, "pjrt.clj:74");
static_assert(sizeof(PJRT_Error_Message_Args) == 40, "pjrt.clj:69");
static_assert(sizeof(PJRT_NamedValue) == 56, "pjrt_c_api.h PJRT_NamedValue");
static_assert(offsetof(PJRT_NamedValue, name) == 16, "pjrt.clj:233");
static_assert(offsetof(PJRT_NamedValue, name_size) == 24, "pjrt.clj:234");
static_assert(offsetof(PJRT_NamedValue, type) == 32, "pjrt.clj:238");
static_assert(offsetof(PJRT_NamedValue, string_value) == 40, "pjrt.clj:239");
static_assert(offsetof(PJRT_NamedValue, value_size) == 48, "pjrt.clj:240");
static_assert(offsetof(PJRT_Plugin_Attributes_Args, attributes) == 16, "pjrt.clj:125");
static_assert(offsetof(PJRT_Plugin_Attributes_Args, num_attributes) == 24, "pjrt.clj:126");
static_assert(offsetof(PJRT_Event_Await_Args, event) == 16, "pjrt.clj:425");
static_assert(sizeof(PJRT_Client_Create_Args) == 88, "pjrt.clj:267");
static_assert(offsetof(PJRT_Client_Create_Args, create_options) == 16, "pjrt.clj:271");
static_assert(offsetof(PJRT_Client_Create_Args, num_options) == 24, "pjrt.clj:272");
static_assert(offsetof(PJRT_Client_Create_Args, client) == 64, "pjrt.clj:275");
static_assert(offsetof(PJRT_Client_PlatformName_Args, platform_name) == 24, "pjrt.clj:288");
static_assert(offsetof(PJRT_Client_PlatformName_Args, platform_name_size) == 32, "pjrt.clj:289");
static_assert(offsetof(PJRT_Client_AddressableDevices_Args, addressable_devices) == 24, "pjrt.clj:304");
static_assert(offsetof(PJRT_Client_AddressableDevices_Args, num_addressable_devices) == 32, "pjrt.clj:305");
static_assert(sizeof(PJRT_Program) == 48, "pjrt.clj:321");
static_assert(offsetof(PJRT_Program, code) == 16, "pjrt.clj:323");
static_assert(offsetof(PJRT_Program, code_size) == 24, "pjrt.clj:324");
static_assert(offsetof(PJRT_Program, format) == 32, "pjrt.clj:325");
static_assert(sizeof(PJRT_Client_Compile_Args) == 56, "pjrt.clj:329");
static_assert(offsetof(PJRT_Client_Compile_Args, program) == 24, "pjrt.clj:332");
static_assert(offsetof(PJRT_Client_Compile_Args, compile_options) == 32, "pjrt.clj:333");
static_assert(offsetof(PJRT_Client_Compile_Args, executable) == 48, "pjrt.clj:340");
static_assert(sizeof(PJRT_Client_BufferFromHostBuffer_Args) == 120, "pjrt.clj:390");
static_assert(offsetof(PJRT_Client_BufferFromHostBuffer_Args, data) == 24, "pjrt.clj:394");
static_assert(offsetof(PJRT_Client_BufferFromHostBuffer_Args, type) == 32, "pjrt.clj:395");
static_assert(offsetof(PJRT_Client_BufferFromHostBuffer_Args, dims) == 40, "pjrt.clj:396");
static_assert(offsetof(PJRT_Client_BufferFromHostBuffer_Args, num_dims) == 48, "pjrt.clj:397");
static_assert(offsetof(PJRT_Client_BufferFromHostBuffer_Args, byte_strides) == 56, "pjrt.clj:409");
static_assert(offsetof(PJRT_Client_BufferFromHostBuffer_Args, num_byte_strides) == 64, "pjrt.clj:410");
static_assert(offsetof(PJRT_Client_BufferFromHostBuffer_Args, host_buffer_semantics) == 72, "pjrt.clj:414");
static_assert(offsetof(PJRT_Client_BufferFromHostBuffer_Args, device) == 80, "pjrt.clj:416");
static_assert(offsetof(PJRT_Client_BufferFromHostBuffer_Args, done_with_host_buffer) == 104, "pjrt.clj:420");
static_assert(offsetof(PJRT_Client_BufferFromHostBuffer_Args, buffer) == 112, "pjrt.clj:421");
static_assert(offsetof(PJRT_ExecuteOptions, non_donatable_input_indices) == 56, "pjrt.clj:488");
static_assert(offsetof(PJRT_ExecuteOptions, num_non_donatable_input_indices) == 64, "pjrt.clj:489");
static_assert(sizeof(PJRT_ExecuteOptions) == 112, "pjrt.clj:487");
static_assert(sizeof(PJRT_LoadedExecutable_Execute_Args) == 80, "pjrt.clj:492");
static_assert(offsetof(PJRT_LoadedExecutable_Execute_Args, executable) == 16, "pjrt.clj:493");
static_assert(offsetof(PJRT_LoadedExecutable_Execute_Args, options) == 24, "pjrt.clj:494");
static_assert(offsetof(PJRT_LoadedExecutable_Execute_Args, argument_lists) == 32, "pjrt.clj:495");
static_assert(offsetof(PJRT_LoadedExecutable_Execute_Args, num_devices) == 40, "pjrt.clj:496");
static_assert(offsetof(PJRT_LoadedExecutable_Execute_Args, num_args) == 48, "pjrt.clj:497");
static_assert(offsetof(PJRT_LoadedExecutable_Execute_Args, output_lists) == 56, "pjrt.clj:498");
static_assert(offsetof(PJRT_LoadedExecutable_Execute_Args, device_complete_events) == 64, "pjrt.clj:501");
static_assert(offsetof(PJRT_Buffer_Destroy_Args, buffer) == 16, "pjrt.clj:448");
static_assert(sizeof(PJRT_Buffer_ToHostBuffer_Args) == 56, "pjrt.clj:538");
static_assert(offsetof(PJRT_Buffer_ToHostBuffer_Args, src) == 16, "pjrt.clj:541");
static_assert(offsetof(PJRT_Buffer_ToHostBuffer_Args, host_layout) == 24, "pjrt.clj:542");
static_assert(offsetof(PJRT_Buffer_ToHostBuffer_Args, dst) == 32, "pjrt.clj:543");
static_assert(offsetof(PJRT_Buffer_ToHostBuffer_Args, dst_size) == 40, "pjrt.clj:544");
static_assert(offsetof(PJRT_Buffer_ToHostBuffer_Args, event) == 48, "pjrt.clj:548");
#endif

#endif  /* CLJXLA_PJRT_ABI_H_ */
