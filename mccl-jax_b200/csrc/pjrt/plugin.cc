// plugin.cc — PJRT C-API v0.55 implementation for B200 (the drop-in boundary).
//
// Mirrors the reference plugin's surface and error behaviour (src/pjrt/api/pjrt_c_api.cc): the same
// entry points are real, the same ones answer UNIMPLEMENTED (:833-873), errors carry the same codes
// (INVALID_ARGUMENT for bad arguments and "jam compile: ..." compile failures, RESOURCE_EXHAUSTED for
// allocation, INTERNAL for execute / communicator failures).  What changes is underneath: buffers
// live in HBM (stream-ordered CUDA pool), transfers are cudaMemcpyAsync on the device stream, events
// are CUDA events, Execute enqueues asynchronously and returns events that complete on the GPU.
#include <cuda_runtime.h>

#include <atomic>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../../include/b200_kernels.h"
#include "../../../include/pjrt_b200.h"
#include "../comm/comm.h"
#include "../jam/runtime.h"

struct PJRT_Error {
  PJRT_Error_Code code = PJRT_Error_Code_UNKNOWN;
  std::string message;
};

namespace {

PJRT_Error* Err(PJRT_Error_Code c, const std::string& m) { return new PJRT_Error{c, m}; }

// Shared completion state: a PJRT_Event and any waiter threads hold it.
struct EventState {
  std::mutex mu;
  std::condition_variable cv;
  bool ready = false;
  bool has_error = false;
  PJRT_Error_Code code = PJRT_Error_Code_UNKNOWN;
  std::string message;
  cudaEvent_t ev = nullptr;
  int device = -1;
  bool check_kernels = false;   // read the tensor-core kernels' timeout flag on completion
  std::vector<std::pair<PJRT_Event_OnReadyCallback, void*>> callbacks;

  ~EventState() {
    if (ev) cudaEventDestroy(ev);
  }
  // Blocks until the GPU work is done; idempotent.
  void Complete() {
    std::vector<std::pair<PJRT_Event_OnReadyCallback, void*>> cbs;
    {
      std::unique_lock<std::mutex> lock(mu);
      if (ready) return;
    }
    if (ev) {
      cudaSetDevice(device);
      cudaError_t e = cudaEventSynchronize(ev);
      std::lock_guard<std::mutex> lock(mu);
      if (e != cudaSuccess) {
        has_error = true;
        code = PJRT_Error_Code_INTERNAL;
        message = std::string("device execution failed: ") + cudaGetErrorString(e);
      } else if (check_kernels) {
        int k = b200_take_device_error();
        if (k) {
          has_error = true;
          code = PJRT_Error_Code_DEADLINE_EXCEEDED;
          message = "a tensor-core kernel gave up waiting on a pipeline barrier (code " + std::to_string(k) + ")";
        }
      }
    }
    {
      std::lock_guard<std::mutex> lock(mu);
      ready = true;
      cbs.swap(callbacks);
    }
    cv.notify_all();
    for (auto& cb : cbs) cb.first(MakeError(), cb.second);
  }
  bool Poll() {
    {
      std::lock_guard<std::mutex> lock(mu);
      if (ready) return true;
    }
    if (ev) {
      cudaSetDevice(device);
      if (cudaEventQuery(ev) == cudaErrorNotReady) return false;
    }
    Complete();
    return true;
  }
  PJRT_Error* MakeError() {
    return has_error ? Err(code, message) : nullptr;
  }
};

std::shared_ptr<EventState> ReadyState() {
  auto s = std::make_shared<EventState>();
  s->ready = true;
  return s;
}

std::shared_ptr<EventState> RecordState(int device, cudaStream_t st, bool check_kernels = false) {
  auto s = std::make_shared<EventState>();
  s->device = device;
  s->check_kernels = check_kernels;
  if (cudaEventCreateWithFlags(&s->ev, cudaEventDisableTiming) != cudaSuccess || cudaEventRecord(s->ev, st) != cudaSuccess) {
    cudaGetLastError();
    if (s->ev) cudaEventDestroy(s->ev);
    s->ev = nullptr;
    cudaStreamSynchronize(st);
    s->ready = true;
  }
  return s;
}

}  // namespace

struct PJRT_Event {
  std::shared_ptr<EventState> s;
};

struct PJRT_DeviceDescription {
  int id = 0;
  int process_index = 0;
  std::string kind = "NVIDIA B200";
  std::string debug_string;
  std::string to_string;
  std::vector<PJRT_NamedValue> attrs;
  std::vector<std::string> attr_names;
  std::string cc;
  int64_t core_count = 0;
};

struct PJRT_Device {
  PJRT_DeviceDescription description;
  PJRT_Client* client = nullptr;
  int local_hardware_id = -1;
  bool addressable = false;
  std::vector<PJRT_Memory*> memories;
  PJRT_Memory* default_memory = nullptr;
  b200::DeviceState state;
  std::mutex exec_mu;
};

struct PJRT_Memory {
  int id = 0;
  std::string kind;
  int kind_id = 0;
  std::string debug_string;
  std::string to_string;
  std::vector<PJRT_Device*> devices;
};

struct PJRT_TopologyDescription {
  std::string platform_name = "b200";
  std::string platform_version;
  std::vector<std::unique_ptr<PJRT_DeviceDescription>> owned;
  std::vector<PJRT_DeviceDescription*> descriptions;
};

struct PJRT_Client {
  std::string platform_name = "b200";
  std::string platform_version;
  int process_index = 0;
  int num_processes = 1;
  std::vector<std::unique_ptr<PJRT_Device>> owned_devices;
  std::vector<PJRT_Device*> devices;
  std::vector<PJRT_Device*> addressable_devices;
  std::vector<std::unique_ptr<PJRT_Memory>> owned_memories;
  std::vector<PJRT_Memory*> memories;
  std::unique_ptr<PJRT_TopologyDescription> topology;
  std::unique_ptr<b200::Comm> comm;
  ~PJRT_Client() {
    // drain the compute and communication streams before the communicator goes away
    for (PJRT_Device* d : addressable_devices) {
      cudaSetDevice(d->state.ordinal);
      if (d->state.stream) cudaStreamSynchronize(d->state.stream);
      if (d->state.comm_stream) cudaStreamSynchronize(d->state.comm_stream);
    }
    comm.reset();
    for (PJRT_Device* d : addressable_devices) {
      cudaSetDevice(d->state.ordinal);
      if (d->state.stream) cudaStreamDestroy(d->state.stream);
      if (d->state.comm_stream) cudaStreamDestroy(d->state.comm_stream);
    }
  }
};

struct PJRT_Buffer {
  PJRT_Client* client = nullptr;
  PJRT_Device* device = nullptr;
  PJRT_Memory* memory = nullptr;
  PJRT_Buffer_Type type = PJRT_Buffer_Type_INVALID;
  std::vector<int64_t> dims;
  size_t nbytes = 0;
  void* data = nullptr;
  std::shared_ptr<EventState> ready;
  int external_refs = 0;
  bool delete_requested = false;
  bool deleted = false;
};

struct PJRT_ExecuteContext {};

struct PJRT_Executable {
  std::shared_ptr<b200::Executable> program;
  std::string name;
  std::vector<PJRT_Buffer_Type> out_types;
  std::vector<int64_t> out_dims_flat;
  std::vector<size_t> out_dim_sizes;
  std::vector<std::string> out_mem_kinds;
  std::vector<const char*> out_mem_kind_ptrs;
  std::vector<size_t> out_mem_kind_sizes;
};

struct PJRT_LoadedExecutable {
  PJRT_Client* client = nullptr;
  std::shared_ptr<b200::Executable> program;
  std::vector<PJRT_Device*> devices;
  bool deleted = false;
};

namespace {

const char* kVersion = "pjrt-b200 0.1.0 (PJRT 0.55, sm_100a)";

size_t ByteWidth(PJRT_Buffer_Type t) {
  switch (t) {
    case PJRT_Buffer_Type_PRED: case PJRT_Buffer_Type_S8: case PJRT_Buffer_Type_U8:
    case PJRT_Buffer_Type_F8E5M2: case PJRT_Buffer_Type_F8E4M3FN: case PJRT_Buffer_Type_F8E4M3B11FNUZ:
    case PJRT_Buffer_Type_F8E5M2FNUZ: case PJRT_Buffer_Type_F8E4M3FNUZ: case PJRT_Buffer_Type_F8E4M3:
    case PJRT_Buffer_Type_F8E3M4:
      return 1;
    case PJRT_Buffer_Type_S16: case PJRT_Buffer_Type_U16: case PJRT_Buffer_Type_F16: case PJRT_Buffer_Type_BF16:
      return 2;
    case PJRT_Buffer_Type_S32: case PJRT_Buffer_Type_U32: case PJRT_Buffer_Type_F32:
      return 4;
    case PJRT_Buffer_Type_S64: case PJRT_Buffer_Type_U64: case PJRT_Buffer_Type_F64: case PJRT_Buffer_Type_C64:
      return 8;
    case PJRT_Buffer_Type_C128:
      return 16;
    default:
      return 0;
  }
}

PJRT_Buffer_Type ToPjrt(b200::DT d) {
  using b200::DT;
  switch (d) {
    case DT::kPred: return PJRT_Buffer_Type_PRED;
    case DT::kS8: return PJRT_Buffer_Type_S8;
    case DT::kS16: return PJRT_Buffer_Type_S16;
    case DT::kS32: return PJRT_Buffer_Type_S32;
    case DT::kS64: return PJRT_Buffer_Type_S64;
    case DT::kU8: return PJRT_Buffer_Type_U8;
    case DT::kU16: return PJRT_Buffer_Type_U16;
    case DT::kU32: return PJRT_Buffer_Type_U32;
    case DT::kU64: return PJRT_Buffer_Type_U64;
    case DT::kF16: return PJRT_Buffer_Type_F16;
    case DT::kBF16: return PJRT_Buffer_Type_BF16;
    case DT::kF32: return PJRT_Buffer_Type_F32;
    case DT::kF64: return PJRT_Buffer_Type_F64;
    default: return PJRT_Buffer_Type_INVALID;
  }
}

std::string DimsStr(const std::vector<int64_t>& d) {
  std::string s = "[";
  for (size_t i = 0; i < d.size(); ++i) s += (i ? "," : "") + std::to_string(d[i]);
  return s + "]";
}

PJRT_Error* MakeUnimplemented(const char* name) {
  return Err(PJRT_Error_Code_UNIMPLEMENTED, std::string(name) + " is not implemented by the B200 plugin");
}

int GetIntEnv(const char* n, int dflt) {
  const char* v = std::getenv(n);
  return v && *v ? std::atoi(v) : dflt;
}

// ------------------------------------------------------------------------------------------ errors
void ErrorDestroy(PJRT_Error_Destroy_Args* a) { delete a->error; }
void ErrorMessage(PJRT_Error_Message_Args* a) {
  a->message = a->error->message.c_str();
  a->message_size = a->error->message.size();
}
PJRT_Error* ErrorGetCode(PJRT_Error_GetCode_Args* a) {
  a->code = a->error->code;
  return nullptr;
}

// ------------------------------------------------------------------------------------------ events
PJRT_Event* NewEvent(std::shared_ptr<EventState> s) { return new PJRT_Event{std::move(s)}; }

PJRT_Error* EventDestroy(PJRT_Event_Destroy_Args* a) {
  delete a->event;
  return nullptr;
}
PJRT_Error* EventIsReady(PJRT_Event_IsReady_Args* a) {
  a->is_ready = a->event->s->Poll();
  return nullptr;
}
PJRT_Error* EventError(PJRT_Event_Error_Args* a) {
  std::lock_guard<std::mutex> lock(a->event->s->mu);
  return a->event->s->MakeError();
}
PJRT_Error* EventAwait(PJRT_Event_Await_Args* a) {
  a->event->s->Complete();
  std::lock_guard<std::mutex> lock(a->event->s->mu);
  return a->event->s->MakeError();
}
PJRT_Error* EventOnReady(PJRT_Event_OnReady_Args* a) {
  std::shared_ptr<EventState> s = a->event->s;
  {
    std::unique_lock<std::mutex> lock(s->mu);
    if (!s->ready) {
      s->callbacks.emplace_back(a->callback, a->user_arg);
      lock.unlock();
      std::thread([s] { s->Complete(); }).detach();
      return nullptr;
    }
  }
  a->callback(s->MakeError(), a->user_arg);
  return nullptr;
}

// ------------------------------------------------------------------------------------------ plugin
PJRT_Error* PluginInitialize(PJRT_Plugin_Initialize_Args*) { return nullptr; }
PJRT_Error* PluginAttributes(PJRT_Plugin_Attributes_Args* a) {
  a->attributes = nullptr;
  a->num_attributes = 0;
  return nullptr;
}

// ------------------------------------------------------------------------------------------ client
void FillDescription(PJRT_DeviceDescription* d, int id, int ordinal, bool local) {
  d->id = id;
  d->process_index = id;
  d->to_string = "B200Device(id=" + std::to_string(id) + ")";
  d->debug_string = "b200:" + std::to_string(id);
  int major = 10, minor = 0, sms = 148;
  if (local) {
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, ordinal) == cudaSuccess) {
      d->kind = p.name;
      major = p.major;
      minor = p.minor;
      sms = p.multiProcessorCount;
    }
  }
  d->cc = std::to_string(major) + "." + std::to_string(minor);
  d->core_count = sms;
  d->attr_names = {"compute_capability", "core_count", "device_vendor"};
  d->attrs.resize(3);
  for (auto& nv : d->attrs) {
    std::memset(&nv, 0, sizeof(nv));
    nv.struct_size = sizeof(PJRT_NamedValue);
  }
  static const char* vendor = "NVIDIA";
  d->attrs[0].name = d->attr_names[0].c_str();
  d->attrs[0].name_size = d->attr_names[0].size();
  d->attrs[0].type = PJRT_NamedValue_kString;
  d->attrs[0].string_value = d->cc.c_str();
  d->attrs[0].value_size = d->cc.size();
  d->attrs[1].name = d->attr_names[1].c_str();
  d->attrs[1].name_size = d->attr_names[1].size();
  d->attrs[1].type = PJRT_NamedValue_kInt64;
  d->attrs[1].int64_value = d->core_count;
  d->attrs[1].value_size = 1;
  d->attrs[2].name = d->attr_names[2].c_str();
  d->attrs[2].name_size = d->attr_names[2].size();
  d->attrs[2].type = PJRT_NamedValue_kString;
  d->attrs[2].string_value = vendor;
  d->attrs[2].value_size = 6;
}

// Builds `num_nodes` devices of which `node_id` is addressable (the reference's process model,
// src/pjrt/api/pjrt_c_api.cc:129-171), bound to CUDA device `ordinal`.
PJRT_Client* CreateClient(int num_nodes, int node_id, int ordinal) {
  auto client = std::make_unique<PJRT_Client>();
  client->process_index = node_id;
  client->num_processes = num_nodes;
  client->platform_version = kVersion;
  for (int k = 0; k < num_nodes; ++k) {
    const std::string ks = std::to_string(k);
    auto device = std::make_unique<PJRT_Device>();
    device->client = client.get();
    device->addressable = (k == node_id);
    device->local_hardware_id = device->addressable ? ordinal : -1;
    FillDescription(&device->description, k, ordinal, device->addressable);
    PJRT_Device* dev = device.get();
    auto hbm = std::make_unique<PJRT_Memory>();
    hbm->id = k * 2;
    hbm->kind = "device";
    hbm->kind_id = 0;
    hbm->debug_string = "hbm:" + ks;
    hbm->to_string = "HbmMemory(id=" + ks + ")";
    hbm->devices.push_back(dev);
    auto host = std::make_unique<PJRT_Memory>();
    host->id = k * 2 + 1;
    host->kind = "pinned_host";
    host->kind_id = 1;
    host->debug_string = "host:" + ks;
    host->to_string = "PinnedHostMemory(id=" + ks + ")";
    host->devices.push_back(dev);
    dev->memories = {hbm.get(), host.get()};
    dev->default_memory = hbm.get();
    if (dev->addressable) {
      client->memories = {hbm.get(), host.get()};
      client->addressable_devices.push_back(dev);
      dev->state.ordinal = ordinal;
    }
    client->owned_memories.push_back(std::move(hbm));
    client->owned_memories.push_back(std::move(host));
    client->devices.push_back(dev);
    client->owned_devices.push_back(std::move(device));
  }
  auto topo = std::make_unique<PJRT_TopologyDescription>();
  topo->platform_version = kVersion;
  for (PJRT_Device* d : client->devices) topo->descriptions.push_back(&d->description);
  client->topology = std::move(topo);
  return client.release();
}

PJRT_Error* ClientCreate(PJRT_Client_Create_Args* a) {
  int node_id = 0, num_nodes = 1, ordinal = -1;
  for (size_t i = 0; i < a->num_options; ++i) {
    const PJRT_NamedValue& nv = a->create_options[i];
    const std::string name(nv.name, nv.name_size);
    if (nv.type == PJRT_NamedValue_kInt64) {
      if (name == "node_id") node_id = (int)nv.int64_value;
      else if (name == "num_nodes") num_nodes = (int)nv.int64_value;
      else if (name == "device_ordinal") ordinal = (int)nv.int64_value;
    }
  }
  if (num_nodes < 1) num_nodes = 1;
  if (node_id < 0 || node_id >= num_nodes) node_id = 0;
  int count = 0;
  cudaError_t ce = cudaGetDeviceCount(&count);
  if (ce != cudaSuccess || count == 0) {
    cudaGetLastError();
    return Err(PJRT_Error_Code_FAILED_PRECONDITION, "no CUDA device is visible to the B200 plugin");
  }
  if (ordinal < 0) ordinal = GetIntEnv("LOCAL_RANK", node_id % count);
  if (ordinal >= count) return Err(PJRT_Error_Code_INVALID_ARGUMENT, "device_ordinal " + std::to_string(ordinal) + " out of range");
  std::unique_ptr<PJRT_Client> client(CreateClient(num_nodes, node_id, ordinal));
  PJRT_Device* local = client->addressable_devices[0];
  cudaSetDevice(ordinal);
  if (cudaStreamCreateWithFlags(&local->state.stream, cudaStreamNonBlocking) != cudaSuccess)
    return Err(PJRT_Error_Code_INTERNAL, "cudaStreamCreate failed");
  // keep freed pool memory cached (stream-ordered reuse instead of returning it to the driver)
  cudaMemPool_t pool;
  if (cudaDeviceGetDefaultMemPool(&pool, ordinal) == cudaSuccess) {
    uint64_t thr = UINT64_MAX;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
  }
  if (num_nodes > 1) {
    b200::KvStore kv;
    if (a->kv_put_callback && a->kv_get_callback) {
      auto put_cb = a->kv_put_callback;
      void* put_arg = a->kv_put_user_arg;
      auto get_cb = a->kv_get_callback;
      void* get_arg = a->kv_get_user_arg;
      kv.put = [put_cb, put_arg](const std::string& k, const std::string& v) -> std::string {
        PJRT_KeyValuePutCallback_Args pa;
        std::memset(&pa, 0, sizeof(pa));
        pa.struct_size = sizeof(pa);
        pa.key = k.data();
        pa.key_size = k.size();
        pa.value = v.data();
        pa.value_size = v.size();
        pa.user_arg = put_arg;
        PJRT_Error* e = put_cb(&pa);
        if (!e) return "";
        std::string m = "kv_put callback failed";
        return m;
      };
      kv.get = [get_cb, get_arg](const std::string& k, int timeout_ms, std::string* out) -> std::string {
        PJRT_KeyValueGetCallback_Args ga;
        std::memset(&ga, 0, sizeof(ga));
        ga.struct_size = sizeof(ga);
        ga.key = k.data();
        ga.key_size = k.size();
        ga.timeout_in_ms = timeout_ms;
        ga.user_arg = get_arg;
        PJRT_Error* e = get_cb(&ga);
        if (e) return "kv_get callback failed";
        out->assign(ga.value, ga.value_size);
        if (ga.value_deleter_callback) ga.value_deleter_callback(ga.value);
        return "";
      };
    }
    std::string err;
    client->comm = b200::Comm::Create(num_nodes, node_id, ordinal, kv, GetIntEnv("B200_COMM_TIMEOUT_MS", 120000), &err);
    if (!client->comm) return Err(err.find("timed out") != std::string::npos ? PJRT_Error_Code_DEADLINE_EXCEEDED : PJRT_Error_Code_INTERNAL,
                                  "NCCL communicator init failed: " + err);
  }
  a->client = client.release();
  return nullptr;
}

PJRT_Error* ClientDestroy(PJRT_Client_Destroy_Args* a) {
  delete a->client;
  return nullptr;
}
PJRT_Error* ClientPlatformName(PJRT_Client_PlatformName_Args* a) {
  a->platform_name = a->client->platform_name.c_str();
  a->platform_name_size = a->client->platform_name.size();
  return nullptr;
}
PJRT_Error* ClientPlatformVersion(PJRT_Client_PlatformVersion_Args* a) {
  a->platform_version = a->client->platform_version.c_str();
  a->platform_version_size = a->client->platform_version.size();
  return nullptr;
}
PJRT_Error* ClientProcessIndex(PJRT_Client_ProcessIndex_Args* a) {
  a->process_index = a->client->process_index;
  return nullptr;
}
PJRT_Error* ClientDevices(PJRT_Client_Devices_Args* a) {
  a->devices = a->client->devices.data();
  a->num_devices = a->client->devices.size();
  return nullptr;
}
PJRT_Error* ClientAddressableDevices(PJRT_Client_AddressableDevices_Args* a) {
  a->addressable_devices = a->client->addressable_devices.data();
  a->num_addressable_devices = a->client->addressable_devices.size();
  return nullptr;
}
PJRT_Error* ClientAddressableMemories(PJRT_Client_AddressableMemories_Args* a) {
  a->addressable_memories = a->client->memories.data();
  a->num_addressable_memories = a->client->memories.size();
  return nullptr;
}
PJRT_Error* ClientLookupDevice(PJRT_Client_LookupDevice_Args* a) {
  for (PJRT_Device* d : a->client->devices)
    if (d->description.id == a->id) { a->device = d; return nullptr; }
  return Err(PJRT_Error_Code_INVALID_ARGUMENT, "no device with that id");
}
PJRT_Error* ClientLookupAddressableDevice(PJRT_Client_LookupAddressableDevice_Args* a) {
  for (PJRT_Device* d : a->client->addressable_devices)
    if (d->local_hardware_id == a->local_hardware_id) { a->addressable_device = d; return nullptr; }
  return Err(PJRT_Error_Code_INVALID_ARGUMENT, "no addressable device with that local hardware id");
}
PJRT_Error* ClientDefaultDeviceAssignment(PJRT_Client_DefaultDeviceAssignment_Args* a) {
  const size_t n = (size_t)a->num_replicas * (size_t)a->num_partitions;
  const size_t nd = a->client->devices.size();
  for (size_t i = 0; i < n && i < a->default_assignment_size; ++i) a->default_assignment[i] = (int)(i % nd);
  return nullptr;
}
PJRT_Error* ClientTopologyDescription(PJRT_Client_TopologyDescription_Args* a) {
  a->topology = a->client->topology.get();
  return nullptr;
}

// ------------------------------------------------------------------------------------------ devices
PJRT_Error* DeviceGetDescription(PJRT_Device_GetDescription_Args* a) {
  a->device_description = &a->device->description;
  return nullptr;
}
PJRT_Error* DeviceIsAddressable(PJRT_Device_IsAddressable_Args* a) {
  a->is_addressable = a->device->addressable;
  return nullptr;
}
PJRT_Error* DeviceLocalHardwareId(PJRT_Device_LocalHardwareId_Args* a) {
  a->local_hardware_id = a->device->local_hardware_id;
  return nullptr;
}
PJRT_Error* DeviceAddressableMemories(PJRT_Device_AddressableMemories_Args* a) {
  a->memories = a->device->memories.data();
  a->num_memories = a->device->memories.size();
  return nullptr;
}
PJRT_Error* DeviceDefaultMemory(PJRT_Device_DefaultMemory_Args* a) {
  a->memory = a->device->default_memory;
  return nullptr;
}
PJRT_Error* DeviceMemoryStats(PJRT_Device_MemoryStats_Args* a) {
  size_t free_b = 0, total = 0;
  if (a->device->addressable) {
    cudaSetDevice(a->device->state.ordinal);
    cudaMemGetInfo(&free_b, &total);
  }
  a->bytes_in_use = (int64_t)(total - free_b);
  a->peak_bytes_in_use_is_set = false;
  a->num_allocs_is_set = false;
  a->largest_alloc_size_is_set = false;
  a->bytes_limit = (int64_t)total;
  a->bytes_limit_is_set = total != 0;
  a->bytes_reserved_is_set = false;
  a->peak_bytes_reserved_is_set = false;
  a->bytes_reservable_limit_is_set = false;
  a->largest_free_block_bytes_is_set = false;
  a->pool_bytes_is_set = false;
  a->peak_pool_bytes_is_set = false;
  return nullptr;
}

PJRT_Error* DescId(PJRT_DeviceDescription_Id_Args* a) {
  a->id = a->device_description->id;
  return nullptr;
}
PJRT_Error* DescProcessIndex(PJRT_DeviceDescription_ProcessIndex_Args* a) {
  a->process_index = a->device_description->process_index;
  return nullptr;
}
PJRT_Error* DescAttributes(PJRT_DeviceDescription_Attributes_Args* a) {
  a->num_attributes = a->device_description->attrs.size();
  a->attributes = a->device_description->attrs.data();
  return nullptr;
}
PJRT_Error* DescKind(PJRT_DeviceDescription_Kind_Args* a) {
  a->device_kind = a->device_description->kind.c_str();
  a->device_kind_size = a->device_description->kind.size();
  return nullptr;
}
PJRT_Error* DescDebugString(PJRT_DeviceDescription_DebugString_Args* a) {
  a->debug_string = a->device_description->debug_string.c_str();
  a->debug_string_size = a->device_description->debug_string.size();
  return nullptr;
}
PJRT_Error* DescToString(PJRT_DeviceDescription_ToString_Args* a) {
  a->to_string = a->device_description->to_string.c_str();
  a->to_string_size = a->device_description->to_string.size();
  return nullptr;
}

// ------------------------------------------------------------------------------------------ memories
PJRT_Error* MemoryId(PJRT_Memory_Id_Args* a) { a->id = a->memory->id; return nullptr; }
PJRT_Error* MemoryKind(PJRT_Memory_Kind_Args* a) {
  a->kind = a->memory->kind.c_str();
  a->kind_size = a->memory->kind.size();
  return nullptr;
}
PJRT_Error* MemoryKindId(PJRT_Memory_Kind_Id_Args* a) { a->kind_id = a->memory->kind_id; return nullptr; }
PJRT_Error* MemoryDebugString(PJRT_Memory_DebugString_Args* a) {
  a->debug_string = a->memory->debug_string.c_str();
  a->debug_string_size = a->memory->debug_string.size();
  return nullptr;
}
PJRT_Error* MemoryToString(PJRT_Memory_ToString_Args* a) {
  a->to_string = a->memory->to_string.c_str();
  a->to_string_size = a->memory->to_string.size();
  return nullptr;
}
PJRT_Error* MemoryAddressableByDevices(PJRT_Memory_AddressableByDevices_Args* a) {
  a->devices = a->memory->devices.data();
  a->num_devices = a->memory->devices.size();
  return nullptr;
}

// ------------------------------------------------------------------------------------------ topology
PJRT_Error* TopologyCreate(PJRT_TopologyDescription_Create_Args* a) {
  auto* t = new PJRT_TopologyDescription();
  t->platform_version = kVersion;
  auto d = std::make_unique<PJRT_DeviceDescription>();
  FillDescription(d.get(), 0, 0, false);
  t->descriptions.push_back(d.get());
  t->owned.push_back(std::move(d));
  a->topology = t;
  return nullptr;
}
PJRT_Error* TopologyDestroy(PJRT_TopologyDescription_Destroy_Args* a) {
  delete a->topology;
  return nullptr;
}
PJRT_Error* TopologyPlatformName(PJRT_TopologyDescription_PlatformName_Args* a) {
  a->platform_name = a->topology->platform_name.c_str();
  a->platform_name_size = a->topology->platform_name.size();
  return nullptr;
}
PJRT_Error* TopologyPlatformVersion(PJRT_TopologyDescription_PlatformVersion_Args* a) {
  a->platform_version = a->topology->platform_version.c_str();
  a->platform_version_size = a->topology->platform_version.size();
  return nullptr;
}
PJRT_Error* TopologyGetDeviceDescriptions(PJRT_TopologyDescription_GetDeviceDescriptions_Args* a) {
  a->descriptions = a->topology->descriptions.data();
  a->num_descriptions = a->topology->descriptions.size();
  return nullptr;
}
PJRT_Error* TopologyAttributes(PJRT_TopologyDescription_Attributes_Args* a) {
  a->attributes = nullptr;
  a->num_attributes = 0;
  return nullptr;
}

PJRT_Error* ExecuteContextCreate(PJRT_ExecuteContext_Create_Args* a) {
  a->context = new PJRT_ExecuteContext();
  return nullptr;
}
PJRT_Error* ExecuteContextDestroy(PJRT_ExecuteContext_Destroy_Args* a) {
  delete a->context;
  return nullptr;
}

// ------------------------------------------------------------------------------------------ buffers
PJRT_Error* ClientBufferFromHostBuffer(PJRT_Client_BufferFromHostBuffer_Args* a) {
  const size_t width = ByteWidth(a->type);
  if (width == 0) return Err(PJRT_Error_Code_UNIMPLEMENTED, "BufferFromHostBuffer: unsupported element type");
  size_t count = 1;
  for (size_t i = 0; i < a->num_dims; ++i) {
    if (a->dims[i] < 0) return Err(PJRT_Error_Code_INVALID_ARGUMENT, "BufferFromHostBuffer: negative dimension");
    count *= (size_t)a->dims[i];
  }
  const size_t nbytes = count * width;
  if (a->num_byte_strides) {
    // only dense row-major host layouts (the reference assumes the same, pjrt_c_api.cc:492-522)
    int64_t expect = (int64_t)width;
    for (int i = (int)a->num_dims - 1; i >= 0; --i) {
      if (a->dims[i] > 1 && a->byte_strides[i] != expect)
        return Err(PJRT_Error_Code_UNIMPLEMENTED, "BufferFromHostBuffer: non-dense host strides");
      expect *= a->dims[i];
    }
  }
  PJRT_Device* device = a->device;
  PJRT_Memory* memory = a->memory;
  if (!device && memory && !memory->devices.empty()) device = memory->devices.front();
  if (!device) device = a->client->addressable_devices.front();
  if (!memory) memory = device->default_memory;
  if (!device->addressable) return Err(PJRT_Error_Code_INVALID_ARGUMENT, "BufferFromHostBuffer: device is not addressable");
  cudaSetDevice(device->state.ordinal);
  cudaStream_t st = device->state.stream;
  void* d = nullptr;
  std::string e = b200::DeviceAlloc(nbytes, st, &d);
  if (!e.empty()) return Err(PJRT_Error_Code_RESOURCE_EXHAUSTED, "BufferFromHostBuffer: " + e);
  if (nbytes && cudaMemcpyAsync(d, a->data, nbytes, cudaMemcpyHostToDevice, st) != cudaSuccess) {
    cudaGetLastError();
    b200::DeviceFree(d, st);
    return Err(PJRT_Error_Code_INTERNAL, "BufferFromHostBuffer: host to device copy failed");
  }
  auto ev = RecordState(device->state.ordinal, st);
  if (a->host_buffer_semantics == PJRT_HostBufferSemantics_kImmutableOnlyDuringCall) ev->Complete();
  auto* buf = new PJRT_Buffer();
  buf->client = a->client;
  buf->device = device;
  buf->memory = memory;
  buf->type = a->type;
  buf->dims.assign(a->dims, a->dims + a->num_dims);
  buf->nbytes = nbytes;
  buf->data = d;
  buf->ready = ev;
  a->done_with_host_buffer = NewEvent(ev);
  a->buffer = buf;
  return nullptr;
}

PJRT_Error* BufferToHostBuffer(PJRT_Buffer_ToHostBuffer_Args* a) {
  PJRT_Buffer* b = a->src;
  if (a->dst == nullptr) {
    a->dst_size = b->nbytes;
    a->event = NewEvent(ReadyState());
    return nullptr;
  }
  if (b->deleted || !b->data) return Err(PJRT_Error_Code_INVALID_ARGUMENT, "ToHostBuffer: buffer has been deleted");
  if (a->dst_size < b->nbytes) return Err(PJRT_Error_Code_INVALID_ARGUMENT, "ToHostBuffer: dst_size too small");
  cudaSetDevice(b->device->state.ordinal);
  cudaStream_t st = b->device->state.stream;
  if (b->nbytes && cudaMemcpyAsync(a->dst, b->data, b->nbytes, cudaMemcpyDeviceToHost, st) != cudaSuccess) {
    cudaGetLastError();
    return Err(PJRT_Error_Code_INTERNAL, "ToHostBuffer: device to host copy failed");
  }
  a->event = NewEvent(RecordState(b->device->state.ordinal, st, true));
  return nullptr;
}

PJRT_Buffer* CopyBuffer(PJRT_Buffer* src, PJRT_Device* dev, PJRT_Memory* mem, std::string* err) {
  if (!dev || !dev->addressable) { *err = "destination device is not addressable"; return nullptr; }
  cudaSetDevice(dev->state.ordinal);
  void* d = nullptr;
  *err = b200::DeviceAlloc(src->nbytes, dev->state.stream, &d);
  if (!err->empty()) return nullptr;
  if (src->device == dev) {
    cudaMemcpyAsync(d, src->data, src->nbytes, cudaMemcpyDeviceToDevice, dev->state.stream);
  } else {
    src->ready->Complete();
    cudaMemcpyPeerAsync(d, dev->state.ordinal, src->data, src->device->state.ordinal, src->nbytes, dev->state.stream);
  }
  auto* b = new PJRT_Buffer();
  b->client = src->client;
  b->device = dev;
  b->memory = mem ? mem : dev->default_memory;
  b->type = src->type;
  b->dims = src->dims;
  b->nbytes = src->nbytes;
  b->data = d;
  b->ready = RecordState(dev->state.ordinal, dev->state.stream);
  return b;
}

PJRT_Error* BufferCopyToMemory(PJRT_Buffer_CopyToMemory_Args* a) {
  if (a->buffer->deleted) return Err(PJRT_Error_Code_INVALID_ARGUMENT, "CopyToMemory: deleted buffer");
  PJRT_Memory* mem = a->dst_memory;
  PJRT_Device* dev = (mem && !mem->devices.empty()) ? mem->devices.front() : a->buffer->device;
  std::string err;
  PJRT_Buffer* nb = CopyBuffer(a->buffer, dev, mem, &err);
  if (!nb) return Err(PJRT_Error_Code_RESOURCE_EXHAUSTED, "CopyToMemory: " + err);
  a->dst_buffer = nb;
  return nullptr;
}
PJRT_Error* BufferCopyToDevice(PJRT_Buffer_CopyToDevice_Args* a) {
  if (a->buffer->deleted) return Err(PJRT_Error_Code_INVALID_ARGUMENT, "CopyToDevice: deleted buffer");
  std::string err;
  PJRT_Buffer* nb = CopyBuffer(a->buffer, a->dst_device, nullptr, &err);
  if (!nb) return Err(PJRT_Error_Code_RESOURCE_EXHAUSTED, "CopyToDevice: " + err);
  a->dst_buffer = nb;
  return nullptr;
}

void ReleaseStorage(PJRT_Buffer* b) {
  if (b->data) {
    cudaSetDevice(b->device->state.ordinal);
    b200::DeviceFree(b->data, b->device->state.stream);
    b->data = nullptr;
  }
}

PJRT_Error* BufferDestroy(PJRT_Buffer_Destroy_Args* a) {
  ReleaseStorage(a->buffer);
  delete a->buffer;
  return nullptr;
}
PJRT_Error* BufferDelete(PJRT_Buffer_Delete_Args* a) {
  a->buffer->deleted = true;
  if (a->buffer->external_refs == 0) ReleaseStorage(a->buffer);
  else a->buffer->delete_requested = true;
  return nullptr;
}
PJRT_Error* BufferIsDeleted(PJRT_Buffer_IsDeleted_Args* a) {
  a->is_deleted = a->buffer->deleted;
  return nullptr;
}
PJRT_Error* BufferElementType(PJRT_Buffer_ElementType_Args* a) {
  a->type = a->buffer->type;
  return nullptr;
}
PJRT_Error* BufferDimensions(PJRT_Buffer_Dimensions_Args* a) {
  a->dims = a->buffer->dims.data();
  a->num_dims = a->buffer->dims.size();
  return nullptr;
}
PJRT_Error* BufferUnpaddedDimensions(PJRT_Buffer_UnpaddedDimensions_Args* a) {
  a->unpadded_dims = a->buffer->dims.data();
  a->num_dims = a->buffer->dims.size();
  return nullptr;
}
PJRT_Error* BufferDynamicDimensionIndices(PJRT_Buffer_DynamicDimensionIndices_Args* a) {
  a->dynamic_dim_indices = nullptr;
  a->num_dynamic_dims = 0;
  return nullptr;
}
PJRT_Error* BufferOnDeviceSizeInBytes(PJRT_Buffer_OnDeviceSizeInBytes_Args* a) {
  a->on_device_size_in_bytes = a->buffer->nbytes;
  return nullptr;
}
PJRT_Error* BufferDevice(PJRT_Buffer_Device_Args* a) {
  a->device = a->buffer->device;
  return nullptr;
}
PJRT_Error* BufferMemory(PJRT_Buffer_Memory_Args* a) {
  a->memory = a->buffer->memory;
  return nullptr;
}
PJRT_Error* BufferIsOnCpu(PJRT_Buffer_IsOnCpu_Args* a) {
  a->is_on_cpu = false;
  return nullptr;
}
PJRT_Error* BufferReadyEvent(PJRT_Buffer_ReadyEvent_Args* a) {
  a->event = NewEvent(a->buffer->ready ? a->buffer->ready : ReadyState());
  return nullptr;
}
PJRT_Error* BufferUnsafePointer(PJRT_Buffer_UnsafePointer_Args* a) {
  a->buffer_pointer = reinterpret_cast<uintptr_t>(a->buffer->data);
  return nullptr;
}
PJRT_Error* BufferOpaqueDeviceMemoryDataPointer(PJRT_Buffer_OpaqueDeviceMemoryDataPointer_Args* a) {
  a->device_memory_ptr = a->buffer->data;
  return nullptr;
}
PJRT_Error* BufferIncreaseExternalReferenceCount(PJRT_Buffer_IncreaseExternalReferenceCount_Args* a) {
  ++a->buffer->external_refs;
  return nullptr;
}
PJRT_Error* BufferDecreaseExternalReferenceCount(PJRT_Buffer_DecreaseExternalReferenceCount_Args* a) {
  if (a->buffer->external_refs > 0) --a->buffer->external_refs;
  if (a->buffer->external_refs == 0 && a->buffer->delete_requested) ReleaseStorage(a->buffer);
  return nullptr;
}

// ------------------------------------------------------------------------------------------ compile / execute
void CacheExecutableOutputs(PJRT_Executable* e) {
  const b200::Plan& p = e->program->plan();
  for (const auto& t : p.out_types) {
    e->out_types.push_back(ToPjrt(t.dt));
    e->out_dim_sizes.push_back(t.dims.size());
    for (int64_t d : t.dims) e->out_dims_flat.push_back(d);
    e->out_mem_kinds.push_back("device");
  }
  for (const auto& k : e->out_mem_kinds) {
    e->out_mem_kind_ptrs.push_back(k.c_str());
    e->out_mem_kind_sizes.push_back(k.size());
  }
}

PJRT_Error* ClientCompile(PJRT_Client_Compile_Args* a) {
  const PJRT_Program* p = a->program;
  if (!p || !p->code) return Err(PJRT_Error_Code_INVALID_ARGUMENT, "jam compile: empty program");
  std::string fmt(p->format ? p->format : "", p->format_size);
  if (!fmt.empty() && fmt != "mlir") return Err(PJRT_Error_Code_INVALID_ARGUMENT, "jam compile: unsupported program format '" + fmt + "'");
  if (const char* dump = std::getenv("JAM_DUMP_ARTIFACT")) {
    if (FILE* f = std::fopen(dump, "wb")) {
      std::fwrite(p->code, 1, p->code_size, f);
      std::fclose(f);
    }
  }
  b200::CompileOptions opt;
  opt.num_processes = a->client->num_processes;
  opt.rank = a->client->process_index;
  opt.fuse_attention = std::getenv("B200_NO_FLASH") == nullptr;
  std::unique_ptr<b200::Executable> ex;
  std::string err = b200::Executable::Build(p->code, p->code_size, opt, &ex);
  if (!err.empty()) return Err(PJRT_Error_Code_INVALID_ARGUMENT, "jam compile: " + err);
  auto le = std::make_unique<PJRT_LoadedExecutable>();
  le->client = a->client;
  le->program = std::shared_ptr<b200::Executable>(std::move(ex));
  le->devices = a->client->addressable_devices;
  a->executable = le.release();
  return nullptr;
}

PJRT_Error* LoadedGetExecutable(PJRT_LoadedExecutable_GetExecutable_Args* a) {
  if (!a->loaded_executable->program) return Err(PJRT_Error_Code_INVALID_ARGUMENT, "GetExecutable: deleted executable");
  auto* e = new PJRT_Executable();
  e->program = a->loaded_executable->program;
  e->name = e->program->name();
  CacheExecutableOutputs(e);
  a->executable = e;
  return nullptr;
}
PJRT_Error* ExecutableDestroy(PJRT_Executable_Destroy_Args* a) {
  delete a->executable;
  return nullptr;
}
PJRT_Error* ExecutableName(PJRT_Executable_Name_Args* a) {
  a->executable_name = a->executable->name.c_str();
  a->executable_name_size = a->executable->name.size();
  return nullptr;
}
PJRT_Error* ExecutableNumReplicas(PJRT_Executable_NumReplicas_Args* a) {
  a->num_replicas = 1;
  return nullptr;
}
PJRT_Error* ExecutableNumPartitions(PJRT_Executable_NumPartitions_Args* a) {
  a->num_partitions = (size_t)a->executable->program->plan().num_partitions;
  return nullptr;
}
PJRT_Error* ExecutableNumOutputs(PJRT_Executable_NumOutputs_Args* a) {
  a->num_outputs = a->executable->program->plan().out_types.size();
  return nullptr;
}
PJRT_Error* ExecutableOutputElementTypes(PJRT_Executable_OutputElementTypes_Args* a) {
  a->output_types = a->executable->out_types.data();
  a->num_output_types = a->executable->out_types.size();
  return nullptr;
}
PJRT_Error* ExecutableOutputDimensions(PJRT_Executable_OutputDimensions_Args* a) {
  auto* e = a->executable;
  a->num_outputs = e->out_dim_sizes.size();
  a->dims = e->out_dims_flat.data();
  a->dim_sizes = e->out_dim_sizes.data();
  return nullptr;
}
PJRT_Error* ExecutableOutputMemoryKinds(PJRT_Executable_OutputMemoryKinds_Args* a) {
  auto* e = a->executable;
  a->num_outputs = e->out_mem_kind_ptrs.size();
  a->memory_kinds = e->out_mem_kind_ptrs.data();
  a->memory_kind_sizes = e->out_mem_kind_sizes.data();
  return nullptr;
}
PJRT_Error* LoadedDestroy(PJRT_LoadedExecutable_Destroy_Args* a) {
  delete a->executable;
  return nullptr;
}
PJRT_Error* LoadedDelete(PJRT_LoadedExecutable_Delete_Args* a) {
  a->executable->deleted = true;
  a->executable->program.reset();
  return nullptr;
}
PJRT_Error* LoadedIsDeleted(PJRT_LoadedExecutable_IsDeleted_Args* a) {
  a->is_deleted = a->executable->deleted;
  return nullptr;
}
PJRT_Error* LoadedAddressableDevices(PJRT_LoadedExecutable_AddressableDevices_Args* a) {
  a->addressable_devices = a->executable->devices.data();
  a->num_addressable_devices = a->executable->devices.size();
  return nullptr;
}

PJRT_Error* LoadedExecute(PJRT_LoadedExecutable_Execute_Args* a) {
  PJRT_LoadedExecutable* le = a->executable;
  if (!le->program) return Err(PJRT_Error_Code_INVALID_ARGUMENT, "Execute: deleted executable");
  const b200::Plan& plan = le->program->plan();
  if (a->num_args != plan.arg_types.size())
    return Err(PJRT_Error_Code_INVALID_ARGUMENT, "Execute: expected " + std::to_string(plan.arg_types.size()) +
                                                     " arguments, got " + std::to_string(a->num_args));
  if (a->num_devices < 1) return Err(PJRT_Error_Code_INVALID_ARGUMENT, "Execute: no devices");
  for (size_t d = 0; d < a->num_devices; ++d) {
    PJRT_Device* dev = a->execute_device;
    if (!dev) dev = le->devices[d % le->devices.size()];
    if (!dev->addressable) return Err(PJRT_Error_Code_INVALID_ARGUMENT, "Execute: device is not addressable");
    std::vector<const void*> args;
    for (size_t i = 0; i < a->num_args; ++i) {
      PJRT_Buffer* b = a->argument_lists[d][i];
      const b200::TensorType& want = plan.arg_types[i];
      if (!b || b->deleted || (!b->data && b->nbytes))
        return Err(PJRT_Error_Code_INVALID_ARGUMENT, "Execute: argument " + std::to_string(i) + " is deleted");
      if (b->type != ToPjrt(want.dt) || b->dims != want.dims)
        return Err(PJRT_Error_Code_INVALID_ARGUMENT, "Execute: argument " + std::to_string(i) + " has shape " +
                                                         DimsStr(b->dims) + ", expected " + want.str());
      if (b->device != dev) {
        if (b->ready) b->ready->Complete();
      }
      args.push_back(b->data);
    }
    std::vector<void*> outs;
    {
      std::lock_guard<std::mutex> lock(dev->exec_mu);
      cudaSetDevice(dev->state.ordinal);
      std::string err = le->program->Run(dev->state, args, &outs, le->client->comm.get());
      if (!err.empty()) return Err(PJRT_Error_Code_INTERNAL, err);
    }
    auto ev = RecordState(dev->state.ordinal, dev->state.stream, true);
    for (size_t i = 0; i < outs.size(); ++i) {
      auto* ob = new PJRT_Buffer();
      ob->client = le->client;
      ob->device = dev;
      ob->memory = dev->default_memory;
      ob->type = ToPjrt(plan.out_types[i].dt);
      ob->dims = plan.out_types[i].dims;
      ob->nbytes = (size_t)plan.out_types[i].bytes();
      ob->data = outs[i];
      ob->ready = ev;
      a->output_lists[d][i] = ob;
    }
    if (a->device_complete_events) a->device_complete_events[d] = NewEvent(ev);
  }
  return nullptr;
}

#define B200_UNIMPLEMENTED(X)                                                                      \
  X(Executable_SizeOfGeneratedCodeInBytes) X(Executable_GetCostAnalysis) X(Executable_OptimizedProgram) \
  X(Executable_Serialize) X(Executable_DeserializeAndLoad) X(LoadedExecutable_Fingerprint)           \
  X(Buffer_GetMemoryLayout) X(CopyToDeviceStream_Destroy) X(CopyToDeviceStream_AddChunk)              \
  X(CopyToDeviceStream_TotalBytes) X(CopyToDeviceStream_GranuleSize) X(CopyToDeviceStream_CurrentBytes) \
  X(TopologyDescription_Serialize) X(Compile) X(Client_CreateViewOfDeviceBuffer) X(Executable_Fingerprint) \
  X(Executable_GetCompiledMemoryStats)

#define B200_DEFINE_STUB(name) \
  PJRT_Error* name##_Stub(PJRT_##name##_Args*) { return MakeUnimplemented(#name); }
B200_UNIMPLEMENTED(B200_DEFINE_STUB)
#undef B200_DEFINE_STUB

}  // namespace

extern "C" __attribute__((visibility("default"))) const PJRT_Api* GetPjrtApi(void) {
  static PJRT_Api api = [] {
    PJRT_Api a;
    std::memset(&a, 0, sizeof(a));
    a.struct_size = sizeof(PJRT_Api);
    a.pjrt_api_version.struct_size = sizeof(PJRT_Api_Version);
    a.pjrt_api_version.major_version = PJRT_API_MAJOR;
    a.pjrt_api_version.minor_version = PJRT_API_MINOR;

    a.PJRT_Error_Destroy = ErrorDestroy;
    a.PJRT_Error_Message = ErrorMessage;
    a.PJRT_Error_GetCode = ErrorGetCode;
    a.PJRT_Event_Destroy = EventDestroy;
    a.PJRT_Event_IsReady = EventIsReady;
    a.PJRT_Event_Error = EventError;
    a.PJRT_Event_Await = EventAwait;
    a.PJRT_Event_OnReady = EventOnReady;
    a.PJRT_Plugin_Initialize = PluginInitialize;
    a.PJRT_Plugin_Attributes = PluginAttributes;

    a.PJRT_Client_Create = ClientCreate;
    a.PJRT_Client_Destroy = ClientDestroy;
    a.PJRT_Client_PlatformName = ClientPlatformName;
    a.PJRT_Client_PlatformVersion = ClientPlatformVersion;
    a.PJRT_Client_ProcessIndex = ClientProcessIndex;
    a.PJRT_Client_Devices = ClientDevices;
    a.PJRT_Client_AddressableDevices = ClientAddressableDevices;
    a.PJRT_Client_AddressableMemories = ClientAddressableMemories;
    a.PJRT_Client_LookupDevice = ClientLookupDevice;
    a.PJRT_Client_LookupAddressableDevice = ClientLookupAddressableDevice;
    a.PJRT_Client_DefaultDeviceAssignment = ClientDefaultDeviceAssignment;
    a.PJRT_Client_TopologyDescription = ClientTopologyDescription;
    a.PJRT_Client_BufferFromHostBuffer = ClientBufferFromHostBuffer;
    a.PJRT_Client_Compile = ClientCompile;

    a.PJRT_Device_GetDescription = DeviceGetDescription;
    a.PJRT_Device_IsAddressable = DeviceIsAddressable;
    a.PJRT_Device_LocalHardwareId = DeviceLocalHardwareId;
    a.PJRT_Device_AddressableMemories = DeviceAddressableMemories;
    a.PJRT_Device_DefaultMemory = DeviceDefaultMemory;
    a.PJRT_Device_MemoryStats = DeviceMemoryStats;
    a.PJRT_DeviceDescription_Id = DescId;
    a.PJRT_DeviceDescription_ProcessIndex = DescProcessIndex;
    a.PJRT_DeviceDescription_Attributes = DescAttributes;
    a.PJRT_DeviceDescription_Kind = DescKind;
    a.PJRT_DeviceDescription_DebugString = DescDebugString;
    a.PJRT_DeviceDescription_ToString = DescToString;

    a.PJRT_Memory_Id = MemoryId;
    a.PJRT_Memory_Kind = MemoryKind;
    a.PJRT_Memory_Kind_Id = MemoryKindId;
    a.PJRT_Memory_DebugString = MemoryDebugString;
    a.PJRT_Memory_ToString = MemoryToString;
    a.PJRT_Memory_AddressableByDevices = MemoryAddressableByDevices;

    a.PJRT_TopologyDescription_Create = TopologyCreate;
    a.PJRT_TopologyDescription_Destroy = TopologyDestroy;
    a.PJRT_TopologyDescription_PlatformName = TopologyPlatformName;
    a.PJRT_TopologyDescription_PlatformVersion = TopologyPlatformVersion;
    a.PJRT_TopologyDescription_GetDeviceDescriptions = TopologyGetDeviceDescriptions;
    a.PJRT_TopologyDescription_Attributes = TopologyAttributes;

    a.PJRT_ExecuteContext_Create = ExecuteContextCreate;
    a.PJRT_ExecuteContext_Destroy = ExecuteContextDestroy;

    a.PJRT_Buffer_Destroy = BufferDestroy;
    a.PJRT_Buffer_Delete = BufferDelete;
    a.PJRT_Buffer_IsDeleted = BufferIsDeleted;
    a.PJRT_Buffer_ElementType = BufferElementType;
    a.PJRT_Buffer_Dimensions = BufferDimensions;
    a.PJRT_Buffer_UnpaddedDimensions = BufferUnpaddedDimensions;
    a.PJRT_Buffer_DynamicDimensionIndices = BufferDynamicDimensionIndices;
    a.PJRT_Buffer_OnDeviceSizeInBytes = BufferOnDeviceSizeInBytes;
    a.PJRT_Buffer_Device = BufferDevice;
    a.PJRT_Buffer_Memory = BufferMemory;
    a.PJRT_Buffer_IsOnCpu = BufferIsOnCpu;
    a.PJRT_Buffer_ReadyEvent = BufferReadyEvent;
    a.PJRT_Buffer_ToHostBuffer = BufferToHostBuffer;
    a.PJRT_Buffer_CopyToMemory = BufferCopyToMemory;
    a.PJRT_Buffer_CopyToDevice = BufferCopyToDevice;
    a.PJRT_Buffer_UnsafePointer = BufferUnsafePointer;
    a.PJRT_Buffer_OpaqueDeviceMemoryDataPointer = BufferOpaqueDeviceMemoryDataPointer;
    a.PJRT_Buffer_IncreaseExternalReferenceCount = BufferIncreaseExternalReferenceCount;
    a.PJRT_Buffer_DecreaseExternalReferenceCount = BufferDecreaseExternalReferenceCount;

    a.PJRT_Executable_Destroy = ExecutableDestroy;
    a.PJRT_Executable_Name = ExecutableName;
    a.PJRT_Executable_NumReplicas = ExecutableNumReplicas;
    a.PJRT_Executable_NumPartitions = ExecutableNumPartitions;
    a.PJRT_Executable_NumOutputs = ExecutableNumOutputs;
    a.PJRT_Executable_OutputElementTypes = ExecutableOutputElementTypes;
    a.PJRT_Executable_OutputDimensions = ExecutableOutputDimensions;
    a.PJRT_Executable_OutputMemoryKinds = ExecutableOutputMemoryKinds;
    a.PJRT_LoadedExecutable_Destroy = LoadedDestroy;
    a.PJRT_LoadedExecutable_GetExecutable = LoadedGetExecutable;
    a.PJRT_LoadedExecutable_AddressableDevices = LoadedAddressableDevices;
    a.PJRT_LoadedExecutable_Delete = LoadedDelete;
    a.PJRT_LoadedExecutable_IsDeleted = LoadedIsDeleted;
    a.PJRT_LoadedExecutable_Execute = LoadedExecute;

#define B200_BIND_STUB(name) a.PJRT_##name = name##_Stub;
    B200_UNIMPLEMENTED(B200_BIND_STUB)
#undef B200_BIND_STUB
    return a;
  }();
  return &api;
}
