// plugin.cc — the PJRT C API (v0.55) over B200 devices: the plugin's drop-in boundary, GetPjrtApi.
//
// The reference plugin (src/pjrt/api/pjrt_c_api.cc) fixes what a caller sees: which entry points
// work and which answer UNIMPLEMENTED (its list at :833-873), the error codes (INVALID_ARGUMENT for
// bad arguments and "jam compile: ..." failures, RESOURCE_EXHAUSTED for allocation, INTERNAL for
// execution and communicator failures), one addressable device per process, and two memories per
// device ("device", "pinned_host").  The implementation here is its own:
//
//   PJRT_Client   the process's view of a job of `world` processes: one device per process, the local
//                 one bound to a CUDA ordinal; the NCCL communicator when world > 1.
//   PJRT_Device   a global device id with its two memory spaces embedded (HBM and page-locked host
//                 memory) and, for the local device, the executor's CUDA state.
//   PJRT_Buffer   typed, shaped storage in one memory space -- HBM from the executor's stream-ordered
//                 pool, or cudaHostAlloc'd host memory -- with a completion for its contents and a
//                 pin count for external references.
//   PJRT_Event    a Completion: a CUDA event the host can poll, await or attach callbacks to.
//   PJRT_(Loaded)Executable   a compiled b200::Executable and its output signature.
// The API table is bound from small lambdas grouped by object (Bind* below).
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstddef>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <functional>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <tuple>
#include <vector>

#include "../../../include/b200_kernels.h"
#include "../../../include/pjrt_b200.h"
#include "../comm/comm.h"
#include "../jam/runtime.h"
#include "compile_options.h"

struct PJRT_Error {
  PJRT_Error_Code code;
  std::string text;
};

namespace b200pj {

PJRT_Error* Fail(PJRT_Error_Code code, std::string text) { return new PJRT_Error{code, std::move(text)}; }
PJRT_Error* BadArg(std::string text) { return Fail(PJRT_Error_Code_INVALID_ARGUMENT, std::move(text)); }

// Writes a plugin-owned string into a (pointer, size) pair of an Args struct.
inline void Put(const std::string& s, const char** p, size_t* n) {
  *p = s.data();
  *n = s.size();
}

const std::string kPlatform = "b200";
const std::string kPlatformVersion = "pjrt-b200 0.2.0 (PJRT 0.55, sm_100a)";

// ------------------------------------------------------------------------------------ completions
// The state behind a PJRT_Event: done once the CUDA event it recorded has completed on the GPU (or
// at once, for host-side work).  Callbacks run when it completes; a completion that follows kernel
// launches also reads the tensor-core kernels' timed-out-wait flag and turns it into an error.
class Completion {
 public:
  static std::shared_ptr<Completion> Done() {
    auto c = std::make_shared<Completion>();
    c->done_ = true;
    return c;
  }
  // Records an event on `stream`; falls back to a stream synchronize if that fails.
  static std::shared_ptr<Completion> After(int ordinal, cudaStream_t stream, bool reads_kernel_flags) {
    auto c = std::make_shared<Completion>();
    c->ordinal_ = ordinal;
    c->reads_kernel_flags_ = reads_kernel_flags;
    if (cudaEventCreateWithFlags(&c->event_, cudaEventDisableTiming) == cudaSuccess &&
        cudaEventRecord(c->event_, stream) == cudaSuccess)
      return c;
    cudaGetLastError();
    if (c->event_) cudaEventDestroy(c->event_);
    c->event_ = nullptr;
    cudaStreamSynchronize(stream);
    c->done_ = true;
    return c;
  }
  ~Completion() {
    if (event_) cudaEventDestroy(event_);
  }
  // For work that includes collectives: if it has not completed `ms` after a wait starts, run
  // `on_expiry` (which aborts the communicator, so the NCCL kernels waiting on it return) and report
  // DEADLINE_EXCEEDED.
  void SetDeadline(int ms, std::function<void()> on_expiry) {
    deadline_ms_ = ms;
    on_expiry_ = std::move(on_expiry);
  }

  // Blocks until done, then runs the callbacks (once).
  void Wait() {
    {
      std::lock_guard<std::mutex> g(mu_);
      if (done_) return;
    }
    PJRT_Error_Code code = PJRT_Error_Code_UNKNOWN;
    std::string problem;
    if (event_) {
      cudaSetDevice(ordinal_);
      bool expired = false;
      if (deadline_ms_ > 0) {
        const auto until = std::chrono::steady_clock::now() + std::chrono::milliseconds(deadline_ms_);
        const auto spin_until = std::chrono::steady_clock::now() + std::chrono::milliseconds(5);
        while (cudaEventQuery(event_) == cudaErrorNotReady) {
          const auto now = std::chrono::steady_clock::now();
          if (now > until) {
            expired = true;
            if (on_expiry_) on_expiry_();
            break;
          }
          if (now < spin_until) std::this_thread::yield();     // short waits: no sleep latency
          else std::this_thread::sleep_for(std::chrono::microseconds(100));
        }
      }
      const cudaError_t e = cudaEventSynchronize(event_);
      if (expired) {
        code = PJRT_Error_Code_DEADLINE_EXCEEDED;
        problem = "the execution's collectives did not complete within " + std::to_string(deadline_ms_) +
                  " ms; the communicator was aborted";
      } else if (e != cudaSuccess) {
        code = PJRT_Error_Code_INTERNAL;
        problem = std::string("device execution failed: ") + cudaGetErrorString(e);
      } else if (reads_kernel_flags_) {
        if (const int k = b200_take_device_error()) {
          code = PJRT_Error_Code_DEADLINE_EXCEEDED;
          problem = "a tensor-core kernel gave up waiting on a pipeline barrier (code " + std::to_string(k) + ")";
        }
      }
    }
    std::vector<std::pair<PJRT_Event_OnReadyCallback, void*>> run;
    {
      std::lock_guard<std::mutex> g(mu_);
      if (done_) return;
      done_ = true;
      failed_ = !problem.empty();
      code_ = code;
      problem_ = problem;
      run.swap(callbacks_);
    }
    for (auto& cb : run) cb.first(Status(), cb.second);
  }
  bool Ready() {
    {
      std::lock_guard<std::mutex> g(mu_);
      if (done_) return true;
    }
    if (event_) {
      cudaSetDevice(ordinal_);
      if (cudaEventQuery(event_) == cudaErrorNotReady) return false;
    }
    Wait();
    return true;
  }
  // A new PJRT_Error for a failed completion (the caller owns it), null otherwise.
  PJRT_Error* Status() {
    std::lock_guard<std::mutex> g(mu_);
    return failed_ ? Fail(code_, problem_) : nullptr;
  }
  // Runs `cb` now if done, else when done (a helper thread waits for the GPU).
  void Then(PJRT_Event_OnReadyCallback cb, void* arg, const std::shared_ptr<Completion>& self) {
    {
      std::lock_guard<std::mutex> g(mu_);
      if (!done_) {
        callbacks_.emplace_back(cb, arg);
        std::thread([self] { self->Wait(); }).detach();
        return;
      }
    }
    cb(Status(), arg);
  }

 private:
  std::mutex mu_;
  bool done_ = false, failed_ = false, reads_kernel_flags_ = false;
  PJRT_Error_Code code_ = PJRT_Error_Code_UNKNOWN;
  std::string problem_;
  cudaEvent_t event_ = nullptr;
  int ordinal_ = 0;
  int deadline_ms_ = 0;
  std::function<void()> on_expiry_;
  std::vector<std::pair<PJRT_Event_OnReadyCallback, void*>> callbacks_;
};

using CompletionRef = std::shared_ptr<Completion>;

// ------------------------------------------------------------------------------------ element types
// Bytes per element of each PJRT_Buffer_Type, indexed by the enum value (0: not storable here).
constexpr uint8_t kElementBytes[] = {
    /*INVALID*/ 0, /*PRED*/ 1, /*S8*/ 1, /*S16*/ 2, /*S32*/ 4, /*S64*/ 8, /*U8*/ 1, /*U16*/ 2, /*U32*/ 4, /*U64*/ 8,
    /*F16*/ 2, /*F32*/ 4, /*F64*/ 8, /*BF16*/ 2, /*C64*/ 8, /*C128*/ 16, /*F8E5M2*/ 1, /*F8E4M3FN*/ 1,
    /*F8E4M3B11FNUZ*/ 1, /*F8E5M2FNUZ*/ 1, /*F8E4M3FNUZ*/ 1, /*S4*/ 0, /*U4*/ 0, /*TOKEN*/ 0, /*S2*/ 0, /*U2*/ 0,
    /*F8E4M3*/ 1, /*F8E3M4*/ 1};

size_t ElementBytes(PJRT_Buffer_Type t) {
  const size_t i = (size_t)t;
  return i < sizeof(kElementBytes) ? kElementBytes[i] : 0;
}

// The compiler's element types and the PJRT ones (same names, PJRT numbering).
PJRT_Buffer_Type PjrtTypeOf(b200::DT d) {
  static const PJRT_Buffer_Type kMap[] = {
      PJRT_Buffer_Type_PRED, PJRT_Buffer_Type_S8,  PJRT_Buffer_Type_S16,  PJRT_Buffer_Type_S32, PJRT_Buffer_Type_S64,
      PJRT_Buffer_Type_U8,   PJRT_Buffer_Type_U16, PJRT_Buffer_Type_U32,  PJRT_Buffer_Type_U64, PJRT_Buffer_Type_F16,
      PJRT_Buffer_Type_BF16, PJRT_Buffer_Type_F32, PJRT_Buffer_Type_F64};
  const size_t i = (size_t)d;
  return i < sizeof(kMap) / sizeof(kMap[0]) ? kMap[i] : PJRT_Buffer_Type_INVALID;
}

std::string ShapeText(PJRT_Buffer_Type t, const std::vector<int64_t>& dims) {
  std::string s = "type " + std::to_string((int)t) + " [";
  for (size_t i = 0; i < dims.size(); ++i) s += (i ? "x" : "") + std::to_string(dims[i]);
  return s + "]";
}

// The two memory spaces every device has.
enum class Space : int { kHbm = 0, kPinnedHost = 1 };
const std::string kSpaceKind[2] = {"device", "pinned_host"};

int EnvInt(const char* name, int fallback) {
  const char* v = std::getenv(name);
  return v && *v ? std::atoi(v) : fallback;
}

// Named values the plugin reports (device attributes); owns the strings the entries point at.
class Attributes {
 public:
  void AddString(const std::string& name, const std::string& value) {
    Entry& e = Push(name);
    e.text = value;
    e.nv.type = PJRT_NamedValue_kString;
  }
  void AddInt(const std::string& name, int64_t value) {
    Entry& e = Push(name);
    e.nv.type = PJRT_NamedValue_kInt64;
    e.nv.int64_value = value;
    e.nv.value_size = 1;
  }
  // The PJRT_NamedValue array (pointers into this object; valid while it lives unchanged).
  const PJRT_NamedValue* Values() {
    flat_.clear();
    for (Entry& e : entries_) {
      e.nv.name = e.name.c_str();
      e.nv.name_size = e.name.size();
      if (e.nv.type == PJRT_NamedValue_kString) {
        e.nv.string_value = e.text.c_str();
        e.nv.value_size = e.text.size();
      }
      flat_.push_back(e.nv);
    }
    return flat_.data();
  }
  size_t Count() const { return entries_.size(); }

 private:
  struct Entry {
    std::string name, text;
    PJRT_NamedValue nv;
  };
  Entry& Push(const std::string& name) {
    entries_.emplace_back();
    Entry& e = entries_.back();
    std::memset(&e.nv, 0, sizeof(e.nv));
    e.nv.struct_size = sizeof(PJRT_NamedValue);
    e.name = name;
    return e;
  }
  std::deque<Entry> entries_;
  std::vector<PJRT_NamedValue> flat_;
};

// The output signature of a compiled program in the shapes PJRT returns it.
struct Signature {
  std::vector<PJRT_Buffer_Type> types;
  std::vector<size_t> ranks;
  std::vector<int64_t> dims;                   // all outputs' dims, concatenated
  std::vector<const char*> kinds;
  std::vector<size_t> kind_sizes;
  explicit Signature(const b200::Plan& plan) {
    for (const b200::TensorType& t : plan.out_types) {
      types.push_back(PjrtTypeOf(t.dt));
      ranks.push_back(t.dims.size());
      dims.insert(dims.end(), t.dims.begin(), t.dims.end());
      kinds.push_back(kSpaceKind[0].c_str());
      kind_sizes.push_back(kSpaceKind[0].size());
    }
  }
};

}  // namespace b200pj

using namespace b200pj;

// ======================================================================================= objects
struct PJRT_Event {
  CompletionRef done;
};

struct PJRT_DeviceDescription {
  int global_id = 0;
  int process = 0;
  std::string kind = "NVIDIA B200";
  std::string summary;       // ToString
  std::string detail;        // DebugString
  Attributes attributes;
  const PJRT_NamedValue* attribute_values = nullptr;

  // Fills the description of global device `id`; `ordinal` >= 0 reads the local GPU's properties.
  void Describe(int id, int ordinal) {
    global_id = id;
    process = id;                 // one device per process
    int major = 10, minor = 0, sms = 148;
    size_t hbm = 0;
    cudaDeviceProp prop;
    if (ordinal >= 0 && cudaGetDeviceProperties(&prop, ordinal) == cudaSuccess) {
      kind = prop.name;
      major = prop.major;
      minor = prop.minor;
      sms = prop.multiProcessorCount;
      hbm = prop.totalGlobalMem;
    }
    summary = "B200(id=" + std::to_string(id) + ", process=" + std::to_string(process) + ")";
    detail = "b200 device " + std::to_string(id) + (ordinal >= 0 ? " on cuda:" + std::to_string(ordinal) : " (remote)") +
             ", sm_" + std::to_string(major) + std::to_string(minor) + "a, " + std::to_string(sms) + " SMs";
    attributes.AddString("compute_capability", std::to_string(major) + "." + std::to_string(minor));
    attributes.AddInt("core_count", sms);
    attributes.AddString("device_vendor", "NVIDIA");
    if (hbm) attributes.AddInt("hbm_bytes", (int64_t)hbm);
    attribute_values = attributes.Values();
  }
};

struct PJRT_Memory {
  Space space = Space::kHbm;
  int id = 0;
  std::string summary, detail;
  PJRT_Device* owner[1] = {nullptr};
  const std::string& kind() const { return kSpaceKind[(int)space]; }
};

// Pinned host staging for small host-to-device uploads: the caller's bytes are copied here at once,
// so the call can release the caller's memory without waiting for the device stream to reach the
// copy (which queues behind every execution already enqueued).  A ring of 16 MiB; a range is
// reused once the copy that last read it has completed.
struct UploadStaging {
  static constexpr size_t kCap = 16u << 20, kMaxItem = 1u << 20;
  std::mutex mu;
  uint8_t* base = nullptr;
  size_t head = 0;
  std::deque<std::tuple<size_t, size_t, cudaEvent_t>> busy;   // (offset, bytes, copy done)
  ~UploadStaging() {
    for (auto& b : busy) cudaEventDestroy(std::get<2>(b));
    if (base) cudaFreeHost(base);
  }
};

struct PJRT_Device {
  PJRT_DeviceDescription desc;
  PJRT_Client* client = nullptr;
  int ordinal = -1;                     // CUDA device, -1 unless this process's device
  PJRT_Memory spaces[2];
  PJRT_Memory* space_list[2] = {nullptr, nullptr};
  b200::DeviceState cuda;               // executor state of the local device
  std::mutex launch_mu;                 // serializes Execute's enqueue on this device
  UploadStaging staging;
  bool local() const { return ordinal >= 0; }
  PJRT_Memory* hbm() { return &spaces[(int)Space::kHbm]; }
};

struct PJRT_TopologyDescription {
  std::vector<PJRT_DeviceDescription*> descriptions;
  std::deque<PJRT_DeviceDescription> owned;   // only for a topology created without a client
};

struct PJRT_Client {
  int rank = 0, world = 1;
  std::deque<PJRT_Device> fleet;              // every device of the job, by global id
  std::vector<PJRT_Device*> all, mine;
  std::vector<PJRT_Memory*> my_memories;
  PJRT_TopologyDescription topology;
  std::unique_ptr<b200::Comm> comm;

  PJRT_Device* local() { return mine.front(); }
  ~PJRT_Client() {
    for (PJRT_Device* d : mine) {                 // let queued work drain before the communicator goes
      cudaSetDevice(d->ordinal);
      if (d->cuda.stream) cudaStreamSynchronize(d->cuda.stream);
      if (d->cuda.comm_stream) cudaStreamSynchronize(d->cuda.comm_stream);
    }
    comm.reset();
    for (PJRT_Device* d : mine) {
      cudaSetDevice(d->ordinal);
      if (d->cuda.stream) cudaStreamDestroy(d->cuda.stream);
      if (d->cuda.comm_stream) cudaStreamDestroy(d->cuda.comm_stream);
    }
  }
};

struct PJRT_Buffer {
  enum class Life { kLive, kFreeWhenUnpinned, kFreed };
  PJRT_Client* client = nullptr;
  PJRT_Memory* where = nullptr;               // memory space, and through it the device
  PJRT_Buffer_Type etype = PJRT_Buffer_Type_INVALID;
  std::vector<int64_t> dims;
  size_t bytes = 0;
  void* ptr = nullptr;                         // device pointer (HBM) or host pointer (pinned host)
  CompletionRef ready;                         // contents are written once this completes
  int pins = 0;                                // external references
  Life life = Life::kLive;

  PJRT_Device* device() const { return where->owner[0]; }
  bool on_host() const { return where->space == Space::kPinnedHost; }
  bool usable() const { return life == Life::kLive && (ptr || bytes == 0); }
};

struct PJRT_ExecuteContext {};

struct PJRT_Executable {
  std::shared_ptr<b200::Executable> program;
  Signature outputs;
  explicit PJRT_Executable(std::shared_ptr<b200::Executable> p) : program(std::move(p)), outputs(program->plan()) {}
};

struct PJRT_LoadedExecutable {
  PJRT_Client* client = nullptr;
  std::shared_ptr<b200::Executable> program;   // null once deleted
  std::vector<PJRT_Device*> devices;
};

namespace {

// ======================================================================================= storage
// Allocates `bytes` in memory space `m`: HBM from the executor's stream-ordered pool on the owning
// device's stream, pinned host memory with cudaHostAlloc.
std::string Allocate(PJRT_Memory* m, size_t bytes, void** out) {
  *out = nullptr;
  PJRT_Device* d = m->owner[0];
  cudaSetDevice(d->ordinal);
  if (m->space == Space::kHbm) return b200::DeviceAlloc(bytes, d->cuda.stream, out);
  if (bytes == 0) return "";
  if (cudaHostAlloc(out, bytes, cudaHostAllocPortable) != cudaSuccess) {
    cudaGetLastError();
    *out = nullptr;
    return "pinned host allocation of " + std::to_string(bytes) + " bytes failed";
  }
  return "";
}

// Returns a buffer's storage.  HBM goes back to the pool stream-ordered; pinned host memory is freed
// once the device's stream has finished any copy that may still touch it.
void Release(PJRT_Buffer* b) {
  if (!b->ptr) return;
  PJRT_Device* d = b->device();
  cudaSetDevice(d->ordinal);
  if (b->on_host()) {
    cudaStreamSynchronize(d->cuda.stream);
    cudaFreeHost(b->ptr);
  } else {
    b200::DeviceFree(b->ptr, d->cuda.stream);
  }
  b->ptr = nullptr;
  b->life = PJRT_Buffer::Life::kFreed;
}

PJRT_Buffer* NewBuffer(PJRT_Client* c, PJRT_Memory* m, PJRT_Buffer_Type t, std::vector<int64_t> dims, size_t bytes,
                       void* ptr, CompletionRef ready) {
  auto* b = new PJRT_Buffer();
  b->client = c;
  b->where = m;
  b->etype = t;
  b->dims = std::move(dims);
  b->bytes = bytes;
  b->ptr = ptr;
  b->ready = std::move(ready);
  return b;
}

// A copy of `src` in memory space `dst` (same or another device, either space).
PJRT_Error* CopyInto(PJRT_Buffer* src, PJRT_Memory* dst, PJRT_Buffer** out) {
  if (!src->usable()) return BadArg("copy of a deleted buffer");
  PJRT_Device* to = dst->owner[0];
  if (!to->local()) return BadArg("copy to a device this process does not address");
  void* p = nullptr;
  std::string e = Allocate(dst, src->bytes, &p);
  if (!e.empty()) return Fail(PJRT_Error_Code_RESOURCE_EXHAUSTED, "buffer copy: " + e);
  PJRT_Device* from = src->device();
  cudaStream_t st = to->cuda.stream;
  if (from != to) src->ready->Wait();          // another device's stream: wait on the host
  cudaError_t ce = cudaSuccess;
  if (src->bytes) {
    if (from != to && !src->on_host() && dst->space == Space::kHbm)
      ce = cudaMemcpyPeerAsync(p, to->ordinal, src->ptr, from->ordinal, src->bytes, st);
    else
      ce = cudaMemcpyAsync(p, src->ptr, src->bytes, cudaMemcpyDefault, st);   // UVA: any space to any space
  }
  if (ce != cudaSuccess) {
    cudaGetLastError();
    PJRT_Buffer failed;
    failed.where = dst;
    failed.ptr = p;
    Release(&failed);
    return Fail(PJRT_Error_Code_INTERNAL, std::string("buffer copy failed: ") + cudaGetErrorString(ce));
  }
  CompletionRef done = Completion::After(to->ordinal, st, false);
  if (dst->space == Space::kPinnedHost) done->Wait();
  *out = NewBuffer(src->client, dst, src->etype, src->dims, src->bytes, p, done);
  return nullptr;
}

// ======================================================================================= client
// Builds the job's devices: `world` of them, device `rank` local on CUDA device `ordinal`.  Memory
// ids: HBM of device k is k, its pinned host memory world + k.
std::unique_ptr<PJRT_Client> MakeClient(int world, int rank, int ordinal) {
  auto c = std::make_unique<PJRT_Client>();
  c->rank = rank;
  c->world = world;
  for (int k = 0; k < world; ++k) {
    c->fleet.emplace_back();
    PJRT_Device& d = c->fleet.back();
    d.client = c.get();
    d.ordinal = k == rank ? ordinal : -1;
    d.desc.Describe(k, d.ordinal);
    for (int s = 0; s < 2; ++s) {
      PJRT_Memory& m = d.spaces[s];
      m.space = (Space)s;
      m.id = s * world + k;
      m.owner[0] = &d;
      m.summary = (s == 0 ? "HBM(device=" : "PinnedHost(device=") + std::to_string(k) + ")";
      m.detail = m.kind() + " memory " + std::to_string(m.id) + " of b200 device " + std::to_string(k);
      d.space_list[s] = &m;
    }
    d.cuda.ordinal = d.local() ? ordinal : 0;
    c->all.push_back(&d);
    c->topology.descriptions.push_back(&d.desc);
    if (d.local()) {
      c->mine.push_back(&d);
      c->my_memories = {&d.spaces[0], &d.spaces[1]};
    }
  }
  return c;
}

// The kv_put / kv_get callbacks of PJRT_Client_Create as the communicator's key-value store.
b200::KvStore StoreFrom(const PJRT_Client_Create_Args* a) {
  b200::KvStore kv;
  if (!a->kv_put_callback || !a->kv_get_callback) return kv;
  PJRT_KeyValuePutCallback put = a->kv_put_callback;
  PJRT_KeyValueGetCallback get = a->kv_get_callback;
  void* put_arg = a->kv_put_user_arg;
  void* get_arg = a->kv_get_user_arg;
  kv.put = [put, put_arg](const std::string& key, const std::string& value) -> std::string {
    PJRT_KeyValuePutCallback_Args x;
    std::memset(&x, 0, sizeof(x));
    x.struct_size = sizeof(x);
    x.key = key.data();
    x.key_size = key.size();
    x.value = value.data();
    x.value_size = value.size();
    x.user_arg = put_arg;
    return put(&x) ? "the kv_put callback reported an error" : "";
  };
  kv.get = [get, get_arg](const std::string& key, int timeout_ms, std::string* value) -> std::string {
    PJRT_KeyValueGetCallback_Args x;
    std::memset(&x, 0, sizeof(x));
    x.struct_size = sizeof(x);
    x.key = key.data();
    x.key_size = key.size();
    x.timeout_in_ms = timeout_ms;
    x.user_arg = get_arg;
    if (get(&x)) return "the kv_get callback reported an error";
    value->assign(x.value, x.value_size);
    if (x.value_deleter_callback) x.value_deleter_callback(x.value);
    return "";
  };
  return kv;
}

PJRT_Error* CreateClient(PJRT_Client_Create_Args* a) {
  // recognised int64 options; anything else is ignored, as jax passes options for other backends
  int64_t rank = 0, world = 1, ordinal = -1, nccl_max_ctas = 0;
  struct Known { const char* name; int64_t* slot; } known[] = {{"node_id", &rank}, {"num_nodes", &world},
                                                                {"device_ordinal", &ordinal},
                                                                {"nccl_max_ctas", &nccl_max_ctas}};
  for (size_t i = 0; i < a->num_options; ++i) {
    const PJRT_NamedValue& nv = a->create_options[i];
    if (nv.type != PJRT_NamedValue_kInt64) continue;
    for (const Known& k : known)
      if (nv.name_size == std::strlen(k.name) && std::memcmp(nv.name, k.name, nv.name_size) == 0) *k.slot = nv.int64_value;
  }
  world = std::max<int64_t>(world, 1);
  if (rank < 0 || rank >= world) rank = 0;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cudaGetLastError();
    return Fail(PJRT_Error_Code_FAILED_PRECONDITION, "no CUDA device is visible to the B200 plugin");
  }
  if (ordinal < 0) ordinal = EnvInt("LOCAL_RANK", (int)(rank % count));
  if (ordinal >= count) return BadArg("device_ordinal " + std::to_string(ordinal) + " out of range");
  std::unique_ptr<PJRT_Client> c = MakeClient((int)world, (int)rank, (int)ordinal);
  PJRT_Device* d = c->local();
  cudaSetDevice((int)ordinal);
  if (cudaStreamCreateWithFlags(&d->cuda.stream, cudaStreamNonBlocking) != cudaSuccess)
    return Fail(PJRT_Error_Code_INTERNAL, "cudaStreamCreate failed");
  // freed pool memory stays cached for stream-ordered reuse instead of going back to the driver
  cudaMemPool_t pool;
  if (cudaDeviceGetDefaultMemPool(&pool, (int)ordinal) == cudaSuccess) {
    uint64_t keep = UINT64_MAX;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
  }
  if (world > 1) {
    std::string err;
    c->comm = b200::Comm::Create((int)world, (int)rank, (int)ordinal, StoreFrom(a), EnvInt("B200_COMM_TIMEOUT_MS", 120000),
                                 &err, (int)nccl_max_ctas);
    if (!c->comm)
      return Fail(err.find("timed out") != std::string::npos ? PJRT_Error_Code_DEADLINE_EXCEEDED : PJRT_Error_Code_INTERNAL,
                  "NCCL communicator init failed: " + err);
  }
  a->client = c.release();
  return nullptr;
}

// ======================================================================================= transfers
// Copies `bytes` of host data into device d's staging ring (waiting, rarely, for the copy that last
// read the range) and returns its address in *src; the ring stays locked until StagedCopyIssued
// records the completion of the copy that reads it.
bool Stage(PJRT_Device* d, const void* data, size_t bytes, const void** src) {
  UploadStaging& g = d->staging;
  g.mu.lock();
  if (!g.base) {
    void* b = nullptr;
    if (cudaHostAlloc(&b, UploadStaging::kCap, cudaHostAllocPortable) != cudaSuccess) {
      cudaGetLastError();
      g.mu.unlock();
      return false;
    }
    g.base = (uint8_t*)b;
  }
  size_t off = (g.head + 255) & ~(size_t)255;
  if (off + bytes > UploadStaging::kCap) off = 0;
  // wait for (and forget) the earlier copies that read any byte of [off, off + bytes)
  for (auto it = g.busy.begin(); it != g.busy.end();) {
    const size_t o = std::get<0>(*it), n = std::get<1>(*it);
    if (o < off + bytes && off < o + n) {
      cudaEventSynchronize(std::get<2>(*it));
      cudaEventDestroy(std::get<2>(*it));
      it = g.busy.erase(it);
    } else {
      ++it;
    }
  }
  std::memcpy(g.base + off, data, bytes);
  g.head = off + bytes;
  g.busy.push_back({off, bytes, nullptr});
  *src = g.base + off;
  return true;
}

void StagedCopyIssued(PJRT_Device* d) {
  UploadStaging& g = d->staging;
  cudaEvent_t e = nullptr;
  if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) == cudaSuccess) {
    cudaEventRecord(e, d->cuda.stream);
    std::get<2>(g.busy.back()) = e;
  } else {
    cudaGetLastError();
    cudaStreamSynchronize(d->cuda.stream);    // no event: let the copy finish before the range is reused
    g.busy.pop_back();
  }
  g.mu.unlock();
}

PJRT_Error* FromHost(PJRT_Client_BufferFromHostBuffer_Args* a) {
  const size_t width = ElementBytes(a->type);
  if (width == 0) return Fail(PJRT_Error_Code_UNIMPLEMENTED, "BufferFromHostBuffer: unsupported element type");
  size_t count = 1;
  for (size_t i = 0; i < a->num_dims; ++i) {
    if (a->dims[i] < 0) return BadArg("BufferFromHostBuffer: negative dimension");
    count *= (size_t)a->dims[i];
  }
  if (a->num_byte_strides) {
    // dense row-major host data only: each stride is the bytes of the dimensions after it
    size_t dense = width;
    for (size_t i = a->num_dims; i-- > 0;) {
      if (a->dims[i] > 1 && a->byte_strides[i] != (int64_t)dense)
        return Fail(PJRT_Error_Code_UNIMPLEMENTED, "BufferFromHostBuffer: non-dense host strides");
      dense *= (size_t)a->dims[i];
    }
  }
  PJRT_Memory* m = a->memory;
  if (!m) m = (a->device ? a->device : a->client->local())->hbm();
  if (a->device && m->owner[0] != a->device) return BadArg("BufferFromHostBuffer: memory is not on the given device");
  PJRT_Device* d = m->owner[0];
  if (!d->local()) return BadArg("BufferFromHostBuffer: device is not addressable");
  const size_t bytes = count * width;
  void* p = nullptr;
  std::string e = Allocate(m, bytes, &p);
  if (!e.empty()) return Fail(PJRT_Error_Code_RESOURCE_EXHAUSTED, "BufferFromHostBuffer: " + e);
  CompletionRef done;
  if (m->space == Space::kPinnedHost) {
    if (bytes) std::memcpy(p, a->data, bytes);
    done = Completion::Done();
  } else {
    const void* src = a->data;
    bool staged = false;
    if (bytes && bytes <= UploadStaging::kMaxItem) staged = Stage(d, a->data, bytes, &src);
    if (bytes && cudaMemcpyAsync(p, src, bytes, cudaMemcpyHostToDevice, d->cuda.stream) != cudaSuccess) {
      cudaGetLastError();
      if (staged) {
        d->staging.busy.pop_back();
        d->staging.mu.unlock();
      }
      b200::DeviceFree(p, d->cuda.stream);
      return Fail(PJRT_Error_Code_INTERNAL, "BufferFromHostBuffer: host to device copy failed");
    }
    done = Completion::After(d->ordinal, d->cuda.stream, false);
    if (staged) {
      StagedCopyIssued(d);
      a->buffer = NewBuffer(a->client, m, a->type, std::vector<int64_t>(a->dims, a->dims + a->num_dims), bytes, p, done);
      a->done_with_host_buffer = new PJRT_Event{Completion::Done()};   // the caller's bytes are copied
      return nullptr;
    }
    // the caller may reuse its host memory when this call returns
    if (a->host_buffer_semantics == PJRT_HostBufferSemantics_kImmutableOnlyDuringCall) done->Wait();
  }
  a->buffer = NewBuffer(a->client, m, a->type, std::vector<int64_t>(a->dims, a->dims + a->num_dims), bytes, p, done);
  a->done_with_host_buffer = new PJRT_Event{done};
  return nullptr;
}

PJRT_Error* ToHost(PJRT_Buffer_ToHostBuffer_Args* a) {
  PJRT_Buffer* b = a->src;
  if (!a->dst) {                                 // size query
    a->dst_size = b->bytes;
    a->event = new PJRT_Event{Completion::Done()};
    return nullptr;
  }
  if (!b->usable()) return BadArg("ToHostBuffer: buffer has been deleted");
  if (a->dst_size < b->bytes) return BadArg("ToHostBuffer: dst_size too small");
  PJRT_Device* d = b->device();
  if (b->on_host()) {
    b->ready->Wait();
    if (b->bytes) std::memcpy(a->dst, b->ptr, b->bytes);
    a->event = new PJRT_Event{Completion::Done()};
    return nullptr;
  }
  cudaSetDevice(d->ordinal);
  if (b->bytes && cudaMemcpyAsync(a->dst, b->ptr, b->bytes, cudaMemcpyDeviceToHost, d->cuda.stream) != cudaSuccess) {
    cudaGetLastError();
    return Fail(PJRT_Error_Code_INTERNAL, "ToHostBuffer: device to host copy failed");
  }
  a->event = new PJRT_Event{Completion::After(d->ordinal, d->cuda.stream, true)};
  return nullptr;
}

// ======================================================================================= execute
PJRT_Error* Execute(PJRT_LoadedExecutable_Execute_Args* a) {
  PJRT_LoadedExecutable* le = a->executable;
  if (!le->program) return BadArg("Execute: deleted executable");
  const b200::Plan& plan = le->program->plan();
  if (a->num_args != plan.arg_types.size())
    return BadArg("Execute: expected " + std::to_string(plan.arg_types.size()) + " arguments, got " +
                  std::to_string(a->num_args));
  if (a->num_devices < 1) return BadArg("Execute: no devices");
  // donation: an argument the program marks donatable (tf.aliasing_output / jax.buffer_donor) is
  // given up unless the options list it as non-donatable
  std::vector<bool> donatable(a->num_args, false);
  for (size_t i = 0; i < a->num_args && i < plan.arg_donor.size(); ++i) donatable[i] = plan.arg_donor[i];
  if (a->options && a->options->non_donatable_input_indices)
    for (size_t j = 0; j < a->options->num_non_donatable_input_indices; ++j) {
      const int64_t i = a->options->non_donatable_input_indices[j];
      if (i >= 0 && (size_t)i < donatable.size()) donatable[i] = false;
    }
  for (size_t k = 0; k < a->num_devices; ++k) {
    PJRT_Device* dev = a->execute_device ? a->execute_device : le->devices[k % le->devices.size()];
    if (!dev->local()) return BadArg("Execute: device is not addressable");
    std::vector<const void*> args(a->num_args);
    for (size_t i = 0; i < a->num_args; ++i) {
      PJRT_Buffer* b = a->argument_lists[k][i];
      const b200::TensorType& want = plan.arg_types[i];
      if (!b || !b->usable()) return BadArg("Execute: argument " + std::to_string(i) + " is deleted");
      if (b->etype != PjrtTypeOf(want.dt) || b->dims != want.dims)
        return BadArg("Execute: argument " + std::to_string(i) + " is " + ShapeText(b->etype, b->dims) + ", expected " +
                      want.str());
      if (b->on_host())
        return BadArg("Execute: argument " + std::to_string(i) +
                      " is in pinned_host memory; executables read device memory (copy it there first)");
      if (b->device() != dev) b->ready->Wait();   // written on another device's stream
      args[i] = b->ptr;
    }
    std::vector<bool> donated(a->num_args, false);
    for (size_t i = 0; i < a->num_args; ++i) {
      if (!donatable[i]) continue;
      PJRT_Buffer* b = a->argument_lists[k][i];
      if (b->pins > 0)
        return BadArg("Execute: argument " + std::to_string(i) + " is donated but has external references");
      for (size_t j = 0; j < a->num_args; ++j)
        if (j != i && a->argument_lists[k][j] == b)
          return BadArg("Execute: argument " + std::to_string(i) + " is donated and also passed as argument " +
                        std::to_string(j));
      donated[i] = b->device() == dev;           // a buffer on another device is copied, not given up
    }
    std::vector<void*> outs;
    std::vector<bool> taken;
    {
      std::lock_guard<std::mutex> g(dev->launch_mu);
      cudaSetDevice(dev->ordinal);
      std::string err = le->program->Run(dev->cuda, args, &outs, le->client->comm.get(), &donated, &taken);
      if (!err.empty())
        return Fail(err.find("timed out") != std::string::npos ? PJRT_Error_Code_DEADLINE_EXCEEDED : PJRT_Error_Code_INTERNAL,
                    err);
    }
    CompletionRef done = Completion::After(dev->ordinal, dev->cuda.stream, true);
    if (b200::Comm* comm = le->client->comm.get()) {
      bool collectives = false;
      for (const b200::Step& st : plan.steps) collectives = collectives || st.kind == b200::StepKind::kCollective;
      if (collectives)
        done->SetDeadline(EnvInt("B200_COLLECTIVE_TIMEOUT_MS", 600000), [comm] {
          comm->Abort("a collective did not complete within its deadline");
        });
    }
    for (size_t i = 0; i < outs.size(); ++i) {
      const b200::TensorType& t = plan.out_types[i];
      a->output_lists[k][i] = NewBuffer(le->client, dev->hbm(), PjrtTypeOf(t.dt), t.dims, (size_t)t.bytes(), outs[i], done);
    }
    // donated arguments are deleted: their memory is now a result's, or goes back to the pool once
    // the execution is done with it (stream-ordered)
    for (size_t i = 0; i < a->num_args; ++i) {
      if (!donated[i]) continue;
      PJRT_Buffer* b = a->argument_lists[k][i];
      if (i < taken.size() && taken[i]) {
        b->ptr = nullptr;
        b->life = PJRT_Buffer::Life::kFreed;
      } else {
        Release(b);
      }
    }
    if (a->device_complete_events) a->device_complete_events[k] = new PJRT_Event{done};
  }
  return nullptr;
}

PJRT_Error* CompileProgram(PJRT_Client_Compile_Args* a) {
  const PJRT_Program* p = a->program;
  if (!p || !p->code) return BadArg("jam compile: empty program");
  const std::string format(p->format ? p->format : "", p->format_size);
  if (!format.empty() && format != "mlir") return BadArg("jam compile: unsupported program format '" + format + "'");
  if (const char* path = std::getenv("JAM_DUMP_ARTIFACT")) {   // the reference's artifact dump switch
    if (FILE* f = std::fopen(path, "wb")) {
      std::fwrite(p->code, 1, p->code_size, f);
      std::fclose(f);
    }
  }
  // the partitioning jax asks for (xla.CompileOptionsProto), checked against this client's job
  b200::CompileOptionsInfo co;
  if (a->compile_options && a->compile_options_size) {
    const std::string e = b200::ParseCompileOptions((const uint8_t*)a->compile_options, a->compile_options_size, &co);
    if (!e.empty()) return BadArg("jam compile: compile_options: " + e);
  }
  const int64_t want = std::max<int64_t>(co.num_replicas, 1) * std::max<int64_t>(co.num_partitions, 1);
  if (want > a->client->world)
    return BadArg("jam compile: the compile options ask for " + std::to_string(want) +
                  " devices (num_replicas x num_partitions); this job has " + std::to_string(a->client->world));
  for (const auto& ids : co.da_devices)
    for (int64_t id : ids)
      if (id < 0 || id >= a->client->world)
        return BadArg("jam compile: the device assignment names device " + std::to_string(id) + ", outside the job");
  b200::CompileOptions opt;
  opt.num_processes = a->client->world;
  opt.rank = a->client->rank;
  opt.fuse_attention = std::getenv("B200_NO_FLASH") == nullptr;
  std::unique_ptr<b200::Executable> ex;
  const std::string err = b200::Executable::Build(p->code, p->code_size, opt, &ex);
  if (!err.empty()) return BadArg("jam compile: " + err);
  const int module_parts = ex->plan().num_partitions;
  if (co.num_partitions > 1 && module_parts > 1 && co.num_partitions != module_parts)
    return BadArg("jam compile: compile options say num_partitions = " + std::to_string(co.num_partitions) +
                  ", the module says " + std::to_string(module_parts));
  auto* le = new PJRT_LoadedExecutable();
  le->client = a->client;
  le->program = std::move(ex);
  le->devices = a->client->mine;
  a->executable = le;
  return nullptr;
}

// ======================================================================================= the table
PJRT_Error* NotProvided(const char* what) {
  return Fail(PJRT_Error_Code_UNIMPLEMENTED, std::string(what) + " is not implemented by the B200 plugin");
}

void BindErrorsAndEvents(PJRT_Api& t) {
  t.PJRT_Error_Destroy = [](PJRT_Error_Destroy_Args* a) { delete a->error; };
  t.PJRT_Error_Message = [](PJRT_Error_Message_Args* a) { Put(a->error->text, &a->message, &a->message_size); };
  t.PJRT_Error_GetCode = [](PJRT_Error_GetCode_Args* a) -> PJRT_Error* {
    a->code = a->error->code;
    return nullptr;
  };
  t.PJRT_Event_Destroy = [](PJRT_Event_Destroy_Args* a) -> PJRT_Error* {
    delete a->event;
    return nullptr;
  };
  t.PJRT_Event_IsReady = [](PJRT_Event_IsReady_Args* a) -> PJRT_Error* {
    a->is_ready = a->event->done->Ready();
    return nullptr;
  };
  t.PJRT_Event_Error = [](PJRT_Event_Error_Args* a) -> PJRT_Error* { return a->event->done->Status(); };
  t.PJRT_Event_Await = [](PJRT_Event_Await_Args* a) -> PJRT_Error* {
    a->event->done->Wait();
    return a->event->done->Status();
  };
  t.PJRT_Event_OnReady = [](PJRT_Event_OnReady_Args* a) -> PJRT_Error* {
    a->event->done->Then(a->callback, a->user_arg, a->event->done);
    return nullptr;
  };
  t.PJRT_Plugin_Initialize = [](PJRT_Plugin_Initialize_Args*) -> PJRT_Error* { return nullptr; };
  t.PJRT_Plugin_Attributes = [](PJRT_Plugin_Attributes_Args* a) -> PJRT_Error* {
    a->attributes = nullptr;
    a->num_attributes = 0;
    return nullptr;
  };
}

void BindClient(PJRT_Api& t) {
  t.PJRT_Client_Create = CreateClient;
  t.PJRT_Client_Destroy = [](PJRT_Client_Destroy_Args* a) -> PJRT_Error* {
    delete a->client;
    return nullptr;
  };
  t.PJRT_Client_PlatformName = [](PJRT_Client_PlatformName_Args* a) -> PJRT_Error* {
    Put(kPlatform, &a->platform_name, &a->platform_name_size);
    return nullptr;
  };
  t.PJRT_Client_PlatformVersion = [](PJRT_Client_PlatformVersion_Args* a) -> PJRT_Error* {
    Put(kPlatformVersion, &a->platform_version, &a->platform_version_size);
    return nullptr;
  };
  t.PJRT_Client_ProcessIndex = [](PJRT_Client_ProcessIndex_Args* a) -> PJRT_Error* {
    a->process_index = a->client->rank;
    return nullptr;
  };
  t.PJRT_Client_Devices = [](PJRT_Client_Devices_Args* a) -> PJRT_Error* {
    a->devices = a->client->all.data();
    a->num_devices = a->client->all.size();
    return nullptr;
  };
  t.PJRT_Client_AddressableDevices = [](PJRT_Client_AddressableDevices_Args* a) -> PJRT_Error* {
    a->addressable_devices = a->client->mine.data();
    a->num_addressable_devices = a->client->mine.size();
    return nullptr;
  };
  t.PJRT_Client_AddressableMemories = [](PJRT_Client_AddressableMemories_Args* a) -> PJRT_Error* {
    a->addressable_memories = a->client->my_memories.data();
    a->num_addressable_memories = a->client->my_memories.size();
    return nullptr;
  };
  t.PJRT_Client_LookupDevice = [](PJRT_Client_LookupDevice_Args* a) -> PJRT_Error* {
    if (a->id < 0 || a->id >= (int)a->client->all.size()) return BadArg("no device with id " + std::to_string(a->id));
    a->device = a->client->all[a->id];
    return nullptr;
  };
  t.PJRT_Client_LookupAddressableDevice = [](PJRT_Client_LookupAddressableDevice_Args* a) -> PJRT_Error* {
    for (PJRT_Device* d : a->client->mine)
      if (d->ordinal == a->local_hardware_id) {
        a->addressable_device = d;
        return nullptr;
      }
    return BadArg("no addressable device with local hardware id " + std::to_string(a->local_hardware_id));
  };
  t.PJRT_Client_DefaultDeviceAssignment = [](PJRT_Client_DefaultDeviceAssignment_Args* a) -> PJRT_Error* {
    // replica-major over the job's devices, wrapping when the program asks for more than exist
    const size_t want = (size_t)a->num_replicas * (size_t)a->num_partitions;
    for (size_t i = 0; i < want && i < a->default_assignment_size; ++i)
      a->default_assignment[i] = a->client->all[i % a->client->all.size()]->desc.global_id;
    return nullptr;
  };
  t.PJRT_Client_TopologyDescription = [](PJRT_Client_TopologyDescription_Args* a) -> PJRT_Error* {
    a->topology = &a->client->topology;
    return nullptr;
  };
  t.PJRT_Client_BufferFromHostBuffer = FromHost;
  t.PJRT_Client_Compile = CompileProgram;
}

void BindDevicesAndMemories(PJRT_Api& t) {
  t.PJRT_Device_GetDescription = [](PJRT_Device_GetDescription_Args* a) -> PJRT_Error* {
    a->device_description = &a->device->desc;
    return nullptr;
  };
  t.PJRT_Device_IsAddressable = [](PJRT_Device_IsAddressable_Args* a) -> PJRT_Error* {
    a->is_addressable = a->device->local();
    return nullptr;
  };
  t.PJRT_Device_LocalHardwareId = [](PJRT_Device_LocalHardwareId_Args* a) -> PJRT_Error* {
    a->local_hardware_id = a->device->ordinal;
    return nullptr;
  };
  t.PJRT_Device_AddressableMemories = [](PJRT_Device_AddressableMemories_Args* a) -> PJRT_Error* {
    a->memories = a->device->space_list;
    a->num_memories = 2;
    return nullptr;
  };
  t.PJRT_Device_DefaultMemory = [](PJRT_Device_DefaultMemory_Args* a) -> PJRT_Error* {
    a->memory = a->device->hbm();
    return nullptr;
  };
  t.PJRT_Device_MemoryStats = [](PJRT_Device_MemoryStats_Args* a) -> PJRT_Error* {
    // what the driver reports for the whole GPU; the per-allocator statistics are left unset
    size_t free_bytes = 0, total = 0;
    if (a->device->local()) {
      cudaSetDevice(a->device->ordinal);
      cudaMemGetInfo(&free_bytes, &total);
    }
    // every output field (and its *_is_set flag) starts cleared
    std::memset(reinterpret_cast<char*>(a) + offsetof(PJRT_Device_MemoryStats_Args, bytes_in_use), 0,
                sizeof(PJRT_Device_MemoryStats_Args) - offsetof(PJRT_Device_MemoryStats_Args, bytes_in_use));
    a->bytes_in_use = (int64_t)(total - free_bytes);
    a->bytes_limit = (int64_t)total;
    a->bytes_limit_is_set = total != 0;
    return nullptr;
  };
  t.PJRT_DeviceDescription_Id = [](PJRT_DeviceDescription_Id_Args* a) -> PJRT_Error* {
    a->id = a->device_description->global_id;
    return nullptr;
  };
  t.PJRT_DeviceDescription_ProcessIndex = [](PJRT_DeviceDescription_ProcessIndex_Args* a) -> PJRT_Error* {
    a->process_index = a->device_description->process;
    return nullptr;
  };
  t.PJRT_DeviceDescription_Attributes = [](PJRT_DeviceDescription_Attributes_Args* a) -> PJRT_Error* {
    a->attributes = a->device_description->attribute_values;
    a->num_attributes = a->device_description->attributes.Count();
    return nullptr;
  };
  t.PJRT_DeviceDescription_Kind = [](PJRT_DeviceDescription_Kind_Args* a) -> PJRT_Error* {
    Put(a->device_description->kind, &a->device_kind, &a->device_kind_size);
    return nullptr;
  };
  t.PJRT_DeviceDescription_DebugString = [](PJRT_DeviceDescription_DebugString_Args* a) -> PJRT_Error* {
    Put(a->device_description->detail, &a->debug_string, &a->debug_string_size);
    return nullptr;
  };
  t.PJRT_DeviceDescription_ToString = [](PJRT_DeviceDescription_ToString_Args* a) -> PJRT_Error* {
    Put(a->device_description->summary, &a->to_string, &a->to_string_size);
    return nullptr;
  };
  t.PJRT_Memory_Id = [](PJRT_Memory_Id_Args* a) -> PJRT_Error* {
    a->id = a->memory->id;
    return nullptr;
  };
  t.PJRT_Memory_Kind = [](PJRT_Memory_Kind_Args* a) -> PJRT_Error* {
    Put(a->memory->kind(), &a->kind, &a->kind_size);
    return nullptr;
  };
  t.PJRT_Memory_Kind_Id = [](PJRT_Memory_Kind_Id_Args* a) -> PJRT_Error* {
    a->kind_id = (int)a->memory->space;
    return nullptr;
  };
  t.PJRT_Memory_DebugString = [](PJRT_Memory_DebugString_Args* a) -> PJRT_Error* {
    Put(a->memory->detail, &a->debug_string, &a->debug_string_size);
    return nullptr;
  };
  t.PJRT_Memory_ToString = [](PJRT_Memory_ToString_Args* a) -> PJRT_Error* {
    Put(a->memory->summary, &a->to_string, &a->to_string_size);
    return nullptr;
  };
  t.PJRT_Memory_AddressableByDevices = [](PJRT_Memory_AddressableByDevices_Args* a) -> PJRT_Error* {
    a->devices = a->memory->owner;
    a->num_devices = 1;
    return nullptr;
  };
}

void BindTopology(PJRT_Api& t) {
  t.PJRT_TopologyDescription_Create = [](PJRT_TopologyDescription_Create_Args* a) -> PJRT_Error* {
    // a topology without a client: one (remote-described) B200
    auto* topo = new PJRT_TopologyDescription();
    topo->owned.emplace_back();
    topo->owned.back().Describe(0, -1);
    topo->descriptions.push_back(&topo->owned.back());
    a->topology = topo;
    return nullptr;
  };
  t.PJRT_TopologyDescription_Destroy = [](PJRT_TopologyDescription_Destroy_Args* a) -> PJRT_Error* {
    delete a->topology;
    return nullptr;
  };
  t.PJRT_TopologyDescription_PlatformName = [](PJRT_TopologyDescription_PlatformName_Args* a) -> PJRT_Error* {
    Put(kPlatform, &a->platform_name, &a->platform_name_size);
    return nullptr;
  };
  t.PJRT_TopologyDescription_PlatformVersion = [](PJRT_TopologyDescription_PlatformVersion_Args* a) -> PJRT_Error* {
    Put(kPlatformVersion, &a->platform_version, &a->platform_version_size);
    return nullptr;
  };
  t.PJRT_TopologyDescription_GetDeviceDescriptions = [](PJRT_TopologyDescription_GetDeviceDescriptions_Args* a)
      -> PJRT_Error* {
    a->descriptions = a->topology->descriptions.data();
    a->num_descriptions = a->topology->descriptions.size();
    return nullptr;
  };
  t.PJRT_TopologyDescription_Attributes = [](PJRT_TopologyDescription_Attributes_Args* a) -> PJRT_Error* {
    a->attributes = nullptr;
    a->num_attributes = 0;
    return nullptr;
  };
  t.PJRT_ExecuteContext_Create = [](PJRT_ExecuteContext_Create_Args* a) -> PJRT_Error* {
    a->context = new PJRT_ExecuteContext();
    return nullptr;
  };
  t.PJRT_ExecuteContext_Destroy = [](PJRT_ExecuteContext_Destroy_Args* a) -> PJRT_Error* {
    delete a->context;
    return nullptr;
  };
}

void BindBuffers(PJRT_Api& t) {
  t.PJRT_Buffer_Destroy = [](PJRT_Buffer_Destroy_Args* a) -> PJRT_Error* {
    Release(a->buffer);
    delete a->buffer;
    return nullptr;
  };
  t.PJRT_Buffer_Delete = [](PJRT_Buffer_Delete_Args* a) -> PJRT_Error* {
    PJRT_Buffer* b = a->buffer;
    if (b->life != PJRT_Buffer::Life::kLive) return nullptr;
    if (b->pins > 0) b->life = PJRT_Buffer::Life::kFreeWhenUnpinned;   // freed by the last unpin
    else Release(b);
    return nullptr;
  };
  t.PJRT_Buffer_IsDeleted = [](PJRT_Buffer_IsDeleted_Args* a) -> PJRT_Error* {
    a->is_deleted = a->buffer->life != PJRT_Buffer::Life::kLive;
    return nullptr;
  };
  t.PJRT_Buffer_ElementType = [](PJRT_Buffer_ElementType_Args* a) -> PJRT_Error* {
    a->type = a->buffer->etype;
    return nullptr;
  };
  t.PJRT_Buffer_Dimensions = [](PJRT_Buffer_Dimensions_Args* a) -> PJRT_Error* {
    a->dims = a->buffer->dims.data();
    a->num_dims = a->buffer->dims.size();
    return nullptr;
  };
  t.PJRT_Buffer_UnpaddedDimensions = [](PJRT_Buffer_UnpaddedDimensions_Args* a) -> PJRT_Error* {
    a->unpadded_dims = a->buffer->dims.data();            // buffers are dense: no padding
    a->num_dims = a->buffer->dims.size();
    return nullptr;
  };
  t.PJRT_Buffer_DynamicDimensionIndices = [](PJRT_Buffer_DynamicDimensionIndices_Args* a) -> PJRT_Error* {
    a->dynamic_dim_indices = nullptr;                      // static shapes only
    a->num_dynamic_dims = 0;
    return nullptr;
  };
  t.PJRT_Buffer_OnDeviceSizeInBytes = [](PJRT_Buffer_OnDeviceSizeInBytes_Args* a) -> PJRT_Error* {
    a->on_device_size_in_bytes = a->buffer->bytes;
    return nullptr;
  };
  t.PJRT_Buffer_Device = [](PJRT_Buffer_Device_Args* a) -> PJRT_Error* {
    a->device = a->buffer->device();
    return nullptr;
  };
  t.PJRT_Buffer_Memory = [](PJRT_Buffer_Memory_Args* a) -> PJRT_Error* {
    a->memory = a->buffer->where;
    return nullptr;
  };
  t.PJRT_Buffer_IsOnCpu = [](PJRT_Buffer_IsOnCpu_Args* a) -> PJRT_Error* {
    a->is_on_cpu = a->buffer->on_host();
    return nullptr;
  };
  t.PJRT_Buffer_ReadyEvent = [](PJRT_Buffer_ReadyEvent_Args* a) -> PJRT_Error* {
    a->event = new PJRT_Event{a->buffer->ready ? a->buffer->ready : Completion::Done()};
    return nullptr;
  };
  t.PJRT_Buffer_ToHostBuffer = ToHost;
  t.PJRT_Buffer_CopyToMemory = [](PJRT_Buffer_CopyToMemory_Args* a) -> PJRT_Error* {
    return CopyInto(a->buffer, a->dst_memory ? a->dst_memory : a->buffer->where, &a->dst_buffer);
  };
  t.PJRT_Buffer_CopyToDevice = [](PJRT_Buffer_CopyToDevice_Args* a) -> PJRT_Error* {
    if (!a->dst_device) return BadArg("CopyToDevice: no destination device");
    return CopyInto(a->buffer, a->dst_device->hbm(), &a->dst_buffer);
  };
  t.PJRT_Buffer_UnsafePointer = [](PJRT_Buffer_UnsafePointer_Args* a) -> PJRT_Error* {
    a->buffer_pointer = reinterpret_cast<uintptr_t>(a->buffer->ptr);
    return nullptr;
  };
  t.PJRT_Buffer_OpaqueDeviceMemoryDataPointer = [](PJRT_Buffer_OpaqueDeviceMemoryDataPointer_Args* a) -> PJRT_Error* {
    a->device_memory_ptr = a->buffer->ptr;
    return nullptr;
  };
  t.PJRT_Buffer_IncreaseExternalReferenceCount = [](PJRT_Buffer_IncreaseExternalReferenceCount_Args* a) -> PJRT_Error* {
    ++a->buffer->pins;
    return nullptr;
  };
  t.PJRT_Buffer_DecreaseExternalReferenceCount = [](PJRT_Buffer_DecreaseExternalReferenceCount_Args* a) -> PJRT_Error* {
    PJRT_Buffer* b = a->buffer;
    if (b->pins == 0) return BadArg("DecreaseExternalReferenceCount: the buffer has no external references");
    if (--b->pins == 0 && b->life == PJRT_Buffer::Life::kFreeWhenUnpinned) Release(b);
    return nullptr;
  };
}

void BindExecutables(PJRT_Api& t) {
  t.PJRT_LoadedExecutable_GetExecutable = [](PJRT_LoadedExecutable_GetExecutable_Args* a) -> PJRT_Error* {
    if (!a->loaded_executable->program) return BadArg("GetExecutable: deleted executable");
    a->executable = new PJRT_Executable(a->loaded_executable->program);
    return nullptr;
  };
  t.PJRT_LoadedExecutable_Destroy = [](PJRT_LoadedExecutable_Destroy_Args* a) -> PJRT_Error* {
    delete a->executable;
    return nullptr;
  };
  t.PJRT_LoadedExecutable_Delete = [](PJRT_LoadedExecutable_Delete_Args* a) -> PJRT_Error* {
    a->executable->program.reset();
    return nullptr;
  };
  t.PJRT_LoadedExecutable_IsDeleted = [](PJRT_LoadedExecutable_IsDeleted_Args* a) -> PJRT_Error* {
    a->is_deleted = !a->executable->program;
    return nullptr;
  };
  t.PJRT_LoadedExecutable_AddressableDevices = [](PJRT_LoadedExecutable_AddressableDevices_Args* a) -> PJRT_Error* {
    a->addressable_devices = a->executable->devices.data();
    a->num_addressable_devices = a->executable->devices.size();
    return nullptr;
  };
  t.PJRT_LoadedExecutable_Execute = Execute;
  t.PJRT_Executable_Destroy = [](PJRT_Executable_Destroy_Args* a) -> PJRT_Error* {
    delete a->executable;
    return nullptr;
  };
  t.PJRT_Executable_Name = [](PJRT_Executable_Name_Args* a) -> PJRT_Error* {
    Put(a->executable->program->name(), &a->executable_name, &a->executable_name_size);
    return nullptr;
  };
  t.PJRT_Executable_NumReplicas = [](PJRT_Executable_NumReplicas_Args* a) -> PJRT_Error* {
    a->num_replicas = 1;
    return nullptr;
  };
  t.PJRT_Executable_NumPartitions = [](PJRT_Executable_NumPartitions_Args* a) -> PJRT_Error* {
    a->num_partitions = (size_t)a->executable->program->plan().num_partitions;
    return nullptr;
  };
  t.PJRT_Executable_NumOutputs = [](PJRT_Executable_NumOutputs_Args* a) -> PJRT_Error* {
    a->num_outputs = a->executable->outputs.types.size();
    return nullptr;
  };
  t.PJRT_Executable_OutputElementTypes = [](PJRT_Executable_OutputElementTypes_Args* a) -> PJRT_Error* {
    a->output_types = a->executable->outputs.types.data();
    a->num_output_types = a->executable->outputs.types.size();
    return nullptr;
  };
  t.PJRT_Executable_OutputDimensions = [](PJRT_Executable_OutputDimensions_Args* a) -> PJRT_Error* {
    const Signature& s = a->executable->outputs;
    a->num_outputs = s.ranks.size();
    a->dims = s.dims.data();
    a->dim_sizes = s.ranks.data();
    return nullptr;
  };
  t.PJRT_Executable_OutputMemoryKinds = [](PJRT_Executable_OutputMemoryKinds_Args* a) -> PJRT_Error* {
    const Signature& s = a->executable->outputs;
    a->num_outputs = s.kinds.size();
    a->memory_kinds = s.kinds.data();
    a->memory_kind_sizes = s.kind_sizes.data();
    return nullptr;
  };
}

// The entry points the reference also leaves UNIMPLEMENTED (src/pjrt/api/pjrt_c_api.cc:833-873).
#define B200_NOT_PROVIDED(slot) \
  t.PJRT_##slot = [](PJRT_##slot##_Args*) -> PJRT_Error* { return NotProvided(#slot); };

void BindUnimplemented(PJRT_Api& t) {
  B200_NOT_PROVIDED(Executable_SizeOfGeneratedCodeInBytes)
  B200_NOT_PROVIDED(Executable_GetCostAnalysis)
  B200_NOT_PROVIDED(Executable_OptimizedProgram)
  B200_NOT_PROVIDED(Executable_Serialize)
  B200_NOT_PROVIDED(Executable_DeserializeAndLoad)
  B200_NOT_PROVIDED(Executable_Fingerprint)
  B200_NOT_PROVIDED(Executable_GetCompiledMemoryStats)
  B200_NOT_PROVIDED(LoadedExecutable_Fingerprint)
  B200_NOT_PROVIDED(Buffer_GetMemoryLayout)
  B200_NOT_PROVIDED(CopyToDeviceStream_Destroy)
  B200_NOT_PROVIDED(CopyToDeviceStream_AddChunk)
  B200_NOT_PROVIDED(CopyToDeviceStream_TotalBytes)
  B200_NOT_PROVIDED(CopyToDeviceStream_GranuleSize)
  B200_NOT_PROVIDED(CopyToDeviceStream_CurrentBytes)
  B200_NOT_PROVIDED(TopologyDescription_Serialize)
  B200_NOT_PROVIDED(Compile)
  B200_NOT_PROVIDED(Client_CreateViewOfDeviceBuffer)
}
#undef B200_NOT_PROVIDED

}  // namespace

extern "C" __attribute__((visibility("default"))) const PJRT_Api* GetPjrtApi(void) {
  static const PJRT_Api table = [] {
    PJRT_Api t;
    std::memset(&t, 0, sizeof(t));
    t.struct_size = sizeof(PJRT_Api);
    t.pjrt_api_version.struct_size = sizeof(PJRT_Api_Version);
    t.pjrt_api_version.major_version = PJRT_API_MAJOR;
    t.pjrt_api_version.minor_version = PJRT_API_MINOR;
    BindErrorsAndEvents(t);
    BindClient(t);
    BindDevicesAndMemories(t);
    BindTopology(t);
    BindBuffers(t);
    BindExecutables(t);
    BindUnimplemented(t);
    return t;
  }();
  return &table;
}
