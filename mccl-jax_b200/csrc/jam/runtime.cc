// runtime.cc — plan execution on a device (see runtime.h).
#include "runtime.h"

#include <cuda.h>
#include <nvrtc.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <functional>
#include <thread>

#include <nvtx3/nvToolsExt.h>

#include "../../../include/b200_kernels.h"
#include "../comm/comm.h"
#include "../kernels/kernels.h"


namespace b200 {
namespace {

// ---- driver API through the runtime's entry points (the plugin does not link libcuda) ----
typedef CUresult (*FnModuleLoadData)(CUmodule*, const void*);
typedef CUresult (*FnModuleGetFunction)(CUfunction*, CUmodule, const char*);
typedef CUresult (*FnLaunchKernel)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned,
                                   CUstream, void**, void**);
typedef CUresult (*FnModuleUnload)(CUmodule);
typedef CUresult (*FnOccupancy)(int*, CUfunction, int, size_t);

typedef CUresult (*FnLaunchKernelEx)(const CUlaunchConfig*, CUfunction, void**, void**);
struct Driver {
  FnModuleLoadData load = nullptr;
  FnModuleGetFunction get = nullptr;
  FnLaunchKernel launch = nullptr;
  FnLaunchKernelEx launch_ex = nullptr;      // programmatic dependent launches (optional)
  FnModuleUnload unload = nullptr;
  FnOccupancy occupancy = nullptr;
  bool ok = false;
};

const Driver& Drv() {
  static Driver d;
  static std::once_flag once;
  std::call_once(once, [] {
    auto sym = [](const char* name) -> void* {
      void* p = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
        return nullptr;
      return p;
    };
    d.load = (FnModuleLoadData)sym("cuModuleLoadData");
    d.get = (FnModuleGetFunction)sym("cuModuleGetFunction");
    d.launch = (FnLaunchKernel)sym("cuLaunchKernel");
    d.launch_ex = (FnLaunchKernelEx)sym("cuLaunchKernelEx");
    d.unload = (FnModuleUnload)sym("cuModuleUnload");
    d.occupancy = (FnOccupancy)sym("cuOccupancyMaxActiveBlocksPerMultiprocessor");
    d.ok = d.load && d.get && d.launch && d.unload && d.occupancy;
  });
  return d;
}

std::string Nvrtc(const std::string& src, std::vector<char>* cubin) {
  nvrtcProgram prog;
  nvrtcResult r = nvrtcCreateProgram(&prog, src.c_str(), "b200_fusions.cu", 0, nullptr, nullptr);
  if (r != NVRTC_SUCCESS) return std::string("nvrtcCreateProgram: ") + nvrtcGetErrorString(r);
  const char* opts[] = {"--gpu-architecture=sm_100a", "--std=c++17", "-default-device", "-lineinfo", "--fmad=true"};
  r = nvrtcCompileProgram(prog, 5, opts);
  if (r != NVRTC_SUCCESS) {
    size_t n = 0;
    nvrtcGetProgramLogSize(prog, &n);
    std::string log(n, '\0');
    nvrtcGetProgramLog(prog, &log[0]);
    nvrtcDestroyProgram(&prog);
    if (const char* dump = std::getenv("B200_DUMP_CUDA")) std::ofstream(dump) << src;
    return "NVRTC compile of generated kernels failed: " + log.substr(0, 4000);
  }
  size_t n = 0;
  nvrtcGetCUBINSize(prog, &n);
  cubin->resize(n);
  nvrtcGetCUBIN(prog, cubin->data());
  nvrtcDestroyProgram(&prog);
  return "";
}

int PjrtType(DT t) { return KernelTypeCode(t); }

struct StepTimer {
  bool on = std::getenv("B200_TIME") != nullptr;
  std::map<std::string, double> ms;
  double host_ms = 0;          // time the host spends enqueueing one execution
  int runs = 0;
};

std::atomic<long long> g_graph_captures{0}, g_graph_launches{0};

// Execution timer (b200_exec_timer): a start event recorded by the first execution after a reset
// and an end event re-recorded by every execution, both on the device stream.  In per-execution
// mode every execution records its own pair instead and the reading is the sum of their spans:
// the device time of the executions without the gaps between them.
struct ExecTimer {
  std::mutex mu;
  bool armed = false, started = false, per_exec = false;
  int device = -1;
  cudaEvent_t start = nullptr, end = nullptr;
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> pairs;
  size_t used = 0;
  bool open = false;           // a pair's start is recorded and its end is not
};
ExecTimer& GetExecTimer() {
  static ExecTimer t;
  return t;
}

void ExecTimerMarkStart(int device, cudaStream_t st) {
  ExecTimer& t = GetExecTimer();
  std::lock_guard<std::mutex> lock(t.mu);
  if (t.armed && t.per_exec) {
    if (t.started && t.device != device) return;
    if (t.used == t.pairs.size()) {
      cudaEvent_t a, b;
      if (cudaEventCreate(&a) != cudaSuccess) return;
      if (cudaEventCreate(&b) != cudaSuccess) { cudaEventDestroy(a); return; }
      t.pairs.push_back({a, b});
    }
    cudaEventRecord(t.pairs[t.used].first, st);
    t.device = device;
    t.started = true;
    t.open = true;
    return;
  }
  if (!t.armed || t.started) return;
  if (!t.start) {
    cudaEventCreate(&t.start);
    cudaEventCreate(&t.end);
  }
  cudaEventRecord(t.start, st);
  t.device = device;
  t.started = true;
}

void ExecTimerMarkEnd(int device, cudaStream_t st) {
  ExecTimer& t = GetExecTimer();
  std::lock_guard<std::mutex> lock(t.mu);
  if (t.armed && t.per_exec) {
    if (t.open && t.device == device) {
      cudaEventRecord(t.pairs[t.used++].second, st);
      t.open = false;
    }
    return;
  }
  if (t.armed && t.started && t.device == device) cudaEventRecord(t.end, st);
}

}  // namespace

std::string DeviceAlloc(size_t bytes, cudaStream_t stream, void** out) {
  *out = nullptr;
  cudaError_t e = cudaMallocAsync(out, bytes < 16 ? 16 : bytes, stream);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return std::string("device allocation of ") + std::to_string(bytes) + " bytes failed: " + cudaGetErrorString(e);
  }
  return "";
}

void DeviceFree(void* p, cudaStream_t stream) {
  if (p) cudaFreeAsync(p, stream);
}

std::string Executable::Build(const char* text, size_t n, const CompileOptions& opt, std::unique_ptr<Executable>* out) {
  std::unique_ptr<Executable> ex(new Executable());
  Graph g;
  std::string err = ParseModule(text, n, &g);
  if (!err.empty()) return err;
  err = Lower(g, opt, &ex->plan_);
  if (!err.empty()) return err;
  ex->name_ = g.name.empty() ? "b200.main" : g.name;
  if (std::getenv("B200_DUMP_PLAN")) std::fprintf(stderr, "%s", ex->plan_.dump().c_str());
  if (const char* dump = std::getenv("B200_DUMP_CUDA")) std::ofstream(dump) << ex->plan_.cuda_source;
  // NVRTC: the generated kernels are split into groups compiled as separate modules on parallel
  // threads (one large module of a train step takes tens of seconds on one thread).
  const auto& ks = ex->plan_.kernel_sources;
  if (!ks.empty()) {
    unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    size_t groups = std::min<size_t>(std::min<size_t>(hw, 32), (ks.size() + 7) / 8);
    groups = std::max<size_t>(groups, 1);
    std::vector<std::string> srcs(groups, ex->plan_.cuda_prelude);
    size_t total = 0;
    for (const auto& k : ks) total += k.size();
    size_t per = total / groups + 1, g = 0, acc = 0;
    for (const auto& k : ks) {
      if (acc > per && g + 1 < groups) { ++g; acc = 0; }
      srcs[g] += k;
      acc += k.size();
    }
    ex->cubins_.assign(groups, {});
    std::vector<std::string> errs(groups);
    std::vector<std::thread> th;
    for (size_t i = 0; i < groups; ++i)
      th.emplace_back([&, i] { errs[i] = Nvrtc(srcs[i], &ex->cubins_[i]); });
    for (auto& t : th) t.join();
    for (auto& e : errs)
      if (!e.empty()) return e;
  }
  *out = std::move(ex);
  return "";
}

// The slots a step reads or writes.
// Arguments and results up to this size are staged at fixed addresses (PerDevice::stage).
constexpr int64_t kStageMax = 256;

static void StepSlots(const Step& S, std::vector<int>* out) {
  out->clear();
  auto add = [&](std::initializer_list<int> l) { for (int s : l) if (s >= 0) out->push_back(s); };
  switch (S.kind) {
    case StepKind::kFusion:
      for (const Launch& L : S.launches) {
        for (int s : L.in_slots) add({s});
        for (int s : L.out_slots) add({s});
        add({L.scratch});
      }
      break;
    case StepKind::kGemm: add({S.gemm.a, S.gemm.b, S.gemm.c, S.gemm.ws, S.gemm.split_ws}); break;
    case StepKind::kAttention: add({S.attn.q, S.attn.k, S.attn.v, S.attn.o, S.attn.lse}); break;
    case StepKind::kAttentionBwd:
      add({S.bwd.q, S.bwd.k, S.bwd.v, S.bwd.o, S.bwd.dout, S.bwd.lse, S.bwd.dq, S.bwd.dk, S.bwd.dv, S.bwd.dq_acc, S.bwd.delta});
      break;
    case StepKind::kScatterAdd: add({S.scatter.base, S.scatter.idx, S.scatter.upd, S.scatter.out}); break;
    case StepKind::kCollective:
      add({S.coll.in, S.coll.out});
      for (int s : S.coll.packed_in) add({s});
      for (int s : S.coll.packed_out) add({s});
      break;
    case StepKind::kCopy: add({S.copy.src, S.copy.dst}); break;
  }
}

// Arena layout: every intermediate slot (not an argument, constant or output) gets an offset such
// that slots with overlapping live ranges [first step touching it, last step reading it] do not
// share bytes.  Greedy: largest first, lowest offset that clears the placed slots it overlaps.
static int64_t LayoutArena(const Plan& P, std::vector<int64_t>* off) {
  const size_t n = P.slots.size();
  std::vector<int> first(n, -1), last(n, -1);
  std::vector<int> ss;
  for (size_t i = 0; i < P.steps.size(); ++i) {
    StepSlots(P.steps[i], &ss);
    for (int s : ss) {
      if (first[s] < 0) first[s] = (int)i;
      last[s] = std::max(last[s], (int)i);
    }
  }
  off->assign(n, -1);
  // a slot living inside a bucket (alias_of) takes no space of its own; the bucket lives from the
  // first to the last step touching any of its members
  for (size_t s = 0; s < n; ++s) {
    const int b = P.slots[s].alias_of;
    if (b < 0 || first[s] < 0) continue;
    last[s] = std::max(last[s], P.slots[s].last_use);
    first[b] = first[b] < 0 ? first[s] : std::min(first[b], first[s]);
    last[b] = std::max(last[b], last[s]);
  }
  std::vector<int> order;
  for (size_t s = 0; s < n; ++s) {
    const Slot& sl = P.slots[s];
    if (sl.arg_index >= 0 || sl.const_index >= 0 || sl.output || sl.alias_of >= 0 || first[s] < 0) continue;
    last[s] = std::max(last[s], sl.last_use);
    order.push_back((int)s);
  }
  std::sort(order.begin(), order.end(), [&](int a, int b) { return P.slots[a].bytes > P.slots[b].bytes; });
  auto align = [](int64_t x) { return (x + 255) & ~(int64_t)255; };
  int64_t total = 0;
  std::vector<int> placed;
  std::vector<std::pair<int64_t, int64_t>> busy;
  for (int s : order) {
    const int64_t sz = align(std::max<int64_t>(P.slots[s].bytes, 16));
    busy.clear();
    for (int q : placed)
      if (first[q] <= last[s] && first[s] <= last[q]) busy.push_back({(*off)[q], (*off)[q] + align(std::max<int64_t>(P.slots[q].bytes, 16))});
    std::sort(busy.begin(), busy.end());
    int64_t at = 0;
    for (auto& b : busy) {
      if (at + sz <= b.first) break;
      at = std::max(at, b.second);
    }
    (*off)[s] = at;
    total = std::max(total, at + sz);
    placed.push_back(s);
  }
  return total;
}

const std::vector<Executable::Piece>& Executable::Pieces() {
  std::call_once(pieces_once_, [this] {
    const std::vector<Step>& steps = plan_.steps;
    auto launches = [](const Step& S) { return S.kind == StepKind::kFusion ? (int)S.launches.size() : 1; };
    Piece cur;
    auto close = [&](int at) {
      if (at > cur.begin) {
        cur.end = at;
        pieces_.push_back(cur);
      }
      cur = Piece();
      cur.begin = at;
    };
    for (int i = 0; i < (int)steps.size(); ++i) {
      if (steps[i].kind == StepKind::kCollective) {
        close(i);
        Piece c;
        c.begin = i;
        c.end = i + 1;
        c.coll = true;
        pieces_.push_back(c);
        cur.begin = i + 1;
        continue;
      }
      if (!steps[i].wait_coll.empty()) close(i);     // the wait goes in front of a piece
      cur.launches += launches(steps[i]);
    }
    close((int)steps.size());
  });
  return pieces_;
}

Executable::~Executable() {
  const Driver& d = Drv();
  for (auto& kv : per_dev_) {
    cudaSetDevice(kv.first);
    for (auto& g : kv.second.graphs)
      for (cudaGraphExec_t x : g.execs)
        if (x) cudaGraphExecDestroy(x);
    if (kv.second.arena) cudaFree(kv.second.arena);
    if (kv.second.gemm_counters) cudaFree(kv.second.gemm_counters);
    if (kv.second.stage) cudaFree(kv.second.stage);
    for (void* p : kv.second.consts) cudaFree(p);
    if (d.ok)
      for (void* m : kv.second.modules) d.unload((CUmodule)m);
  }
}

std::string Executable::Load(DeviceState& dev, PerDevice** pd) {
  std::lock_guard<std::mutex> lock(mu_);
  auto it = per_dev_.find(dev.ordinal);
  if (it != per_dev_.end()) { *pd = &it->second; return ""; }
  PerDevice p;
  if (!cubins_.empty()) {
    const Driver& d = Drv();
    if (!d.ok) return "CUDA driver entry points unavailable";
    for (const auto& cubin : cubins_) {
      CUmodule m;
      CUresult r = d.load(&m, cubin.data());
      if (r != CUDA_SUCCESS) return "cuModuleLoadData failed (" + std::to_string((int)r) + ")";
      p.modules.push_back(m);
    }
    for (const Step& s : plan_.steps)
      for (const Launch& L : s.launches) {
        if (p.fns.count(L.fn)) continue;
        CUfunction f = nullptr;
        for (void* m : p.modules)
          if (d.get(&f, (CUmodule)m, L.fn.c_str()) == CUDA_SUCCESS) break;
        if (!f) return "generated kernel " + L.fn + " not found";
        p.fns[L.fn] = f;
        if (L.grid_stride) {
          // one full wave: a grid-stride kernel gains nothing from CTAs that wait for a free SM
          int per_sm = 0, sms = 0;
          cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev.ordinal);
          if (d.occupancy(&per_sm, f, L.block, (size_t)L.smem) == CUDA_SUCCESS && per_sm > 0 && sms > 0)
            p.wave[L.fn] = (int64_t)per_sm * sms;
        }
      }
  }
  const int64_t arena_bytes = LayoutArena(plan_, &p.arena_off);
  if (arena_bytes > 0 && cudaMalloc(&p.arena, (size_t)arena_bytes) != cudaSuccess) {
    cudaGetLastError();
    return "device allocation of the " + std::to_string(arena_bytes) + "-byte intermediate arena failed";
  }
  // fixed homes for small arguments and results (see PerDevice::stage)
  p.stage_off.assign(plan_.slots.size(), -1);
  int64_t stage_bytes = 0;
  auto stage_slot = [&](int s) {
    const int64_t b = plan_.slots[s].bytes;
    if (b <= 0 || b > kStageMax || p.stage_off[s] >= 0) return;
    p.stage_off[s] = stage_bytes;
    stage_bytes += (b + 255) & ~(int64_t)255;
  };
  for (int s : plan_.arg_slots) stage_slot(s);
  for (int s : plan_.out_slots)
    if (plan_.slots[s].arg_index < 0 && plan_.slots[s].const_index < 0) stage_slot(s);
  if (stage_bytes > 0 && cudaMalloc(&p.stage, (size_t)stage_bytes) != cudaSuccess) {
    cudaGetLastError();
    return "device allocation of the small-value stage failed";
  }
  // one work-unit counter per GEMM step, zeroed at the start of every execution -- in programs with
  // collectives only: there NCCL kernels hold SMs while GEMMs run, and CTAs that start late should
  // find their units taken; alone on the GPU the static walk is faster (no atomic before the first
  // tile: 0.25 ms per DP step)
  p.gemm_slot.assign(plan_.steps.size(), -1);
  int n_gemm = 0;
  bool coll = false;
  for (size_t i = 0; i < plan_.steps.size(); ++i) {
    if (plan_.steps[i].kind == StepKind::kGemm) p.gemm_slot[i] = n_gemm++;
    coll = coll || plan_.steps[i].kind == StepKind::kCollective;
  }
  const char* units = std::getenv("B200_GEMM_STATIC_UNITS");
  if (n_gemm > 0 && (units ? units[0] == '0' : coll)) {
    if (cudaMalloc(&p.gemm_counters, (size_t)n_gemm * sizeof(int)) != cudaSuccess) {
      cudaGetLastError();
      return "device allocation of the GEMM work-unit counters failed";
    }
    p.n_gemm = n_gemm;
  }
  for (const ConstBlob& c : plan_.consts) {
    void* ptr = nullptr;
    if (cudaMalloc(&ptr, c.bytes.empty() ? 16 : c.bytes.size()) != cudaSuccess) return "constant upload: out of memory";
    if (!c.bytes.empty()) cudaMemcpy(ptr, c.bytes.data(), c.bytes.size(), cudaMemcpyHostToDevice);
    p.consts.push_back(ptr);
  }
  per_dev_[dev.ordinal] = std::move(p);
  *pd = &per_dev_[dev.ordinal];
  return "";
}

namespace {
// B200_NVTX=1: an NVTX range around each execution and each of its steps (host enqueue side), for
// profilers that record NVTX; without a profiler attached the calls do nothing.
bool NvtxOn() {
  static const bool on = std::getenv("B200_NVTX") != nullptr;
  return on;
}
struct NvtxRange {
  bool on;
  NvtxRange(bool enable, const std::string& name) : on(enable) {
    if (on) nvtxRangePushA(name.c_str());
  }
  ~NvtxRange() {
    if (on) nvtxRangePop();
  }
};
}  // namespace

std::string Executable::Run(DeviceState& dev, const std::vector<const void*>& args, std::vector<void*>* outs, Comm* comm,
                            const std::vector<bool>* donated, std::vector<bool>* taken) {
  NvtxRange run_range(NvtxOn(), "execute " + name_);
  cudaSetDevice(dev.ordinal);
  PerDevice* pd = nullptr;
  std::string err = Load(dev, &pd);
  if (!err.empty()) return err;
  const Plan& P = plan_;
  if (args.size() != P.arg_slots.size()) return "wrong number of arguments";
  std::vector<void*> ptr(P.slots.size(), nullptr);
  std::vector<bool> owned(P.slots.size(), false);
  for (size_t k = 0; k < args.size(); ++k) ptr[P.arg_slots[k]] = const_cast<void*>(args[k]);
  for (size_t s = 0; s < P.slots.size(); ++s) {
    if (P.slots[s].const_index >= 0) ptr[s] = pd->consts[P.slots[s].const_index];
    else if (pd->arena_off[s] >= 0) ptr[s] = (char*)pd->arena + pd->arena_off[s];
  }
  // slots that live inside a packed bucket
  for (size_t s = 0; s < P.slots.size(); ++s) {
    const int b = P.slots[s].alias_of;
    if (b < 0) continue;
    if (!ptr[b]) {
      std::string e = DeviceAlloc((size_t)P.slots[b].bytes, dev.stream, &ptr[b]);
      if (!e.empty()) return e;
      owned[b] = true;
    }
    ptr[s] = (char*)ptr[b] + P.slots[s].alias_off;
  }
  // results written in place of donated arguments
  std::vector<bool> in_place(args.size(), false);
  if (donated && donated->size() == args.size())
    for (size_t k = 0; k < P.out_inplace_arg.size(); ++k) {
      const int i = P.out_inplace_arg[k];
      if (i < 0 || !(*donated)[i] || !args[i]) continue;
      ptr[P.out_slots[k]] = const_cast<void*>(args[i]);
      in_place[i] = true;
    }
  if (taken) *taken = in_place;
  cudaStream_t st = dev.stream;
  auto slot = [&](int s) -> std::string {
    if (s < 0 || ptr[s]) return "";
    std::string e = DeviceAlloc((size_t)P.slots[s].bytes, st, &ptr[s]);
    if (e.empty()) owned[s] = true;
    return e;
  };
  std::function<void()> abort_capture;
  auto fail = [&](const std::string& e) {
    if (abort_capture) abort_capture();
    for (size_t s = 0; s < ptr.size(); ++s)
      if (owned[s]) DeviceFree(ptr[s], st);
    return e;
  };
  bool has_coll = false;
  for (const Step& S : P.steps) has_coll = has_coll || S.kind == StepKind::kCollective;
  if (has_coll && comm) {
    if (comm->broken()) return "the communicator is unusable: " + comm->broken_reason();
    // optional host-side rendezvous of all ranks before any collective of this execution is enqueued
    static const int handshake_ms = std::getenv("B200_EXEC_HANDSHAKE_MS") ? std::atoi(std::getenv("B200_EXEC_HANDSHAKE_MS")) : 0;
    if (handshake_ms > 0) {
      std::string e = comm->Handshake(handshake_ms);
      if (!e.empty()) return e;
    }
  }
  ExecTimerMarkStart(dev.ordinal, st);
  if (pd->gemm_counters && cudaMemsetAsync(pd->gemm_counters, 0, (size_t)pd->n_gemm * sizeof(int), st) != cudaSuccess)
    return fail("zeroing the GEMM work-unit counters failed");
  static StepTimer timer;
  const auto host_t0 = std::chrono::steady_clock::now();
  std::vector<cudaEvent_t> evs;
  if (timer.on) {
    evs.resize(P.steps.size() + 1);
    for (auto& e : evs) cudaEventCreate(&e);
    cudaEventRecord(evs[0], st);
  }
  const Driver& drv = Drv();
  std::vector<cudaEvent_t> coll_done(P.steps.size(), nullptr);   // async collectives in flight
  auto release_events = [&]() {
    for (auto& e : coll_done)
      if (e) { cudaEventDestroy(e); e = nullptr; }
  };
  // CUDA graphs.  An execution is a sequence of pieces: runs of steps between collectives (cut
  // again where a step waits for an earlier collective, that wait being done before the piece),
  // and the collective steps themselves.  When the arguments and outputs sit at the addresses of an
  // earlier execution (intermediates are at fixed arena offsets), each piece of two or more
  // launches replays as one graph: the first execution with a set of addresses runs eagerly (lazy
  // set-up happens there), the second captures, later ones launch the graphs.  Collectives always
  // run eagerly on the communication stream, so every rank issues the same NCCL calls in the same
  // way whether or not its pieces replay; a program without collectives is one piece.
  const std::vector<Piece>& pieces = Pieces();
  size_t n_launch = 0;
  for (const Step& S : P.steps) n_launch += S.kind == StepKind::kFusion ? S.launches.size() : 1;
  const bool graphs = n_launch >= 8 && !timer.on && !std::getenv("B200_NO_GRAPHS") &&
                      !(has_coll && std::getenv("B200_NO_COLL_GRAPHS"));
  GraphEntry* ge = nullptr;
  bool capturing = false;          // this execution captures its pieces' graphs
  std::vector<int> staged_outs;    // results computed in the stage, copied out at the end
  if (graphs && pd->stage) {
    for (size_t k = 0; k < args.size(); ++k) {
      const int s = P.arg_slots[k];
      if (pd->stage_off[s] < 0 || !args[k] || in_place[k]) continue;
      void* home = (char*)pd->stage + pd->stage_off[s];
      if (cudaMemcpyAsync(home, args[k], (size_t)P.slots[s].bytes, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return fail("staging a small argument failed");
      ptr[s] = home;
    }
    for (int s : P.out_slots) {
      if (pd->stage_off[s] < 0 || ptr[s]) continue;
      ptr[s] = (char*)pd->stage + pd->stage_off[s];
      staged_outs.push_back(s);
    }
  }
  if (graphs) {
    for (int s : P.out_slots) {
      err = slot(s);
      if (!err.empty()) return fail(err);
    }
    std::vector<void*> key;
    for (int s : P.arg_slots) key.push_back(ptr[s]);
    for (int s : P.out_slots) key.push_back(ptr[s]);
    for (auto& g : pd->graphs)
      if (g.key == key) ge = &g;
    if (ge) {
      capturing = !ge->captured && !ge->no_graph;
      ge->last = ++pd->graph_clock;
    } else {
      if (pd->graphs.size() >= 4) {   // forget the least recently used address set
        auto old = std::min_element(pd->graphs.begin(), pd->graphs.end(),
                                    [](const GraphEntry& a, const GraphEntry& b) { return a.last < b.last; });
        for (cudaGraphExec_t x : old->execs)
          if (x) cudaGraphExecDestroy(x);
        pd->graphs.erase(old);
      }
      pd->graphs.push_back(GraphEntry{key});
      pd->graphs.back().last = ++pd->graph_clock;
    }
  }
  bool capture = false;            // a piece is being captured right now
  abort_capture = [&]() {
    if (!capture) return;
    capture = false;
    cudaGraph_t g = nullptr;
    cudaStreamEndCapture(st, &g);
    if (g) cudaGraphDestroy(g);
    cudaGetLastError();
  };
  // programmatic dependent launch of generated kernels: off unless asked for (B200_PDL=1); on the
  // DP step it measured 0.07 ms slower per step than plain stream order
  static const bool pdl = std::getenv("B200_PDL") != nullptr;
  auto wait_for_collectives = [&](const Step& S) {
    for (int k : S.wait_coll)
      if (coll_done[k]) cudaStreamWaitEvent(st, coll_done[k], 0);
  };
  // enqueues steps [begin, end); `waits`: also the waits for earlier collectives (a captured piece
  // has them done before the capture starts)
  auto run_steps = [&](int begin, int end, bool waits) -> std::string {
    for (int i = begin; i < end; ++i) {
      const Step& S = P.steps[i];
      NvtxRange step_range(NvtxOn(), S.label);
      if (waits) wait_for_collectives(S);
      switch (S.kind) {
        case StepKind::kFusion: {
          for (const Launch& L : S.launches) {
            std::vector<void*> vals;
            for (int s : L.in_slots) { err = slot(s); if (!err.empty()) return fail(err); vals.push_back(ptr[s]); }
            for (int s : L.out_slots) { err = slot(s); if (!err.empty()) return fail(err); vals.push_back(ptr[s]); }
            if (L.scratch >= 0) { err = slot(L.scratch); if (!err.empty()) return fail(err); vals.push_back(ptr[L.scratch]); }
            std::vector<void*> params;
            for (void*& v : vals) params.push_back(&v);
            int64_t gx = L.grid_x;
            if (L.grid_stride) {
              auto w = pd->wave.find(L.fn);
              if (w != pd->wave.end()) gx = std::max<int64_t>(1, std::min(gx, w->second));
            }
            CUresult r;
            if (drv.launch_ex && pdl) {
              // may start while the previous kernel drains; the kernel waits (griddepcontrol.wait)
              // before it reads anything
              CUlaunchAttribute attr[1];
              attr[0].id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
              attr[0].value.programmaticStreamSerializationAllowed = 1;
              CUlaunchConfig cfg = {};
              cfg.gridDimX = (unsigned)gx;
              cfg.gridDimY = (unsigned)L.grid_y;
              cfg.gridDimZ = (unsigned)L.grid_z;
              cfg.blockDimX = L.block;
              cfg.blockDimY = 1;
              cfg.blockDimZ = 1;
              cfg.sharedMemBytes = L.smem;
              cfg.hStream = (CUstream)st;
              cfg.attrs = attr;
              cfg.numAttrs = 1;
              r = drv.launch_ex(&cfg, (CUfunction)pd->fns.at(L.fn), params.data(), nullptr);
            } else {
              r = drv.launch((CUfunction)pd->fns.at(L.fn), (unsigned)gx, (unsigned)L.grid_y, (unsigned)L.grid_z, L.block, 1, 1,
                             L.smem, (CUstream)st, params.data(), nullptr);
            }
            if (r != CUDA_SUCCESS) return fail("launch of " + L.fn + " failed (" + std::to_string((int)r) + ")");
            b200k::CountLaunches();
          }
          break;
        }
        case StepKind::kGemm: {
          const GemmStep& g = S.gemm;
          for (int s : {g.a, g.b, g.c, g.ws, g.split_ws}) { err = slot(s); if (!err.empty()) return fail(err); }
          const long long lda = g.lda ? g.lda : (g.a_mn ? g.M : g.K), ldb = g.ldb ? g.ldb : (g.b_mn ? g.N : g.K);
          int* counter = pd->gemm_counters ? pd->gemm_counters + pd->gemm_slot[i] : nullptr;
          int rc = g.split
              ? b200k::GemmSplit(ptr[g.a], lda, g.a_mn, PjrtType(g.a_dt), ptr[g.b], ldb, g.b_mn, PjrtType(g.b_dt), ptr[g.c],
                                 g.batch, g.M, g.N, g.K, PjrtType(g.out), st, g.split_ws >= 0 ? ptr[g.split_ws] : nullptr,
                                 (size_t)g.split_ws_bytes, g.ldc, counter)
              : b200k::Gemm(ptr[g.a], lda, g.a_mn, ptr[g.b], ldb, g.b_mn, ptr[g.c], g.batch, g.M, g.N, g.K, PjrtType(g.ab),
                            PjrtType(g.out), st, g.ws >= 0 ? (float*)ptr[g.ws] : nullptr, g.ldc, counter);
          if (rc != 0) return fail("gemm launch failed (" + std::to_string(rc) + ") for " + S.label);
          break;
        }
        case StepKind::kAttention: {
          const AttentionStep& a = S.attn;
          for (int s : {a.q, a.k, a.v, a.o, a.lse}) { err = slot(s); if (!err.empty()) return fail(err); }
          int rc = a.lse >= 0 ? b200k::AttentionFwdLse(ptr[a.q], ptr[a.k], ptr[a.v], ptr[a.o], (float*)ptr[a.lse], a.B, a.H, a.S,
                                                       a.D, a.causal, a.scale, st)
                              : b200k::AttentionFwd(ptr[a.q], ptr[a.k], ptr[a.v], ptr[a.o], a.B, a.H, a.S, a.D, a.causal, a.scale, st);
          if (rc != 0) return fail("attention launch failed (" + std::to_string(rc) + ")");
          break;
        }
        case StepKind::kAttentionBwd: {
          const AttentionBwdStep& b = S.bwd;
          for (int s : {b.q, b.k, b.v, b.o, b.dout, b.lse, b.dq, b.dk, b.dv, b.dq_acc, b.delta}) {
            err = slot(s);
            if (!err.empty()) return fail(err);
          }
          int rc = b200k::AttentionBwd(ptr[b.q], ptr[b.k], ptr[b.v], ptr[b.o], ptr[b.dout], (const float*)ptr[b.lse],
                                     b.dq >= 0 ? ptr[b.dq] : nullptr,
                                       ptr[b.dk], ptr[b.dv], (float*)ptr[b.dq_acc], (float*)ptr[b.delta], b.B, b.H, b.S, b.D,
                                       b.causal, b.scale, st, b.dk_t ? 1 : 0);
          if (rc != 0) return fail("attention backward launch failed (" + std::to_string(rc) + ")");
          break;
        }
        case StepKind::kScatterAdd: {
          const ScatterStep& s = S.scatter;
          for (int q : {s.base, s.idx, s.upd, s.out}) { err = slot(q); if (!err.empty()) return fail(err); }
          size_t bytes = (size_t)s.rows * s.row_len * DTBytes(s.dt);
          if (ptr[s.out] != ptr[s.base]) cudaMemcpyAsync(ptr[s.out], ptr[s.base], bytes, cudaMemcpyDeviceToDevice, st);
          int rc = b200_scatter_add_rows(ptr[s.idx], ptr[s.upd], ptr[s.out], s.n_upd, s.row_len, s.rows, PjrtType(s.dt),
                                         PjrtType(s.idx_dt), st);
          if (rc != 0) return fail("scatter-add launch failed");
          break;
        }
        case StepKind::kCollective: {
          const CollectiveStep& c = S.coll;
          for (int q : {c.in, c.out}) { err = slot(q); if (!err.empty()) return fail(err); }
          if (!comm) return fail("collective in a single-process program without a communicator");
          // a group is a run of consecutive collective steps with one group id: one NCCL group
          auto same_group = [&](size_t j) {
            return j < P.steps.size() && P.steps[j].kind == StepKind::kCollective && P.steps[j].coll.group == c.group;
          };
          const bool opens = c.group < 0 || i == 0 || !same_group(i - 1);
          const bool closes = c.group < 0 || !same_group(i + 1);
          cudaStream_t cs = st;
          if (S.async) {
            // on the communication stream, after everything enqueued so far on the compute stream
            if (!dev.comm_stream && cudaStreamCreateWithFlags(&dev.comm_stream, cudaStreamNonBlocking) != cudaSuccess)
              return fail("cannot create the communication stream");
            if (opens) {
              cudaEvent_t ready;
              cudaEventCreateWithFlags(&ready, cudaEventDisableTiming);
              cudaEventRecord(ready, st);
              cudaStreamWaitEvent(dev.comm_stream, ready, 0);
              cudaEventDestroy(ready);
            }
            cs = dev.comm_stream;
          }
          if (c.group >= 0 && opens) {
            err = comm->GroupStart();
            if (!err.empty()) { release_events(); return fail(err); }
          }
          if (c.op == CollKind::kAllReduce) err = comm->AllReduce(ptr[c.in], ptr[c.out], c.send_count, c.dt, c.reduce, cs);
          else if (c.op == CollKind::kAllGather) err = comm->AllGather(ptr[c.in], ptr[c.out], c.send_count, c.dt, cs);
          else err = comm->ReduceScatter(ptr[c.in], ptr[c.out], c.recv_count, c.dt, c.reduce, cs);
          if (c.group >= 0 && (closes || !err.empty())) {
            const std::string e2 = comm->GroupEnd();
            if (err.empty()) err = e2;
          }
          if (!err.empty()) { release_events(); return fail(err); }
          if (S.async && closes) {
            // every member of the group completes with the group
            for (size_t k = i; ; --k) {
              cudaEventCreateWithFlags(&coll_done[k], cudaEventDisableTiming);
              cudaEventRecord(coll_done[k], cs);
              if (c.group < 0 || k == 0 || !same_group(k - 1)) break;
            }
          }
          break;
        }
        case StepKind::kCopy: {
          for (int q : {S.copy.src, S.copy.dst}) { err = slot(q); if (!err.empty()) return fail(err); }
          // a result that is a donated argument itself is already in place
          if (ptr[S.copy.dst] != ptr[S.copy.src])
            cudaMemcpyAsync(ptr[S.copy.dst], ptr[S.copy.src], (size_t)S.copy.bytes, cudaMemcpyDeviceToDevice, st);
          break;
        }
      }
      if (timer.on) cudaEventRecord(evs[i + 1], st);
    }
    return std::string();
  };
  for (size_t k = 0; k < pieces.size(); ++k) {
    const Piece& pc = pieces[k];
    const bool graphable = ge && !pc.coll && pc.launches >= 2;
    if (graphable && ge->captured && k < ge->execs.size() && ge->execs[k]) {
      wait_for_collectives(P.steps[pc.begin]);
      if (cudaGraphLaunch(ge->execs[k], st) != cudaSuccess) return fail("graph launch failed");
      b200k::CountLaunches(ge->kernels[k]);
      continue;
    }
    if (graphable && capturing) {
      wait_for_collectives(P.steps[pc.begin]);
      capture = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
      if (!capture) cudaGetLastError();
      const long long launches0 = b200k::g_kernel_launches.load();
      err = run_steps(pc.begin, pc.end, false);
      if (!err.empty()) return err;
      if (capture) {
        capture = false;
        cudaGraph_t g = nullptr;
        cudaGraphExec_t ex = nullptr;
        if (cudaStreamEndCapture(st, &g) == cudaSuccess && g && cudaGraphInstantiate(&ex, g, 0) == cudaSuccess) {
          ge->execs.resize(pieces.size(), nullptr);
          ge->kernels.resize(pieces.size(), 0);
          ge->execs[k] = ex;
          ge->kernels[k] = b200k::g_kernel_launches.load() - launches0;
          g_graph_captures.fetch_add(1);
        }
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        if (ex) {
          if (cudaGraphLaunch(ex, st) != cudaSuccess) return fail("graph launch failed");
          continue;
        }
        ge->no_graph = true;             // capture failed: this address set runs eagerly from now on
        capturing = false;
      }
      err = run_steps(pc.begin, pc.end, false);     // the captured launches did not run: run them now
      if (!err.empty()) return err;
      continue;
    }
    err = run_steps(pc.begin, pc.end, true);
    if (!err.empty()) return err;
  }
  if (ge) {
    if (capturing) ge->captured = true;
    else if (ge->captured) g_graph_launches.fetch_add(1);
  }
  abort_capture = nullptr;
  // the execution completes on the compute stream only after its collectives
  for (auto& e : coll_done)
    if (e) cudaStreamWaitEvent(st, e, 0);
  release_events();
  outs->clear();
  for (int s : P.out_slots) {
    if (std::find(staged_outs.begin(), staged_outs.end(), s) != staged_outs.end()) {
      void* own = nullptr;
      err = DeviceAlloc((size_t)P.slots[s].bytes, st, &own);
      if (!err.empty()) return fail(err);
      if (cudaMemcpyAsync(own, ptr[s], (size_t)P.slots[s].bytes, cudaMemcpyDeviceToDevice, st) != cudaSuccess) {
        DeviceFree(own, st);
        return fail("copying a small result out of the stage failed");
      }
      outs->push_back(own);
      continue;
    }
    if (!ptr[s]) { err = slot(s); if (!err.empty()) return fail(err); }
    outs->push_back(ptr[s]);
    owned[s] = false;
  }
  for (size_t s = 0; s < P.slots.size(); ++s)
    if (owned[s]) DeviceFree(ptr[s], st);
  ExecTimerMarkEnd(dev.ordinal, st);
  cudaError_t ce = cudaGetLastError();
  if (ce != cudaSuccess) return std::string("CUDA error during execute: ") + cudaGetErrorString(ce);
  if (timer.on) {
    timer.host_ms += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - host_t0).count();
    cudaEventSynchronize(evs.back());
    for (size_t i = 0; i < P.steps.size(); ++i) {
      float ms = 0;
      cudaEventElapsedTime(&ms, evs[i], evs[i + 1]);
      timer.ms[P.steps[i].label.substr(0, 48)] += ms;
    }
    for (auto& e : evs) cudaEventDestroy(e);
    if (++timer.runs % 20 == 0) {
      std::fprintf(stderr, "[b200 timing] %s: per-run ms by step label (avg over %d runs); host enqueue %.3f ms\n",
                   name_.c_str(), timer.runs, timer.host_ms / timer.runs);
      for (auto& kv : timer.ms) std::fprintf(stderr, "  %10.4f  %s\n", kv.second / timer.runs, kv.first.c_str());
    }
  }
  return "";
}

}  // namespace b200

// ------------------------------------------------------------------------------------------------
#include "../../../include/b200_compiler.h"

extern "C" int b200_compile_report(const char* text, size_t size, int num_processes, int nvrtc, char* out, size_t out_size) {
  std::string report;
  int rc = 0;
  b200::CompileOptions opt;
  opt.num_processes = num_processes;
  opt.fuse_attention = std::getenv("B200_NO_FLASH") == nullptr;
  if (nvrtc == 2) {
    b200::Graph g;
    std::string err = b200::ParseModule(text, size, &g);
    if (!err.empty()) { report = "error: " + err; rc = 1; }
    else report = b200::DumpGraph(g);
  } else if (nvrtc) {
    std::unique_ptr<b200::Executable> ex;
    std::string err = b200::Executable::Build(text, size, opt, &ex);
    if (!err.empty()) { report = "error: " + err; rc = 1; }
    else report = ex->plan().dump();
  } else {
    b200::Graph g;
    b200::Plan plan;
    std::string err = b200::ParseModule(text, size, &g);
    if (err.empty()) err = b200::Lower(g, opt, &plan);
    if (!err.empty()) { report = "error: " + err; rc = 1; }
    else report = plan.dump();
  }
  if (report.size() + 1 > out_size) return -1;
  std::memcpy(out, report.c_str(), report.size() + 1);
  return rc;
}

#include "../pjrt/compile_options.h"

extern "C" int b200_compile_options_report(const void* data, size_t size, char* out, size_t out_size) {
  b200::CompileOptionsInfo co;
  const std::string e = b200::ParseCompileOptions((const uint8_t*)data, size, &co);
  std::string r;
  if (!e.empty()) {
    r = "error: " + e;
  } else {
    r = "replicas=" + std::to_string(co.num_replicas) + " partitions=" + std::to_string(co.num_partitions) +
        " assignment=" + std::to_string(co.da_replicas) + "x" + std::to_string(co.da_computations) + " devices=";
    for (size_t c = 0; c < co.da_devices.size(); ++c) {
      r += c ? ";" : "";
      for (size_t k = 0; k < co.da_devices[c].size(); ++k) r += (k ? "," : "") + std::to_string(co.da_devices[c][k]);
    }
  }
  if (!out || r.size() + 1 > out_size) return -1;
  std::memcpy(out, r.c_str(), r.size() + 1);
  return e.empty() ? 0 : 1;
}

extern "C" long long b200_graph_stats(int which) {
  return which == 0 ? b200::g_graph_captures.load() : b200::g_graph_launches.load();
}

extern "C" double b200_exec_timer(int action) {
  b200::ExecTimer& t = b200::GetExecTimer();
  std::lock_guard<std::mutex> lock(t.mu);
  if (action == 0 || action == 2) {   // 0: first start to last end; 2: sum over executions
    t.armed = true;
    t.started = false;
    t.per_exec = action == 2;
    t.used = 0;
    t.open = false;
    return 0.0;
  }
  if (!t.armed || !t.started) return -1.0;
  cudaSetDevice(t.device);
  if (t.per_exec) {
    if (t.used == 0) return -1.0;
    cudaEventSynchronize(t.pairs[t.used - 1].second);
    double total = 0;
    for (size_t i = 0; i < t.used; ++i) {
      float ms = 0.f;
      if (cudaEventElapsedTime(&ms, t.pairs[i].first, t.pairs[i].second) != cudaSuccess) return -1.0;
      total += ms;
    }
    return total;
  }
  cudaEventSynchronize(t.end);
  float ms = 0.f;
  if (cudaEventElapsedTime(&ms, t.start, t.end) != cudaSuccess) return -1.0;
  return ms;
}
