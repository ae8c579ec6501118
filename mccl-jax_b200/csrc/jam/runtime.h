// runtime.h — executes a compiled plan on one device: the B200 counterpart of the reference's
// segmented MPSGraph runner (src/jam/jam_run.mm:130-344, Run :346-419).
//
// Differences that matter on B200: every step is enqueued asynchronously on the device's stream
// (the reference runs each segment synchronously, jam_run.mm:305); slot memory comes from CUDA's
// stream-ordered pool (cudaMallocAsync / cudaFreeAsync after the last use) instead of a size-keyed
// buffer pool (jam_run.mm:74-112); generated kernels are compiled once per executable with NVRTC for
// sm_100a and loaded per device.
#pragma once

#include <cuda_runtime.h>

#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "plan.h"

namespace b200 {

class Comm;

struct DeviceState {
  int ordinal = 0;
  cudaStream_t stream = nullptr;
  cudaStream_t comm_stream = nullptr;   // collectives overlapped with compute (created on first use)
};

class Executable {
 public:
  // Parses, lowers and NVRTC-compiles a StableHLO text module.  Returns "" or the error.
  static std::string Build(const char* text, size_t n, const CompileOptions& opt, std::unique_ptr<Executable>* out);
  ~Executable();

  const Plan& plan() const { return plan_; }
  const std::string& name() const { return name_; }

  // Enqueues one execution on `dev`.  `args` are device pointers of the argument buffers (sizes were
  // checked against plan().arg_types by the caller); on success `outs` receives newly allocated
  // device buffers (stream-ordered on dev.stream) that the caller owns.
  // `donated` (per argument, may be null): the caller gives up these argument buffers.  A result the
  // plan writes in place of a donated argument is written into that argument's memory; `taken`
  // reports which donated buffers became results this way (the caller releases the others).
  std::string Run(DeviceState& dev, const std::vector<const void*>& args, std::vector<void*>* outs, Comm* comm,
                  const std::vector<bool>* donated = nullptr, std::vector<bool>* taken = nullptr);

 private:
  // A run of steps enqueued as a unit: steps [begin, end) between collectives (replayable as one
  // CUDA graph), or one collective step (always eager).
  struct Piece {
    int begin = 0, end = 0;
    bool coll = false;
    int launches = 0;                        // kernel launches of the piece (graphs need >= 2)
  };
  const std::vector<Piece>& Pieces();
  struct GraphEntry {
    std::vector<void*> key;                  // argument then output addresses
    std::vector<cudaGraphExec_t> execs;      // per piece; null for pieces run eagerly
    std::vector<long long> kernels;          // kernel launches each captured piece recorded
    bool captured = false;                   // set by the second execution with these addresses
    bool no_graph = false;                   // capture failed once: run eagerly
    uint64_t last = 0;
  };
  struct PerDevice {
    std::vector<void*> modules;              // CUmodule per NVRTC group
    std::map<std::string, void*> fns;        // CUfunction by kernel name
    std::map<std::string, int64_t> wave;     // grid-stride kernels: resident CTAs on the device
    std::vector<void*> consts;               // uploaded constants
    // Intermediates live at fixed offsets in one arena allocated at load: slots whose live ranges
    // (first to last step that touches them) do not overlap share bytes.  Executions on a device
    // are stream-ordered, so each reuses the arena; only outputs are allocated per execution.
    void* arena = nullptr;
    std::vector<int64_t> arena_off;          // per slot, -1 when not in the arena
    std::vector<GraphEntry> graphs;          // captured executions by argument / output addresses
    // Small arguments and results (scalars: step counters, bias corrections, a loss) live at fixed
    // offsets of `stage` inside executions that may replay CUDA graphs: arguments are copied in
    // first, results copied out into their own buffers last, so the graphs' addresses -- and the
    // cache key -- do not change with the fresh small buffers a caller passes every step.
    void* stage = nullptr;
    std::vector<int64_t> stage_off;          // per slot, -1 when not staged
    int* gemm_counters = nullptr;            // per GEMM step: its launch's work-unit counter
    int n_gemm = 0;
    std::vector<int> gemm_slot;              // step index -> its counter (-1: not a GEMM)
    uint64_t graph_clock = 0;
  };
  std::string Load(DeviceState& dev, PerDevice** pd);

  Plan plan_;
  std::vector<Piece> pieces_;
  std::once_flag pieces_once_;
  std::string name_;
  std::vector<std::vector<char>> cubins_;
  std::mutex mu_;
  std::map<int, PerDevice> per_dev_;
};

// Frees memory allocated by Run / the allocator on `stream` (stream-ordered).
void DeviceFree(void* p, cudaStream_t stream);
// Allocates `bytes` stream-ordered from the device pool (never returns null for bytes == 0).
std::string DeviceAlloc(size_t bytes, cudaStream_t stream, void** out);

}  // namespace b200
