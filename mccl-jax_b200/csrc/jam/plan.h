// plan.h — the compiled form of a StableHLO program: buffer slots + an ordered list of device steps.
//
// The reference compiles `@main` into MPSGraph "segments" separated by collective steps and binds
// values to numbered slots (src/jam/program_impl.h:14-51, src/jam/lower.mm:460-566).  Here a program
// becomes a flat list of B200 steps — generated fused kernels (NVRTC, sm_100a), tcgen05 GEMMs, the
// fused attention kernel, scatter-add, NCCL collectives and copies — over slots that the runtime
// allocates stream-ordered on first definition and frees after last use.
#pragma once

#include <string>
#include <vector>

#include "ir.h"

namespace b200 {

struct Slot {
  int64_t bytes = 0;
  int arg_index = -1;          // bound to @main argument k (not owned)
  int const_index = -1;        // bound to uploaded constant k (owned by the executable)
  bool output = false;         // handed to the caller as an output buffer
  int last_use = -1;           // index of the last step that reads it (-1: never read)
  int alias_of = -1;           // lives inside slot alias_of, at byte offset alias_off (a packed bucket)
  int64_t alias_off = 0;
};

enum class StepKind { kFusion, kGemm, kAttention, kAttentionBwd, kScatterAdd, kCollective, kCopy };

// One generated kernel launch (loop fusion, or one stage of a reduction).
struct Launch {
  std::string fn;              // kernel name inside the NVRTC module
  std::vector<int> in_slots;   // pointer params first, in this order
  std::vector<int> out_slots;  // then output pointers
  int scratch = -1;            // scratch slot appended as the last pointer (-1: none)
  int64_t grid_x = 1, grid_y = 1, grid_z = 1;
  int block = 256;
  int smem = 0;
  bool grid_stride = false;    // any grid size is correct: launched with at most one wave of CTAs
  // (input slot, output slot) pairs this kernel may run with the output in the input's memory: the
  // input is read only at the element the same thread then writes (or not at all), and the kernel
  // declares those two pointers without __restrict__
  std::vector<std::pair<int, int>> inplace;
};

struct GemmStep {
  int a = -1, b = -1, c = -1;  // A[batch,M,K], B[batch,N,K] (K-major), C[batch,M,N] row-major
  int64_t batch = 1, M = 0, N = 0, K = 0;
  int64_t lda = 0, ldb = 0;    // row pitch of A / B in elements (>= K; K rounded up to 8 for TMA)
  int64_t ldc = 0;             // row pitch of C in elements (0: N; padded to 16 bytes for TMA stores)
  bool a_mn = false, b_mn = false;  // operand stored MN-major: A[batch,K,M] / B[batch,K,N], pitch M / N
  int ws = -1;                 // f32 [batch,M,N] workspace when a 16-bit result is computed split-K
  DT ab = DT::kBF16, out = DT::kF32;
  // f32-accurate product of f32 operands on the tensor cores (b200k::GemmSplit): the operands keep
  // their stored types a_dt / b_dt; split_ws holds their bf16 pieces
  bool split = false;
  DT a_dt = DT::kBF16, b_dt = DT::kBF16;
  int split_ws = -1;
  int64_t split_ws_bytes = 0;
};

struct AttentionStep {
  int q = -1, k = -1, v = -1, o = -1;   // [B,H,S,D] each, D contiguous
  int B = 0, H = 0, S = 0, D = 0;
  bool causal = false;
  float scale = 1.f;
  DT dt = DT::kBF16;
  int lse = -1;                          // training forward: lse2 [B*H*S] f32 for the backward
};

// dQ, dK, dV of an attention whose forward ran as an AttentionStep with lse.
struct AttentionBwdStep {
  int q = -1, k = -1, v = -1, o = -1, dout = -1, lse = -1;   // inputs, [B,H,S,D] bf16 (lse [B*H*S] f32)
  int dq = -1, dk = -1, dv = -1;                            // outputs bf16; dk is [B,H,D,S] when dk_t
  int dq_acc = -1, delta = -1;                 // scratch
  bool dk_t = false;
  int B = 0, H = 0, S = 0, D = 0;
  bool causal = false;
  float scale = 1.f;
};

struct ScatterStep {           // out = base; out[idx[i], :] += upd[i, :]
  int base = -1, idx = -1, upd = -1, out = -1;
  int64_t rows = 0, row_len = 0, n_upd = 0;
  DT dt = DT::kF32, idx_dt = DT::kS32;
};

enum class CollKind { kAllReduce, kAllGather, kReduceScatter };

struct CollectiveStep {
  CollKind op = CollKind::kAllReduce;
  ReduceKind reduce = ReduceKind::kAdd;
  int in = -1, out = -1;
  int64_t send_count = 0, recv_count = 0;
  DT dt = DT::kF32;
  int group = -1;              // consecutive steps with one group id go to NCCL as one group
  // a packed all-reduce: in = out = a bucket slot holding these members' inputs (reduced in place
  // into their outputs, which alias the same bytes)
  std::vector<int> packed_in, packed_out;
};

struct CopyStep {
  int src = -1, dst = -1;
  int64_t bytes = 0;
};

struct Step {
  StepKind kind;
  std::vector<Launch> launches;      // kFusion: one or two (reduction stage 2) launches
  GemmStep gemm;
  AttentionStep attn;
  AttentionBwdStep bwd;
  ScatterStep scatter;
  CollectiveStep coll;
  CopyStep copy;
  bool async = false;                // kCollective: runs on the communication stream
  std::vector<int> wait_coll;        // async collective steps that must finish before this step
  std::string label;                 // for dumps / timing
};

struct ConstBlob {
  std::vector<uint8_t> bytes;
};

struct Plan {
  std::vector<Slot> slots;
  std::vector<Step> steps;
  std::vector<ConstBlob> consts;
  std::string cuda_prelude;          // helpers every generated kernel uses
  std::vector<std::string> kernel_sources;  // one entry per generated kernel (or reduction pair)
  std::string cuda_source;           // prelude + every kernel (for dumps)
  std::vector<int> arg_slots;        // per @main argument
  std::vector<TensorType> arg_types; // after shard_map retyping
  std::vector<int> out_slots;        // per @main result
  std::vector<TensorType> out_types;
  // buffer donation: per argument, the result its buffer may become (-1: none) and whether the
  // caller gives the buffer up at all; per result, the argument whose memory it is written into when
  // that argument is donated (-1: a fresh buffer)
  std::vector<int> arg_alias;
  std::vector<bool> arg_donor;
  std::vector<int> out_inplace_arg;
  int num_partitions = 1;
  std::string dump() const;
};

struct CompileOptions {
  int num_processes = 1;             // ranks in the communicator (1: collectives are identities)
  int rank = 0;                      // this process's rank (the value of partition_id / replica_id)
  bool fuse_attention = true;        // B200_NO_FLASH=1 turns the attention pattern match off
};

// Lowers a parsed graph into a plan.  Returns "" on success, else the error (unsupported op ...).
std::string Lower(Graph& g, const CompileOptions& opt, Plan* plan);

}  // namespace b200
