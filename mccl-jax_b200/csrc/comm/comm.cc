// comm.cc — NCCL communicator (see comm.h).  Collective calls follow the reference's typed wrappers
// (src/mccl/collective/collectives.cc:113-132); the dtype / reduce-op mapping mirrors
// src/pjrt/api/pjrt_c_api.cc:645-666.
#include "comm.h"

#include <nccl.h>

#include <chrono>
#include <cstring>
#include <thread>

namespace b200 {
namespace {

bool NcclType(DT t, ncclDataType_t* out) {
  switch (t) {
    case DT::kS8: *out = ncclInt8; return true;
    case DT::kU8: case DT::kPred: *out = ncclUint8; return true;
    case DT::kS32: *out = ncclInt32; return true;
    case DT::kU32: *out = ncclUint32; return true;
    case DT::kS64: *out = ncclInt64; return true;
    case DT::kU64: *out = ncclUint64; return true;
    case DT::kF16: *out = ncclFloat16; return true;
    case DT::kBF16: *out = ncclBfloat16; return true;
    case DT::kF32: *out = ncclFloat32; return true;
    case DT::kF64: *out = ncclFloat64; return true;
    default: return false;
  }
}

bool NcclOp(ReduceKind k, ncclRedOp_t* out) {
  switch (k) {
    case ReduceKind::kAdd: *out = ncclSum; return true;
    case ReduceKind::kMul: *out = ncclProd; return true;
    case ReduceKind::kMax: *out = ncclMax; return true;
    case ReduceKind::kMin: *out = ncclMin; return true;
    default: return false;
  }
}

std::string Hex(const void* p, size_t n) {
  static const char* d = "0123456789abcdef";
  std::string s;
  for (size_t i = 0; i < n; ++i) {
    uint8_t b = ((const uint8_t*)p)[i];
    s.push_back(d[b >> 4]);
    s.push_back(d[b & 15]);
  }
  return s;
}

bool Unhex(const std::string& s, void* p, size_t n) {
  if (s.size() != 2 * n) return false;
  for (size_t i = 0; i < n; ++i) ((uint8_t*)p)[i] = (uint8_t)std::stoul(s.substr(2 * i, 2), nullptr, 16);
  return true;
}

}  // namespace

std::unique_ptr<Comm> Comm::Create(int world, int rank, int device, const KvStore& kv, int timeout_ms, std::string* err,
                                   int max_ctas) {
  if (!kv.put || !kv.get) {
    *err = "no key-value store to exchange the NCCL id (pass kv_put / kv_get callbacks to PJRT_Client_Create)";
    return nullptr;
  }
  ncclUniqueId id;
  const std::string key = "b200_pjrt/nccl_id";
  if (rank == 0) {
    ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) { *err = std::string("ncclGetUniqueId: ") + ncclGetErrorString(r); return nullptr; }
    std::string e = kv.put(key, Hex(&id, sizeof(id)));
    if (!e.empty()) { *err = "kv_put: " + e; return nullptr; }
  } else {
    std::string v;
    std::string e = kv.get(key, timeout_ms, &v);
    if (!e.empty()) { *err = "kv_get: " + e; return nullptr; }
    if (!Unhex(v, &id, sizeof(id))) { *err = "malformed NCCL id in the key-value store"; return nullptr; }
  }
  cudaSetDevice(device);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  if (max_ctas > 0) cfg.maxCTAs = max_ctas;
  ncclComm_t comm = nullptr;
  ncclResult_t r = ncclCommInitRankConfig(&comm, world, id, rank, &cfg);
  auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
  while (r == ncclInProgress || r == ncclSuccess) {
    ncclResult_t a = ncclSuccess;
    if (comm) ncclCommGetAsyncError(comm, &a);
    if (a == ncclSuccess) break;
    if (a != ncclInProgress) { r = a; break; }
    if (std::chrono::steady_clock::now() > deadline) {
      ncclCommAbort(comm);
      *err = "NCCL communicator init timed out after " + std::to_string(timeout_ms) + " ms (a rank did not join)";
      return nullptr;
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(1));
  }
  if (r != ncclSuccess && r != ncclInProgress) {
    if (comm) ncclCommAbort(comm);
    *err = std::string("ncclCommInitRankConfig: ") + ncclGetErrorString(r);
    return nullptr;
  }
  std::unique_ptr<Comm> c(new Comm());
  c->comm_ = comm;
  c->rank_ = rank;
  c->world_ = world;
  c->kv_ = kv;
  c->enqueue_timeout_ms_ = timeout_ms;
  return c;
}

Comm::~Comm() {
  if (comm_) ncclCommDestroy((ncclComm_t)comm_);     // an aborted communicator has none left
}

void Comm::AbortLocked(const std::string& why) {
  if (!broken_.empty()) return;
  broken_ = why.empty() ? "communicator aborted" : why;
  if (comm_) ncclCommAbort((ncclComm_t)comm_);
  comm_ = nullptr;
}

void Comm::Abort(const std::string& why) {
  std::lock_guard<std::mutex> g(mu_);
  AbortLocked(why);
}

bool Comm::broken() {
  std::lock_guard<std::mutex> g(mu_);
  return !broken_.empty();
}

std::string Comm::broken_reason() {
  std::lock_guard<std::mutex> g(mu_);
  return broken_;
}

// Non-blocking communicator: an enqueue may return ncclInProgress until NCCL has taken the call.
// The wait is bounded; past the bound the communicator is aborted.
std::string Comm::Finish(int result, const char* what) {
  ncclResult_t r = (ncclResult_t)result;
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(enqueue_timeout_ms_);
  while (r == ncclInProgress) {
    ncclCommGetAsyncError((ncclComm_t)comm_, &r);
    if (r != ncclInProgress) break;
    if (std::chrono::steady_clock::now() > deadline) {
      AbortLocked(std::string(what) + " timed out after " + std::to_string(enqueue_timeout_ms_) + " ms");
      return broken_;
    }
    std::this_thread::yield();
  }
  return r == ncclSuccess ? std::string() : std::string(what) + ": " + ncclGetErrorString(r);
}

std::string Comm::AllReduce(const void* send, void* recv, size_t count, DT dt, ReduceKind op, cudaStream_t st) {
  std::lock_guard<std::mutex> g(mu_);
  if (!broken_.empty()) return broken_;
  ncclDataType_t t;
  ncclRedOp_t o;
  if (!NcclType(dt, &t) || !NcclOp(op, &o)) return "all_reduce: unsupported dtype or reducer";
  return Finish(ncclAllReduce(send, recv, count, t, o, (ncclComm_t)comm_, st), "ncclAllReduce");
}

std::string Comm::AllGather(const void* send, void* recv, size_t send_count, DT dt, cudaStream_t st) {
  std::lock_guard<std::mutex> g(mu_);
  if (!broken_.empty()) return broken_;
  ncclDataType_t t;
  if (!NcclType(dt, &t)) return "all_gather: unsupported dtype";
  return Finish(ncclAllGather(send, recv, send_count, t, (ncclComm_t)comm_, st), "ncclAllGather");
}

std::string Comm::ReduceScatter(const void* send, void* recv, size_t recv_count, DT dt, ReduceKind op, cudaStream_t st) {
  std::lock_guard<std::mutex> g(mu_);
  if (!broken_.empty()) return broken_;
  ncclDataType_t t;
  ncclRedOp_t o;
  if (!NcclType(dt, &t) || !NcclOp(op, &o)) return "reduce_scatter: unsupported dtype or reducer";
  return Finish(ncclReduceScatter(send, recv, recv_count, t, o, (ncclComm_t)comm_, st), "ncclReduceScatter");
}

std::string Comm::GroupStart() {
  std::lock_guard<std::mutex> g(mu_);
  if (!broken_.empty()) return broken_;
  const ncclResult_t r = ncclGroupStart();
  return r == ncclSuccess ? std::string() : std::string("ncclGroupStart: ") + ncclGetErrorString(r);
}

std::string Comm::GroupEnd() {
  std::lock_guard<std::mutex> g(mu_);
  if (!broken_.empty()) {
    ncclGroupEnd();                                  // close the host-side group either way
    return broken_;
  }
  return Finish(ncclGroupEnd(), "ncclGroupEnd");
}

std::string Comm::Handshake(int timeout_ms) {
  if (broken()) return broken_reason();
  if (!kv_.put || !kv_.get) return "";
  const long long n = ++handshakes_;
  const std::string base = "b200_pjrt/execution/" + std::to_string(n) + "/";
  std::string e = kv_.put(base + std::to_string(rank_), "1");
  if (!e.empty()) {
    Abort("execution handshake: " + e);
    return broken_reason();
  }
  for (int r = 0; r < world_; ++r) {
    if (r == rank_) continue;
    std::string v;
    e = kv_.get(base + std::to_string(r), timeout_ms, &v);
    if (!e.empty()) {
      Abort("execution handshake timed out after " + std::to_string(timeout_ms) + " ms: rank " + std::to_string(r) +
            " did not arrive at execution " + std::to_string(n) + " (" + e + ")");
      return broken_reason();
    }
  }
  return "";
}

}  // namespace b200
