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

std::unique_ptr<Comm> Comm::Create(int world, int rank, int device, const KvStore& kv, int timeout_ms, std::string* err) {
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
  return c;
}

Comm::~Comm() {
  if (comm_) ncclCommDestroy((ncclComm_t)comm_);
}

static std::string Wait(ncclComm_t comm, ncclResult_t r, const char* what) {
  // non-blocking communicator: enqueue may return ncclInProgress
  while (r == ncclInProgress) {
    ncclCommGetAsyncError(comm, &r);
    if (r == ncclInProgress) std::this_thread::yield();
  }
  return r == ncclSuccess ? std::string() : std::string(what) + ": " + ncclGetErrorString(r);
}

std::string Comm::AllReduce(const void* send, void* recv, size_t count, DT dt, ReduceKind op, cudaStream_t st) {
  ncclDataType_t t;
  ncclRedOp_t o;
  if (!NcclType(dt, &t) || !NcclOp(op, &o)) return "all_reduce: unsupported dtype or reducer";
  return Wait((ncclComm_t)comm_, ncclAllReduce(send, recv, count, t, o, (ncclComm_t)comm_, st), "ncclAllReduce");
}

std::string Comm::AllGather(const void* send, void* recv, size_t send_count, DT dt, cudaStream_t st) {
  ncclDataType_t t;
  if (!NcclType(dt, &t)) return "all_gather: unsupported dtype";
  return Wait((ncclComm_t)comm_, ncclAllGather(send, recv, send_count, t, (ncclComm_t)comm_, st), "ncclAllGather");
}

std::string Comm::ReduceScatter(const void* send, void* recv, size_t recv_count, DT dt, ReduceKind op, cudaStream_t st) {
  ncclDataType_t t;
  ncclRedOp_t o;
  if (!NcclType(dt, &t) || !NcclOp(op, &o)) return "reduce_scatter: unsupported dtype or reducer";
  return Wait((ncclComm_t)comm_, ncclReduceScatter(send, recv, recv_count, t, o, (ncclComm_t)comm_, st), "ncclReduceScatter");
}

}  // namespace b200
