// comm.h — the collective backend: NCCL over NVLink / NVSwitch, one rank per device.
//
// Replaces the reference's libmccl wrapper (src/mccl/collective/comm.h:14-40, collectives.h:33-56):
// the same Create(n, rank) / typed AllReduce / AllGather / ReduceScatter surface, returning a status
// string instead of aborting.  Bootstrap exchanges the NCCL unique id through a key-value callback
// (the PJRT client's kv_put / kv_get, which the reference ignores, src/pjrt/api/pjrt_c_api.cc:239-266)
// and initialises non-blocking so that a rank that never joins ends in a deadline error, not a hang.
#pragma once

#include <cuda_runtime.h>

#include <functional>
#include <memory>
#include <mutex>
#include <string>

#include "../jam/ir.h"

namespace b200 {

struct KvStore {
  std::function<std::string(const std::string& key, const std::string& value)> put;   // "" on success
  std::function<std::string(const std::string& key, int timeout_ms, std::string* value)> get;
};

class Comm {
 public:
  // Creates the communicator of `world` ranks; every rank must call it.  `timeout_ms` bounds the
  // wait for the other ranks.  On failure returns null and sets *err.
  // `max_ctas` > 0 caps the CTAs (SMs) an NCCL collective may occupy: gradients all-reduced while
  // the backward pass runs need little bandwidth, and every SM a collective holds is one the
  // persistent one-CTA-per-SM kernels running beside it cannot use.
  static std::unique_ptr<Comm> Create(int world, int rank, int device, const KvStore& kv, int timeout_ms,
                                      std::string* err, int max_ctas = 0);
  ~Comm();

  int rank() const { return rank_; }
  int world() const { return world_; }

  std::string AllReduce(const void* send, void* recv, size_t count, DT dt, ReduceKind op, cudaStream_t st);
  std::string AllGather(const void* send, void* recv, size_t send_count, DT dt, cudaStream_t st);
  std::string ReduceScatter(const void* send, void* recv, size_t recv_count, DT dt, ReduceKind op, cudaStream_t st);

  // Collectives enqueued between GroupStart and GroupEnd go to NCCL as one group (one launch for
  // the set instead of one per call).
  std::string GroupStart();
  std::string GroupEnd();

  // Host-side rendezvous before an execution that runs collectives: this rank posts its arrival at
  // the next execution through the key-value store and waits up to `timeout_ms` for every other
  // rank's.  A rank that has left makes it fail ("timed out") before any collective is enqueued; the
  // communicator is then aborted, with no NCCL work of this rank in flight.
  std::string Handshake(int timeout_ms);

  // Ends the communicator (ncclCommAbort: NCCL kernels still waiting on it return); later calls fail
  // with `why`.  Used when a rank is gone or a collective ran past its deadline.
  // Safe to call from another thread while this one is enqueueing (the calls are serialized).
  void Abort(const std::string& why);
  bool broken();
  std::string broken_reason();

  // Bound on the host-side waits of one enqueue (ncclInProgress on the non-blocking communicator).
  void set_enqueue_timeout_ms(int ms) { enqueue_timeout_ms_ = ms; }

 private:
  Comm() = default;
  std::string Finish(int result, const char* what);   // waits out ncclInProgress, bounded (mu_ held)
  void AbortLocked(const std::string& why);
  std::mutex mu_;         // serializes NCCL calls on comm_ with Abort
  void* comm_ = nullptr;  // ncclComm_t
  int rank_ = 0, world_ = 1;
  KvStore kv_;
  long long handshakes_ = 0;
  int enqueue_timeout_ms_ = 120000;
  std::string broken_;
};

}  // namespace b200
