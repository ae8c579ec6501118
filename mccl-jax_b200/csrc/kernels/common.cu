// common.cu — driver entry points shared by the kernels, the device error flag readout, and the
// row scatter-add used for the VJP of an embedding take.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <mutex>

#include "kernels.h"
#include "tc_common.cuh"
#include "../../../include/b200_kernels.h"

namespace b200k {

std::atomic<long long> g_kernel_launches{0};

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point (the plugin does not link libcuda,
// so it also loads on hosts without a GPU driver).
EncodeTiledFn GetEncodeTiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)p;
  });
  return fn;
}

static __device__ int g_tc_error_selftest;

// The bounded mbarrier wait of the tensor-core kernels, run on a barrier whose one expected arrival
// never comes: after `budget` cycles the wait gives up, records kErrTimeoutFull in the device flag
// and the kernel returns (the recovery path every pipeline wait takes).
__global__ void wait_timeout_selftest_kernel(long long budget, int* waited_out) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  fence_barrier_init();
  const bool ok = mbar_wait_budget(&bar, 0, kErrTimeoutFull, &g_tc_error_selftest, budget);
  if (waited_out) *waited_out = ok ? 0 : 1;
}

static int TakeSelftestError() {
  int v = 0, z = 0;
  cudaMemcpyFromSymbol(&v, g_tc_error_selftest, sizeof(int));
  if (v) cudaMemcpyToSymbol(g_tc_error_selftest, &z, sizeof(int));
  return v;
}

template <typename T, typename I>
__global__ void __launch_bounds__(256) scatter_add_rows_kernel(const I* __restrict__ idx, const T* __restrict__ upd, T* __restrict__ out,
                                                               long long n_upd, long long row_len, long long rows) {
  for (long long i = blockIdx.x; i < n_upd; i += gridDim.x) {
    long long r = (long long)idx[i];
    if (r < 0 || r >= rows) continue;  // out-of-range updates are dropped (StableHLO scatter semantics)
    const T* src = upd + i * row_len;
    T* dst = out + r * row_len;
    for (long long j = threadIdx.x; j < row_len; j += blockDim.x) atomicAdd(dst + j, src[j]);
  }
}

}  // namespace b200k

extern "C" int b200_take_device_error(void) {
  cudaDeviceSynchronize();
  int e = b200k::TakeGemmError();
  int a = b200k::TakeAttnError();
  int b = b200k::TakeAttnBwdError();
  int t = b200k::TakeSelftestError();
  return e ? e : a ? a : b ? b : t;
}

extern "C" int b200_selftest_wait_timeout(long long budget_cycles, int* waited_out, void* stream) {
  if (budget_cycles <= 0) return -1;
  b200k::wait_timeout_selftest_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(budget_cycles, waited_out);
  b200k::CountLaunches();
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

extern "C" long long b200_kernel_launches(void) { return b200k::g_kernel_launches.load(); }

extern "C" int b200_scatter_add_rows(const void* idx, const void* upd, void* out, int64_t n_upd, int64_t row_len,
                                     int64_t rows, int dtype, int idx_type, void* stream) {
  cudaStream_t st = (cudaStream_t)stream;
  if (n_upd <= 0 || row_len <= 0) return 0;
  int grid = (int)std::min<int64_t>(n_upd, 148 * 16);
  int block = row_len >= 256 ? 256 : 128;
  if (dtype == B200_DT_F32 && idx_type == B200_DT_S32)
    b200k::scatter_add_rows_kernel<float, int><<<grid, block, 0, st>>>((const int*)idx, (const float*)upd, (float*)out, n_upd, row_len, rows);
  else if (dtype == B200_DT_F32 && idx_type == B200_DT_S64)
    b200k::scatter_add_rows_kernel<float, long long><<<grid, block, 0, st>>>((const long long*)idx, (const float*)upd, (float*)out, n_upd, row_len, rows);
  else if (dtype == B200_DT_BF16 && idx_type == B200_DT_S32)
    b200k::scatter_add_rows_kernel<__nv_bfloat16, int><<<grid, block, 0, st>>>((const int*)idx, (const __nv_bfloat16*)upd, (__nv_bfloat16*)out, n_upd, row_len, rows);
  else if (dtype == B200_DT_BF16 && idx_type == B200_DT_S64)
    b200k::scatter_add_rows_kernel<__nv_bfloat16, long long><<<grid, block, 0, st>>>((const long long*)idx, (const __nv_bfloat16*)upd, (__nv_bfloat16*)out, n_upd, row_len, rows);
  else
    return -1;
  b200k::CountLaunches();
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
