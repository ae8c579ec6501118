// kernels.h — host-side interface of the hand-written sm_100a kernels (csrc/kernels/*.cu) for the
// compiler and the executor.  The C-ABI entry points for outside callers are in
// include/b200_kernels.h; these are the richer internal forms (operand layouts, pitches, scratch).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <atomic>

namespace b200k {

// Kernel launches issued by this library (the kernels of csrc/kernels and the generated fusion
// kernels); a CUDA-graph replay adds the launches its capture recorded.
extern std::atomic<long long> g_kernel_launches;
inline void CountLaunches(long long n = 1) { g_kernel_launches.fetch_add(n, std::memory_order_relaxed); }

int NumSMs();

// ---- dot_general on the tensor cores (gemm_tc.cu) -----------------------------------------------
// C[b] = A[b] . B[b]^T.  A is [batch, M, >=K] (K-major, row pitch lda) or, with a_mn, [batch, K, >=M]
// (MN-major, pitch lda); B likewise with N, ldb and b_mn.  ab_type: PJRT type code of both operands
// (bf16 / f16 on the tensor cores, f32 on the SIMT kernel).  With `ws` (batch*M*N f32) a 16-bit result
// may be computed split-K; ldc is C's row pitch (0 = N).  `counter` (device int, zero before the
// launch, used by this one launch only; may be null): the CTAs draw their work units from it instead
// of taking every gridDim.x-th, so CTAs that start late take fewer.
int Gemm(const void* A, long long lda, bool a_mn, const void* B, long long ldb, bool b_mn, void* C, int64_t batch, int64_t M,
         int64_t N, int64_t K, int ab_type, int out_type, cudaStream_t st, float* ws, int64_t ldc, int* counter = nullptr);
int Gemm(const void* A, long long lda, const void* B, long long ldb, void* C, int64_t batch, int64_t M, int64_t N,
         int64_t K, int ab_type, int out_type, cudaStream_t st);
void GemmTile(int64_t batch, int64_t M, int64_t N, int64_t K, int sms, int* bn_out, int* splits_out,
              bool* pair_out = nullptr);
int GemmSplitK(int64_t batch, int64_t M, int64_t N, int64_t K, int sms);

// f32-accurate products of f32 (or mixed f32 x 16-bit) operands on the bf16 tensor cores.  Each wide
// operand is split into three bf16 pieces x = x1 + x2 + x3 (x1 = bf16(x), x2 = bf16(x - x1), x3 =
// bf16(x - x1 - x2), exact to f32's 24 bits); the product keeps the terms of order >= 2^-16
// (x1 y1, x1 y2, x2 y1, x2 y2, x1 y3, x3 y1 for two wide operands: "bf16x6"; x1 y, x2 y, x3 y when y
// is bf16 already) accumulated in one f32 TMEM accumulator (Henry, Tang, Heinecke, "Leveraging the
// bfloat16 Artificial Intelligence Datatype For Higher-Precision Computations", ARITH 2019).
// The pieces sit side by side along K, each padded to a multiple of 64, in `scratch`
// (GemmSplitScratchBytes); a bf16 operand that TMA can read in place is not copied.
// a_type / b_type: PJRT type codes (f32, bf16, f16).
size_t GemmSplitScratchBytes(int64_t batch, int64_t M, int64_t N, int64_t K, int a_type, int b_type, bool a_mn, bool b_mn,
                             long long lda, long long ldb);
int GemmSplit(const void* A, long long lda, bool a_mn, int a_type, const void* B, long long ldb, bool b_mn, int b_type,
              void* C, int64_t batch, int64_t M, int64_t N, int64_t K, int out_type, cudaStream_t st, void* scratch,
              size_t scratch_bytes, int64_t ldc, int* counter = nullptr);

// ---- attention (attention_tc.cu, attention_bwd_tc.cu) -------------------------------------------
bool AttentionShapeOk(int B, int H, int S, int D);
int AttentionFwd(const void* q, const void* k, const void* v, void* o, int B, int H, int S, int D, int causal, float scale,
                 cudaStream_t st);
int AttentionFwdLse(const void* q, const void* k, const void* v, void* o, float* lse2, int B, int H, int S, int D,
                    int causal, float scale, cudaStream_t st);
int AttentionFwdWithVt(const void* q, const void* k, const void* v, void* vt, void* o, int B, int H, int S, int D,
                       int causal, float scale, cudaStream_t st);
int AttentionBwd(const void* q, const void* k, const void* v, const void* o, const void* dout, const float* lse2,
                 void* dq, void* dk, void* dv, float* dq_acc, float* delta, int B, int H, int S, int D, int causal,
                 float scale, cudaStream_t st, int dk_t);

// ---- device error flags of the bounded waits ----------------------------------------------------
int TakeGemmError();
int TakeAttnError();
int TakeAttnBwdError();

}  // namespace b200k
