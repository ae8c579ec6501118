/* b200_kernels.h — direct C-ABI entry points to the plugin's hand-written sm_100a kernels.
 *
 * The drop-in boundary is `GetPjrtApi()` (include/pjrt_b200.h); these entry points expose the same
 * kernels that PJRT_LoadedExecutable_Execute launches, on caller-owned device memory and a caller
 * stream, so that tests and benchmarks can time one kernel on HBM-resident inputs.  They have no
 * counterpart in the reference (whose kernels are MPSGraph nodes chosen inside Apple's framework);
 * each comment names the reference call site whose work the kernel performs.
 *
 * All pointers are device pointers; `stream` is a cudaStream_t (NULL = legacy default stream).
 * Element types use the PJRT_Buffer_Type codes below.  Functions return 0 on success, a negative
 * code on invalid arguments or launch failure; asynchronous kernel faults are reported by
 * b200_take_device_error().
 */
#ifndef B200_KERNELS_H_
#define B200_KERNELS_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200_API __attribute__((visibility("default")))

#define B200_DT_F16 10  /* PJRT_Buffer_Type_F16 */
#define B200_DT_F32 11  /* PJRT_Buffer_Type_F32 */
#define B200_DT_BF16 13 /* PJRT_Buffer_Type_BF16 */
#define B200_DT_S32 4   /* PJRT_Buffer_Type_S32 */
#define B200_DT_S64 5   /* PJRT_Buffer_Type_S64 */

/* C[b] = A[b] . B[b]^T : A [batch, M, K] and B [batch, N, K] row-major (K contiguous), C [batch, M, N].
 * ab_type in {BF16, F16, F32}; out_type in {F32, BF16, F16}.  bf16/f16 with K % 8 == 0 run on the
 * tcgen05 tensor-core kernel; other cases on a SIMT kernel.
 * Replaces: DotGeneral's matmulWithPrimaryTensor, src/jam/ops/linalg.mm:47-105 (call at :98). */
B200_API int b200_gemm(const void* A, const void* B, void* C, int64_t batch, int64_t M, int64_t N, int64_t K,
              int ab_type, int out_type, void* stream);

/* f32-accurate C[b] = A[b] . B[b]^T on the bf16 tensor cores, for f32 operands or an f32 operand
 * with a bf16 / f16 one (A [batch, M, K] of a_type, B [batch, N, K] of b_type, K contiguous; C
 * [batch, M, N] of out_type).  Each f32 / f16 operand is split into three bf16 pieces that sum to it
 * exactly; the product keeps the terms down to 2^-16 relative (six for two f32 operands, three for
 * f32 x bf16) in one f32 accumulator: the f32 arithmetic of a dot_general, within the f32 bar
 * (normwise 1e-5), at bf16 tensor-core throughput.  `scratch` (256-byte aligned device memory of
 * b200_gemm_split_scratch_bytes(...) bytes) holds the pieces; A and B must be 16-byte aligned.  Returns 0, -1 (bad arguments), -4 (scratch too small or misaligned), or a launch
 * failure code.
 * Replaces: DotGeneral's matmul for f32 operands, src/jam/ops/linalg.mm:47-105 (call at :98). */
B200_API size_t b200_gemm_split_scratch_bytes(int64_t batch, int64_t M, int64_t N, int64_t K, int a_type, int b_type);
B200_API int b200_gemm_split(const void* A, int a_type, const void* B, int b_type, void* C, int64_t batch, int64_t M,
                             int64_t N, int64_t K, int out_type, void* scratch, size_t scratch_bytes, void* stream);

/* O = softmax(scale * Q K^T [causal mask]) V, fp32 softmax, for bf16 Q, K, V, O of shape [B, H, S, D]
 * (D contiguous), D = 64, S a multiple of 256.  Fused flash-style kernel on tcgen05; allocates nothing.
 * Replaces: the dot_general -> softMaxWithTensor -> dot_general chain, src/jam/ops/linalg.mm:98 and
 * src/jam/ops/elementwise.mm:71-89 (TrySoftmax). */
B200_API int b200_attention_fwd(const void* q, const void* k, const void* v, void* o, int B, int H, int S, int D,
                       int causal, float scale, void* stream);

/* b200_attention_fwd that also writes lse2 [B, H, S] (f32): per query row, log2 of sum_j
 * 2^(scale * log2(e) * s_j) over the keys it sees, which the backward uses to recompute P.
 * Replaces: the forward half of the same chain when its intermediates feed a backward pass
 * (reference: softmax and dot_general VJPs as separate MPSGraph ops, src/jam/ops/linalg.mm:47-105,
 * src/jam/ops/elementwise.mm:71-123). */
B200_API int b200_attention_fwd_lse(const void* q, const void* k, const void* v, void* o, float* lse2, int B, int H,
                                    int S, int D, int causal, float scale, void* stream);

/* dQ, dK, dV of O = softmax(scale * Q K^T [causal]) V from Q, K, V, O, dO (bf16 [B, H, S, D]) and
 * the forward's lse2, D = 64, S a multiple of 128.  Scores are recomputed per 128 x 128 tile on
 * tcgen05; dQ accumulates in the caller's f32 scratch dq_acc [B, H, S, D] and is rounded into dq
 * (with dq NULL it stays there, unrounded, for a caller that rounds on read); delta [B, H, S] f32
 * is scratch too.  Allocates nothing.
 * Replaces: the VJP of the attention chain, which the reference runs as the transposed
 * dot_generals (src/jam/ops/linalg.mm:47-105) and the elementwise softmax VJP ops
 * (src/jam/ops/elementwise.mm:91-191, src/jam/ops/reduce.mm:45-109) over full S x S tensors. */
B200_API int b200_attention_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout,
                                const float* lse2, void* dq, void* dk, void* dv, float* dq_acc, float* delta, int B,
                                int H, int S, int D, int causal, float scale, void* stream);

/* The same attention with V first transposed into the caller's scratch `vt` (B*H*S*D bf16 elements)
 * and consumed K-major: an independent operand layout for cross-checking b200_attention_fwd.
 * No counterpart in the reference. */
B200_API int b200_attention_fwd_vt(const void* q, const void* k, const void* v, void* vt, void* o, int B, int H, int S,
                                   int D, int causal, float scale, void* stream);

/* b200_attention_fwd_vt without the caller-provided scratch: for callers that cannot allocate device
 * memory — code running under a framework whose caching allocator owns the whole device budget, or
 * a latency-critical path where cudaMalloc / cudaFree (which can synchronize the device) are not
 * allowed.  No counterpart in the reference.
 * The transposed V goes to a static 32 MiB device array built into the library; the function calls
 * no cudaMalloc, cudaFree or other allocating routine.  Limit: B*H*S*D*2 bytes <= 32 MiB (e.g.
 * [4,16,4096,64]); larger problems return -5 without launching anything.  The array's device address
 * is looked up on the first call on each device (with that device current), so make that first call
 * before any stream capture.  All calls share the one array and it keeps the previous call's
 * contents (each call overwrites the part it uses before reading it): calls that overlap on the GPU
 * (different streams, or different host threads on one device) race on it and must be serialized by
 * the caller.  Returns 0, -1 (bad shape), -5 (too large for the scratch), -6 (scratch address lookup
 * failed), or the attention kernel's launch codes. */
B200_API int b200_attention_fwd_noalloc(const void* q, const void* k, const void* v, void* o, int B, int H, int S,
                                        int D, int causal, float scale, void* stream);

/* out[idx[i], :] += upd[i, :] for i < n_upd (rows of length row_len; out has `rows` rows; indices
 * outside [0, rows) are skipped).  dtype in {F32, BF16}; idx_type in {S32, S64}.
 * Replaces: Scatter (add region), src/jam/ops/gather_scatter.mm:262-335. */
B200_API int b200_scatter_add_rows(const void* idx, const void* upd, void* out, int64_t n_upd, int64_t row_len, int64_t rows,
                          int dtype, int idx_type, void* stream);

/* Returns and clears the first error code recorded by a bounded wait inside a tensor-core kernel on
 * the current device (0 = none).  Synchronizes the device. */
B200_API int b200_take_device_error(void);

/* Runs the tensor-core kernels' bounded mbarrier wait on a barrier whose arrival never comes, with a
 * budget of `budget_cycles` SM clock cycles: the wait gives up, records its error code (1, a timed-out
 * pipeline wait) for b200_take_device_error and the kernel returns, leaving the context usable.
 * `waited_out` (device int, may be NULL) receives 1 when the wait gave up.  For tests of the timeout
 * path; no counterpart in the reference.  Returns 0 or a launch failure code. */
B200_API int b200_selftest_wait_timeout(long long budget_cycles, int* waited_out, void* stream);

/* Number of kernel launches this library has issued since it was loaded: its hand-written kernels,
 * the generated fusion kernels of PJRT executions, and the kernels of each CUDA-graph replay. */
B200_API long long b200_kernel_launches(void);

#ifdef __cplusplus
}
#endif

#endif /* B200_KERNELS_H_ */
