/* b200_compiler.h — compile-only entry point of the B200 plugin's StableHLO compiler.
 *
 * No counterpart in the reference (its compiler, src/jam/jam.cc:8-24, is reachable only through
 * PJRT_Client_Compile).  It runs the same parse -> lower -> NVRTC pipeline as PJRT_Client_Compile
 * without creating a client or touching a GPU, and reports the plan, so the compiler can be tested
 * on hosts with no GPU.
 */
#ifndef B200_COMPILER_H_
#define B200_COMPILER_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Compiles StableHLO (MLIR text or bytecode) for `num_processes` ranks.  Writes a NUL-terminated report into
 * out[0..out_size): on success the plan dump ("plan: ...\n" then one line per step); on failure
 * "error: <message>".  Returns 0 on success, 1 on a compile error, -1 if `out` is too small.
 * `nvrtc` = 0 skips the NVRTC step (parse + lower only); `nvrtc` = 2 only parses and reports the
 * parsed op graph (one line per op with its attributes and a checksum of constant data) instead of
 * the plan.  `text` may also be MLIR bytecode (it starts with "ML\xefR"). */
__attribute__((visibility("default"))) int b200_compile_report(const char* text, size_t size, int num_processes,
                                                               int nvrtc, char* out, size_t out_size);

/* Decodes the partitioning fields of an xla.CompileOptionsProto (the compile_options bytes of
 * PJRT_Client_Compile) the way PJRT_Client_Compile does, without a client: writes
 * "replicas=R partitions=P assignment=RxC devices=d,d;d,d" (-1 for fields not present) or
 * "error: <message>".  Returns 0, 1 on malformed input, -1 if `out` is too small.  No counterpart in
 * the reference (which ignores compile_options, src/pjrt/api/pjrt_c_api.cc:681-697). */
__attribute__((visibility("default"))) int b200_compile_options_report(const void* data, size_t size, char* out,
                                                                       size_t out_size);

/* Device-time measurement of PJRT executions (no counterpart in the reference, whose runner timed
 * segments with host clocks under MCCL_JAX_TIME, src/jam/jam_run.mm:114-126).
 * b200_exec_timer(0): reset — the next LoadedExecutable_Execute records a CUDA event on the device
 *   stream before its first step;
 * b200_exec_timer(2): reset into per-execution mode — every execution records its own start and end;
 * b200_exec_timer(1): returns the device milliseconds from that event to the end of the most recent
 *   execution (waits for it), or in per-execution mode the sum of the executions' own spans (the
 *   gaps between executions left out), or -1 if nothing was recorded since the reset. */
__attribute__((visibility("default"))) double b200_exec_timer(int action);

/* CUDA-graph replay of executions (no counterpart in the reference): a program without collectives
 * whose argument and output buffers sit at the addresses of an earlier execution is captured once
 * and replayed as one graph (B200_NO_GRAPHS=1 turns this off).
 * b200_graph_stats(0): graphs captured so far; b200_graph_stats(1): executions replayed from one. */
__attribute__((visibility("default"))) long long b200_graph_stats(int which);

#ifdef __cplusplus
}
#endif

#endif /* B200_COMPILER_H_ */
