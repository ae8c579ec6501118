/* pjrt_b200.h — the drop-in boundary of the B200 PJRT plugin (libpjrt_b200.so).
 *
 * Like the reference's libpjrt_metal.dylib (src/pjrt/api/pjrt_c_api.h:6, CMakeLists.txt:8-10), the
 * library's one PJRT entry point is GetPjrtApi(), returning the static PJRT v0.55 function table
 * (reference: GetPjrtApi, src/pjrt/api/pjrt_c_api.cc:877-989).  jax binds it with
 * `jax._src.xla_bridge.register_plugin("b200", library_path=".../libpjrt_b200.so")`; the C++ and
 * ctypes harnesses in this repository bind it the way src/pjrt/pjrt_e2e.cc:60-181 does.
 *
 * Platform identity: platform name "b200", device kind "NVIDIA B200" (the CUDA device name), two
 * memories per device ("device", kind id 0; "pinned_host", kind id 1) as at pjrt_c_api.cc:146-156.
 * Client create options (PJRT_NamedValue, int64): "node_id", "num_nodes" (pjrt_c_api.cc:241-249) and
 * "device_ordinal" (CUDA device of this process; default: env LOCAL_RANK, else node_id modulo the
 * device count).  With num_nodes > 1 the NCCL unique id travels through the kv_put / kv_get
 * callbacks of PJRT_Client_Create.
 * Compile input: PJRT_Program format "mlir" holding StableHLO as MLIR text.
 */
#ifndef PJRT_B200_H_
#define PJRT_B200_H_

#include "pjrt_b200_abi.h"

#ifdef __cplusplus
extern "C" {
#endif

/* The PJRT function table (static storage, thread-safe initialisation). */
__attribute__((visibility("default"))) const PJRT_Api* GetPjrtApi(void);

#ifdef __cplusplus
}
#endif

#endif /* PJRT_B200_H_ */
