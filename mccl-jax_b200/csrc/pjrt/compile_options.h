// compile_options.h — the parts of xla.CompileOptionsProto (PJRT_Client_Compile's compile_options
// bytes) that decide how a program is partitioned.
//
// The reference ignores compile_options (src/pjrt/api/pjrt_c_api.cc:681-697) and reads the partition
// count from the module only.  jax sends the proto on every compile; for a shard_map program its
// executable_build_options carry num_replicas / num_partitions and the device assignment, which the
// plugin checks against the module's mhlo.num_partitions and the client's process count.
//
// Read from the protobuf wire format (varints, length-delimited fields; unknown fields skipped):
//   CompileOptionsProto         field 3  executable_build_options (message)
//   ExecutableBuildOptionsProto field 4  num_replicas (int64)
//                               field 5  num_partitions (int64)
//                               field 9  device_assignment (message)
//   DeviceAssignmentProto       field 1  replica_count (int32), field 2 computation_count (int32),
//                               field 3  computation_devices (repeated message)
//   ComputationDevice           field 1  replica_device_ids (repeated int64, packed or not)
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <string>
#include <vector>

namespace b200 {

struct CompileOptionsInfo {
  int64_t num_replicas = -1;        // -1: not stated
  int64_t num_partitions = -1;
  int64_t da_replicas = -1, da_computations = -1;          // device assignment shape, if given
  std::vector<std::vector<int64_t>> da_devices;           // per computation: device id per replica
};

// Decodes `data`; returns "" or a description of the malformed input.
std::string ParseCompileOptions(const uint8_t* data, size_t size, CompileOptionsInfo* out);

}  // namespace b200
