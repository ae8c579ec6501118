"""Writes tests/golden/compile_options.json: xla.CompileOptionsProto messages serialized by the protobuf
library, for the plugin's own decoder of PJRT_Client_Compile's compile_options bytes.

jax / jaxlib and the XLA .proto files are not on this image, so the messages are declared here with
the field numbers of openxla's xla/pjrt/proto/compile_options.proto and xla/xla_data.proto (only the
fields the plugin reads, plus a few it must skip): CompileOptionsProto {1 argument_layouts (message,
repeated), 2 parameter_is_tupled_arguments (bool), 3 executable_build_options, 4
compile_portable_executable (bool), 5 profile_version (int64)}; ExecutableBuildOptionsProto {1
device_ordinal, 4 num_replicas, 5 num_partitions, 6 use_spmd_partitioning (bool), 9
device_assignment}; DeviceAssignmentProto {1 replica_count, 2 computation_count, 3
computation_devices}; ComputationDevice {1 replica_device_ids (repeated int64)}.  The protobuf
library does the encoding (varints, packed repeated fields, nested lengths).

    python tests/golden/make_compile_options.py
"""
import json
import os

from google.protobuf import descriptor_pb2, descriptor_pool, message_factory

HERE = os.path.dirname(os.path.abspath(__file__))
F = descriptor_pb2.FieldDescriptorProto


def _messages():
    fd = descriptor_pb2.FileDescriptorProto(name="b200_compile_options_fixture.proto", package="fixture", syntax="proto3")

    def msg(name, fields):
        m = fd.message_type.add(name=name)
        for fname, num, ftype, label, tname in fields:
            f = m.field.add(name=fname, number=num, type=ftype, label=label)
            if tname:
                f.type_name = tname
    opt, rep = F.LABEL_OPTIONAL, F.LABEL_REPEATED
    msg("ShapeProto", [("element_type", 2, F.TYPE_INT32, opt, None), ("dimensions", 3, F.TYPE_INT64, rep, None)])
    msg("ComputationDevice", [("replica_device_ids", 1, F.TYPE_INT64, rep, None)])
    msg("DeviceAssignmentProto", [("replica_count", 1, F.TYPE_INT32, opt, None),
                                  ("computation_count", 2, F.TYPE_INT32, opt, None),
                                  ("computation_devices", 3, F.TYPE_MESSAGE, rep, ".fixture.ComputationDevice")])
    msg("ExecutableBuildOptionsProto", [("device_ordinal", 1, F.TYPE_INT64, opt, None),
                                        ("num_replicas", 4, F.TYPE_INT64, opt, None),
                                        ("num_partitions", 5, F.TYPE_INT64, opt, None),
                                        ("use_spmd_partitioning", 6, F.TYPE_BOOL, opt, None),
                                        ("device_assignment", 9, F.TYPE_MESSAGE, opt, ".fixture.DeviceAssignmentProto")])
    msg("CompileOptionsProto", [("argument_layouts", 1, F.TYPE_MESSAGE, rep, ".fixture.ShapeProto"),
                                ("parameter_is_tupled_arguments", 2, F.TYPE_BOOL, opt, None),
                                ("executable_build_options", 3, F.TYPE_MESSAGE, opt, ".fixture.ExecutableBuildOptionsProto"),
                                ("compile_portable_executable", 4, F.TYPE_BOOL, opt, None),
                                ("profile_version", 5, F.TYPE_INT64, opt, None)])
    pool = descriptor_pool.DescriptorPool()
    pool.Add(fd)
    return {n: message_factory.GetMessageClass(pool.FindMessageTypeByName("fixture." + n))
            for n in ("CompileOptionsProto", "ExecutableBuildOptionsProto", "DeviceAssignmentProto", "ComputationDevice",
                      "ShapeProto")}


def cases():
    M = _messages()
    out = []

    def add(name, msg, expect):
        out.append({"name": name, "hex": msg.SerializeToString().hex(), "expect": expect})

    add("empty", M["CompileOptionsProto"](), "replicas=-1 partitions=-1 assignment=-1x-1 devices=")
    one = M["CompileOptionsProto"](profile_version=7)
    one.executable_build_options.num_replicas = 1
    one.executable_build_options.num_partitions = 1
    one.executable_build_options.device_ordinal = -1
    add("single_device_jit", one, "replicas=1 partitions=1 assignment=-1x-1 devices=")
    sm = M["CompileOptionsProto"](parameter_is_tupled_arguments=False, compile_portable_executable=True)
    sm.argument_layouts.add(element_type=11, dimensions=[8, 1024])
    b = sm.executable_build_options
    b.num_replicas, b.num_partitions, b.use_spmd_partitioning = 1, 8, True
    b.device_assignment.replica_count, b.device_assignment.computation_count = 1, 8
    for d in range(8):
        b.device_assignment.computation_devices.add(replica_device_ids=[d])
    add("shard_map_8", sm, "replicas=1 partitions=8 assignment=1x8 devices=0;1;2;3;4;5;6;7")
    rp = M["CompileOptionsProto"]()
    rp.executable_build_options.num_replicas = 2
    rp.executable_build_options.num_partitions = 2
    da = rp.executable_build_options.device_assignment
    da.replica_count, da.computation_count = 2, 2
    da.computation_devices.add(replica_device_ids=[0, 2])
    da.computation_devices.add(replica_device_ids=[1, 3])
    add("replicas_2_partitions_2", rp, "replicas=2 partitions=2 assignment=2x2 devices=0,2;1,3")
    return out


if __name__ == "__main__":
    with open(os.path.join(HERE, "compile_options.json"), "w") as f:
        json.dump(cases(), f, indent=1)
        f.write("\n")
