"""ctypes binding of the PJRT C API exported by libpjrt_b200.so — the Python-side harness.

It drives the plugin exactly the way a PJRT client does (and the way the reference's C++ harness
src/pjrt/pjrt_e2e.cc:60-181 does): GetPjrtApi -> Client_Create -> BufferFromHostBuffer ->
Client_Compile(format "mlir") -> LoadedExecutable_Execute -> Buffer_ToHostBuffer, with every
PJRT_Error turned into a `PjrtError(code, message)`.  jax is not installed on this image; this
binding stands in for jaxlib's loader, through the same C ABI.
"""
from __future__ import annotations

import ctypes as C
import os
import threading
from typing import Callable, Dict, List, Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
DEFAULT_LIB = os.path.join(os.path.dirname(HERE), "lib", "libpjrt_b200.so")

# PJRT_Buffer_Type codes
TYPES = {"pred": 1, "i8": 2, "i16": 3, "i32": 4, "i64": 5, "u8": 6, "u16": 7, "u32": 8, "u64": 9,
         "f16": 10, "f32": 11, "f64": 12, "bf16": 13}
CODE_NAMES = {1: "CANCELLED", 2: "UNKNOWN", 3: "INVALID_ARGUMENT", 4: "DEADLINE_EXCEEDED", 5: "NOT_FOUND",
              6: "ALREADY_EXISTS", 7: "PERMISSION_DENIED", 8: "RESOURCE_EXHAUSTED", 9: "FAILED_PRECONDITION",
              10: "ABORTED", 11: "OUT_OF_RANGE", 12: "UNIMPLEMENTED", 13: "INTERNAL", 14: "UNAVAILABLE",
              15: "DATA_LOSS", 16: "UNAUTHENTICATED"}

# Function-table slot order of PJRT_Api v0.55 (after struct_size, extension_start, version).
API_FIELDS = [
    "Error_Destroy", "Error_Message", "Error_GetCode", "Plugin_Initialize", "Plugin_Attributes",
    "Event_Destroy", "Event_IsReady", "Event_Error", "Event_Await", "Event_OnReady",
    "Client_Create", "Client_Destroy", "Client_PlatformName", "Client_ProcessIndex", "Client_PlatformVersion",
    "Client_Devices", "Client_AddressableDevices", "Client_LookupDevice", "Client_LookupAddressableDevice",
    "Client_AddressableMemories", "Client_Compile", "Client_DefaultDeviceAssignment", "Client_BufferFromHostBuffer",
    "DeviceDescription_Id", "DeviceDescription_ProcessIndex", "DeviceDescription_Attributes", "DeviceDescription_Kind",
    "DeviceDescription_DebugString", "DeviceDescription_ToString",
    "Device_GetDescription", "Device_IsAddressable", "Device_LocalHardwareId", "Device_AddressableMemories",
    "Device_DefaultMemory", "Device_MemoryStats",
    "Memory_Id", "Memory_Kind", "Memory_DebugString", "Memory_ToString", "Memory_AddressableByDevices",
    "Executable_Destroy", "Executable_Name", "Executable_NumReplicas", "Executable_NumPartitions",
    "Executable_NumOutputs", "Executable_SizeOfGeneratedCodeInBytes", "Executable_GetCostAnalysis",
    "Executable_OutputMemoryKinds", "Executable_OptimizedProgram", "Executable_Serialize",
    "LoadedExecutable_Destroy", "LoadedExecutable_GetExecutable", "LoadedExecutable_AddressableDevices",
    "LoadedExecutable_Delete", "LoadedExecutable_IsDeleted", "LoadedExecutable_Execute",
    "Executable_DeserializeAndLoad", "LoadedExecutable_Fingerprint",
    "Buffer_Destroy", "Buffer_ElementType", "Buffer_Dimensions", "Buffer_UnpaddedDimensions",
    "Buffer_DynamicDimensionIndices", "Buffer_GetMemoryLayout", "Buffer_OnDeviceSizeInBytes", "Buffer_Device",
    "Buffer_Memory", "Buffer_Delete", "Buffer_IsDeleted", "Buffer_CopyToDevice", "Buffer_ToHostBuffer",
    "Buffer_IsOnCpu", "Buffer_ReadyEvent", "Buffer_UnsafePointer", "Buffer_IncreaseExternalReferenceCount",
    "Buffer_DecreaseExternalReferenceCount", "Buffer_OpaqueDeviceMemoryDataPointer",
    "CopyToDeviceStream_Destroy", "CopyToDeviceStream_AddChunk", "CopyToDeviceStream_TotalBytes",
    "CopyToDeviceStream_GranuleSize", "CopyToDeviceStream_CurrentBytes",
    "TopologyDescription_Create", "TopologyDescription_Destroy", "TopologyDescription_PlatformName",
    "TopologyDescription_PlatformVersion", "TopologyDescription_GetDeviceDescriptions",
    "TopologyDescription_Serialize", "TopologyDescription_Attributes",
    "Compile", "Executable_OutputElementTypes", "Executable_OutputDimensions", "Buffer_CopyToMemory",
    "Client_CreateViewOfDeviceBuffer", "Executable_Fingerprint", "Client_TopologyDescription",
    "Executable_GetCompiledMemoryStats", "Memory_Kind_Id", "ExecuteContext_Create", "ExecuteContext_Destroy",
]

P = C.c_void_p
SZ = C.c_size_t


def _args(name, fields):
    return type(name, (C.Structure,), {"_fields_": [("struct_size", SZ), ("extension_start", P)] + fields})


class NamedValue(C.Structure):
    class _V(C.Union):
        _fields_ = [("string_value", C.c_char_p), ("int64_value", C.c_int64), ("int64_array_value", P),
                    ("float_value", C.c_float), ("bool_value", C.c_bool)]
    _anonymous_ = ("v",)
    _fields_ = [("struct_size", SZ), ("extension_start", P), ("name", C.c_char_p), ("name_size", SZ),
                ("type", C.c_int), ("v", _V), ("value_size", SZ)]


ErrorDestroyArgs = _args("ErrorDestroyArgs", [("error", P)])
ErrorMessageArgs = _args("ErrorMessageArgs", [("error", P), ("message", P), ("message_size", SZ)])
ErrorGetCodeArgs = _args("ErrorGetCodeArgs", [("error", P), ("code", C.c_int)])
EventArgs = _args("EventArgs", [("event", P)])
EventIsReadyArgs = _args("EventIsReadyArgs", [("event", P), ("is_ready", C.c_bool)])
KvGetArgs = _args("KvGetArgs", [("key", P), ("key_size", SZ), ("timeout_in_ms", C.c_int), ("callback_error", P),
                                ("user_arg", P), ("value", P), ("value_size", SZ), ("value_deleter_callback", P)])
KvPutArgs = _args("KvPutArgs", [("key", P), ("key_size", SZ), ("value", P), ("value_size", SZ),
                                ("callback_error", P), ("user_arg", P)])
KV_GET_FN = C.CFUNCTYPE(P, C.POINTER(KvGetArgs))
KV_PUT_FN = C.CFUNCTYPE(P, C.POINTER(KvPutArgs))
DELETER_FN = C.CFUNCTYPE(None, P)
ClientCreateArgs = _args("ClientCreateArgs", [("create_options", P), ("num_options", SZ), ("kv_get_callback", KV_GET_FN),
                                              ("kv_get_user_arg", P), ("kv_put_callback", KV_PUT_FN),
                                              ("kv_put_user_arg", P), ("client", P)])
ClientArgs = _args("ClientArgs", [("client", P)])
ClientStrArgs = _args("ClientStrArgs", [("client", P), ("s", P), ("n", SZ)])
ClientListArgs = _args("ClientListArgs", [("client", P), ("items", C.POINTER(P)), ("n", SZ)])
Program = _args("Program", [("code", P), ("code_size", SZ), ("format", C.c_char_p), ("format_size", SZ)])
CompileArgs = _args("CompileArgs", [("client", P), ("program", C.POINTER(Program)), ("compile_options", P),
                                    ("compile_options_size", SZ), ("executable", P)])
FromHostArgs = _args("FromHostArgs", [("client", P), ("data", P), ("type", C.c_int), ("dims", C.POINTER(C.c_int64)),
                                      ("num_dims", SZ), ("byte_strides", P), ("num_byte_strides", SZ),
                                      ("host_buffer_semantics", C.c_int), ("device", P), ("memory", P),
                                      ("device_layout", P), ("done_with_host_buffer", P), ("buffer", P)])
BufferArgs = _args("BufferArgs", [("buffer", P)])
BufferDimsArgs = _args("BufferDimsArgs", [("buffer", P), ("dims", C.POINTER(C.c_int64)), ("num_dims", SZ)])
BufferTypeArgs = _args("BufferTypeArgs", [("buffer", P), ("type", C.c_int)])
ToHostArgs = _args("ToHostArgs", [("src", P), ("host_layout", P), ("dst", P), ("dst_size", SZ), ("event", P)])
BufferPtrArgs = _args("BufferPtrArgs", [("buffer", P), ("ptr", C.c_uint64)])
LoadedArgs = _args("LoadedArgs", [("executable", P)])
GetExecArgs = _args("GetExecArgs", [("loaded_executable", P), ("executable", P)])
ExecNumOutArgs = _args("ExecNumOutArgs", [("executable", P), ("num_outputs", SZ)])
ExecNameArgs = _args("ExecNameArgs", [("executable", P), ("name", P), ("name_size", SZ)])
ExecuteOptions = _args("ExecuteOptions", [("send_callbacks", P), ("recv_callbacks", P), ("num_send_ops", SZ),
                                          ("num_recv_ops", SZ), ("launch_id", C.c_int),
                                          ("non_donatable_input_indices", P), ("num_non_donatable_input_indices", SZ)])
ExecuteArgs = _args("ExecuteArgs", [("executable", P), ("options", C.POINTER(ExecuteOptions)),
                                    ("argument_lists", C.POINTER(C.POINTER(P))), ("num_devices", SZ), ("num_args", SZ),
                                    ("output_lists", C.POINTER(C.POINTER(P))), ("device_complete_events", C.POINTER(P)),
                                    ("execute_device", P)])
DeviceDescArgs = _args("DeviceDescArgs", [("device", P), ("description", P)])
DescStrArgs = _args("DescStrArgs", [("description", P), ("s", P), ("n", SZ)])
DescIdArgs = _args("DescIdArgs", [("description", P), ("id", C.c_int)])
DescAttrArgs = _args("DescAttrArgs", [("description", P), ("num_attributes", SZ), ("attributes", C.POINTER(NamedValue))])
DeviceBoolArgs = _args("DeviceBoolArgs", [("device", P), ("value", C.c_bool)])
DeviceIntArgs = _args("DeviceIntArgs", [("device", P), ("value", C.c_int)])
DeviceMemsArgs = _args("DeviceMemsArgs", [("device", P), ("memories", C.POINTER(P)), ("n", SZ)])
MemoryStrArgs = _args("MemoryStrArgs", [("memory", P), ("s", P), ("n", SZ)])
MemoryIntArgs = _args("MemoryIntArgs", [("memory", P), ("value", C.c_int)])
BufferMemArgs = _args("BufferMemArgs", [("buffer", P), ("memory", P)])
BufferBoolArgs = _args("BufferBoolArgs", [("buffer", P), ("value", C.c_bool)])
CopyToMemoryArgs = _args("CopyToMemoryArgs", [("buffer", P), ("dst_memory", P), ("dst_buffer", P)])
LookupDeviceArgs = _args("LookupDeviceArgs", [("client", P), ("id", C.c_int), ("device", P)])
AssignArgs = _args("AssignArgs", [("client", P), ("num_replicas", C.c_int), ("num_partitions", C.c_int),
                                  ("size", SZ), ("assignment", C.POINTER(C.c_int))])


class PjrtError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"{CODE_NAMES.get(code, code)}: {message}")
        self.code = code
        self.code_name = CODE_NAMES.get(code, str(code))
        self.message = message


def np_type_code(a: np.ndarray) -> int:
    import ml_dtypes
    dt = a.dtype
    if dt == ml_dtypes.bfloat16:
        return TYPES["bf16"]
    return {np.dtype(np.bool_): 1, np.dtype(np.int8): 2, np.dtype(np.int16): 3, np.dtype(np.int32): 4,
            np.dtype(np.int64): 5, np.dtype(np.uint8): 6, np.dtype(np.uint16): 7, np.dtype(np.uint32): 8,
            np.dtype(np.uint64): 9, np.dtype(np.float16): 10, np.dtype(np.float32): 11,
            np.dtype(np.float64): 12}[np.dtype(dt)]


def np_dtype_of(code: int):
    import ml_dtypes
    return {1: np.bool_, 2: np.int8, 3: np.int16, 4: np.int32, 5: np.int64, 6: np.uint8, 7: np.uint16, 8: np.uint32,
            9: np.uint64, 10: np.float16, 11: np.float32, 12: np.float64, 13: ml_dtypes.bfloat16}[code]


class Api:
    """The loaded plugin and its function table."""

    def __init__(self, path: str = DEFAULT_LIB):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} not built: run `python mccl-jax_b200/build.py`")
        self.lib = C.CDLL(path)
        self.lib.GetPjrtApi.restype = P
        self.ptr = self.lib.GetPjrtApi()
        head = C.cast(self.ptr, C.POINTER(C.c_size_t))
        self.struct_size = head[0]
        self.version = (C.cast(self.ptr + 32, C.POINTER(C.c_int))[0], C.cast(self.ptr + 36, C.POINTER(C.c_int))[0])
        table = C.cast(self.ptr + 40, C.POINTER(P))
        self.fn: Dict[str, P] = {name: table[i] for i, name in enumerate(API_FIELDS)}

    def call(self, name: str, args: C.Structure):
        args.struct_size = C.sizeof(args)
        f = C.CFUNCTYPE(P, C.c_void_p)(self.fn[name])
        err = f(C.addressof(args))
        if err:
            raise self._error(err)
        return args

    def _error(self, err) -> PjrtError:
        m = ErrorMessageArgs(error=err)
        m.struct_size = C.sizeof(m)
        C.CFUNCTYPE(None, C.c_void_p)(self.fn["Error_Message"])(C.addressof(m))
        msg = C.string_at(m.message, m.message_size).decode(errors="replace")
        g = ErrorGetCodeArgs(error=err)
        g.struct_size = C.sizeof(g)
        C.CFUNCTYPE(P, C.c_void_p)(self.fn["Error_GetCode"])(C.addressof(g))
        d = ErrorDestroyArgs(error=err)
        d.struct_size = C.sizeof(d)
        C.CFUNCTYPE(None, C.c_void_p)(self.fn["Error_Destroy"])(C.addressof(d))
        return PjrtError(g.code, msg)

    # events
    def await_event(self, ev):
        if not ev:
            return
        try:
            self.call("Event_Await", EventArgs(event=ev))
        finally:
            self.call("Event_Destroy", EventArgs(event=ev))

    def event_ready(self, ev) -> bool:
        return bool(self.call("Event_IsReady", EventIsReadyArgs(event=ev)).is_ready)


class Buffer:
    def __init__(self, client: "Client", handle):
        self.client, self.h = client, handle

    @property
    def api(self):
        return self.client.api

    def shape(self):
        a = self.api.call("Buffer_Dimensions", BufferDimsArgs(buffer=self.h))
        return tuple(a.dims[i] for i in range(a.num_dims))

    def type_code(self):
        return self.api.call("Buffer_ElementType", BufferTypeArgs(buffer=self.h)).type

    def device_pointer(self) -> int:
        return self.api.call("Buffer_UnsafePointer", BufferPtrArgs(buffer=self.h)).ptr

    def to_numpy(self, out: Optional[np.ndarray] = None) -> np.ndarray:
        shape = self.shape()
        dt = np_dtype_of(self.type_code())
        if out is None:
            out = np.empty(shape, dtype=dt)
        a = self.api.call("Buffer_ToHostBuffer", ToHostArgs(src=self.h, dst=out.ctypes.data, dst_size=out.nbytes))
        self.api.await_event(a.event)
        return out

    def memory(self):
        return self.api.call("Buffer_Memory", BufferMemArgs(buffer=self.h)).memory

    def is_on_cpu(self) -> bool:
        return bool(self.api.call("Buffer_IsOnCpu", BufferBoolArgs(buffer=self.h)).value)

    def is_deleted(self) -> bool:
        return bool(self.api.call("Buffer_IsDeleted", BufferBoolArgs(buffer=self.h)).value)

    def copy_to_memory(self, memory) -> "Buffer":
        a = self.api.call("Buffer_CopyToMemory", CopyToMemoryArgs(buffer=self.h, dst_memory=memory))
        return Buffer(self.client, a.dst_buffer)

    def add_external_ref(self, delta: int):
        name = "Buffer_IncreaseExternalReferenceCount" if delta > 0 else "Buffer_DecreaseExternalReferenceCount"
        self.api.call(name, BufferArgs(buffer=self.h))

    def mark_deleted(self):
        """PJRT_Buffer_Delete: storage released (now, or at the last external reference's release);
        the handle stays valid until destroyed."""
        self.api.call("Buffer_Delete", BufferArgs(buffer=self.h))

    def delete(self):
        # a buffer outliving its client is dropped without a call: the client freed the device
        if self.h and self.client.h:
            self.api.call("Buffer_Destroy", BufferArgs(buffer=self.h))
        self.h = None

    def __del__(self):
        try:
            self.delete()
        except Exception:
            pass


class Executable:
    def __init__(self, client: "Client", handle):
        self.client, self.h = client, handle
        api = client.api
        g = api.call("LoadedExecutable_GetExecutable", GetExecArgs(loaded_executable=handle))
        self.num_outputs = api.call("Executable_NumOutputs", ExecNumOutArgs(executable=g.executable)).num_outputs
        n = api.call("Executable_Name", ExecNameArgs(executable=g.executable))
        self.name = C.string_at(n.name, n.name_size).decode()
        api.call("Executable_Destroy", LoadedArgs(executable=g.executable))

    def execute(self, args: Sequence[Buffer], wait: bool = True, non_donatable: Sequence[int] = ()) -> List[Buffer]:
        """LoadedExecutable_Execute on one device.  Arguments the program marks donated
        (tf.aliasing_output / jax.buffer_donor) are given up -- deleted after the call, their memory
        reused by the aliased result where the plan allows -- unless listed in `non_donatable`."""
        api = self.client.api
        arg_arr = (P * max(1, len(args)))(*[b.h for b in args])
        arg_lists = (C.POINTER(P) * 1)(C.cast(arg_arr, C.POINTER(P)))
        out_arr = (P * max(1, self.num_outputs))()
        out_lists = (C.POINTER(P) * 1)(C.cast(out_arr, C.POINTER(P)))
        evs = (P * 1)()
        opts = ExecuteOptions()
        opts.struct_size = C.sizeof(opts)
        nd = (C.c_int64 * max(1, len(non_donatable)))(*non_donatable)
        if non_donatable:
            opts.non_donatable_input_indices = C.cast(nd, P)
            opts.num_non_donatable_input_indices = len(non_donatable)
        api.call("LoadedExecutable_Execute", ExecuteArgs(executable=self.h, options=C.pointer(opts), argument_lists=arg_lists,
                                                          num_devices=1, num_args=len(args), output_lists=out_lists,
                                                          device_complete_events=evs))
        outs = [Buffer(self.client, out_arr[i]) for i in range(self.num_outputs)]
        if wait:
            api.await_event(evs[0])
        elif evs[0]:
            # asynchronous: the outputs carry their own ready events; drop the completion event
            api.call("Event_Destroy", EventArgs(event=evs[0]))
        return outs

    def destroy(self):
        if self.h and self.client.h:
            self.client.api.call("LoadedExecutable_Destroy", LoadedArgs(executable=self.h))
        self.h = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


class Client:
    """One PJRT client: `node_id` of `num_nodes` processes, bound to CUDA device `device_ordinal`."""

    def __init__(self, api: Optional[Api] = None, node_id: int = 0, num_nodes: int = 1,
                 device_ordinal: Optional[int] = None, kv_put: Optional[Callable[[str, bytes], None]] = None,
                 kv_get: Optional[Callable[[str, int], bytes]] = None, nccl_max_ctas: int = 0):
        self.api = api or Api()
        opts = [("node_id", node_id), ("num_nodes", num_nodes)]
        if device_ordinal is not None:
            opts.append(("device_ordinal", device_ordinal))
        if nccl_max_ctas:
            opts.append(("nccl_max_ctas", nccl_max_ctas))
        arr = (NamedValue * len(opts))()
        self._names = []
        for i, (k, v) in enumerate(opts):
            kb = k.encode()
            self._names.append(kb)
            arr[i].struct_size = C.sizeof(NamedValue)
            arr[i].name = kb
            arr[i].name_size = len(kb)
            arr[i].type = 1  # kInt64
            arr[i].int64_value = int(v)
            arr[i].value_size = 1
        args = ClientCreateArgs(create_options=C.cast(arr, P), num_options=len(opts))
        self._keep = []
        if kv_put and kv_get:
            held: Dict[int, C.Array] = {}

            def put_cb(pa):
                a = pa.contents
                try:
                    kv_put(C.string_at(a.key, a.key_size).decode(), C.string_at(a.value, a.value_size))
                    return None
                except Exception:
                    return 1  # non-null: the plugin treats it as a failed callback

            def get_cb(ga):
                a = ga.contents
                try:
                    v = kv_get(C.string_at(a.key, a.key_size).decode(), a.timeout_in_ms)
                except Exception:
                    return 1
                buf = C.create_string_buffer(v, len(v))
                held[C.addressof(buf)] = buf
                a.value = C.addressof(buf)
                a.value_size = len(v)
                a.value_deleter_callback = C.cast(deleter, P)
                return None

            def del_cb(p):
                held.pop(p, None)

            deleter = DELETER_FN(del_cb)
            g, pcb = KV_GET_FN(get_cb), KV_PUT_FN(put_cb)
            self._keep += [deleter, g, pcb, held]
            args.kv_get_callback, args.kv_put_callback = g, pcb
        self.h = self.api.call("Client_Create", args).client
        self._arr = arr

    def platform_name(self) -> str:
        a = self.api.call("Client_PlatformName", ClientStrArgs(client=self.h))
        return C.string_at(a.s, a.n).decode()

    def platform_version(self) -> str:
        a = self.api.call("Client_PlatformVersion", ClientStrArgs(client=self.h))
        return C.string_at(a.s, a.n).decode()

    def devices(self, addressable=False):
        a = self.api.call("Client_AddressableDevices" if addressable else "Client_Devices", ClientListArgs(client=self.h))
        return [a.items[i] for i in range(a.n)]

    def device_kind(self, dev) -> str:
        d = self.api.call("Device_GetDescription", DeviceDescArgs(device=dev)).description
        a = self.api.call("DeviceDescription_Kind", DescStrArgs(description=d))
        return C.string_at(a.s, a.n).decode()

    def memories(self):
        a = self.api.call("Client_AddressableMemories", ClientListArgs(client=self.h))
        return [a.items[i] for i in range(a.n)]

    def memory_kind(self, mem) -> str:
        a = self.api.call("Memory_Kind", MemoryStrArgs(memory=mem))
        return C.string_at(a.s, a.n).decode()

    def memory_id(self, mem) -> int:
        return self.api.call("Memory_Id", MemoryIntArgs(memory=mem)).value

    def lookup_device(self, global_id: int):
        return self.api.call("Client_LookupDevice", LookupDeviceArgs(client=self.h, id=global_id)).device

    def default_device_assignment(self, replicas: int, partitions: int):
        out = (C.c_int * (replicas * partitions))()
        self.api.call("Client_DefaultDeviceAssignment", AssignArgs(client=self.h, num_replicas=replicas,
                                                                   num_partitions=partitions,
                                                                   size=replicas * partitions, assignment=out))
        return list(out)

    def compile(self, program) -> Executable:
        """`program`: StableHLO as MLIR text (str) or MLIR bytecode (bytes); format "mlir" covers both."""
        code = program.encode() if isinstance(program, str) else bytes(program)
        buf = C.create_string_buffer(code, len(code))
        prog = Program(code=C.addressof(buf), code_size=len(code), format=b"mlir", format_size=4)
        prog.struct_size = C.sizeof(prog)
        a = self.api.call("Client_Compile", CompileArgs(client=self.h, program=C.pointer(prog)))
        return Executable(self, a.executable)

    def buffer_from_host(self, x: np.ndarray, device=None, semantics: int = 1, memory=None) -> Buffer:
        x = np.ascontiguousarray(x).reshape(np.shape(x))   # (ascontiguousarray turns 0-d into 1-d)
        dims = (C.c_int64 * max(1, x.ndim))(*x.shape)
        a = self.api.call("Client_BufferFromHostBuffer", FromHostArgs(
            client=self.h, data=x.ctypes.data, type=np_type_code(x), dims=dims, num_dims=x.ndim,
            host_buffer_semantics=semantics, device=device if device or memory else self.devices(True)[0],
            memory=memory))
        self.api.await_event(a.done_with_host_buffer)
        return Buffer(self, a.buffer)

    def run(self, text_or_exe, inputs: Sequence[np.ndarray]) -> List[np.ndarray]:
        exe = self.compile(text_or_exe) if isinstance(text_or_exe, (str, bytes)) else text_or_exe
        bufs, outs = [], []
        try:
            bufs = [self.buffer_from_host(x) for x in inputs]
            outs = exe.execute(bufs)
            return [o.to_numpy() for o in outs]
        finally:
            for b in bufs + outs:
                b.delete()
            if isinstance(text_or_exe, str):
                exe.destroy()

    def close(self):
        if self.h:
            self.api.call("Client_Destroy", ClientArgs(client=self.h))
            self.h = None
