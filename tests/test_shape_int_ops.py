"""Shape, bit and special-function ops of the reference's lowering beyond the configs' own programs:
broadcast (structural.mm), reverse, dynamic_slice, dynamic_update_slice, bitcast_convert (src/jam/ops/shape.mm), popcnt and the
three shifts (unary.mm, binary.mm), count_leading_zeros and reduce_precision (hard_limit.mm:15-52),
erf (chlo.erf, or custom_call @mhlo.erf as hard_limit.mm:65-67 reads it) and partition_id
(collectives.mm:16-29).

CPU: the oracle's integer ops against Python integer arithmetic (StableHLO's width rules: shift
amounts read as unsigned, >= width gives 0 or the sign fill), the other ops against independent
numpy / scipy computations; every op compiles through NVRTC; the generic op form parses to the
pretty form's graph.  GPU: each op through PJRT against the oracle, bit-exact for integer and bit
results, f32 rel 1e-5 / bf16 rel 2e-2 for erf.
"""
import ctypes
import os
import sys

import ml_dtypes
import numpy as np
import pytest
import scipy.special

from conftest import RTOL_BF16, RTOL_F32, assert_close
from oracle.interp import run as oracle_run

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
import mlir_generic  # noqa: E402

INT_TYPES = {"i8": np.int8, "i16": np.int16, "i32": np.int32, "i64": np.int64,
             "ui8": np.uint8, "ui32": np.uint32, "ui64": np.uint64}
NP = dict(INT_TYPES, f32=np.float32, f64=np.float64, f16=np.float16, bf16=ml_dtypes.bfloat16, ui16=np.uint16)
SHAPE = (8, 128)


def prog(body, ins, out, attrs=""):
    sig = ", ".join(f"%arg{i}: {t}" for i, t in enumerate(ins))
    return (f"module @jit_ops {attrs}{{\n  func.func public @main({sig}) -> ({out}) {{\n{body}\n"
            f"    return %0 : {out}\n  }}\n}}\n")


def T(dt, shape=SHAPE):
    return "tensor<" + "".join(f"{d}x" for d in shape) + dt + ">"


def int_inputs(dt, seed):
    npd = INT_TYPES[dt]
    info, w = np.iinfo(npd), 8 * np.dtype(npd).itemsize
    rng = np.random.default_rng(seed)
    x = rng.integers(info.min, info.max, size=SHAPE, dtype=npd, endpoint=True)
    x[0, :4] = [0, 1, info.max, info.min]
    y = rng.integers(0, w + 3, size=SHAPE).astype(npd)     # amounts around the width
    if info.min < 0:
        y[1, :3] = [-1, -w, w]
    return x, y


def int_program(op, dt):
    t = T(dt)
    if op in ("popcnt", "count_leading_zeros"):
        return prog(f"    %0 = stablehlo.{op} %arg0 : {t}", [t], t)
    return prog(f"    %0 = stablehlo.{op} %arg0, %arg1 : {t}", [t, t], t)


def python_int_op(op, a, b, w):
    ua, ub = int(a) & ((1 << w) - 1), int(b) & ((1 << w) - 1)
    if op == "popcnt":
        return bin(ua).count("1")
    if op == "count_leading_zeros":
        return w - ua.bit_length()
    if op == "shift_left":
        return 0 if ub >= w else (ua << ub) & ((1 << w) - 1)
    if op == "shift_right_logical":
        return 0 if ub >= w else ua >> ub
    sa = ua - (1 << w) if ua >> (w - 1) else ua
    return (sa >> min(ub, w - 1)) & ((1 << w) - 1)


INT_OPS = ["popcnt", "count_leading_zeros", "shift_left", "shift_right_logical", "shift_right_arithmetic"]
INT_CASES = [(op, dt) for op in INT_OPS for dt in ["i8", "i16", "i32", "i64", "ui8", "ui32"]]

BITCASTS = [("f32", "i32"), ("i32", "f32"), ("bf16", "i16"), ("f16", "ui16"), ("f64", "i64"), ("f32", "ui32")]

F = T("f32")
OTHER = {
    "broadcast": (prog(f"    %0 = stablehlo.broadcast %arg0, sizes = [3] : ({F}) -> {T('f32', (3, 8, 128))}", [F],
                       T("f32", (3, 8, 128))), ["f32"]),
    "reverse_1": (prog(f"    %0 = stablehlo.reverse %arg0, dims = [1] : {F}", [F], F), ["f32"]),
    "reverse_01": (prog(f"    %0 = stablehlo.reverse %arg0, dims = [0, 1] : {F}", [F], F), ["f32"]),
    "dynamic_slice": (prog(f"    %0 = stablehlo.dynamic_slice %arg0, %arg1, %arg2, sizes = [4, 64] : "
                           f"({F}, tensor<i32>, tensor<i32>) -> {T('f32', (4, 64))}",
                           [F, "tensor<i32>", "tensor<i32>"], T("f32", (4, 64))), ["f32", "s", "s"]),
    # unsigned 64-bit starts: 2^64 - 5 (from -5) is a large value and clamps to dim - window
    "dynamic_slice_u64": (prog(f"    %0 = stablehlo.dynamic_slice %arg0, %arg1, %arg2, sizes = [4, 64] : "
                               f"({F}, tensor<ui64>, tensor<ui64>) -> {T('f32', (4, 64))}",
                               [F, "tensor<ui64>", "tensor<ui64>"], T("f32", (4, 64))), ["f32", "u", "u"]),
    "dynamic_update_slice": (prog(f"    %0 = stablehlo.dynamic_update_slice %arg0, %arg1, %arg2, %arg3 : "
                                  f"({F}, {T('f32', (4, 64))}, tensor<i32>, tensor<i32>) -> {F}",
                                  [F, T("f32", (4, 64)), "tensor<i32>", "tensor<i32>"], F), ["f32", "f32u", "s", "s"]),
    "reduce_precision_e8m7": (prog(f"    %0 = stablehlo.reduce_precision %arg0, format = e8m7 : {F}", [F], F), ["f32w"]),
    "reduce_precision_e5m10": (prog(f"    %0 = stablehlo.reduce_precision %arg0, format = e5m10 : {F}", [F], F), ["f32w"]),
    "erf_chlo": (prog(f"    %0 = chlo.erf %arg0 : {F} -> {F}", [F], F), ["f32"]),
    "erf_custom_call": (prog(f"    %0 = stablehlo.custom_call @mhlo.erf(%arg0) : ({F}) -> {F}", [F], F), ["f32"]),
    "erf_bf16": (prog(f"    %0 = chlo.erf %arg0 : {T('bf16')} -> {T('bf16')}", [T("bf16")], T("bf16")), ["bf16"]),
    "partition_id": (prog("    %p = stablehlo.partition_id : tensor<ui32>\n"
                          "    %c = stablehlo.convert %p : (tensor<ui32>) -> tensor<f32>\n"
                          f"    %b = stablehlo.broadcast_in_dim %c, dims = [] : (tensor<f32>) -> {F}\n"
                          f"    %0 = stablehlo.add %arg0, %b : {F}", [F], F), ["f32"]),
}


def other_inputs(kinds, seed, starts=(3, 100)):
    rng = np.random.default_rng(seed)
    out, k = [], 0
    for kind in kinds:
        if kind == "s":
            out.append(np.array(starts[k], np.int32))
            k += 1
        elif kind == "u":
            out.append(np.array(starts[k] % 2 ** 64, np.uint64))
            k += 1
        elif kind == "f32u":
            out.append(rng.standard_normal((4, 64)).astype(np.float32) + 10)
        elif kind == "f32w":   # wide range: f16 overflow, f16 subnormals, ties
            x = (rng.standard_normal(SHAPE) * np.exp2(rng.integers(-30, 20, SHAPE))).astype(np.float32)
            x[0, :4] = [65520.0, 1e-7, -3.0e-8, 1.00390625]
            out.append(x)
        elif kind == "bf16":
            out.append(rng.standard_normal(SHAPE).astype(ml_dtypes.bfloat16))
        else:
            out.append(rng.standard_normal(SHAPE).astype(np.float32))
    return out


def bitcast_input(a, seed):
    rng = np.random.default_rng(seed)
    if a in ("f32", "f64"):
        return rng.standard_normal(SHAPE).astype(NP[a])
    if a == "bf16":
        return rng.standard_normal(SHAPE).astype(ml_dtypes.bfloat16)
    if a == "f16":
        return rng.standard_normal(SHAPE).astype(np.float16)
    bits = rng.integers(0, 1 << 62, size=SHAPE, dtype=np.int64)
    x = bits.astype(np.uint64).astype(np.dtype("u%d" % np.dtype(NP[a]).itemsize)).view(NP[a])
    if a in ("i32", "ui32"):        # keep clear of f32 NaN bit patterns (payloads are not compared)
        x = np.where((x.view(np.uint32) & 0x7F800000) == 0x7F800000, x ^ np.array(0x40000000, x.dtype), x)
    return x


# ------------------------------------------------------------------------------------- CPU tests
@pytest.mark.parametrize("op,dt", INT_CASES)
def test_oracle_int_ops_follow_integer_arithmetic(op, dt):
    x, y = int_inputs(dt, 7)
    ins = [x] if op in ("popcnt", "count_leading_zeros") else [x, y]
    r = oracle_run(int_program(op, dt), ins)[0]
    w = 8 * x.dtype.itemsize
    got = [int(v) & ((1 << w) - 1) for v in r.ravel()]
    exp = [python_int_op(op, a, b, w) for a, b in zip(x.ravel(), y.ravel())]
    assert got == exp


def test_oracle_reduce_precision_erf_and_dynamic_slices():
    x = other_inputs(["f32w"], 3)[0]
    # round to nearest even at bf16's 7 mantissa bits, on the bits (finite inputs)
    u = x.view(np.uint32).astype(np.uint64)
    e8m7 = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32).view(np.float32)
    np.testing.assert_array_equal(oracle_run(OTHER["reduce_precision_e8m7"][0], [x])[0], e8m7)
    with np.errstate(over="ignore"):
        e5m10 = np.array([float(np.float16(v)) for v in x.ravel()], np.float32).reshape(x.shape)
    np.testing.assert_array_equal(oracle_run(OTHER["reduce_precision_e5m10"][0], [x])[0], e5m10)
    y = other_inputs(["f32"], 4)[0]
    np.testing.assert_allclose(oracle_run(OTHER["erf_chlo"][0], [y])[0], scipy.special.erf(y.astype(np.float64)), rtol=1e-6)
    np.testing.assert_allclose(oracle_run(OTHER["erf_custom_call"][0], [y])[0], scipy.special.erf(y.astype(np.float64)), rtol=1e-6)
    # offsets clamp so the window stays inside: (3, 100) -> (3, 64); (-5, 7) -> (0, 7)
    for starts, clamped in [((3, 100), (3, 64)), ((-5, 7), (0, 7))]:
        ins = other_inputs(OTHER["dynamic_slice"][1], 5, starts)
        r = oracle_run(OTHER["dynamic_slice"][0], ins)[0]
        np.testing.assert_array_equal(r, ins[0][clamped[0]:clamped[0] + 4, clamped[1]:clamped[1] + 64])
        ins = other_inputs(OTHER["dynamic_update_slice"][1], 6, starts)
        r = oracle_run(OTHER["dynamic_update_slice"][0], ins)[0]
        exp = ins[0].copy()
        exp[clamped[0]:clamped[0] + 4, clamped[1]:clamped[1] + 64] = ins[1]
        np.testing.assert_array_equal(r, exp)
    # unsigned starts never count as negative: 2^64 - 5 clamps to the last window, 2^63 + 1 too
    for starts, clamped in [((2 ** 64 - 5, 7), (4, 7)), ((1, 2 ** 63 + 1), (1, 64))]:
        ins = other_inputs(OTHER["dynamic_slice_u64"][1], 5, starts)
        r = oracle_run(OTHER["dynamic_slice_u64"][0], ins)[0]
        np.testing.assert_array_equal(r, ins[0][clamped[0]:clamped[0] + 4, clamped[1]:clamped[1] + 64])


@pytest.fixture(scope="module")
def report(lib_path):
    lib = ctypes.CDLL(lib_path)
    buf = ctypes.create_string_buffer(1 << 22)

    def run(text, mode=1):
        t = text.encode()
        rc = lib.b200_compile_report(t, len(t), 1, mode, buf, len(buf))
        return rc, buf.value.decode()
    return run


def test_all_ops_compile_with_nvrtc(report):
    texts = [int_program(op, dt) for op, dt in INT_CASES]
    texts += [prog(f"    %0 = stablehlo.bitcast_convert %arg0 : ({T(a)}) -> {T(b)}", [T(a)], T(b)) for a, b in BITCASTS]
    texts += [t for t, _ in OTHER.values()]
    for t in texts:
        rc, rep = report(t)
        assert rc == 0, rep + "\n" + t


@pytest.mark.parametrize("text,msg", [
    (prog(f"    %0 = stablehlo.reduce_precision %arg0, format = e4m3 : {F}", [F], F), "reduce_precision to e4m3"),
    (prog(f"    %0 = stablehlo.bitcast_convert %arg0 : ({F}) -> {T('i16', (8, 128, 2))}", [F], T("i16", (8, 128, 2))),
     "same width"),
    (prog(f"    %0 = stablehlo.popcnt %arg0 : {F}", [F], F), "popcnt"),
])
def test_unsupported_variants_fail_at_compile_time(report, text, msg):
    rc, rep = report(text, mode=0)
    assert rc == 1 and msg in rep, rep


def test_generic_form_of_these_ops_gives_the_same_graph(report):
    texts = [int_program(op, "i32") for op in INT_OPS] + [t for t, _ in OTHER.values()]
    for t in texts:
        rc_p, rep_p = report(t, mode=2)
        rc_g, rep_g = report(mlir_generic.convert(t), mode=2)
        assert rc_p == 0 and rc_g == 0, rep_g
        assert rep_g == rep_p, t


# ------------------------------------------------------------------------------------- GPU tests
@pytest.mark.gpu
@pytest.mark.parametrize("op,dt", INT_CASES)
def test_int_ops_bit_exact(client, op, dt):
    x, y = int_inputs(dt, 11)
    ins = [x] if op in ("popcnt", "count_leading_zeros") else [x, y]
    text = int_program(op, dt)
    got = client.run(text, ins)[0]
    ref = oracle_run(text, ins)[0]
    np.testing.assert_array_equal(got.view(np.dtype("u%d" % got.dtype.itemsize)),
                                  ref.view(np.dtype("u%d" % ref.dtype.itemsize)))


@pytest.mark.gpu
@pytest.mark.parametrize("a,b", BITCASTS)
def test_bitcast_convert_bit_exact(client, a, b):
    text = prog(f"    %0 = stablehlo.bitcast_convert %arg0 : ({T(a)}) -> {T(b)}", [T(a)], T(b))
    x = bitcast_input(a, 13)
    got = client.run(text, [x])[0]
    ref = oracle_run(text, [x])[0]
    u = np.dtype("u%d" % got.dtype.itemsize)
    np.testing.assert_array_equal(got.view(u), ref.view(u))


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(OTHER))
def test_shape_and_special_ops_vs_oracle(client, name):
    text, kinds = OTHER[name]
    for starts in [(3, 100), (-5, 7)]:
        ins = other_inputs(kinds, 17, starts)
        got = client.run(text, ins)[0]
        ref = oracle_run(text, ins)[0]
        if name.startswith("erf"):
            assert_close(got, ref, RTOL_BF16 if name == "erf_bf16" else RTOL_F32, name)
        else:
            np.testing.assert_array_equal(got, ref)
        if "s" not in kinds and "u" not in kinds:
            break
