"""A small tracer that writes StableHLO *text* in the form jax's `jit(f).lower(...).as_text()` prints.

jax is not installed on this image, so the programs the plugin compiles are produced here: each
`Builder` records ops on `T` handles and `Builder.text()` renders an MLIR module with one public
`@main`.  The op spellings follow the StableHLO assembly formats jax emits (pretty form for
elementwise/shape/reduce/dot ops, generic form for gather/scatter/all_reduce), so the plugin's
parser reads the same text a jaxlib front end would hand it (as MLIR text rather than bytecode).

`grad()` is reverse-mode autodiff over the recorded graph (the VJP rules jax applies for the ~25 ops
these configs use), so train steps (`value_and_grad` + optimizer) are written as in jax.
"""
from __future__ import annotations

import math
import struct
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

# MLIR element type spellings
DTYPES = {"pred": "i1", "i8": "i8", "i16": "i16", "i32": "i32", "i64": "i64",
          "u8": "ui8", "u16": "ui16", "u32": "ui32", "u64": "ui64",
          "f16": "f16", "bf16": "bf16", "f32": "f32", "f64": "f64"}
FLOATS = ("f16", "bf16", "f32", "f64")


def mlir_type(shape, dtype):
    dims = "x".join(str(int(d)) for d in shape)
    return f"tensor<{dims + 'x' if dims else ''}{DTYPES[dtype]}>"


def _fmt_float(x, dtype):
    x = float(x)
    if math.isnan(x) or math.isinf(x):
        if dtype == "f32":
            return "0x%08X" % struct.unpack("<I", struct.pack("<f", x))[0]
        if dtype == "bf16":
            return "0x%04X" % (struct.unpack("<I", struct.pack("<f", x))[0] >> 16)
        if dtype == "f16":
            return "0x%04X" % np.array(x, np.float16).view(np.uint16)
        return "0x%016X" % struct.unpack("<Q", struct.pack("<d", x))[0]
    return "%.6e" % x if dtype != "f64" else repr(x)


def _fmt_scalar(x, dtype):
    if dtype == "pred":
        return "true" if x else "false"
    if dtype in FLOATS:
        return _fmt_float(x, dtype)
    return str(int(x))


def _dims(lst):
    return "[" + ", ".join(str(int(d)) for d in lst) + "]"


class T:
    """A traced tensor value."""
    __slots__ = ("b", "name", "shape", "dtype", "op", "inputs", "attrs")

    def __init__(self, b, name, shape, dtype, op=None, inputs=(), attrs=None):
        self.b, self.name, self.shape, self.dtype = b, name, tuple(int(d) for d in shape), dtype
        self.op, self.inputs, self.attrs = op, tuple(inputs), attrs or {}

    @property
    def ndim(self):
        return len(self.shape)

    @property
    def type(self):
        return mlir_type(self.shape, self.dtype)

    # arithmetic sugar (numpy-style broadcasting, scalars become constants)
    def _bin(self, other, op, rev=False):
        a, c = self.b._coerce(self, other)
        return self.b.binary(op, c, a) if rev else self.b.binary(op, a, c)

    def __add__(self, o): return self._bin(o, "add")
    def __radd__(self, o): return self._bin(o, "add", True)
    def __sub__(self, o): return self._bin(o, "subtract")
    def __rsub__(self, o): return self._bin(o, "subtract", True)
    def __mul__(self, o): return self._bin(o, "multiply")
    def __rmul__(self, o): return self._bin(o, "multiply", True)
    def __truediv__(self, o): return self._bin(o, "divide")
    def __rtruediv__(self, o): return self._bin(o, "divide", True)
    def __neg__(self): return self.b.unary("negate", self)
    def __matmul__(self, o): return self.b.matmul(self, o)


class Builder:
    def __init__(self, name="jit_main", num_partitions=1, num_replicas=1):
        self.name = name
        self.num_partitions, self.num_replicas = num_partitions, num_replicas
        self.args: List[T] = []
        self.ops: List[T] = []          # in program order (each records one line)
        self.lines: Dict[int, str] = {}
        self._n = 0
        self._nc = 0
        self._const_cache = {}

    # ------------------------------------------------------------------ naming / emission
    def _fresh(self, const=False):
        if const:
            name = "%cst" if self._nc == 0 else f"%cst_{self._nc - 1}"
            self._nc += 1
            return name
        name = f"%{self._n}"
        self._n += 1
        return name

    def _emit(self, t: T, line: str):
        self.ops.append(t)
        self.lines[id(t)] = line
        return t

    # ------------------------------------------------------------------ leaves
    def arg(self, shape, dtype="f32"):
        t = T(self, f"%arg{len(self.args)}", shape, dtype, op="arg")
        self.args.append(t)
        return t

    def const(self, value, dtype="f32", shape=()):
        """Constant; scalars are emitted as 0-d constants and broadcast to `shape` (as jax does)."""
        arr = np.asarray(value)
        if arr.ndim == 0:
            key = (float(arr) if dtype in FLOATS else int(arr), dtype)
            if key not in self._const_cache:
                t = T(self, self._fresh(const=True), (), dtype, op="constant",
                      attrs={"value": arr.item()})
                self._emit(t, f"{t.name} = stablehlo.constant dense<{_fmt_scalar(arr.item(), dtype)}> : {t.type}")
                self._const_cache[key] = t
            t = self._const_cache[key]
            return self.broadcast_in_dim(t, shape, []) if tuple(shape) else t
        return self.const_array(arr, dtype)

    def const_array(self, arr, dtype):
        arr = np.asarray(arr)
        t = T(self, self._fresh(const=True), arr.shape, dtype, op="constant", attrs={"value": arr})

        def rec(a):
            if a.ndim == 0:
                return _fmt_scalar(a.item(), dtype)
            return "[" + ", ".join(rec(x) for x in a) + "]"
        return self._emit(t, f"{t.name} = stablehlo.constant dense<{rec(arr)}> : {t.type}")

    def iota(self, shape, dim, dtype="i32"):
        t = T(self, self._fresh(), shape, dtype, op="iota", attrs={"dim": dim})
        return self._emit(t, f"{t.name} = stablehlo.iota dim = {dim} : {t.type}")

    # ------------------------------------------------------------------ elementwise
    def unary(self, op, x, dtype=None):
        t = T(self, self._fresh(), x.shape, dtype or x.dtype, op=op, inputs=(x,))
        if t.dtype == x.dtype:
            return self._emit(t, f"{t.name} = stablehlo.{op} {x.name} : {t.type}")
        return self._emit(t, f"{t.name} = stablehlo.{op} {x.name} : ({x.type}) -> {t.type}")

    def binary(self, op, a, c):
        assert a.shape == c.shape, (op, a.shape, c.shape)
        assert a.dtype == c.dtype, (op, a.dtype, c.dtype)
        t = T(self, self._fresh(), a.shape, a.dtype, op=op, inputs=(a, c))
        return self._emit(t, f"{t.name} = stablehlo.{op} {a.name}, {c.name} : {t.type}")

    def convert(self, x, dtype):
        if x.dtype == dtype:
            return x
        t = T(self, self._fresh(), x.shape, dtype, op="convert", inputs=(x,))
        return self._emit(t, f"{t.name} = stablehlo.convert {x.name} : ({x.type}) -> {t.type}")

    def compare(self, a, c, direction):
        a, c = self._coerce(a, c)
        ctype = "FLOAT" if a.dtype in FLOATS else ("UNSIGNED" if a.dtype.startswith("u") or a.dtype == "pred" else "SIGNED")
        t = T(self, self._fresh(), a.shape, "pred", op="compare", inputs=(a, c),
              attrs={"direction": direction, "type": ctype})
        return self._emit(t, f"{t.name} = stablehlo.compare  {direction}, {a.name}, {c.name},  {ctype} : "
                             f"({a.type}, {c.type}) -> {t.type}")

    def select(self, p, a, c):
        shape = np.broadcast_shapes(p.shape, a.shape if isinstance(a, T) else (), c.shape if isinstance(c, T) else ())
        dt = a.dtype if isinstance(a, T) else c.dtype
        p = self.broadcast_to(p, shape)
        a = self.broadcast_to(a if isinstance(a, T) else self.const(a, dt), shape)
        c = self.broadcast_to(c if isinstance(c, T) else self.const(c, dt), shape)
        t = T(self, self._fresh(), shape, a.dtype, op="select", inputs=(p, a, c))
        return self._emit(t, f"{t.name} = stablehlo.select {p.name}, {a.name}, {c.name} : {p.type}, {t.type}")

    def maximum(self, a, c):
        a, c = self._coerce(a, c)
        return self.binary("maximum", a, c)

    def minimum(self, a, c):
        a, c = self._coerce(a, c)
        return self.binary("minimum", a, c)

    def exp(self, x): return self.unary("exponential", x)
    def log(self, x): return self.unary("log", x)
    def tanh(self, x): return self.unary("tanh", x)
    def sqrt(self, x): return self.unary("sqrt", x)
    def rsqrt(self, x): return self.unary("rsqrt", x)

    def power(self, x, p):
        x, pc = self._coerce(x, p)
        return self.binary("power", x, pc)

    # ------------------------------------------------------------------ shape ops
    def broadcast_in_dim(self, x, shape, dims):
        shape = tuple(int(s) for s in shape)
        if x.shape == shape and list(dims) == list(range(len(shape))):
            return x
        t = T(self, self._fresh(), shape, x.dtype, op="broadcast_in_dim", inputs=(x,), attrs={"dims": tuple(dims)})
        return self._emit(t, f"{t.name} = stablehlo.broadcast_in_dim {x.name}, dims = {_dims(dims)} : ({x.type}) -> {t.type}")

    def broadcast_to(self, x, shape):
        shape = tuple(shape)
        if x.shape == shape:
            return x
        nd = len(shape)
        # numpy rule: align trailing dims; size-1 dims are squeezed via reshape first (jax style)
        lead = nd - x.ndim
        keep = [i for i, s in enumerate(x.shape) if s == shape[lead + i]]
        if len(keep) != x.ndim:
            x = self.reshape(x, [x.shape[i] for i in keep])
        return self.broadcast_in_dim(x, shape, [lead + i for i in keep])

    def reshape(self, x, shape):
        shape = tuple(int(s) for s in shape)
        if x.shape == shape:
            return x
        assert int(np.prod(shape)) == int(np.prod(x.shape)), (x.shape, shape)
        t = T(self, self._fresh(), shape, x.dtype, op="reshape", inputs=(x,))
        return self._emit(t, f"{t.name} = stablehlo.reshape {x.name} : ({x.type}) -> {t.type}")

    def transpose(self, x, perm):
        perm = tuple(perm)
        if perm == tuple(range(x.ndim)):
            return x
        shape = tuple(x.shape[p] for p in perm)
        t = T(self, self._fresh(), shape, x.dtype, op="transpose", inputs=(x,), attrs={"perm": perm})
        return self._emit(t, f"{t.name} = stablehlo.transpose {x.name}, dims = {_dims(perm)} : ({x.type}) -> {t.type}")

    def slice(self, x, start, limit, strides=None):
        strides = strides or [1] * x.ndim
        shape = tuple((l - s + st - 1) // st for s, l, st in zip(start, limit, strides))
        t = T(self, self._fresh(), shape, x.dtype, op="slice", inputs=(x,),
              attrs={"start": tuple(start), "limit": tuple(limit), "strides": tuple(strides)})
        sl = ", ".join(f"{s}:{l}" + (f":{st}" if st != 1 else "") for s, l, st in zip(start, limit, strides))
        return self._emit(t, f"{t.name} = stablehlo.slice {x.name} [{sl}] : ({x.type}) -> {t.type}")

    def pad(self, x, value, low, high, interior=None):
        interior = interior or [0] * x.ndim
        shape = tuple(x.shape[i] + low[i] + high[i] + max(x.shape[i] - 1, 0) * interior[i] for i in range(x.ndim))
        v = value if isinstance(value, T) else self.const(value, x.dtype)
        t = T(self, self._fresh(), shape, x.dtype, op="pad", inputs=(x, v),
              attrs={"low": tuple(low), "high": tuple(high), "interior": tuple(interior)})
        return self._emit(t, f"{t.name} = stablehlo.pad {x.name}, {v.name}, low = {_dims(low)}, high = {_dims(high)}, "
                             f"interior = {_dims(interior)} : ({x.type}, {v.type}) -> {t.type}")

    def stop_gradient(self, x):
        """Same value, no gradient (jax.lax.stop_gradient lowers to nothing in StableHLO)."""
        return T(self, x.name, x.shape, x.dtype, op="stop_gradient", inputs=(x,))

    def concatenate(self, xs, dim):
        shape = list(xs[0].shape)
        shape[dim] = sum(x.shape[dim] for x in xs)
        t = T(self, self._fresh(), shape, xs[0].dtype, op="concatenate", inputs=tuple(xs), attrs={"dim": dim})
        return self._emit(t, f"{t.name} = stablehlo.concatenate {', '.join(x.name for x in xs)}, dim = {dim} : "
                             f"({', '.join(x.type for x in xs)}) -> {t.type}")

    # ------------------------------------------------------------------ reductions
    def reduce(self, x, dims, kind="add", init=None):
        dims = sorted(d % x.ndim for d in dims)
        body = {"add": "add", "max": "maximum", "min": "minimum", "mul": "multiply", "and": "and", "or": "or"}[kind]
        if init is None:
            init = {"add": 0, "mul": 1, "max": -np.inf, "min": np.inf, "and": 1, "or": 0}[kind]
            if x.dtype not in FLOATS and kind in ("max", "min"):
                info = np.iinfo(np.int32)
                init = info.min if kind == "max" else info.max
        c = self.const(init, x.dtype)
        shape = tuple(s for i, s in enumerate(x.shape) if i not in dims)
        t = T(self, self._fresh(), shape, x.dtype, op="reduce", inputs=(x, c), attrs={"dims": tuple(dims), "kind": kind})
        return self._emit(t, f"{t.name} = stablehlo.reduce({x.name} init: {c.name}) applies stablehlo.{body} across "
                             f"dimensions = {_dims(dims)} : ({x.type}, {c.type}) -> {t.type}")

    def argreduce(self, x, axis, kind="max", index_dtype="i32"):
        """(max|min over `axis`, its index) as jnp.argmax / argmin lower it: a two-operand reduce of
        (x, iota) whose reducer keeps the larger (smaller) value, a NaN first, and on ties the smaller
        index.  Returns the (value, index) pair."""
        axis %= x.ndim
        idx = self.iota(x.shape, axis, index_dtype)
        fl = x.dtype in FLOATS
        if fl:
            vinit = -np.inf if kind == "max" else np.inf
        else:
            info = np.iinfo(np.dtype({"i8": "int8", "i16": "int16", "i32": "int32", "i64": "int64"}[x.dtype]))
            vinit = info.min if kind == "max" else info.max
        cv, ci = self.const(vinit, x.dtype), self.const(0, index_dtype)
        name = self._fresh()
        shape = tuple(s for i, s in enumerate(x.shape) if i != axis)
        tv = T(self, name + "#0", shape, x.dtype, op="argreduce", inputs=(x, idx, cv, ci), attrs={"axis": axis})
        ti = T(self, name + "#1", shape, index_dtype, op="argreduce", inputs=(x, idx, cv, ci), attrs={"axis": axis})
        st, it = mlir_type((), x.dtype), mlir_type((), index_dtype)
        ctype = "FLOAT" if fl else "SIGNED"
        d = "GT" if kind == "max" else "LT"
        nan = f"      %n = stablehlo.compare  NE, %a0, %a0,  {ctype} : ({st}, {st}) -> tensor<i1>\n" if fl else ""
        pick = "stablehlo.or %g, %n" if fl else None
        body = (f"{name}:2 = stablehlo.reduce({x.name} init: {cv.name}), ({idx.name} init: {ci.name}) across dimensions = "
                f"[{axis}] : ({x.type}, {idx.type}, {st}, {it}) -> ({tv.type}, {ti.type})\n"
                f"     reducer(%a0: {st}, %b0: {st}) (%a1: {it}, %b1: {it})  {{\n"
                f"      %g = stablehlo.compare  {d}, %a0, %b0,  {ctype} : ({st}, {st}) -> tensor<i1>\n" + nan +
                (f"      %p = {pick} : tensor<i1>\n" if fl else "      %p = stablehlo.or %g, %g : tensor<i1>\n") +
                f"      %e = stablehlo.compare  EQ, %a0, %b0,  {ctype} : ({st}, {st}) -> tensor<i1>\n"
                f"      %l = stablehlo.compare  LT, %a1, %b1,  SIGNED : ({it}, {it}) -> tensor<i1>\n"
                f"      %q = stablehlo.and %e, %l : tensor<i1>\n"
                f"      %r = stablehlo.or %p, %q : tensor<i1>\n"
                f"      %v = stablehlo.select %p, %a0, %b0 : tensor<i1>, {st}\n"
                f"      %w = stablehlo.select %r, %a1, %b1 : tensor<i1>, {it}\n"
                f"      stablehlo.return %v, %w : {st}, {it}\n"
                f"    }}")
        self._emit(tv, body)
        self.ops.append(ti)                     # second result of the same op (no line of its own)
        return tv, ti

    def sum(self, x, axis, keepdims=False):
        return self._keep(self.reduce(x, _axes(axis, x.ndim), "add"), x, axis, keepdims)

    def max(self, x, axis, keepdims=False):
        return self._keep(self.reduce(x, _axes(axis, x.ndim), "max"), x, axis, keepdims)

    def mean(self, x, axis, keepdims=False):
        axes = _axes(axis, x.ndim)
        n = int(np.prod([x.shape[a] for a in axes]))
        s = self.sum(x, axes, keepdims)
        return s / self.const(float(n), x.dtype, s.shape)

    def _keep(self, r, x, axis, keepdims):
        if not keepdims:
            return r
        axes = _axes(axis, x.ndim)
        return self.reshape(r, [1 if i in axes else s for i, s in enumerate(x.shape)])

    # ------------------------------------------------------------------ contractions
    def dot_general(self, a, c, batch=((), ()), contract=((), ()), out_dtype=None):
        lb, rb = list(batch[0]), list(batch[1])
        lc, rc = list(contract[0]), list(contract[1])
        lf = [i for i in range(a.ndim) if i not in lb + lc]
        rf = [i for i in range(c.ndim) if i not in rb + rc]
        shape = [a.shape[i] for i in lb] + [a.shape[i] for i in lf] + [c.shape[i] for i in rf]
        dt = out_dtype or a.dtype
        t = T(self, self._fresh(), shape, dt, op="dot_general", inputs=(a, c),
              attrs={"lb": tuple(lb), "rb": tuple(rb), "lc": tuple(lc), "rc": tuple(rc)})
        parts = []
        if lb:
            parts.append(f"batching_dims = {_dims(lb)} x {_dims(rb)}")
        parts.append(f"contracting_dims = {_dims(lc)} x {_dims(rc)}")
        parts.append("precision = [DEFAULT, DEFAULT]")
        return self._emit(t, f"{t.name} = stablehlo.dot_general {a.name}, {c.name}, {', '.join(parts)} : "
                             f"({a.type}, {c.type}) -> {t.type}")

    def matmul(self, a, c, out_dtype=None):
        """a[..., M, K] @ c[K, N] (weights) or batched a[..., M, K] @ c[..., K, N] with equal batch dims."""
        if c.ndim == 2:
            return self.dot_general(a, c, contract=([a.ndim - 1], [0]), out_dtype=out_dtype)
        nb = a.ndim - 2
        assert c.ndim == a.ndim
        return self.dot_general(a, c, batch=(list(range(nb)), list(range(nb))),
                                contract=([a.ndim - 1], [nb]), out_dtype=out_dtype)

    # ------------------------------------------------------------------ gather / scatter (embedding take)
    def take(self, table, ids):
        """table[V, D] gathered by integer ids[...] -> [..., D] (jnp.take(table, ids, axis=0))."""
        idx = self.reshape(ids, tuple(ids.shape) + (1,))
        shape = tuple(ids.shape) + (table.shape[1],)
        t = T(self, self._fresh(), shape, table.dtype, op="gather", inputs=(table, idx),
              attrs={"offset_dims": (ids.ndim,), "collapsed": (0,), "start_index_map": (0,),
                     "index_vector_dim": ids.ndim, "slice_sizes": (1, table.shape[1])})
        return self._emit(t, f'{t.name} = "stablehlo.gather"({table.name}, {idx.name}) <{{dimension_numbers = '
                             f'#stablehlo.gather<offset_dims = [{ids.ndim}], collapsed_slice_dims = [0], '
                             f'start_index_map = [0], index_vector_dim = {ids.ndim}>, indices_are_sorted = false, '
                             f'slice_sizes = array<i64: 1, {table.shape[1]}>}}> : ({table.type}, {idx.type}) -> {t.type}')

    def scatter_add(self, base, ids, upd):
        """base[V, D] += upd[..., D] at rows ids[...] (the VJP of take)."""
        idx = self.reshape(ids, tuple(ids.shape) + (1,))
        t = T(self, self._fresh(), base.shape, base.dtype, op="scatter", inputs=(base, idx, upd),
              attrs={"update_window_dims": (ids.ndim,), "inserted_window_dims": (0,),
                     "scatter_dims_to_operand_dims": (0,), "index_vector_dim": ids.ndim})
        sc = mlir_type((), base.dtype)
        line = (f'{t.name} = "stablehlo.scatter"({base.name}, {idx.name}, {upd.name}) <{{indices_are_sorted = false, '
                f'scatter_dimension_numbers = #stablehlo.scatter<update_window_dims = [{ids.ndim}], '
                f'inserted_window_dims = [0], scatter_dims_to_operand_dims = [0], index_vector_dim = {ids.ndim}>, '
                f'unique_indices = false}}> ({{\n  ^bb0(%a0: {sc}, %a1: {sc}):\n'
                f'    %s0 = stablehlo.add %a0, %a1 : {sc}\n    stablehlo.return %s0 : {sc}\n  }}) : '
                f'({base.type}, {idx.type}, {upd.type}) -> {t.type}')
        return self._emit(t, line)

    # ------------------------------------------------------------------ collectives (inside shard_map)
    def all_reduce(self, x, n, kind="add"):
        body = {"add": "add", "max": "maximum", "min": "minimum"}[kind]
        groups = "[[" + ", ".join(str(i) for i in range(n)) + "]]"
        sc = mlir_type((), x.dtype)
        t = T(self, self._fresh(), x.shape, x.dtype, op="all_reduce", inputs=(x,), attrs={"kind": kind})
        line = (f'{t.name} = "stablehlo.all_reduce"({x.name}) <{{channel_handle = #stablehlo.channel_handle<handle = 1, '
                f'type = 1>, replica_groups = dense<{groups}> : tensor<1x{n}xi64>, use_global_device_ids}}> ({{\n'
                f'  ^bb0(%r0: {sc}, %r1: {sc}):\n    %s0 = stablehlo.{body} %r0, %r1 : {sc}\n'
                f'    stablehlo.return %s0 : {sc}\n  }}) : ({x.type}) -> {t.type}')
        return self._emit(t, line)

    def all_gather(self, x, n, dim=0):
        shape = list(x.shape)
        shape[dim] *= n
        groups = "[[" + ", ".join(str(i) for i in range(n)) + "]]"
        t = T(self, self._fresh(), shape, x.dtype, op="all_gather", inputs=(x,), attrs={"dim": dim})
        line = (f'{t.name} = "stablehlo.all_gather"({x.name}) <{{all_gather_dim = {dim} : i64, channel_handle = '
                f'#stablehlo.channel_handle<handle = 2, type = 1>, replica_groups = dense<{groups}> : '
                f'tensor<1x{n}xi64>, use_global_device_ids}}> : ({x.type}) -> {t.type}')
        return self._emit(t, line)

    def reduce_scatter(self, x, n, dim=0):
        shape = list(x.shape)
        shape[dim] //= n
        groups = "[[" + ", ".join(str(i) for i in range(n)) + "]]"
        sc = mlir_type((), x.dtype)
        t = T(self, self._fresh(), shape, x.dtype, op="reduce_scatter", inputs=(x,), attrs={"dim": dim})
        line = (f'{t.name} = "stablehlo.reduce_scatter"({x.name}) <{{channel_handle = #stablehlo.channel_handle<handle = 3, '
                f'type = 1>, replica_groups = dense<{groups}> : tensor<1x{n}xi64>, scatter_dimension = {dim} : i64, '
                f'use_global_device_ids}}> ({{\n  ^bb0(%r0: {sc}, %r1: {sc}):\n    %s0 = stablehlo.add %r0, %r1 : {sc}\n'
                f'    stablehlo.return %s0 : {sc}\n  }}) : ({x.type}) -> {t.type}')
        return self._emit(t, line)

    def shard(self, x, shard_shape):
        """shard_map entry: @Sharding + SPMDFullToShardShape, as jax emits at a shard_map boundary."""
        s = T(self, self._fresh(), x.shape, x.dtype, op="custom_call", inputs=(x,), attrs={"target": "Sharding"})
        self._emit(s, f'{s.name} = stablehlo.custom_call @Sharding({x.name}) {{mhlo.sharding = "{{devices=[{self.num_partitions},1]<=[{self.num_partitions}]}}"}} : ({x.type}) -> {s.type}')
        t = T(self, self._fresh(), shard_shape, x.dtype, op="custom_call", inputs=(s,), attrs={"target": "SPMDFullToShardShape"})
        return self._emit(t, f'{t.name} = stablehlo.custom_call @SPMDFullToShardShape({s.name}) {{mhlo.sharding = "{{manual}}"}} : ({s.type}) -> {t.type}')

    def unshard(self, x, full_shape):
        s = T(self, self._fresh(), x.shape, x.dtype, op="custom_call", inputs=(x,), attrs={"target": "Sharding"})
        self._emit(s, f'{s.name} = stablehlo.custom_call @Sharding({x.name}) {{mhlo.sharding = "{{manual}}"}} : ({x.type}) -> {s.type}')
        t = T(self, self._fresh(), full_shape, x.dtype, op="custom_call", inputs=(s,), attrs={"target": "SPMDShardToFullShape"})
        return self._emit(t, f'{t.name} = stablehlo.custom_call @SPMDShardToFullShape({s.name}) {{mhlo.sharding = "{{replicated}}"}} : ({s.type}) -> {t.type}')

    # ------------------------------------------------------------------ helpers
    def _coerce(self, a, c):
        if not isinstance(a, T):
            a = self.const(a, c.dtype)
        if not isinstance(c, T):
            c = self.const(c, a.dtype)
        shape = np.broadcast_shapes(a.shape, c.shape)
        return self.broadcast_to(a, shape), self.broadcast_to(c, shape)

    def text(self, outputs: Sequence[T], aliases=None, donors=()) -> str:
        """The module text.  `aliases` {argument index: result index} marks donated arguments whose
        buffer may become that result (`tf.aliasing_output`, what jax.jit(donate_argnums=...) emits
        when a result matches the argument's type); `donors` marks donated arguments without one
        (`jax.buffer_donor`)."""
        aliases = dict(aliases or {})
        outs = list(outputs)
        live = set()
        stack = list(outs)
        while stack:
            t = stack.pop()
            if id(t) in live:
                continue
            live.add(id(t))
            stack.extend(t.inputs)
        def arg_attr(k):
            if k in aliases:
                return f" {{tf.aliasing_output = {aliases[k]} : i32}}"
            return " {jax.buffer_donor = true}" if k in donors else ""
        sig = ", ".join(f"{a.name}: {a.type}{arg_attr(k)}" for k, a in enumerate(self.args))
        res = ", ".join(f"{o.type}" for o in outs)
        attrs = f"mhlo.num_partitions = {self.num_partitions} : i32, mhlo.num_replicas = {self.num_replicas} : i32"
        body = [f"    {self.lines[id(t)]}".replace("\n", "\n    ") for t in self.ops if id(t) in live and id(t) in self.lines]
        ret = f"    return {', '.join(o.name for o in outs)} : {', '.join(o.type for o in outs)}"
        return (f"module @{self.name} attributes {{{attrs}}} {{\n"
                f"  func.func public @main({sig}) -> ({res}) {{\n" + "\n".join(body) + "\n" + ret + "\n  }\n}\n")


def _axes(axis, nd):
    if isinstance(axis, int):
        return [axis % nd]
    return sorted(a % nd for a in axis)


# ---------------------------------------------------------------------- reverse-mode autodiff
def grad(b: Builder, loss: T, wrt: Sequence[T]) -> List[T]:
    """d loss / d wrt for a scalar f32 loss, by walking the recorded ops in reverse."""
    order = [t for t in b.ops]
    pos = {id(t): i for i, t in enumerate(order)}
    need = set()
    stack = [loss]
    while stack:
        t = stack.pop()
        if id(t) in need:
            continue
        need.add(id(t))
        stack.extend(t.inputs)
    cot: Dict[int, T] = {id(loss): b.const(1.0, loss.dtype, loss.shape)}

    def acc(x, g):
        if x.dtype not in FLOATS or x.op in ("constant", "iota"):
            return
        if id(x) in cot:
            cot[id(x)] = cot[id(x)] + g
        else:
            cot[id(x)] = g

    for t in sorted((t for t in order if id(t) in need), key=lambda t: -pos[id(t)]):
        g = cot.get(id(t))
        if g is None:
            continue
        _vjp(b, t, g, acc)
    out = []
    for w in wrt:
        out.append(cot.get(id(w), None) or b.const(0.0, w.dtype, w.shape))
    return out


def _unbroadcast_bid(b, g, x, dims):
    """VJP of broadcast_in_dim: sum over the broadcast dims, then reshape to x."""
    red = [i for i in range(g.ndim) if i not in dims]
    size1 = [d for j, d in enumerate(dims) if x.shape[j] == 1 and g.shape[d] != 1]
    r = b.reduce(g, sorted(set(red + size1)), "add") if (red or size1) else g
    return b.reshape(r, x.shape)


def _vjp(b: Builder, t: T, g: T, acc):
    op, ins = t.op, t.inputs
    if op in ("arg", "constant", "iota", "compare", "stop_gradient"):
        return
    if op == "slice":
        x = ins[0]
        st, li, sd = t.attrs["start"], t.attrs["limit"], t.attrs["strides"]
        low = list(st)
        interior = [s - 1 for s in sd]
        high = [x.shape[i] - (st[i] + (t.shape[i] - 1) * sd[i] + 1) if t.shape[i] else x.shape[i] - st[i]
                for i in range(x.ndim)]
        acc(x, b.pad(g, 0.0, low, high, interior))
        return
    if op == "add":
        acc(ins[0], g); acc(ins[1], g)
    elif op == "subtract":
        acc(ins[0], g); acc(ins[1], -g)
    elif op == "multiply":
        acc(ins[0], g * ins[1]); acc(ins[1], g * ins[0])
    elif op == "divide":
        acc(ins[0], g / ins[1])
        acc(ins[1], -(g * t) / ins[1])
    elif op == "negate":
        acc(ins[0], -g)
    elif op == "exponential":
        acc(ins[0], g * t)
    elif op == "log":
        acc(ins[0], g / ins[0])
    elif op == "tanh":
        acc(ins[0], g * (1.0 - t * t))
    elif op == "sqrt":
        acc(ins[0], g / (2.0 * t))
    elif op == "rsqrt":
        acc(ins[0], g * (-0.5) * t / ins[0])
    elif op == "maximum":
        m = b.compare(ins[0], ins[1], "GT")
        z = b.const(0.0, g.dtype, g.shape)
        acc(ins[0], b.select(m, g, z)); acc(ins[1], b.select(m, z, g))
    elif op == "minimum":
        m = b.compare(ins[0], ins[1], "LT")
        z = b.const(0.0, g.dtype, g.shape)
        acc(ins[0], b.select(m, g, z)); acc(ins[1], b.select(m, z, g))
    elif op == "power":
        x, p = ins
        acc(x, g * p * b.power(x, p - 1.0))
    elif op == "select":
        z = b.const(0.0, g.dtype, g.shape)
        acc(ins[1], b.select(ins[0], g, z)); acc(ins[2], b.select(ins[0], z, g))
    elif op == "convert":
        if ins[0].dtype in FLOATS:
            acc(ins[0], b.convert(g, ins[0].dtype))
    elif op == "reshape":
        acc(ins[0], b.reshape(g, ins[0].shape))
    elif op == "transpose":
        perm = t.attrs["perm"]
        inv = [0] * len(perm)
        for i, p in enumerate(perm):
            inv[p] = i
        acc(ins[0], b.transpose(g, inv))
    elif op == "broadcast_in_dim":
        acc(ins[0], _unbroadcast_bid(b, g, ins[0], t.attrs["dims"]))
    elif op == "reduce":
        x = ins[0]
        dims = t.attrs["dims"]
        kept = [i for i in range(x.ndim) if i not in dims]
        if t.attrs["kind"] == "add":
            acc(x, b.broadcast_in_dim(g, x.shape, kept))
        elif t.attrs["kind"] == "max":
            # gradient flows to the arg-max positions (ties share it, as jax does for reduce_max)
            tb = b.broadcast_in_dim(t, x.shape, kept)
            m = b.convert(b.compare(x, tb, "EQ"), g.dtype)
            cnt = b.broadcast_in_dim(b.reduce(m, dims, "add"), x.shape, kept)
            acc(x, b.broadcast_in_dim(g, x.shape, kept) * m / cnt)
        else:
            raise NotImplementedError(f"grad of reduce {t.attrs['kind']}")
    elif op == "dot_general":
        a, c = ins
        lb, rb, lc, rc = (list(t.attrs[k]) for k in ("lb", "rb", "lc", "rc"))
        lf = [i for i in range(a.ndim) if i not in lb + lc]
        rf = [i for i in range(c.ndim) if i not in rb + rc]
        nb = len(lb)
        # g dims: [batch (nb), lhs free, rhs free]
        g_lf = list(range(nb, nb + len(lf)))
        g_rf = list(range(nb + len(lf), nb + len(lf) + len(rf)))
        gb = list(range(nb))
        # d a = g . c contracted over rhs free: result dims [batch, lhs_free(g), rhs contract(c)]
        da = b.dot_general(g, c, batch=(gb, rb), contract=(g_rf, rf), out_dtype=a.dtype)
        # da dims order: batch, g_lf (== lf), c's remaining (contract dims in rc order of c indices sorted)
        c_rest = [i for i in range(c.ndim) if i not in rb + rf]  # = rc sorted
        src = lb + lf + [lc[rc.index(i)] for i in c_rest]
        perm = [src.index(i) for i in range(a.ndim)]
        acc(a, b.transpose(da, perm))
        db = b.dot_general(a, g, batch=(lb, gb), contract=(lf, g_lf), out_dtype=c.dtype)
        a_rest = [i for i in range(a.ndim) if i not in lb + lf]  # = lc sorted
        src = rb + [rc[lc.index(i)] for i in a_rest] + rf
        perm = [src.index(i) for i in range(c.ndim)]
        acc(c, b.transpose(db, perm))
    elif op == "gather":
        table, idx = ins
        base = b.const(0.0, table.dtype, table.shape)
        ids = b.reshape(idx, idx.shape[:-1])
        acc(table, b.scatter_add(base, ids, g))
    elif op == "custom_call":
        tgt = t.attrs["target"]
        if tgt == "SPMDFullToShardShape":
            raise NotImplementedError("grad through shard_map entry")
        acc(ins[0], g)
    elif op == "all_reduce":
        acc(ins[0], g)
    else:
        raise NotImplementedError(f"no VJP rule for {op}")
