"""ORACLE (test infrastructure only): a numpy interpreter for StableHLO text — the parity checker.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import this module; the
plugin never routes through it.  The north star names jaxlib's CPU PJRT backend as the oracle; jax is
not installed on this image, so this interpreter restates StableHLO op semantics over the same module
text the plugin compiles.  It follows the reference's lowering choices where they define behaviour:

  * dot_general canonicalisation to [batch, free, contract] (src/jam/ops/linalg.mm:68-104),
    accumulated here in float64 and rounded once to the result type;
  * reduce with the init value applied (the reference ignores it, docs/ops.md:53; src/jam/ops/reduce.mm:45-109),
    accumulated in float64 for floats;
  * compare including the unsigned flip (src/jam/ops/binary.mm:84-111), convert incl. unsigned->float and
    float->int truncation (src/jam/ops/shape.mm:270-293), broadcast_in_dim (shape.mm:163-172),
    bf16 constants rounded to nearest even (src/jam/ops/structural.mm:33-38);
  * gather/scatter with start indices clamped into range (src/jam/ops/gather_scatter.mm:116-121,180-183);
  * collectives: all_reduce = elementwise reduction over ranks, all_gather / reduce_scatter along dim 0
    (src/jam/lower.mm:382-410); with one rank they are the identity (lower.mm:346-352);
  * SPMDFullToShardShape / SPMDShardToFullShape pass the per-device shard through (lower.mm:270-299).

`run(text, inputs)` runs one device; `run_spmd(text, per_rank_inputs)` runs all ranks in lock step so
collectives see every rank's operand.
"""
from __future__ import annotations

import math
import re
import struct
from typing import Callable, Dict, List, Optional

import ml_dtypes
import numpy as np

from .shlo_parse import Block, Module, Op, TType, parse_module

NP = {"i1": np.bool_, "i8": np.int8, "i16": np.int16, "i32": np.int32, "i64": np.int64,
      "ui8": np.uint8, "ui16": np.uint16, "ui32": np.uint32, "ui64": np.uint64,
      "f16": np.float16, "bf16": ml_dtypes.bfloat16, "f32": np.float32, "f64": np.float64}
FLOAT = ("f16", "bf16", "f32", "f64")


def npdt(t: str):
    return np.dtype(NP[t])


def _hi(x: np.ndarray):
    """Working precision for float math: float64."""
    return x.astype(np.float64) if x.dtype.kind == "f" or x.dtype == ml_dtypes.bfloat16 else x


def parse_dense(tok: str, ty: TType) -> np.ndarray:
    body = tok[len("dense<"):-1].strip()
    dt = npdt(ty.dtype)
    shape = ty.dims
    if body.startswith('"0x'):
        raw = bytes.fromhex(body[3:-1])
        arr = np.frombuffer(raw, dtype=dt)
        if arr.size == 1:
            return np.full(shape, arr[0], dtype=dt)
        return arr.reshape(shape).copy()
    if body.startswith("0x"):
        bits = int(body, 16)
        width = dt.itemsize
        raw = bits.to_bytes(width, "little")
        return np.full(shape, np.frombuffer(raw, dtype=dt)[0], dtype=dt)

    def conv(s):
        s = s.strip()
        if s in ("true", "false"):
            return s == "true"
        if s.startswith("0x"):
            raw = int(s, 16).to_bytes(dt.itemsize, "little")
            return np.frombuffer(raw, dtype=dt)[0]
        if ty.dtype in FLOAT:
            return float(s)
        return int(s)

    if body.startswith("["):
        txt = re.sub(r"(true|false|0x[0-9A-Fa-f]+|[-+]?\d+\.?\d*(?:[eE][-+]?\d+)?|inf|nan)", lambda m: repr(str(m.group())), body)
        nested = eval(txt, {"__builtins__": {}})  # list literal of quoted scalars

        def walk(v):
            return [walk(x) for x in v] if isinstance(v, list) else conv(v)
        vals = walk(nested)
        if ty.dtype in FLOAT:
            return np.array(np.array(vals, dtype=np.float64), dtype=dt).reshape(shape)
        return np.array(vals, dtype=dt).reshape(shape)
    v = conv(body)
    if ty.dtype in FLOAT:
        return np.full(shape, np.float64(v)).astype(dt)
    return np.full(shape, v, dtype=dt)


def _cast(x: np.ndarray, t: str) -> np.ndarray:
    dt = npdt(t)
    if x.dtype == dt:
        return x
    if t == "i1":
        return x != 0
    if dt.kind in "iu" and x.dtype.kind == "f" or (dt.kind in "iu" and x.dtype == ml_dtypes.bfloat16):
        xf = x.astype(np.float64)
        xf = np.where(np.isnan(xf), 0, np.trunc(xf))
        info = np.iinfo(dt)
        return np.clip(xf, info.min, info.max).astype(dt)
    if x.dtype == ml_dtypes.bfloat16 or dt == ml_dtypes.bfloat16:
        return x.astype(np.float64 if x.dtype.kind in "fb" or x.dtype == ml_dtypes.bfloat16 else x.dtype).astype(dt) \
            if x.dtype != np.bool_ else x.astype(np.float32).astype(dt)
    return x.astype(dt)


def _binary(name, a, b):
    if name == "stablehlo.add": return a + b
    if name == "stablehlo.subtract": return a - b
    if name == "stablehlo.multiply": return a * b
    if name == "stablehlo.divide":
        if a.dtype.kind in "iu":
            with np.errstate(divide="ignore"):
                q = np.where(b == 0, -1, np.trunc(a.astype(np.float64) / np.where(b == 0, 1, b)))
            return q.astype(a.dtype)
        return a / b
    if name == "stablehlo.remainder":
        return np.fmod(a, b)
    if name == "stablehlo.maximum": return np.maximum(a, b)
    if name == "stablehlo.minimum": return np.minimum(a, b)
    if name == "stablehlo.power": return np.power(a, b)
    if name == "stablehlo.atan2": return np.arctan2(a, b)
    if name == "stablehlo.and": return a & b
    if name == "stablehlo.or": return a | b
    if name == "stablehlo.xor": return a ^ b
    raise NotImplementedError(name)


UNARY = {
    "stablehlo.negate": lambda x: -x,
    "stablehlo.exponential": np.exp,
    "stablehlo.exponential_minus_one": np.expm1,
    "stablehlo.log": np.log,
    "stablehlo.log_plus_one": np.log1p,
    "stablehlo.tanh": np.tanh,
    "stablehlo.sqrt": np.sqrt,
    "stablehlo.rsqrt": lambda x: 1.0 / np.sqrt(x),
    "stablehlo.cbrt": np.cbrt,
    "stablehlo.abs": np.abs,
    "stablehlo.sine": np.sin,
    "stablehlo.cosine": np.cos,
    "stablehlo.tan": np.tan,
    "stablehlo.floor": np.floor,
    "stablehlo.ceil": np.ceil,
    "stablehlo.sign": np.sign,
    "stablehlo.round_nearest_even": np.rint,
    "stablehlo.round_nearest_afz": lambda x: np.sign(x) * np.floor(np.abs(x) + 0.5),
    "stablehlo.logistic": lambda x: 1.0 / (1.0 + np.exp(-x)),
}


def _uview(x: np.ndarray) -> np.ndarray:
    """The two's-complement bits of an integer array as uint64 (only the type's own width set)."""
    return x.view(np.dtype("u%d" % x.dtype.itemsize)).astype(np.uint64)


def _from_bits(u: np.ndarray, dt: np.dtype) -> np.ndarray:
    return u.astype(np.dtype("u%d" % dt.itemsize)).view(dt)


def _popcnt(x):
    """Set bits in each element's own width (StableHLO popcnt)."""
    b = np.unpackbits(np.ascontiguousarray(x).view(np.uint8).reshape(-1, x.dtype.itemsize), axis=1)
    return b.sum(axis=1).reshape(x.shape).astype(x.dtype)


def _clz(x):
    """Leading zero bits in each element's own width; clz(0) = width (StableHLO count_leading_zeros)."""
    v = _uview(x)
    bl = np.zeros(v.shape, np.int64)
    for sh in (32, 16, 8, 4, 2, 1):
        m = v >= (np.uint64(1) << np.uint64(sh))
        bl += m * sh
        v = np.where(m, v >> np.uint64(sh), v)
    bl += (v > 0)
    return (8 * x.dtype.itemsize - bl).astype(x.dtype)


def _shift(name, x, y):
    """StableHLO shifts: the amount is read as unsigned; an amount >= the width gives 0 (the sign
    fill for the arithmetic right shift)."""
    w = 8 * x.dtype.itemsize
    mask = np.uint64((1 << w) - 1) if w < 64 else np.uint64(0xFFFFFFFFFFFFFFFF)
    ux, amt = _uview(x), _uview(y)
    big = amt >= np.uint64(w)
    a = np.where(big, np.uint64(w - 1), amt)
    if name == "stablehlo.shift_left":
        r = np.where(big, np.uint64(0), (ux << a) & mask)
    elif name == "stablehlo.shift_right_logical":
        r = np.where(big, np.uint64(0), ux >> a)
    else:
        sx = x.view(np.dtype("i%d" % x.dtype.itemsize)).astype(np.int64)
        r = (sx >> a.astype(np.int64)).astype(np.uint64) & mask
    return _from_bits(r, x.dtype)


def _reduce_precision(x, fmt, out_dtype):
    """reduce_precision to `eXmY`: the 16-bit float formats (round to bf16 / f16 and back, as the
    reference lowers it, src/jam/ops/hard_limit.mm:38-52) and formats at least as wide as the
    operand's own."""
    m = re.fullmatch(r"e(\d+)m(\d+)", fmt)
    eb, mb = int(m.group(1)), int(m.group(2))
    own = {"f64": (11, 52), "f32": (8, 23), "bf16": (8, 7), "f16": (5, 10)}[out_dtype]
    if eb >= own[0] and mb >= own[1]:
        return x
    h = _hi(x).astype(np.float32)
    if (eb, mb) == (8, 7):
        h = h.astype(ml_dtypes.bfloat16).astype(np.float32)
    elif (eb, mb) == (5, 10):
        with np.errstate(over="ignore"):
            h = h.astype(np.float16).astype(np.float32)
    else:
        raise NotImplementedError(f"reduce_precision {fmt}")
    return _cast(h, out_dtype)


def _dyn_starts(starts, dims, window):
    return [int(min(max(int(np.asarray(s).reshape(())), 0), d - w)) for s, d, w in zip(starts, dims, window)]


def _reducer_kind(block: Block) -> str:
    for op in block.ops:
        for k in ("add", "maximum", "minimum", "multiply", "and", "or"):
            if op.name == f"stablehlo.{k}":
                return k
    raise NotImplementedError("reducer body: " + ", ".join(o.name for o in block.ops))


def _reduce_np(x, dims, kind, init):
    dims = tuple(dims)
    if not dims:
        return x
    if kind == "add":
        r = _hi(x).sum(axis=dims) + _hi(init)
    elif kind == "multiply":
        r = _hi(x).prod(axis=dims) * _hi(init)
    elif kind == "maximum":
        r = np.maximum(_hi(x).max(axis=dims, initial=-np.inf if x.dtype.kind in "fV" or x.dtype == ml_dtypes.bfloat16 else np.iinfo(x.dtype).min), _hi(init))
    elif kind == "minimum":
        r = np.minimum(_hi(x).min(axis=dims, initial=np.inf if x.dtype.kind in "fV" or x.dtype == ml_dtypes.bfloat16 else np.iinfo(x.dtype).max), _hi(init))
    elif kind == "and":
        r = np.logical_and(x.all(axis=dims), init) if x.dtype == np.bool_ else np.bitwise_and.reduce(x, axis=dims) & init
    elif kind == "or":
        r = np.logical_or(x.any(axis=dims), init) if x.dtype == np.bool_ else np.bitwise_or.reduce(x, axis=dims) | init
    else:
        raise NotImplementedError(kind)
    return np.asarray(r)


def dot_general(a, b, lb, rb, lc, rc, out_t):
    lf = [i for i in range(a.ndim) if i not in lb + lc]
    rf = [i for i in range(b.ndim) if i not in rb + rc]
    A = np.transpose(_hi(a), lb + lf + lc)
    B = np.transpose(_hi(b), rb + rc + rf)
    nb = int(np.prod([a.shape[i] for i in lb])) if lb else 1
    M = int(np.prod([a.shape[i] for i in lf])) if lf else 1
    K = int(np.prod([a.shape[i] for i in lc])) if lc else 1
    N = int(np.prod([b.shape[i] for i in rf])) if rf else 1
    C = np.matmul(A.reshape(nb, M, K), B.reshape(nb, K, N))
    shape = [a.shape[i] for i in lb] + [a.shape[i] for i in lf] + [b.shape[i] for i in rf]
    return _cast(C.reshape(shape), out_t)


def _gather(operand, idx, attrs, out_t: TType):
    dn = _dimnums(attrs["dimension_numbers"])
    offset_dims = dn.get("offset_dims", [])
    collapsed = dn.get("collapsed_slice_dims", [])
    start_map = dn.get("start_index_map", [])
    ivd = dn.get("index_vector_dim", idx.ndim)
    slice_sizes = [int(s) for s in re.findall(r"-?\d+", str(attrs["slice_sizes"]).split(":", 1)[-1])]
    if ivd == idx.ndim:
        idx = idx[..., None]
    batch_shape = [s for i, s in enumerate(idx.shape) if i != ivd]
    idx_m = np.moveaxis(idx, ivd, -1).reshape(-1, idx.shape[ivd])
    out = np.zeros(out_t.dims, dtype=operand.dtype)
    batch_dims_out = [i for i in range(len(out_t.dims)) if i not in offset_dims]
    window_operand_dims = [i for i in range(operand.ndim) if i not in collapsed]
    for bi, start in enumerate(idx_m):
        full = [0] * operand.ndim
        for k, od in enumerate(start_map):
            full[od] = int(np.clip(int(start[k]), 0, operand.shape[od] - slice_sizes[od]))
        sl = tuple(slice(full[d], full[d] + slice_sizes[d]) for d in range(operand.ndim))
        win = operand[sl]
        win = win.reshape([slice_sizes[d] for d in window_operand_dims])
        bidx = np.unravel_index(bi, batch_shape) if batch_shape else ()
        o_index = [slice(None)] * len(out_t.dims)
        for k, d in enumerate(batch_dims_out):
            o_index[d] = bidx[k]
        out[tuple(o_index)] = win
    return out


def _scatter(operand, idx, upd, attrs, region: Block):
    dn = _dimnums(attrs["scatter_dimension_numbers"])
    uwd = dn.get("update_window_dims", [])
    inserted = dn.get("inserted_window_dims", [])
    sd2od = dn.get("scatter_dims_to_operand_dims", [])
    ivd = dn.get("index_vector_dim", idx.ndim)
    kind = _reducer_kind(region) if any(o.name != "stablehlo.return" for o in region.ops) else "replace"
    if ivd == idx.ndim:
        idx = idx[..., None]
    idx_m = np.moveaxis(idx, ivd, -1).reshape(-1, idx.shape[ivd])
    upd_scatter_dims = [i for i in range(upd.ndim) if i not in uwd]
    u = np.moveaxis(upd, upd_scatter_dims, list(range(len(upd_scatter_dims))))
    u = u.reshape((-1,) + tuple(upd.shape[d] for d in uwd))
    out = _hi(operand).copy() if kind == "add" else operand.copy()
    win_operand_dims = [i for i in range(operand.ndim) if i not in inserted]
    for bi, start in enumerate(idx_m):
        full = [0] * operand.ndim
        for k, od in enumerate(sd2od):
            full[od] = int(start[k])
        win_sizes = [1] * operand.ndim
        for k, od in enumerate(win_operand_dims):
            win_sizes[od] = u.shape[1 + k]
        if any(full[d] < 0 or full[d] + win_sizes[d] > operand.shape[d] for d in range(operand.ndim)):
            continue                                       # out-of-bounds updates are skipped
        sl = tuple(slice(full[d], full[d] + win_sizes[d]) for d in range(operand.ndim))
        w = u[bi].reshape([win_sizes[d] for d in range(operand.ndim)])
        if kind == "add":
            out[sl] += _hi(w)
        else:
            out[sl] = w
    return out.astype(operand.dtype)


def _dimnums(tok):
    body = str(tok)
    out = {}
    for key, val in re.findall(r"(\w+) = (\[[^\]]*\]|\d+)", body):
        out[key] = [int(x) for x in re.findall(r"-?\d+", val)] if val.startswith("[") else int(val)
    return out


class Interp:
    """Runs one function body; `collective(op_name, kind, array, attrs)` supplies cross-rank results."""

    def __init__(self, module: Module):
        self.m = module

    def call(self, fname: str, args: List[np.ndarray]):
        f = self.m.funcs[fname]
        return (yield from self.block(f.body, f.args, args))

    def block(self, blk: Block, params, args):
        env: Dict[str, np.ndarray] = {}
        for (name, _), a in zip(params, args):
            env[name] = a
        for op in blk.ops:
            if op.name in ("func.return", "stablehlo.return"):
                return [env[v] for v in op.operands]
            ins = [env[v] for v in op.operands]
            outs = yield from self.op(op, ins)
            for r, o in zip(op.results, outs):
                env[r] = o
        return []

    def op(self, op: Op, ins):
        n = op.name
        ot = op.out_types[0] if op.out_types else None
        a = op.attrs
        if n == "func.call":
            return (yield from self.call(a["callee"], ins))
        if n == "stablehlo.constant":
            return [parse_dense(a["value"], ot)]
        if n in ("stablehlo.add", "stablehlo.subtract", "stablehlo.multiply", "stablehlo.divide",
                 "stablehlo.maximum", "stablehlo.minimum", "stablehlo.power", "stablehlo.and",
                 "stablehlo.or", "stablehlo.xor", "stablehlo.remainder", "stablehlo.atan2"):
            x, y = ins
            if x.dtype.kind == "f" or x.dtype == ml_dtypes.bfloat16:
                with np.errstate(all="ignore"):
                    r = _binary(n, _hi(x), _hi(y))
                return [_cast(r, ot.dtype)]
            with np.errstate(all="ignore"):
                return [_binary(n, x, y).astype(npdt(ot.dtype))]
        if n in UNARY:
            with np.errstate(all="ignore"):
                r = UNARY[n](_hi(ins[0]))
            return [_cast(np.asarray(r), ot.dtype)]
        if n in ("stablehlo.shift_left", "stablehlo.shift_right_logical", "stablehlo.shift_right_arithmetic"):
            return [_shift(n, ins[0], ins[1])]
        if n == "stablehlo.popcnt":
            return [_popcnt(ins[0])]
        if n == "stablehlo.count_leading_zeros":
            return [_clz(ins[0])]
        if n in ("chlo.erf", "stablehlo.erf") or (n == "stablehlo.custom_call" and a.get("call_target_name") == "mhlo.erf"):
            r = np.vectorize(math.erf, otypes=[np.float64])(_hi(ins[0]).astype(np.float64))
            return [_cast(r, ot.dtype)]
        if n == "stablehlo.reduce_precision":
            return [_reduce_precision(ins[0], a["format"], ot.dtype)]
        if n == "stablehlo.broadcast":
            x = ins[0]
            return [np.broadcast_to(x, tuple(a["sizes"]) + x.shape).copy()]
        if n == "stablehlo.reverse":
            return [np.flip(ins[0], axis=tuple(a["dims"])).copy()]
        if n == "stablehlo.dynamic_slice":
            x = ins[0]
            st = _dyn_starts(ins[1:], x.shape, a["sizes"])
            return [x[tuple(slice(s0, s0 + w) for s0, w in zip(st, a["sizes"]))].copy()]
        if n == "stablehlo.dynamic_update_slice":
            x, u = ins[0], ins[1]
            st = _dyn_starts(ins[2:], x.shape, u.shape)
            r = x.copy()
            r[tuple(slice(s0, s0 + w) for s0, w in zip(st, u.shape))] = u
            return [r]
        if n == "stablehlo.not":
            x = ins[0]
            return [np.logical_not(x) if x.dtype == np.bool_ else np.invert(x)]
        if n == "stablehlo.is_finite":
            return [np.isfinite(_hi(ins[0]))]
        if n == "stablehlo.convert":
            return [_cast(ins[0], ot.dtype)]
        if n == "stablehlo.bitcast_convert":
            return [ins[0].view(npdt(ot.dtype)).reshape(ot.dims)]
        if n == "stablehlo.compare":
            x, y = ins
            d = a["comparison_direction"]
            ctype = a.get("compare_type", "")
            if ctype == "UNSIGNED" and x.dtype.kind == "i":
                ux = np.dtype("u%d" % x.dtype.itemsize)
                x, y = x.view(ux), y.view(ux)
            x, y = _hi(x), _hi(y)
            fn = {"EQ": np.equal, "NE": np.not_equal, "LT": np.less, "LE": np.less_equal,
                  "GT": np.greater, "GE": np.greater_equal}[d]
            return [fn(x, y)]
        if n == "stablehlo.select":
            p, x, y = ins
            return [np.where(p, x, y).astype(x.dtype)]
        if n == "stablehlo.clamp":
            lo, x, hi = ins
            return [np.minimum(np.maximum(x, lo), hi).astype(x.dtype)]
        if n == "stablehlo.iota":
            d = int(a["dim"])
            shape = ot.dims
            r = np.arange(shape[d]).reshape([-1 if i == d else 1 for i in range(len(shape))])
            return [np.broadcast_to(r, shape).astype(npdt(ot.dtype)).copy()]
        if n == "stablehlo.broadcast_in_dim":
            x = ins[0]
            dims = a["dims"]
            shape = ot.dims
            view = [1] * len(shape)
            for j, d in enumerate(dims):
                view[d] = x.shape[j]
            return [np.broadcast_to(x.reshape(view), shape).copy()]
        if n == "stablehlo.reshape":
            return [ins[0].reshape(ot.dims)]
        if n == "stablehlo.transpose":
            return [np.transpose(ins[0], a["dims"]).copy()]
        if n == "stablehlo.slice":
            sl = tuple(slice(s, l, st) for s, l, st in zip(a["start_indices"], a["limit_indices"], a["strides"]))
            return [ins[0][sl].copy()]
        if n == "stablehlo.concatenate":
            return [np.concatenate(ins, axis=int(a["dim"]))]
        if n == "stablehlo.pad":
            x, v = ins
            lo, hi, it = a["low"], a["high"], a["interior"]
            out = np.full(ot.dims, v, dtype=x.dtype)
            # interior padding then edge padding (negative edges crop)
            big = [x.shape[i] + (x.shape[i] - 1) * it[i] if x.shape[i] else 0 for i in range(x.ndim)]
            tmp = np.full(big, v, dtype=x.dtype)
            tmp[tuple(slice(None, None, it[i] + 1) for i in range(x.ndim))] = x
            src, dst = [], []
            for i in range(x.ndim):
                s0 = max(0, -lo[i]); d0 = max(0, lo[i])
                ln = min(big[i] - s0, ot.dims[i] - d0)
                src.append(slice(s0, s0 + ln)); dst.append(slice(d0, d0 + ln))
            out[tuple(dst)] = tmp[tuple(src)]
            return [out]
        if n == "stablehlo.dot_general":
            lb, rb = a.get("batching_dims", ([], []))
            lc, rc = a["contracting_dims"]
            return [dot_general(ins[0], ins[1], list(lb), list(rb), list(lc), list(rc), ot.dtype)]
        if n == "stablehlo.dot":
            x, y = ins
            return [dot_general(x, y, [], [], [x.ndim - 1], [0], ot.dtype)]
        if n == "stablehlo.reduce":
            k = len(op.out_types)
            xs, inits = ins[:k], ins[k:]
            dims = a["dimensions"]
            if k != 1:
                # general reducer body (argmax / argmin as jnp lowers them): fold it over the reduced
                # positions in index order, accumulator as the left operands, element as the right
                dims = sorted(dims)
                flat = [np.moveaxis(x, dims, list(range(len(dims)))) for x in xs]
                flat = [f.reshape((-1,) + f.shape[len(dims):]) for f in flat]
                acc = [np.broadcast_to(np.asarray(i), flat[0].shape[1:]).astype(i.dtype) for i in inits]
                blk = op.regions[0]
                for j in range(flat[0].shape[0]):
                    acc = yield from self.block(blk, blk.args, acc + [f[j] for f in flat])
                    acc = [np.asarray(v) for v in acc]
                return [_cast(np.asarray(v), t.dtype) for v, t in zip(acc, op.out_types)]
            kind = _reducer_kind(op.regions[0])
            return [_cast(_reduce_np(xs[0], dims, kind, inits[0]), ot.dtype)]
        if n == "stablehlo.gather":
            return [_gather(ins[0], ins[1], a, ot)]
        if n == "stablehlo.scatter":
            return [_scatter(ins[0], ins[1], ins[2], a, op.regions[0])]
        if n == "stablehlo.optimization_barrier":
            return list(ins)
        if n == "stablehlo.custom_call":
            tgt = a["call_target_name"]
            if tgt in ("Sharding", "SPMDFullToShardShape", "SPMDShardToFullShape"):
                return [ins[0]]
            raise NotImplementedError(f"custom_call @{tgt}")
        if n in ("stablehlo.all_reduce", "stablehlo.all_gather", "stablehlo.reduce_scatter", "stablehlo.collective_permute",
                 "stablehlo.collective_broadcast", "stablehlo.all_to_all"):
            kind = _reducer_kind(op.regions[0]) if op.regions else None
            res = yield (n, kind, ins[0], a)
            return [res]
        if n in ("stablehlo.partition_id", "stablehlo.replica_id"):
            res = yield (n, None, None, a)
            return [np.array(res, dtype=np.uint32)]
        raise NotImplementedError(f"oracle: unhandled op {n}")


def _drive(gens):
    """Run rank generators in lock step; at each yield all ranks must be at the same collective."""
    n = len(gens)
    results = [None] * n
    pending = [None] * n
    live = list(range(n))
    sends = [None] * n
    while True:
        msgs = []
        for r in range(n):
            try:
                msgs.append(gens[r].send(sends[r]))
            except StopIteration as e:
                results[r] = e.value
                msgs.append(None)
        if all(m is None for m in msgs):
            return results
        if any(m is None for m in msgs):
            raise RuntimeError("ranks diverged at a collective")
        name = msgs[0][0]
        if name in ("stablehlo.partition_id", "stablehlo.replica_id"):
            sends = list(range(n))
            continue
        kind = msgs[0][1]
        attrs = msgs[0][3]
        arrs = [m[2] for m in msgs]
        sends = [None] * n
        # every collective acts within each replica group on its own (StableHLO semantics; the
        # reference forwards whole-world groups only, src/jam/lower.mm:382-436)
        for grp in _replica_groups(attrs, n, name):
            sub = _collective(name, kind, attrs, [arrs[r] for r in grp])
            for r, out in zip(grp, sub):
                sends[r] = out
        if any(x is None for x in sends):
            raise RuntimeError(f"{name}: a rank belongs to no replica group")


def _replica_groups(attrs, n, name):
    """The replica groups of a collective as lists of ranks; an absent or empty attribute means one
    group of all n ranks.  collective_permute has source_target_pairs instead (one group)."""
    if name == "stablehlo.collective_permute":
        return [list(range(n))]
    txt = str(attrs.get("replica_groups", "")).split(":")[0]
    groups = [[int(v) for v in re.findall(r"-?\d+", g)] for g in re.findall(r"\[([^\[\]]*)\]", txt)]
    groups = [g for g in groups if g]
    if not groups:
        return [list(range(n))]
    seen = sorted(r for g in groups for r in g)
    if seen != list(range(n)):
        raise ValueError(f"{name}: replica_groups {groups} do not partition ranks 0..{n - 1}")
    return groups


def _collective(name, kind, attrs, arrs):
    """One collective over the operands of one group, in group order; returns each member's result."""
    n = len(arrs)
    if name == "stablehlo.all_reduce":
        acc = _hi(arrs[0]).copy()
        for x in arrs[1:]:
            acc = {"add": np.add, "maximum": np.maximum, "minimum": np.minimum,
                   "multiply": np.multiply}[kind](acc, _hi(x))
        out = acc.astype(arrs[0].dtype)
        return [out.copy() for _ in range(n)]
    if name == "stablehlo.all_gather":
        out = np.concatenate(arrs, axis=int(attrs.get("all_gather_dim", 0)))
        return [out.copy() for _ in range(n)]
    if name == "stablehlo.reduce_scatter":
        acc = _hi(arrs[0]).copy()
        for x in arrs[1:]:
            acc = acc + _hi(x)
        return np.split(acc.astype(arrs[0].dtype), n, axis=int(attrs.get("scatter_dimension", 0)))
    if name == "stablehlo.collective_permute":
        # each (source, target) pair moves source's operand to target; a target without a source
        # gets zeros
        nums = [int(v) for v in re.findall(r"-?\d+", str(attrs.get("source_target_pairs", "")).split(":")[0])]
        sends = [np.zeros_like(arrs[0]) for _ in range(n)]
        for k in range(0, len(nums) - 1, 2):
            sends[nums[k + 1]] = arrs[nums[k]].copy()
        return sends
    if name == "stablehlo.collective_broadcast":
        return [arrs[0].copy() for _ in range(n)]        # the group's first member is the source
    if name == "stablehlo.all_to_all":
        sd, cd = int(attrs.get("split_dimension", 0)), int(attrs.get("concat_dimension", 0))
        parts = [np.split(x, n, axis=sd) for x in arrs]
        return [np.concatenate([parts[src][dst] for src in range(n)], axis=cd) for dst in range(n)]
    raise NotImplementedError(name)


def run_spmd(text: str, per_rank_inputs: List[List[np.ndarray]]):
    m = parse_module(text)
    gens = [Interp(m).call("main", list(inp)) for inp in per_rank_inputs]
    # prime: generators start on first send(None)
    return _drive(gens)


def run(text: str, inputs: List[np.ndarray]):
    return run_spmd(text, [inputs])[0]
