"""ORACLE (test infrastructure only): a parser for StableHLO MLIR text, used by oracle/interp.py.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import this package; the
plugin has its own C++ parser (mccl-jax_b200/csrc/jam/parse.cc) and never calls into oracle/.

It reads the pretty and generic op forms that jax's `.as_text()` prints for the op subset of the
five configs, i.e. what the reference deserializes with MLIR at src/jam/parse.cc:53-63 before its
lowering walks `@main` (src/jam/lower.mm:208-314).  `func.call` is kept as an op; the interpreter
inlines it the way the reference's WalkBlock does (lower.mm:245-268).
"""
from __future__ import annotations

import re
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

_TOKEN = re.compile(r"""
    (?P<ws>\s+)
  | (?P<comment>//[^\n]*)
  | (?P<str>"(?:[^"\\]|\\.)*")
  | (?P<val>%[A-Za-z0-9_.$#]+)
  | (?P<sym>@[A-Za-z0-9_.$]+)
  | (?P<bb>\^[A-Za-z0-9_]+)
  | (?P<angled>(?:tensor|dense|array|\#[A-Za-z0-9_.]+|!stablehlo\.[a-z_]+)<)
  | (?P<arrow>->)
  | (?P<num>[-+]?(?:0x[0-9A-Fa-f]+|\d+\.?\d*(?:[eE][-+]?\d+)?|inf|nan))
  | (?P<ident>[A-Za-z_][A-Za-z0-9_.$]*)
  | (?P<punct>[()\[\]{},:=<>*])
""", re.X)


def tokenize(text: str) -> List[str]:
    toks, i, n = [], 0, len(text)
    while i < n:
        m = _TOKEN.match(text, i)
        if not m:
            raise SyntaxError(f"bad character {text[i]!r} at {i}: {text[i:i+40]!r}")
        kind = m.lastgroup
        if kind == "angled":
            # take the whole balanced <...> group as one token
            j, depth = m.end(), 1
            while depth and j < n:
                c = text[j]
                if c == "<":
                    depth += 1
                elif c == ">" and text[j - 1] != "-":
                    depth -= 1
                elif c == '"':
                    j = text.index('"', j + 1)
                j += 1
            toks.append(text[m.start():j])
            i = j
            continue
        if kind not in ("ws", "comment"):
            toks.append(m.group())
        i = m.end()
    return toks


@dataclass
class TType:
    dims: Tuple[int, ...]
    dtype: str                                   # i1 i8 i16 i32 i64 ui8.. f16 bf16 f32 f64


def parse_type(tok: str) -> TType:
    m = re.fullmatch(r"tensor<(.*)>", tok)
    if not m:
        raise SyntaxError(f"expected tensor type, got {tok}")
    body = m.group(1).split(",")[0].strip()
    parts = body.split("x")
    dims = tuple(int(p) for p in parts[:-1])
    return TType(dims, parts[-1])


@dataclass
class Op:
    name: str                                    # e.g. "stablehlo.add"
    results: List[str]
    operands: List[str]
    attrs: Dict[str, object] = field(default_factory=dict)
    in_types: List[TType] = field(default_factory=list)
    out_types: List[TType] = field(default_factory=list)
    regions: List["Block"] = field(default_factory=list)


@dataclass
class Block:
    args: List[Tuple[str, TType]]
    ops: List[Op]


@dataclass
class Func:
    name: str
    args: List[Tuple[str, TType]]
    results: List[TType]
    body: Block


@dataclass
class Module:
    name: str
    attrs: Dict[str, object]
    funcs: Dict[str, Func]


class Parser:
    def __init__(self, text: str):
        self.t = tokenize(text)
        self.i = 0

    # -- token helpers
    def peek(self, k=0):
        j = self.i + k
        return self.t[j] if j < len(self.t) else None

    def next(self):
        tok = self.t[self.i]
        self.i += 1
        return tok

    def expect(self, tok):
        got = self.next()
        if got != tok:
            raise SyntaxError(f"expected {tok!r}, got {got!r} near {' '.join(self.t[self.i-5:self.i+5])}")
        return got

    def accept(self, tok):
        if self.peek() == tok:
            self.i += 1
            return True
        return False

    def skip_balanced(self):
        """Skip one balanced (...)/[...]/{...} group or a single token; return the raw tokens."""
        open_ = self.peek()
        pairs = {"(": ")", "[": "]", "{": "}"}
        if open_ not in pairs:
            return [self.next()]
        out, depth = [], 0
        while True:
            tok = self.next()
            out.append(tok)
            if tok in pairs:
                depth += 1
            elif tok in pairs.values():
                depth -= 1
                if depth == 0:
                    return out

    # -- module structure
    def module(self) -> Module:
        name, attrs = "", {}
        if self.accept("module"):
            if self.peek().startswith("@"):
                name = self.next()[1:]
            if self.accept("attributes"):
                attrs = self.attr_dict()
            self.expect("{")
        funcs = {}
        while self.peek() not in (None, "}"):
            f = self.func()
            funcs[f.name] = f
        return Module(name, attrs, funcs)

    def attr_dict(self):
        d = {}
        self.expect("{")
        while not self.accept("}"):
            key = self.next()
            val = True
            if self.accept("="):
                val = self.attr_value()
            d[key] = val
            self.accept(",")
        return d

    def attr_value(self, typed=True):
        tok = self.peek()
        if tok == "[":
            return self.int_list()
        if tok in ("{", "("):
            return self.skip_balanced()
        val = self.next()
        if typed and self.peek() == ":" and self.peek(1) is not None and re.fullmatch(r"[iuf]\d+|index|tensor<.*>", self.peek(1) or ""):
            self.next(); self.next()            # typed literal `4 : i64`
        return val

    def int_list(self):
        self.expect("[")
        out = []
        while not self.accept("]"):
            tok = self.next()
            if tok == "[":                          # nested list
                self.i -= 1
                out.append(self.int_list())
            elif tok != ",":
                out.append(int(tok) if re.fullmatch(r"-?\d+", tok) else tok)
        return out

    def func(self) -> Func:
        self.expect("func.func")
        if self.peek() in ("public", "private"):
            self.next()
        name = self.next()[1:]
        self.expect("(")
        args = []
        while not self.accept(")"):
            a = self.next()
            self.expect(":")
            ty = parse_type(self.next())
            if self.peek() == "{":
                self.attr_dict()
            args.append((a, ty))
            self.accept(",")
        results = []
        if self.accept("->"):
            if self.accept("("):
                while not self.accept(")"):
                    results.append(parse_type(self.next()))
                    if self.peek() == "{":
                        self.attr_dict()
                    self.accept(",")
            else:
                results.append(parse_type(self.next()))
        if self.accept("attributes"):
            self.attr_dict()
        body = self.block_body([])
        return Func(name, args, results, body)

    def block_body(self, args) -> Block:
        self.expect("{")
        ops = []
        if self.peek() and self.peek().startswith("^"):
            self.next()
            args = self.block_args()
            self.expect(":")
        while not self.accept("}"):
            ops.append(self.op())
        return Block(args, ops)

    def block_args(self):
        args = []
        self.expect("(")
        while not self.accept(")"):
            a = self.next()
            self.expect(":")
            args.append((a, parse_type(self.next())))
            self.accept(",")
        return args

    # -- operations
    def op(self) -> Op:
        results = []
        if self.peek().startswith("%") and (self.peek(1) in ("=", ",") or
                                            (self.peek(1) == ":" and self.peek(3) == "=")):
            while True:
                r = self.next()
                if self.peek() == ":":
                    self.next()
                    results += [f"{r}#{k}" for k in range(int(self.next()))]
                else:
                    results.append(r)
                if not self.accept(","):
                    break
            self.expect("=")
        name = self.next()
        if name.startswith('"'):
            return self.generic_op(name.strip('"'), results)
        if name in ("return", "func.return", "stablehlo.return"):
            operands = []
            while self.peek() and self.peek().startswith("%"):
                operands.append(self.next())
                self.accept(",")
            types = []
            if self.accept(":"):
                types = self.type_list_plain(len(operands))
            return Op("func.return" if name != "stablehlo.return" else name, [], operands, {}, types, [])
        if name in ("call", "func.call"):
            callee = self.next()[1:]
            operands = self.paren_operands()
            self.expect(":")
            ins, outs = self.fn_type()
            return Op("func.call", results, operands, {"callee": callee}, ins, outs)
        if name == "stablehlo.reduce":
            return self.reduce_op(results)
        if name == "stablehlo.custom_call":
            target = self.next()[1:]
            operands = self.paren_operands()
            attrs = {"call_target_name": target}
            if self.peek() == "{":
                attrs.update(self.attr_dict())
            self.expect(":")
            ins, outs = self.fn_type()
            return Op(name, results, operands, attrs, ins, outs)
        return self.pretty_op(name, results)

    def paren_operands(self):
        ops = []
        self.expect("(")
        while not self.accept(")"):
            ops.append(self.next())
            self.accept(",")
        return ops

    def fn_type(self):
        """`(t, t) -> t` or `(t) -> (t, t)` or a single `t` (meaning all operands and result)."""
        if self.accept("("):
            ins = []
            while not self.accept(")"):
                ins.append(parse_type(self.next()))
                self.accept(",")
            self.expect("->")
            return ins, self.result_types()
        ty = parse_type(self.next())
        if self.accept("->"):                    # `: T -> U`, as chlo's unary ops print
            return [ty], [parse_type(self.next())]
        return None, [ty]

    def result_types(self):
        if self.accept("("):
            outs = []
            while not self.accept(")"):
                outs.append(parse_type(self.next()))
                self.accept(",")
            return outs
        return [parse_type(self.next())]

    def type_list_plain(self, n):
        out = [parse_type(self.next())]
        while len(out) < n and self.accept(","):
            out.append(parse_type(self.next()))
        return out

    def pretty_op(self, name, results) -> Op:
        operands, attrs, bare = [], {}, []
        while self.peek() != ":":
            tok = self.peek()
            if tok.startswith("%"):
                operands.append(self.next())
            elif tok == ",":
                self.next()
            elif tok == "[" and name == "stablehlo.slice":
                self.next()
                start, limit, strides = [], [], []
                while not self.accept("]"):
                    parts = [self.next()]
                    while self.peek() == ":":
                        self.next()
                        parts.append(self.next())
                    start.append(int(parts[0])); limit.append(int(parts[1]))
                    strides.append(int(parts[2]) if len(parts) > 2 else 1)
                    self.accept(",")
                attrs.update(start_indices=start, limit_indices=limit, strides=strides)
            elif tok == "{":
                attrs.update(self.attr_dict())
            elif self.peek(1) == "=":
                key = self.next()
                self.next()
                if self.peek() == "[":
                    lhs = self.int_list()
                    if self.peek() == "x":          # `[0] x [1]`
                        self.next()
                        attrs[key] = (lhs, self.int_list())
                    else:
                        attrs[key] = lhs
                else:
                    attrs[key] = self.attr_value(typed=False)
            elif tok.startswith("dense<"):
                attrs["value"] = self.next()
            else:
                bare.append(self.next())
        self.expect(":")
        if name == "stablehlo.compare":
            attrs["comparison_direction"] = bare[0]
            if len(bare) > 1:
                attrs["compare_type"] = bare[1]
        if name == "stablehlo.select" and self.peek() != "(":
            pt = parse_type(self.next())
            self.expect(",")
            rt = parse_type(self.next())
            return Op(name, results, operands, attrs, [pt, rt, rt], [rt])
        ins, outs = self.fn_type()
        if ins is None:
            ins = [outs[0]] * len(operands)
            if name == "stablehlo.optimization_barrier":
                while self.accept(","):
                    outs.append(parse_type(self.next()))
                ins = list(outs)
        return Op(name, results, operands, attrs, ins, outs)

    def reduce_op(self, results) -> Op:
        operands, inits = [], []
        while True:
            self.expect("(")
            operands.append(self.next())
            self.expect("init")
            self.expect(":")
            inits.append(self.next())
            self.expect(")")
            if not self.accept(","):
                break
        attrs = {}
        body_op = None
        if self.accept("applies"):
            body_op = self.next()
        self.expect("across")
        self.expect("dimensions")
        self.expect("=")
        attrs["dimensions"] = self.int_list()
        self.expect(":")
        ins, outs = self.fn_type()
        regions = []
        if body_op is not None:
            scalar = [TType((), t.dtype) for t in outs]
            n = len(outs)
            args = [(f"%__a{k}", scalar[k % n]) for k in range(2 * n)]
            ops = [Op(body_op, ["%__r0"], ["%__a0", "%__a1"], {}, [scalar[0]] * 2, [scalar[0]]),
                   Op("stablehlo.return", [], ["%__r0"], {}, [scalar[0]], [])]
            regions.append(Block(args, ops))
        else:
            self.expect("reducer")
            args = []
            while self.peek() == "(":
                args += self.block_args()
            # reducer args come as pairs (lhs_k, rhs_k) per input; reorder to lhs..., rhs...
            n = len(operands)
            if len(args) == 2 * n:
                args = args[0::2] + args[1::2]
            regions.append(self.block_body(args))
        return Op("stablehlo.reduce", results, operands + inits, attrs, ins, outs, regions)

    def generic_op(self, name, results) -> Op:
        operands = self.paren_operands()
        attrs = {}
        regions = []
        if self.peek() == "<":
            # <{...}> properties: tokenized as '<' '{' ... '}' '>'
            self.next()
            attrs.update(self.attr_dict())
            self.expect(">")
        if self.peek() == "(":
            self.next()
            while not self.accept(")"):
                regions.append(self.block_body([]))
                self.accept(",")
        if self.peek() == "{":
            attrs.update(self.attr_dict())
        self.expect(":")
        ins, outs = self.fn_type()
        return Op(name, results, operands, attrs, ins, outs, regions)


def parse_module(text: str) -> Module:
    return Parser(text).module()
