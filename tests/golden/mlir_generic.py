"""Test tooling: rewrite StableHLO MLIR text from the pretty op forms into MLIR's generic op form.

jax prints (and `pjrt_b200.shlo` writes) the pretty forms, e.g.
    %2 = stablehlo.broadcast_in_dim %1, dims = [0] : (tensor<8xf32>) -> tensor<8x4xf32>
while an MLIR context that does not know the stablehlo dialect -- and any MLIR bytecode reader --
sees every op in the generic form
    %2 = "stablehlo.broadcast_in_dim"(%1) {broadcast_dimensions = array<i64: 0>} : (tensor<8xf32>) -> tensor<8x4xf32>
The attribute names and spellings are StableHLO's own (its op definitions and the generic printer):
broadcast_dimensions, permutation, iota_dimension, dimension, dimensions, start_indices /
limit_indices / strides, edge_padding_low / edge_padding_high / interior_padding,
#stablehlo<comparison_direction ..>, #stablehlo<comparison_type ..>, #stablehlo.dot<...>,
call_target_name, value, dimensions (reverse), slice_sizes, exponent_bits / mantissa_bits.

The tests use it twice: the plugin's parser must give the same plan for both forms, and
`make_bytecode.py` feeds the generic form to an MLIR bytecode writer to make the bytecode fixtures.
It covers the op forms of the five configs' programs, line by line; func.func / return / call stay
in their pretty form (the func dialect is registered in every MLIR context).
"""
from __future__ import annotations

import re
from typing import List

_RES = r"(?P<res>%[\w.#:]+(?:\s*,\s*%[\w.#:]+)*)\s*=\s*"


def _split_top(s: str) -> List[str]:
    """Split on commas outside <>, [], (), {} and quotes."""
    out, depth, cur, q = [], 0, "", False
    for k, c in enumerate(s):
        if q:
            cur += c
            if c == '"' and s[k - 1] != "\\":
                q = False
            continue
        if c == '"':
            q = True
        elif c in "<[({":
            depth += 1
        elif c in ">])}" and not (c == ">" and k and s[k - 1] == "-"):
            depth -= 1
        if c == "," and depth == 0:
            out.append(cur.strip())
            cur = ""
        else:
            cur += c
    if cur.strip():
        out.append(cur.strip())
    return out


def _arr(lst: str) -> str:
    vals = [v.strip() for v in lst.strip()[1:-1].split(",") if v.strip()]
    return "array<i64" + (": " + ", ".join(vals) if vals else "") + ">"


def _fn_type(ty: str, n_operands: int) -> str:
    ty = ty.strip()
    if ty.startswith("("):
        return ty
    return "(" + ", ".join([ty] * n_operands) + ") -> " + ty


def _attrs(d: dict) -> str:
    return "{" + ", ".join(f"{k} = {v}" for k, v in sorted(d.items())) + "}" if d else ""


def _op(res: str, name: str, operands: List[str], attrs: dict, ty: str) -> str:
    a = _attrs(attrs)
    return f'{res} = "stablehlo.{name}"({", ".join(operands)}) {a}{" " if a else ""}: {ty}'


def convert_line(line: str) -> str:
    ind = line[: len(line) - len(line.lstrip())]
    s = line.strip()
    cm = re.match(_RES + r"chlo\.(?P<name>\w+)\s+(?P<x>%[\w.#]+)\s*:\s*(?P<a>tensor<[^>]*>)\s*->\s*(?P<b>tensor<[^>]*>)$", s)
    if cm:   # chlo unary ops print as `chlo.erf %x : T -> U`
        return f'{ind}{cm.group("res")} = "chlo.{cm.group("name")}"({cm.group("x")}) : ({cm.group("a")}) -> {cm.group("b")}'
    m = re.match(_RES + r"stablehlo\.(?P<name>\w+)\s*(?P<rest>.*)$", s)
    if not m:
        m2 = re.match(r"stablehlo\.return\s+(?P<ops>[^:]*):\s*(?P<tys>.*)$", s)
        if m2:
            ops = [o.strip() for o in m2.group("ops").split(",") if o.strip()]
            return f'{ind}"stablehlo.return"({", ".join(ops)}) : ({m2.group("tys").strip()}) -> ()'
        return line
    res, name, rest = m.group("res"), m.group("name"), m.group("rest")
    rest = " " + rest
    body, ty = rest.rsplit(" : ", 1) if " : " in rest else (rest, "")
    parts = _split_top(body)
    operands = [p for p in parts if p.startswith("%")]
    kv = {}
    for p in parts:
        if "=" in p and not p.startswith("%") and not p.startswith("dense<"):
            k, v = p.split("=", 1)
            kv[k.strip()] = v.strip()
    if name == "constant":
        return f'{ind}{res} = "stablehlo.constant"() {{value = {body.strip()} : {ty.strip()}}} : () -> {ty.strip()}'
    if name == "iota":
        return f'{ind}{res} = "stablehlo.iota"() {{iota_dimension = {kv["dim"]} : i64}} : () -> {ty.strip()}'
    if name == "compare":
        direction = [p for p in parts if not p.startswith("%")][0]
        ctype = [p for p in parts if not p.startswith("%")][1:]
        at = {"comparison_direction": f"#stablehlo<comparison_direction {direction}>"}
        if ctype:
            at["compare_type"] = f"#stablehlo<comparison_type {ctype[0]}>"
        return ind + _op(res, name, operands, at, _fn_type(ty, 2))
    if name == "select":
        if not ty.strip().startswith("("):
            pt, rt = _split_top(ty)
            ty = f"({pt}, {rt}, {rt}) -> {rt}"
        return ind + _op(res, name, operands, {}, ty)
    if name == "broadcast_in_dim":
        return ind + _op(res, name, operands, {"broadcast_dimensions": _arr(kv["dims"])}, ty)
    if name == "transpose":
        return ind + _op(res, name, operands, {"permutation": _arr(kv["dims"])}, ty)
    if name == "broadcast":
        return ind + _op(res, name, operands, {"broadcast_sizes": _arr(kv["sizes"])}, ty)
    if name == "reverse":
        return ind + _op(res, name, operands, {"dimensions": _arr(kv["dims"])}, _fn_type(ty, 1))
    if name == "dynamic_slice":
        return ind + _op(res, name, operands, {"slice_sizes": _arr(kv["sizes"])}, ty)
    if name == "reduce_precision":
        fm = re.fullmatch(r"e(\d+)m(\d+)", kv["format"])
        at = {"exponent_bits": f"{fm.group(1)} : i32", "mantissa_bits": f"{fm.group(2)} : i32"}
        return ind + _op(res, name, operands, at, _fn_type(ty, 1))
    if name == "concatenate":
        return ind + _op(res, name, operands, {"dimension": f"{kv['dim']} : i64"}, ty)
    if name == "pad":
        at = {"edge_padding_low": _arr(kv["low"]), "edge_padding_high": _arr(kv["high"]),
              "interior_padding": _arr(kv["interior"])}
        return ind + _op(res, name, operands, at, ty)
    if name == "slice":
        operands = [body.strip().split()[0]]
        sl = re.search(r"\[(.*)\]", body).group(1)
        st, li, sd = [], [], []
        for e in sl.split(","):
            f = [int(x) for x in e.strip().split(":")]
            st.append(f[0]); li.append(f[1] if len(f) > 1 else f[0] + 1); sd.append(f[2] if len(f) > 2 else 1)
        at = {"start_indices": _arr(str(st)), "limit_indices": _arr(str(li)), "strides": _arr(str(sd))}
        return ind + _op(res, name, operands, at, ty)
    if name == "dot_general":
        def pair(key):
            if key not in kv:
                return "[]", "[]"
            lhs, rhs = kv[key].split(" x ")
            return lhs.strip(), rhs.strip()
        lb, rb = pair("batching_dims")
        lc, rc = pair("contracting_dims")
        fields = []
        if lb != "[]":
            fields += [f"lhs_batching_dimensions = {lb}", f"rhs_batching_dimensions = {rb}"]
        fields += [f"lhs_contracting_dimensions = {lc}", f"rhs_contracting_dimensions = {rc}"]
        at = {"dot_dimension_numbers": "#stablehlo.dot<" + ", ".join(fields) + ">"}
        if "precision" in kv:
            ps = [v.strip() for v in kv["precision"].strip()[1:-1].split(",") if v.strip()]
            at["precision_config"] = "[" + ", ".join(f"#stablehlo<precision {v}>" for v in ps) + "]"
        return ind + _op(res, name, operands, at, ty)
    if name == "custom_call":
        cm = re.match(r"@(?P<t>[\w.]+)\((?P<ops>[^)]*)\)\s*(?P<d>\{.*\})?\s*$", body.strip())
        ops = [o.strip() for o in cm.group("ops").split(",") if o.strip()]
        at = {"call_target_name": f'"{cm.group("t")}"'}
        if cm.group("d"):
            for p in _split_top(cm.group("d")[1:-1]):
                k, v = p.split("=", 1)
                at[k.strip()] = v.strip()
        return ind + _op(res, name, ops, at, ty)
    if name == "reduce":
        raise ValueError("reduce is converted by convert()")
    # plain unary / binary elementwise, convert, reshape
    return ind + _op(res, name, operands, {}, _fn_type(ty, len(operands)))


def _props_to_attrs(line: str, pending_props: List[str]) -> str:
    """`"x"(...) <{A}> ...` -> `"x"(...) ... {A}`: an MLIR bytecode writer older than format
    version 5 has no properties section and keeps an unregistered op's attributes only in its
    attribute dictionary."""
    k = line.find("<{")
    if k < 0:
        return line
    depth, j = 0, k + 1
    while j < len(line):
        if line[j] == "{":
            depth += 1
        elif line[j] == "}":
            depth -= 1
            if depth == 0:
                break
        j += 1
    props = line[k + 1:j + 1]
    rest = line[j + 2:]
    if rest.rstrip().endswith("({"):
        pending_props.append(props)
        return line[:k].rstrip() + rest
    head, ty = rest.rsplit(" : ", 1)
    return line[:k].rstrip() + head + " " + props + " : " + ty


def convert(text: str, props_as_attrs: bool = False) -> str:
    """Pretty -> generic for a whole module (see the module docstring).  `props_as_attrs` moves
    `<{...}>` properties into the attribute dictionary (for bytecode versions below 5)."""
    text = "\n".join(_convert(text))
    if not props_as_attrs:
        return text + "\n"
    out, pending = [], []
    for line in text.splitlines():
        if line.strip().startswith("})") and pending and " : " in line:
            head, ty = line.rsplit(" : ", 1)
            line = head + " " + pending.pop() + " : " + ty
        out.append(_props_to_attrs(line, pending))
    return "\n".join(out) + "\n"


def _convert(text: str) -> List[str]:
    out: List[str] = []
    pending: List[tuple] = []          # (depth at which the region closes, trailer text)
    depth = 0
    lines = text.splitlines()
    i = 0
    while i < len(lines):
        line = lines[i]
        s = line.strip()
        ind = line[: len(line) - len(line.lstrip())]
        m = re.match(_RES + r"stablehlo\.reduce\((?P<rest>.*)$", s)
        if m:
            res, rest = m.group("res"), "(" + m.group("rest")
            head, ty = rest.split(" across dimensions = ")
            dims, ty = ty.split(" : ", 1)
            pairs = re.findall(r"\((%[\w.#]+) init: (%[\w.#]+)\)", head)
            xs, inits = [p[0] for p in pairs], [p[1] for p in pairs]
            trailer = f"}}) {{dimensions = {_arr(dims.strip())}}} : {ty.strip()}"
            am = re.search(r"applies stablehlo\.(\w+)", head)
            opnds = ", ".join(xs + inits)
            if am:
                sc = re.match(r"tensor<(?:[\dx]*x)?(\w+)>", _split_top(ty.strip()[1:].split(") ->")[0])[-1])
                st = f"tensor<{sc.group(1)}>"
                out.append(f'{ind}{res} = "stablehlo.reduce"({opnds}) ({{')
                out.append(f"{ind}^bb0(%lhs: {st}, %rhs: {st}):")
                out.append(f'{ind}  %red = "stablehlo.{am.group(1)}"(%lhs, %rhs) : ({st}, {st}) -> {st}')
                out.append(f'{ind}  "stablehlo.return"(%red) : ({st}) -> ()')
                out.append(ind + trailer)
                i += 1
                continue
            # multi-line reducer: next line `reducer(%a0: t, %b0: t) (%a1: u, %b1: u) {`
            i += 1
            rl = lines[i].strip()
            groups = re.findall(r"\(([^()]*)\)", rl[len("reducer"):])
            lhs, rhs = [], []
            for g in groups:
                a, b = _split_top(g)
                lhs.append(a); rhs.append(b)
            out.append(f'{ind}{res} = "stablehlo.reduce"({opnds}) ({{')
            out.append(f"{ind}^bb0({', '.join(lhs + rhs)}):")
            depth += 1
            pending.append((depth, ind + trailer))
            i += 1
            continue
        if s == "}" and pending and pending[-1][0] == depth:
            out.append(pending.pop()[1])
            depth -= 1
            i += 1
            continue
        if s.endswith("({"):
            depth += 1
        elif s.startswith("})"):
            depth -= 1
        out.append(convert_line(line))
        i += 1
    return out
