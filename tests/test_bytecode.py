"""MLIR bytecode input to PJRT_Client_Compile (format "mlir"), on the CPU.

The reference passes the program to MLIR's reader (src/jam/parse.cc:53-63), which accepts text and
bytecode alike.  The plugin decodes bytecode itself (mccl-jax_b200/csrc/jam/bytecode.cc) into MLIR
text that its parser reads.  Pinning: the fixtures under tests/golden/bytecode/ were written by a
real MLIR 20 bytecode writer (tests/golden/make_bytecode.py), format versions 0-6; each must parse
to the same op graph (ops, attributes, constant bytes) and compile to the same plan as the text it
was written from.  The generic op form (what bytecode decodes to) must give the same graph as the
pretty form for every config program, and malformed bytecode must fail with an error, never crash
or hang.
"""
import ctypes
import json
import os
import random
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

import mlir_generic  # noqa: E402
from pjrt_b200 import configs  # noqa: E402
from pjrt_b200.shlo import Builder  # noqa: E402

FIX = os.path.join(HERE, "golden", "bytecode")
INDEX = json.load(open(os.path.join(FIX, "index.json")))
CASES = [(name, v) for name, m in INDEX.items() for v in m["versions"]]

GRAPH, PLAN, FULL = 2, 0, 1      # b200_compile_report modes


@pytest.fixture(scope="module")
def compile_report(lib_path):
    lib = ctypes.CDLL(lib_path)
    buf = ctypes.create_string_buffer(1 << 23)

    def run(data, ranks=1, mode=GRAPH):
        if isinstance(data, str):
            data = data.encode()
        rc = lib.b200_compile_report(data, len(data), ranks, mode, buf, len(buf))
        return rc, buf.value.decode(errors="replace")
    return run


def fixture(name, version):
    m = INDEX[name]
    with open(os.path.join(FIX, m["text"])) as f:
        text = f.read()
    with open(os.path.join(FIX, f"{name}.v{version}.mlirbc"), "rb") as f:
        data = f.read()
    return text, data, m["ranks"]


def test_fixtures_are_mlir_bytecode():
    for name, v in CASES:
        _, data, _ = fixture(name, v)
        assert data[:4] == b"ML\xefR" and data[4] == 2 * v + 1, (name, v)   # magic, varint version


@pytest.mark.parametrize("name,version", CASES)
def test_bytecode_parses_to_the_texts_graph_and_plan(compile_report, name, version):
    text, data, ranks = fixture(name, version)
    for mode in (GRAPH, PLAN):
        rc_t, rep_t = compile_report(text, ranks, mode)
        rc_b, rep_b = compile_report(data, ranks, mode)
        assert rc_t == 0, rep_t
        assert rc_b == 0, rep_b
        assert rep_b == rep_t


@pytest.mark.parametrize("name", ["mlp_step", "attention_causal", "gpt2_tiny_dp2", "misc"])
def test_bytecode_full_compile_matches_text(compile_report, name):
    text, data, ranks = fixture(name, 6)
    rc_t, rep_t = compile_report(text, ranks, FULL)
    rc_b, rep_b = compile_report(data, ranks, FULL)
    assert rc_t == 0 and rc_b == 0, rep_b
    assert rep_b == rep_t


def _argmax():
    b = Builder("jit_argreduce")
    x = b.arg((64, 1000), "bf16")
    v, i = b.argreduce(x, 1, "min")
    return b.text([v, i])


GENERIC_PROGRAMS = [
    ("mlp", lambda: configs.mlp_program(with_inputs=False).text, 1),
    ("attention_causal_4096", lambda: configs.attention_program(S=4096, causal=True, with_inputs=False).text, 1),
    ("attention_full_1024", lambda: configs.attention_program(S=1024, with_inputs=False).text, 1),
    ("gemm_f32", lambda: configs.gemm_program(1024, 1024, 1024, dtype="f32", with_inputs=False).text, 1),
    ("gemm_batched", lambda: configs.gemm_program(2048, 2048, 2048, batch=16, with_inputs=False).text, 1),
    ("psum_8", lambda: configs.psum_program(1 << 20, 8, with_inputs=False).text, 8),
    ("gpt2_small_dp2", lambda: configs.gpt2_program(world=2, with_inputs=False).text, 2),
    ("argmin_bf16", _argmax, 1),
]


@pytest.mark.parametrize("name,make,ranks", GENERIC_PROGRAMS, ids=[g[0] for g in GENERIC_PROGRAMS])
def test_generic_op_form_parses_to_the_pretty_forms_graph(compile_report, name, make, ranks):
    text = make()
    rc_p, rep_p = compile_report(text, ranks, GRAPH)
    rc_g, rep_g = compile_report(mlir_generic.convert(text), ranks, GRAPH)
    assert rc_p == 0 and rc_g == 0, rep_g
    assert rep_g == rep_p


def test_truncated_bytecode_is_an_error(compile_report):
    _, data, _ = fixture("misc", 6)
    for n in range(len(data)):
        rc, rep = compile_report(data[:n])
        assert rc == 1 and rep.startswith("error:"), (n, rep)


@pytest.mark.parametrize("name,version", [("misc", 6), ("misc", 0), ("mlp_step", 3), ("gpt2_tiny_dp2", 6)])
def test_corrupt_bytecode_fails_cleanly(compile_report, name, version):
    """Seeded random byte changes: every result is a clean success or a clean error."""
    _, data, ranks = fixture(name, version)
    rng = random.Random(1234 + version)
    outcomes = {0: 0, 1: 0}
    for _ in range(400):
        d = bytearray(data)
        for _ in range(rng.randint(1, 4)):
            d[rng.randrange(len(d))] = rng.randrange(256)
        rc, rep = compile_report(bytes(d), ranks)
        assert rc in (0, 1), rep
        assert rc == 0 or rep.startswith("error:")
        outcomes[rc] += 1
    assert outcomes[1] > 0


def test_newer_format_version_is_rejected(compile_report):
    _, data, _ = fixture("mlp_step", 6)
    d = bytearray(data)
    d[4] = 2 * 7 + 1
    rc, rep = compile_report(bytes(d))
    assert rc == 1 and "version 7" in rep


def test_text_parser_rejects_unclosed_dimension_list(compile_report):
    # an unclosed `[` inside #stablehlo.dot<...> once sent the dimension-number scan into a loop
    text = mlir_generic.convert(configs.gemm_program(128, 128, 128, with_inputs=False).text)
    bad = text.replace("rhs_contracting_dimensions = [0]", "rhs_contracting_dimensions = [0")
    assert bad != text
    rc, rep = compile_report(bad)
    assert rc == 1 and "malformed dimension numbers" in rep
