"""Generates the MLIR bytecode fixtures under tests/golden/bytecode/ (run from the repo root:
`python tests/golden/make_bytecode.py`).

Each fixture is a StableHLO program (`<name>.mlir`, the pretty text the plugin also compiles) and
its MLIR bytecode (`<name>.v<N>.mlirbc`) written by a real MLIR bytecode writer: the MLIR Python
bindings bundled with the nvidia-cutlass-dsl package (MLIR 20).  That context does not register the
stablehlo dialect, so the program is first rewritten into the generic op form
(tests/golden/mlir_generic.py) and parsed with unregistered dialects allowed; the writer then uses
the builtin dialect's encodings for types / builtin attributes and the textual fallback for the
stablehlo attributes.  Format versions 0-6 are written for two programs (the layouts differ between
versions), version 6 (the writer's default) for the rest.  Below version 5 there is no properties
section, so an op's `<{...}>` properties are written as its attribute dictionary.

`index.json` lists, per fixture, its text file, the number of ranks it is compiled for and the
versions written.  tests/test_bytecode.py checks that the plugin compiles each bytecode file to the
same plan as its text.
"""
import io
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "mccl-jax_b200"))
sys.path.insert(0, HERE)

import mlir_generic  # noqa: E402
from pjrt_b200 import configs  # noqa: E402
from pjrt_b200.shlo import Builder  # noqa: E402

OUT = os.path.join(HERE, "bytecode")

MISC = """module @jit_misc attributes {mhlo.num_partitions = 1 : i32, mhlo.num_replicas = 1 : i32} {
  func.func private @scale(%arg0: tensor<4x8xf32>) -> tensor<4x8xf32> {
    %cst = stablehlo.constant dense<2.500000e-01> : tensor<f32>
    %0 = stablehlo.broadcast_in_dim %cst, dims = [] : (tensor<f32>) -> tensor<4x8xf32>
    %1 = stablehlo.multiply %arg0, %0 : tensor<4x8xf32>
    return %1 : tensor<4x8xf32>
  }
  func.func public @main(%arg0: tensor<4x8xf32>, %arg1: tensor<4x8xui32>, %arg2: tensor<4x8xf16>) -> (tensor<4x8xf32>, tensor<4x8xi1>, tensor<4x16xf16>, tensor<2x8xf32>, tensor<8x4xf32>, tensor<4x8xi32>, tensor<12xi1>, tensor<3xf32>, tensor<4xf32>) {
    %0 = call @scale(%arg0) : (tensor<4x8xf32>) -> tensor<4x8xf32>
    %c = stablehlo.constant dense<[true, false, true, false, true, true, false, false]> : tensor<8xi1>
    %1 = stablehlo.broadcast_in_dim %c, dims = [1] : (tensor<8xi1>) -> tensor<4x8xi1>
    %c_0 = stablehlo.constant dense<7> : tensor<ui32>
    %2 = stablehlo.broadcast_in_dim %c_0, dims = [] : (tensor<ui32>) -> tensor<4x8xui32>
    %3 = stablehlo.compare  GT, %arg1, %2,  UNSIGNED : (tensor<4x8xui32>, tensor<4x8xui32>) -> tensor<4x8xi1>
    %4 = stablehlo.and %1, %3 : tensor<4x8xi1>
    %5 = stablehlo.concatenate %arg2, %arg2, dim = 1 : (tensor<4x8xf16>, tensor<4x8xf16>) -> tensor<4x16xf16>
    %6 = stablehlo.slice %0 [1:3, 0:8] : (tensor<4x8xf32>) -> tensor<2x8xf32>
    %7 = stablehlo.transpose %0, dims = [1, 0] : (tensor<4x8xf32>) -> tensor<8x4xf32>
    %8 = stablehlo.iota dim = 1 : tensor<4x8xi32>
    %c_1 = stablehlo.constant dense<[[1, -2, 3, -4, 5, -6, 7, -8], [0, 0, 0, 0, 0, 0, 0, 0], [9, 9, 9, 9, 9, 9, 9, 9], [-1, -1, -1, -1, -1, -1, -1, -2147483648]]> : tensor<4x8xi32>
    %9 = stablehlo.add %8, %c_1 : tensor<4x8xi32>
    %c_2 = stablehlo.constant dense<true> : tensor<4x8xi1>
    %10 = stablehlo.xor %4, %c_2 : tensor<4x8xi1>
    %c_3 = stablehlo.constant dense<[true, true, false, true, false, false, true, false, true, true, true, false]> : tensor<12xi1>
    %c_4 = stablehlo.constant dense<[false, true, true, true, true, false, true, false, true, false, true, true]> : tensor<12xi1>
    %11 = stablehlo.or %c_3, %c_4 : tensor<12xi1>
    %c_5 = stablehlo.constant dense<[1.5, -2.25, 0x7FC00000]> : tensor<3xf32>
    %c_6 = stablehlo.constant dense<[1.0, -0.5, 3.0, 65504.0]> : tensor<4xbf16>
    %12 = stablehlo.convert %c_6 : (tensor<4xbf16>) -> tensor<4xf32>
    return %0, %10, %5, %6, %7, %9, %11, %c_5, %12 : tensor<4x8xf32>, tensor<4x8xi1>, tensor<4x16xf16>, tensor<2x8xf32>, tensor<8x4xf32>, tensor<4x8xi32>, tensor<12xi1>, tensor<3xf32>, tensor<4xf32>
  }
}
"""


def argmax_text():
    b = Builder("jit_argreduce")
    x = b.arg((16, 100), "f32")
    v, i = b.argreduce(x, 1, "max")
    return b.text([v, i])


def donated_text():
    """An optimizer-style update with donated arguments: two results aliased to their arguments
    (tf.aliasing_output) and one argument donated without an alias (jax.buffer_donor)."""
    b = Builder("jit_donated_update")
    p, g, m = b.arg((64, 64), "f32"), b.arg((64, 64), "f32"), b.arg((64, 64), "f32")
    m1 = m * 0.9 + g
    return b.text([p - m1 * 0.01, m1], aliases={0: 0, 2: 1}, donors=(1,))


def programs():
    """(name, pretty text, ranks, versions)"""
    all_versions = list(range(7))
    return [
        ("mlp_step", configs.mlp_program(with_inputs=False).text, 1, all_versions),
        ("attention_causal", configs.attention_program(B=1, H=2, S=256, causal=True, with_inputs=False).text, 1, [6]),
        ("attention_full", configs.attention_program(B=1, H=2, S=256, causal=False, with_inputs=False).text, 1, [6]),
        ("gemm_bf16", configs.gemm_program(256, 256, 256, dtype="bf16", with_inputs=False).text, 1, [6]),
        ("gemm_f32_batched", configs.gemm_program(128, 128, 128, batch=2, dtype="f32", with_inputs=False).text, 1, [6]),
        ("psum_2", configs.psum_program(1024, 2, with_inputs=False).text, 2, [6]),
        ("gpt2_tiny_dp2", configs.gpt2_program(layers=1, d=128, heads=2, mlp=512, vocab=512, seq=256, batch=2,
                                               world=2, with_inputs=False).text, 2, all_versions),
        ("argmax", argmax_text(), 1, [6]),
        ("misc", MISC, 1, [0, 4, 6]),
        ("donated_update", donated_text(), 1, [0, 6]),
    ]


def write_bytecode(generic_text, version):
    from cutlass._mlir import ir   # the MLIR 20 Python bindings of nvidia-cutlass-dsl
    ctx = ir.Context()
    ctx.allow_unregistered_dialects = True
    with ctx:
        m = ir.Module.parse(generic_text)
        buf = io.BytesIO()
        m.operation.write_bytecode(buf, desired_version=version)
    return buf.getvalue()


def main():
    os.makedirs(OUT, exist_ok=True)
    index = {}
    for name, text, ranks, versions in programs():
        with open(os.path.join(OUT, name + ".mlir"), "w") as f:
            f.write(text)
        for v in versions:
            data = write_bytecode(mlir_generic.convert(text, props_as_attrs=v < 5), v)
            with open(os.path.join(OUT, f"{name}.v{v}.mlirbc"), "wb") as f:
                f.write(data)
        index[name] = {"text": name + ".mlir", "ranks": ranks, "versions": versions}
    with open(os.path.join(OUT, "index.json"), "w") as f:
        json.dump(index, f, indent=1)
    print(f"wrote {sum(len(v['versions']) for v in index.values())} bytecode files to {OUT}")


if __name__ == "__main__":
    main()
