"""Pins the CPU oracle (oracle/interp.py) before it is trusted as the parity checker:
  * against the golden fixtures (tests/golden/make_golden.py, PyTorch CPU) for attention, the MLP
    train step and the GEMMs;
  * against the reference's own known-answer collective tests: src/mccl/collective/smoke.cc:24-40
    (one rank: in-place all-reduce of [1, 2, 3, 4] is the identity) and smoke_multi.cc:32-48 (rank r
    contributes r+1 in each of 1024 floats; every rank reads n(n+1)/2).
"""
import os

import ml_dtypes
import numpy as np
import pytest

from conftest import RTOL_BF16, RTOL_F32, ROOT, assert_close
from oracle.interp import parse_dense, run, run_spmd
from oracle.shlo_parse import TType, parse_module
from pjrt_b200 import configs
from pjrt_b200.shlo import Builder

G = os.path.join(ROOT, "tests", "golden")


def bf(u16):
    return u16.view(ml_dtypes.bfloat16)


@pytest.mark.parametrize("causal", [False, True])
def test_oracle_attention_matches_golden(causal):
    d = np.load(os.path.join(G, f"attention_{'causal' if causal else 'full'}.npz"))
    p = configs.attention_program(B=1, H=2, S=256, D=64, causal=causal, with_inputs=False)
    out = run(p.text, [bf(d["q"]), bf(d["k"]), bf(d["v"])])[0]
    assert out.dtype == ml_dtypes.bfloat16
    assert_close(out.astype(np.float32), d["out"], RTOL_BF16, "attention")


def test_oracle_mlp_step_matches_golden():
    d = np.load(os.path.join(G, "mlp_step.npz"))
    p = configs.mlp_program(batch=32, din=64, hidden=48, classes=10, lr=0.01, with_inputs=False)
    outs = run(p.text, [d[f"in{i}"] for i in range(6)])
    for i, o in enumerate(outs):
        assert_close(o, d[f"out{i}"], RTOL_F32, f"mlp out{i}")


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_oracle_gemm_matches_golden(dtype):
    d = np.load(os.path.join(G, f"gemm_{dtype}.npz"))
    p = configs.gemm_program(M=96, N=80, K=64, dtype=dtype, with_inputs=False)
    a, b = (bf(d["a"]), bf(d["b"])) if dtype == "bf16" else (d["a"], d["b"])
    out = run(p.text, [a, b])[0]
    assert_close(out, d["out"], RTOL_F32, "gemm")


def test_oracle_allreduce_known_answer_single_rank():
    """smoke.cc:24-40: with one rank the all-reduce leaves [1, 2, 3, 4] unchanged."""
    p = configs.psum_program(4, 1, with_inputs=False)
    out = run(p.text, [np.array([1, 2, 3, 4], np.float32)])[0]
    np.testing.assert_array_equal(out, [1, 2, 3, 4])


@pytest.mark.parametrize("n", [2, 4, 8])
def test_oracle_allreduce_known_answer_multi_rank(n):
    """smoke_multi.cc:32-48: rank r contributes r+1 across 1024 floats; all read n(n+1)/2."""
    p = configs.psum_program(1024, n, with_inputs=False)
    res = run_spmd(p.text, [[np.full(1024, r + 1, np.float32)] for r in range(n)])
    for r in range(n):
        np.testing.assert_array_equal(res[r][0], np.full(1024, n * (n + 1) / 2, np.float32))


def test_oracle_integer_compare_iota_bit_exact():
    b = Builder("jit_ints")
    x = b.arg((6, 5), "i32")
    io = b.iota((6, 5), 1)
    m = b.compare(x, io, "GE")
    s = b.select(m, x, io)
    r = b.reduce(s, [1], "max")
    text = b.text([m, s, r])
    xv = np.arange(30, dtype=np.int32).reshape(6, 5) % 7 - 2
    m_o, s_o, r_o = run(text, [xv])
    iov = np.broadcast_to(np.arange(5, dtype=np.int32), (6, 5))
    np.testing.assert_array_equal(m_o, xv >= iov)
    np.testing.assert_array_equal(s_o, np.where(xv >= iov, xv, iov))
    np.testing.assert_array_equal(r_o, np.where(xv >= iov, xv, iov).max(1))


def test_dense_literal_forms():
    assert parse_dense("dense<0xFF800000>", TType((), "f32"))[()] == -np.inf
    np.testing.assert_array_equal(parse_dense("dense<[[1, 2], [3, 4]]>", TType((2, 2), "i32")), [[1, 2], [3, 4]])
    v = parse_dense("dense<1.000000e-01>", TType((3,), "bf16"))
    assert v.dtype == ml_dtypes.bfloat16 and float(v[0]) == float(ml_dtypes.bfloat16(0.1))
    raw = np.array([1.5, -2.0], np.float32).tobytes().hex().upper()
    np.testing.assert_array_equal(parse_dense(f'dense<"0x{raw}">', TType((2,), "f32")), [1.5, -2.0])


def test_parser_handles_generic_reduce_and_call_forms():
    text = """
module @m {
  func.func public @main(%arg0: tensor<4x3xf32>) -> (tensor<4xf32>) {
    %0 = call @inner(%arg0) : (tensor<4x3xf32>) -> tensor<4x3xf32>
    %cst = stablehlo.constant dense<0.000000e+00> : tensor<f32>
    %1 = stablehlo.reduce(%0 init: %cst) across dimensions = [1] : (tensor<4x3xf32>, tensor<f32>) -> tensor<4xf32>
     reducer(%a: tensor<f32>, %b: tensor<f32>)  {
      %2 = stablehlo.add %a, %b : tensor<f32>
      stablehlo.return %2 : tensor<f32>
    }
    return %1 : tensor<4xf32>
  }
  func.func private @inner(%x: tensor<4x3xf32>) -> tensor<4x3xf32> {
    %0 = stablehlo.multiply %x, %x : tensor<4x3xf32>
    return %0 : tensor<4x3xf32>
  }
}
"""
    m = parse_module(text)
    assert set(m.funcs) == {"main", "inner"}
    x = np.arange(12, dtype=np.float32).reshape(4, 3)
    np.testing.assert_allclose(run(text, [x])[0], (x * x).sum(1))


def test_oracle_permute_broadcast_all_to_all():
    """collective_permute / collective_broadcast / all_to_all across simulated ranks, and the
    identity each is at one rank (what the plugin lowers at one process)."""
    def prog(op_text, n):
        t = f"tensor<{2 * n}x4xf32>"
        return ("module @m {\n  func.func public @main(%arg0: " + t + ") -> (" + t + ") {\n"
                f"    %0 = {op_text} : ({t}) -> {t}\n    return %0 : {t}\n  }}\n}}\n")
    perm = '"stablehlo.collective_permute"(%arg0) <{channel_handle = #stablehlo.channel_handle<handle = 1, type = 1>, source_target_pairs = dense<PAIRS> : tensor<NPx2xi64>}>'
    bcast = '"stablehlo.collective_broadcast"(%arg0) <{replica_groups = dense<[[0, 1]]> : tensor<1x2xi64>}>'
    a2a = '"stablehlo.all_to_all"(%arg0) <{concat_dimension = 0 : i64, replica_groups = dense<[[0, 1]]> : tensor<1x2xi64>, split_count = 2 : i64, split_dimension = 0 : i64}>'
    x1 = np.arange(8, dtype=np.float32).reshape(2, 4)
    assert np.array_equal(run(prog(perm.replace("PAIRS", "[[0, 0]]").replace("NP", "1"), 1), [x1])[0], x1)
    xs = [np.full((4, 4), r + 1, np.float32) + np.arange(4, dtype=np.float32)[:, None] for r in range(2)]
    res = run_spmd(prog(perm.replace("PAIRS", "[[0, 1]]").replace("NP", "1"), 2), [[x] for x in xs])
    assert np.array_equal(res[1][0], xs[0]) and np.array_equal(res[0][0], np.zeros_like(xs[0]))
    res = run_spmd(prog(bcast, 2), [[x] for x in xs])
    assert all(np.array_equal(r[0], xs[0]) for r in res)
    res = run_spmd(prog(a2a, 2), [[x] for x in xs])
    for dst in range(2):
        assert np.array_equal(res[dst][0], np.concatenate([xs[src][2 * dst:2 * dst + 2] for src in range(2)], axis=0))


def _coll_prog(op_text, shape_in, shape_out):
    ti, to = f"tensor<{shape_in}xf32>", f"tensor<{shape_out}xf32>"
    return ("module @m {\n  func.func public @main(%arg0: " + ti + ") -> (" + to + ") {\n"
            f"    %0 = {op_text} : ({ti}) -> {to}\n    return %0 : {to}\n  }}\n}}\n")


ADD_REGION = ('({\n      ^bb0(%a: tensor<f32>, %b: tensor<f32>):\n        %s = stablehlo.add %a, %b : tensor<f32>\n'
              '        stablehlo.return %s : tensor<f32>\n      })')


def test_oracle_collectives_act_per_replica_group():
    """StableHLO applies a collective within each replica group: the broadcast source is each
    group's first member, all_reduce sums only within a group, all_gather concatenates in group
    order, reduce_scatter hands the group's i-th part to its i-th member."""
    xs = [np.full((4,), r + 1, np.float32) + np.arange(4, dtype=np.float32) for r in range(4)]
    bcast = '"stablehlo.collective_broadcast"(%arg0) <{replica_groups = dense<[[1, 0]]> : tensor<1x2xi64>}>'
    res = run_spmd(_coll_prog(bcast, "4", "4"), [[x] for x in xs[:2]])
    assert all(np.array_equal(r[0], xs[1]) for r in res)
    ar = ('"stablehlo.all_reduce"(%arg0) <{replica_groups = dense<[[0, 2], [1, 3]]> : tensor<2x2xi64>}> ' + ADD_REGION)
    res = run_spmd(_coll_prog(ar, "4", "4"), [[x] for x in xs])
    for r in range(4):
        np.testing.assert_array_equal(res[r][0], xs[r % 2] + xs[r % 2 + 2])
    ag = '"stablehlo.all_gather"(%arg0) <{all_gather_dim = 0 : i64, replica_groups = dense<[[1, 0], [3, 2]]> : tensor<2x2xi64>}>'
    res = run_spmd(_coll_prog(ag, "4", "8"), [[x] for x in xs])
    np.testing.assert_array_equal(res[0][0], np.concatenate([xs[1], xs[0]]))
    np.testing.assert_array_equal(res[3][0], np.concatenate([xs[3], xs[2]]))
    rs = ('"stablehlo.reduce_scatter"(%arg0) <{replica_groups = dense<[[1, 0]]> : tensor<1x2xi64>, scatter_dimension = 0 : i64}> '
          + ADD_REGION)
    res = run_spmd(_coll_prog(rs, "4", "2"), [[x] for x in xs[:2]])
    np.testing.assert_array_equal(res[1][0], (xs[0] + xs[1])[:2])     # rank 1 is the group's member 0
    np.testing.assert_array_equal(res[0][0], (xs[0] + xs[1])[2:])


def test_oracle_rejects_groups_that_miss_a_rank():
    ar = ('"stablehlo.all_reduce"(%arg0) <{replica_groups = dense<[[0, 1]]> : tensor<1x2xi64>}> ' + ADD_REGION)
    with pytest.raises(ValueError):
        run_spmd(_coll_prog(ar, "4", "4"), [[np.zeros(4, np.float32)] for _ in range(3)])
