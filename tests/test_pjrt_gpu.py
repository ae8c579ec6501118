"""End-to-end through the PJRT C API on a B200, checked against the CPU oracle on the same module
text and the same seeded inputs — the flow of the reference's src/pjrt/pjrt_e2e.cc:60-181."""
import os

import ml_dtypes
import numpy as np
import pytest

from conftest import RTOL_BF16, RTOL_F32, ROOT, assert_close
from oracle.interp import run as oracle_run
from pjrt_b200 import configs, pjrt
from pjrt_b200.shlo import Builder

pytestmark = pytest.mark.gpu
G = os.path.join(ROOT, "tests", "golden")


def test_client_identity(client):
    assert client.platform_name() == "b200"
    assert "PJRT 0.55" in client.platform_version()
    devs = client.devices(addressable=True)
    assert len(devs) == 1
    assert "B200" in client.device_kind(devs[0])


@pytest.mark.parametrize("dt", [np.float32, np.int32, np.bool_, ml_dtypes.bfloat16, np.float16, np.int8])
def test_buffer_roundtrip(client, dt):
    x = (np.arange(3 * 5 * 7) % 11 - 4).reshape(3, 5, 7).astype(dt)
    b = client.buffer_from_host(x)
    assert b.shape() == (3, 5, 7)
    np.testing.assert_array_equal(b.to_numpy(), x)
    b.delete()


def test_empty_buffer(client):
    x = np.zeros((0, 4), np.float32)
    b = client.buffer_from_host(x)
    assert b.shape() == (0, 4)
    assert b.to_numpy().shape == (0, 4)


@pytest.mark.parametrize("causal", [False, True])
def test_attention_golden_through_pjrt(client, causal):
    d = np.load(os.path.join(G, f"attention_{'causal' if causal else 'full'}.npz"))
    p = configs.attention_program(B=1, H=2, S=256, D=64, causal=causal, with_inputs=False)
    ins = [d[k].view(ml_dtypes.bfloat16) for k in ("q", "k", "v")]
    out = client.run(p.text, ins)[0]
    assert out.dtype == ml_dtypes.bfloat16
    assert_close(out.astype(np.float32), d["out"], RTOL_BF16, "attention vs golden")
    ref = oracle_run(p.text, ins)[0]
    assert_close(out.astype(np.float32), ref.astype(np.float32), RTOL_BF16, "attention vs oracle")


@pytest.mark.parametrize("S,causal", [(512, False), (512, True), (1024, True)])
def test_attention_config_shapes_vs_oracle(client, S, causal):
    p = configs.attention_program(B=2, H=4, S=S, D=64, causal=causal, seed=S)
    out = client.run(p.text, p.inputs)[0]
    ref = oracle_run(p.text, p.inputs)[0]
    assert_close(out.astype(np.float32), ref.astype(np.float32), RTOL_BF16, "attention")


def test_attention_unfused_path_vs_oracle(client, monkeypatch):
    monkeypatch.setenv("B200_NO_FLASH", "1")
    p = configs.attention_program(B=1, H=2, S=256, D=64, causal=True, seed=11)
    out = client.run(p.text, p.inputs)[0]
    ref = oracle_run(p.text, p.inputs)[0]
    assert_close(out.astype(np.float32), ref.astype(np.float32), RTOL_BF16, "unfused attention")


def test_mlp_step_golden(client):
    d = np.load(os.path.join(G, "mlp_step.npz"))
    p = configs.mlp_program(batch=32, din=64, hidden=48, classes=10, lr=0.01, with_inputs=False)
    outs = client.run(p.text, [d[f"in{i}"] for i in range(6)])
    for i, o in enumerate(outs):
        assert_close(o, d[f"out{i}"], RTOL_F32, f"mlp out{i}")


def test_mlp_step_config1_vs_oracle(client):
    p = configs.mlp_program()  # [128,784] -> 512 -> 10
    outs = client.run(p.text, p.inputs)
    refs = oracle_run(p.text, p.inputs)
    for i, (o, r) in enumerate(zip(outs, refs)):
        assert_close(o, r, RTOL_F32, f"mlp out{i}")


@pytest.mark.parametrize("version", [6, 0])
def test_mlp_step_from_mlir_bytecode_vs_oracle(client, version):
    """The same MLP step given as MLIR bytecode (written by an MLIR 20 writer,
    tests/golden/make_bytecode.py) runs to the oracle's results on the fixture's text."""
    fx = os.path.join(G, "bytecode")
    with open(os.path.join(fx, f"mlp_step.v{version}.mlirbc"), "rb") as f:
        data = f.read()
    with open(os.path.join(fx, "mlp_step.mlir")) as f:
        text = f.read()
    p = configs.mlp_program()
    assert p.text == text
    outs = client.run(data, p.inputs)
    refs = oracle_run(text, p.inputs)
    assert len(outs) == len(refs)
    for i, (o, r) in enumerate(zip(outs, refs)):
        assert_close(o, r, RTOL_F32, f"mlp (bytecode v{version}) out{i}")


@pytest.mark.parametrize("dtype,M,N,K,batch", [("bf16", 1024, 1024, 1024, 0), ("f32", 256, 192, 320, 0),
                                               ("bf16", 256, 256, 256, 4), ("bf16", 96, 80, 64, 0)])
def test_gemm_vs_oracle(client, dtype, M, N, K, batch):
    p = configs.gemm_program(M, N, K, batch=batch, dtype=dtype, seed=M + K)
    out = client.run(p.text, p.inputs)[0]
    ref = oracle_run(p.text, p.inputs)[0]
    assert_close(out, ref, RTOL_F32 if dtype == "f32" else RTOL_F32 * 10, "gemm")


@pytest.mark.parametrize("pair", ["0", "1"])
@pytest.mark.parametrize("dtype,M,N,K", [("bf16", 2048, 1536, 768), ("bf16", 768, 2304, 8192), ("f32", 1024, 1024, 1024)])
def test_gemm_units_from_a_counter(client, monkeypatch, pair, dtype, M, N, K):
    """Programs with collectives draw GEMM work units from a per-launch counter (CTAs that start late
    take fewer); forced here on one GPU, on one-SM tiles and on CTA pairs (whose even CTA hands each
    unit to its peer), including split-K and the f32 split form."""
    monkeypatch.setenv("B200_GEMM_STATIC_UNITS", "0")
    monkeypatch.setenv("B200_GEMM_PAIR", pair)
    p = configs.gemm_program(M, N, K, dtype=dtype, seed=M + N)
    exe = client.compile(p.text)
    bufs = [client.buffer_from_host(x) for x in p.inputs]
    ref = oracle_run(p.text, p.inputs)[0]
    for _ in range(3):                                  # the counters are zeroed again every execution
        out = exe.execute(bufs)[0]
        assert_close(out.to_numpy(), ref, RTOL_F32 if dtype == "f32" else RTOL_F32 * 10, "gemm with unit counter")
        out.delete()
    exe.destroy()


@pytest.mark.parametrize("K,N,out", [(50, 70, "f32"), (50257 // 41, 333, "bf16"), (768, 1001, "f32"), (1000, 520, "bf16")])
def test_dot_mixed_precision_and_unaligned_shapes(client, K, N, out):
    """bf16 x f32 operands (a backward-pass cotangent meeting bf16 weights).  With an f32 result the
    dot is f32 arithmetic (the f32 operand split into bf16 pieces on the tensor cores) and holds the
    f32 bar; with a bf16 result the f32 operand is rounded to bf16 once and the result holds the bf16
    bar.  K % 8 != 0 takes the padded operand layout; N % 8 != 0 the staged epilogue."""
    b = Builder("jit_mixed_dot")
    x = b.arg((200, K), "bf16")
    w = b.arg((K, N), "f32")
    y = b.dot_general(x, w, contract=([1], [0]), out_dtype=out)
    text = b.text([y])
    rng = np.random.default_rng(K + N)
    ins = [(rng.standard_normal((200, K)) / np.sqrt(K)).astype(ml_dtypes.bfloat16),
           rng.standard_normal((K, N)).astype(np.float32)]
    got = client.run(text, ins)[0]
    ref = oracle_run(text, ins)[0]
    assert_close(np.asarray(got, np.float32), np.asarray(ref, np.float32), RTOL_F32 if out == "f32" else RTOL_BF16,
                 "mixed dot")


@pytest.mark.parametrize("lhs_c,rhs_c", [(1, 0), (0, 0), (1, 1), (0, 1)])
@pytest.mark.parametrize("dtype,M,N,K", [("bf16", 384, 512, 320), ("bf16", 200, 136, 72), ("bf16", 90, 70, 50),
                                         ("f32", 72, 40, 56)])
def test_dot_operand_layouts(client, lhs_c, rhs_c, dtype, M, N, K):
    """Each operand is read where it lies when it is [rows, K] (K-major) or [K, rows] (MN-major, rows
    a multiple of 8); other layouts are copied.  All four contraction placements against the oracle."""
    b = Builder("jit_layouts")
    x = b.arg((M, K) if lhs_c == 1 else (K, M), dtype)
    w = b.arg((N, K) if rhs_c == 1 else (K, N), dtype)
    y = b.dot_general(x, w, contract=([lhs_c], [rhs_c]), out_dtype="f32")
    text = b.text([y])
    rng = np.random.default_rng(M * 7 + N + lhs_c * 2 + rhs_c)
    npdt = ml_dtypes.bfloat16 if dtype == "bf16" else np.float32
    ins = [(rng.standard_normal(x.shape) / np.sqrt(K)).astype(npdt), rng.standard_normal(w.shape).astype(npdt)]
    got = client.run(text, ins)[0]
    ref = oracle_run(text, ins)[0]
    assert_close(got, ref, RTOL_F32 if dtype == "f32" else RTOL_F32 * 10, "dot layouts")


@pytest.mark.parametrize("out", ["bf16", "f32"])
@pytest.mark.parametrize("V", [1001, 1000, 1024])
def test_f32_cotangent_feeding_two_dots(client, V, out):
    """An f32 value read by two dots with bf16 partners (the logits cotangent of an LM head: dX = g W^T,
    dW = x^T g).  With bf16 results it is stored rounded to bf16 (a padded row pitch when V % 8 != 0)
    and read in place, the results held to the bf16 bar; with f32 results the dots are f32-accurate
    (split into bf16 pieces) and held to the f32 bar."""
    b = Builder("jit_cotangent")
    x = b.arg((256, 96), "bf16")
    w = b.arg((V, 96), "bf16")
    z = b.arg((256, V), "f32")
    g = b.exp(z) * 0.5 - z                       # f32 [256, V], produced by a loop kernel
    dx = b.dot_general(g, w, contract=([1], [0]), out_dtype=out)
    dw = b.dot_general(g, x, contract=([0], [0]), out_dtype=out)
    text = b.text([dx, dw])
    rng = np.random.default_rng(V)
    ins = [(rng.standard_normal((256, 96)) * 0.3).astype(ml_dtypes.bfloat16),
           (rng.standard_normal((V, 96)) * 0.3).astype(ml_dtypes.bfloat16),
           (rng.standard_normal((256, V)) * 0.5).astype(np.float32)]
    outs = client.run(text, ins)
    refs = oracle_run(text, ins)
    for o, r, name in zip(outs, refs, ("dx", "dw")):
        assert_close(np.asarray(o, np.float32), np.asarray(r, np.float32), RTOL_F32 if out == "f32" else RTOL_BF16, name)


@pytest.mark.parametrize("splitk", [True, False])
def test_weight_gradient_dot_split_k(client, splitk, monkeypatch):
    """dW = x^T dy with a bf16 result: few output tiles, K = 4096 rows, so the compiler gives the dot
    an f32 split-K workspace (or, disabled, one CTA per tile)."""
    if not splitk:
        monkeypatch.setenv("B200_GEMM_NO_SPLITK", "1")
    b = Builder("jit_dw")
    x = b.arg((4096, 384), "bf16")
    dy = b.arg((4096, 512), "bf16")
    dw = b.dot_general(x, dy, contract=([0], [0]), out_dtype="bf16")
    text = b.text([dw])
    rng = np.random.default_rng(3)
    ins = [(rng.standard_normal((4096, 384)) / 64).astype(ml_dtypes.bfloat16),
           rng.standard_normal((4096, 512)).astype(ml_dtypes.bfloat16)]
    got = client.run(text, ins)[0]
    ref = oracle_run(text, ins)[0]
    assert_close(np.asarray(got, np.float32), np.asarray(ref, np.float32), RTOL_BF16, "dW")


@pytest.mark.parametrize("mn", [True, False])
def test_batched_dot_mn_major_operands(client, mn, monkeypatch):
    """Batched A^T B with both operands MN-major ([b, K, M] and [b, K, N]) against the oracle, and the
    same program with MN-major reads disabled (operands copied K-major)."""
    if not mn:
        monkeypatch.setenv("B200_GEMM_NO_MN", "1")
    b = Builder("jit_bmn")
    x = b.arg((6, 192, 136), "bf16")
    w = b.arg((6, 192, 264), "bf16")
    y = b.dot_general(x, w, batch=([0], [0]), contract=([1], [1]), out_dtype="f32")
    text = b.text([y])
    rng = np.random.default_rng(5)
    ins = [(rng.standard_normal((6, 192, 136)) / 14).astype(ml_dtypes.bfloat16),
           rng.standard_normal((6, 192, 264)).astype(ml_dtypes.bfloat16)]
    got = client.run(text, ins)[0]
    ref = oracle_run(text, ins)[0]
    assert_close(got, ref, RTOL_F32 * 10, "batched mn dot")


def test_psum_single_rank_known_answer(client):
    """smoke.cc:24-40: one rank, all-reduce of [1,2,3,4] is the identity."""
    p = configs.psum_program(4, 1, with_inputs=False)
    out = client.run(p.text, [np.array([1, 2, 3, 4], np.float32)])[0]
    np.testing.assert_array_equal(out, [1, 2, 3, 4])


def test_integer_index_work_bit_exact(client):
    b = Builder("jit_ints")
    x = b.arg((64, 33), "i32")
    io = b.iota((64, 33), 1)
    m = b.compare(x, io, "GE")
    s = b.select(m, x, io)
    r = b.reduce(s, [1], "max")
    c = b.reduce(b.convert(m, "i32"), [0], "add")
    text = b.text([m, s, r, c])
    xv = (np.arange(64 * 33, dtype=np.int32).reshape(64, 33) * 7919) % 61 - 20
    outs = client.run(text, [xv])
    refs = oracle_run(text, [xv])
    for o, rr in zip(outs, refs):
        assert o.dtype == rr.dtype
        np.testing.assert_array_equal(o, rr)


def test_elementwise_and_reductions_vs_oracle(client):
    b = Builder("jit_mix")
    x = b.arg((64, 96), "bf16")
    y = b.arg((96,), "f32")
    xf = b.convert(x, "f32")
    z = b.tanh(xf * 0.5 + y) - b.exp(b.sqrt(b.maximum(xf, 0.0)))
    m = b.compare(b.iota((64, 96), 0), b.iota((64, 96), 1), "LT")
    w = b.select(m, z, b.const(0.0, "f32", (64, 96)))
    text = b.text([b.convert(w, "bf16"), b.sum(w, 1), b.max(w, 0), b.sum(w, [0, 1])])
    rng = np.random.default_rng(1)
    ins = [rng.standard_normal((64, 96)).astype(ml_dtypes.bfloat16), rng.standard_normal(96).astype(np.float32)]
    outs = client.run(text, ins)
    refs = oracle_run(text, ins)
    assert_close(outs[0].astype(np.float32), refs[0].astype(np.float32), RTOL_BF16, "bf16 out")
    for o, r in zip(outs[1:], refs[1:]):
        assert_close(o, r, RTOL_F32, "reduction")


def test_tanh_f32_within_4_ulp(client):
    # a tanh whose result is used as such (not only through 1 +- tanh) compiles to CUDA's tanhf:
    # every binade from 2^-30 to 2^6, signed zeros, infinities and NaN, within 4 ulp of float64
    rng = np.random.default_rng(5)
    mag = np.exp2(rng.uniform(-30, 6, 1 << 20))
    x = (mag * rng.choice([-1.0, 1.0], mag.size)).astype(np.float32)
    x[:6] = [0.0, -0.0, np.inf, -np.inf, np.nan, 0.55]
    b = Builder("jit_tanh")
    a = b.arg(x.shape, "f32")
    y = client.run(b.text([b.tanh(a)]), [x])[0]
    ref = np.tanh(x.astype(np.float64))
    assert np.isnan(y[4]) and np.array_equal(np.signbit(y[:2]), [False, True]) and list(y[2:4]) == [1.0, -1.0]
    fin = np.isfinite(ref)
    ulp = np.abs(y[fin].astype(np.float64) - ref[fin]) / np.spacing(np.abs(ref[fin]).astype(np.float32))
    assert ulp.max() <= 4.0, f"tanh max error {ulp.max():.2f} ulp"


def test_embedding_take_and_scatter_add(client):
    b = Builder("jit_embed")
    table = b.arg((100, 16), "f32")
    ids = b.arg((4, 8), "i32")
    g = b.take(table, ids)                     # [4, 8, 16]
    base = b.const(0.0, "f32", (100, 16))
    s = b.scatter_add(base, ids, g * 2.0)
    text = b.text([g, s])
    rng = np.random.default_rng(2)
    ins = [rng.standard_normal((100, 16)).astype(np.float32), rng.integers(0, 100, (4, 8)).astype(np.int32)]
    outs = client.run(text, ins)
    refs = oracle_run(text, ins)
    np.testing.assert_array_equal(outs[0], refs[0])
    assert_close(outs[1], refs[1], RTOL_F32, "scatter")


def test_wrong_argument_shape_is_invalid_argument(client):
    exe = client.compile(configs.gemm_program(64, 64, 64, dtype="f32", with_inputs=False).text)
    bad = client.buffer_from_host(np.zeros((64, 32), np.float32))
    good = client.buffer_from_host(np.zeros((64, 64), np.float32))
    with pytest.raises(pjrt.PjrtError) as e:
        exe.execute([bad, good])
    assert e.value.code_name == "INVALID_ARGUMENT"
    with pytest.raises(pjrt.PjrtError) as e:
        exe.execute([good])
    assert e.value.code_name == "INVALID_ARGUMENT"
    exe.destroy()


def test_compile_error_names_the_op(client):
    text = """
module @m {
  func.func public @main(%arg0: tensor<8xf32>) -> (tensor<8xf32>) {
    %0 = stablehlo.fft %arg0, type = FFT, length = [8] : (tensor<8xf32>) -> tensor<8xf32>
    return %0 : tensor<8xf32>
  }
}
"""
    with pytest.raises(pjrt.PjrtError) as e:
        client.compile(text)
    assert e.value.code_name == "INVALID_ARGUMENT" and "jam compile" in e.value.message and "fft" in e.value.message


def test_repeated_execution_reuses_executable(client):
    p = configs.attention_program(B=1, H=2, S=256, causal=False, seed=4)
    exe = client.compile(p.text)
    bufs = [client.buffer_from_host(x) for x in p.inputs]
    first = exe.execute(bufs)[0].to_numpy()
    for _ in range(5):
        again = exe.execute(bufs)[0].to_numpy()
        np.testing.assert_array_equal(again.view(np.uint16), first.view(np.uint16))
    exe.destroy()


def test_repeated_executions_replay_a_cuda_graph(client, lib_path):
    """An execution whose buffers sit at the addresses of an earlier one is captured once and then
    replayed as a CUDA graph; every replay gives the eager result and the oracle's."""
    import ctypes
    lib = ctypes.CDLL(lib_path)
    lib.b200_graph_stats.restype = ctypes.c_longlong
    p = configs.mlp_program(seed=3)
    exe = client.compile(p.text)
    bufs = [client.buffer_from_host(x) for x in p.inputs]
    cap0, rep0 = lib.b200_graph_stats(0), lib.b200_graph_stats(1)
    results = []
    for _ in range(6):
        outs = exe.execute(bufs)
        results.append([o.to_numpy() for o in outs])
        for o in outs:
            o.delete()
    assert lib.b200_graph_stats(0) > cap0 and lib.b200_graph_stats(1) > rep0
    for r in results[1:]:
        for a, b in zip(results[0], r):
            np.testing.assert_array_equal(a, b)
    refs = oracle_run(p.text, p.inputs)
    for o, r in zip(results[-1], refs):
        assert_close(np.asarray(o, np.float32), np.asarray(r, np.float32), RTOL_F32 * 10, "mlp step via graph")
    for b in bufs:
        b.delete()
    exe.destroy()


def test_fresh_scalar_arguments_still_replay_the_graph(client, lib_path):
    """A training loop passes new scalar buffers every step (a step count, bias corrections) and
    gets a new scalar loss back: those small values are staged at fixed addresses, so the
    executions keep replaying one captured graph -- and each replay sees its own scalars."""
    import ctypes
    lib = ctypes.CDLL(lib_path)
    lib.b200_graph_stats.restype = ctypes.c_longlong
    b = Builder("jit_scalar_step")
    x, w, c = b.arg((512, 256), "f32"), b.arg((256, 256), "f32"), b.arg((), "f32")
    h = x
    for _ in range(4):                                   # enough launches for graph capture
        h = b.tanh(b.matmul(h, w)) * b.broadcast_to(c, (512, 256))
    text = b.text([h, b.sum(b.sum(h, 1), 0)])
    rng = np.random.default_rng(0)
    xs, ws = rng.standard_normal((512, 256), dtype=np.float32), rng.standard_normal((256, 256), dtype=np.float32) / 16
    exe = client.compile(text)
    bx, bw = client.buffer_from_host(xs), client.buffer_from_host(ws)
    rep0 = lib.b200_graph_stats(1)
    for step in range(8):
        cv = np.array(0.5 + 0.25 * step, np.float32)
        bc = client.buffer_from_host(cv)
        h_out, loss = exe.execute([bx, bw, bc])
        ref = oracle_run(text, [xs, ws, cv])
        assert_close(h_out.to_numpy(), ref[0], RTOL_F32 * 10, f"step {step}")
        assert abs(float(loss.to_numpy()) - float(ref[1])) <= 1e-4 * max(1.0, abs(float(ref[1])))
        for o in (h_out, loss, bc):
            o.delete()
    assert lib.b200_graph_stats(1) - rep0 >= 5
    exe.destroy()


@pytest.mark.parametrize("dt", ["bf16", "f32"])
def test_head_gradients_assembled_into_rows(client, dt):
    """The attention backward's dq / dk / dv ([B, H, S, D]) transposed to [B*S, H*D] and placed side
    by side by pad + add (what autodiff of a slice produces), plus a sliced, offset read: the
    vectorised walk reads four consecutive elements per lane through reshape / transpose / pad /
    slice.  Pure data movement, so bit-exact against the oracle."""
    B, H, S, D = 2, 3, 64, 32
    b = Builder("jit_assemble")
    parts = [b.arg((B, H, S, D), dt) for _ in range(3)]
    rows = []
    for i, p in enumerate(parts):
        r = b.reshape(b.transpose(p, (0, 2, 1, 3)), (B * S, H * D))
        rows.append(b.pad(r, 0.0, [0, i * H * D], [0, (2 - i) * H * D]))
    out = rows[0] + rows[1] + rows[2]
    shifted = b.slice(out, [0, 4], [B * S, 3 * H * D - 4])           # aligned offset
    odd = b.slice(out, [0, 1], [B * S, 3 * H * D - 7])               # unaligned offset
    text = b.text([out, shifted * 2.0, odd])
    rng = np.random.default_rng(9)
    npdt = ml_dtypes.bfloat16 if dt == "bf16" else np.float32
    ins = [rng.standard_normal((B, H, S, D)).astype(npdt) for _ in range(3)]
    outs = client.run(text, ins)
    refs = oracle_run(text, ins)
    for o, r in zip(outs, refs):
        np.testing.assert_array_equal(np.asarray(o, np.float32), np.asarray(r, np.float32))


@pytest.mark.parametrize("V", [1001, 1003, 1024])
def test_unaligned_dot_output_read_by_fused_kernels(client, V):
    """A tensor-core dot whose f32 result rows are not 16-byte multiples (the LM head's logits) is
    written with a padded row pitch; the row kernels (logsumexp, softmax cotangent), a column
    reduction and an elementwise consumer read it through that pitch."""
    b = Builder("jit_lm_head")
    x = b.arg((256, 96), "bf16")
    w = b.arg((V, 96), "bf16")
    lg = b.dot_general(x, w, contract=([1], [1]), out_dtype="f32")        # [256, V] f32
    mx = b.max(lg, 1, keepdims=True)
    z = lg - b.broadcast_to(mx, lg.shape)
    lse = b.log(b.sum(b.exp(z), 1, keepdims=True))
    sm = b.exp(z - b.broadcast_to(lse, lg.shape))
    col = b.sum(lg, 0)
    text = b.text([b.reshape(lse, (256,)), b.convert(sm, "bf16"), col, lg * 2.0])
    rng = np.random.default_rng(V)
    ins = [(rng.standard_normal((256, 96)) * 0.5).astype(ml_dtypes.bfloat16),
           (rng.standard_normal((V, 96)) * 0.5).astype(ml_dtypes.bfloat16)]
    outs = client.run(text, ins)
    refs = oracle_run(text, ins)
    for o, r, name, tol in zip(outs, refs, ("lse", "softmax", "colsum", "2*logits"), (1e-4, RTOL_BF16, 1e-4, 1e-4)):
        assert o.shape == r.shape
        assert_close(np.asarray(o, np.float32), np.asarray(r, np.float32), tol, name)


def test_tanh_read_only_as_one_plus_minus_t(client):
    """tanh(u) whose readers only form 1 + t, 1 - t and 1 - t*t (the tanh-GELU derivative) is
    computed as 1 - 2 / (e^(2u) + 1): those readers agree with the oracle to an absolute 1e-6."""
    b = Builder("jit_tanh_near_one")
    u = b.arg((4096,), "f32")
    t = b.tanh(u)
    text = b.text([1.0 + t, 1.0 - t * t, 2.0 - t])
    rng = np.random.default_rng(2)
    x = np.concatenate([rng.standard_normal(4000) * 3, [0.0, -0.0, 1e-8, -1e-8, 20.0, -20.0, np.inf, -np.inf]]).astype(np.float32)
    x = np.concatenate([x, rng.standard_normal(4096 - x.size)]).astype(np.float32)
    outs = client.run(text, [x])
    refs = oracle_run(text, [x])
    for o, r in zip(outs, refs):
        np.testing.assert_allclose(o, r, atol=1e-6, rtol=0)


@pytest.mark.parametrize("shape,dims", [((640, 96), [0]), ((3, 50, 48), [0, 1]), ((4096, 768), [0])])
def test_sibling_column_reductions_share_a_kernel(client, lib_path, shape, dims):
    """Reductions of one operand shape over the same leading dims (dbeta = sum dy, dgamma =
    sum dy * xhat, plus a max with a non-identity init) run as one kernel reading dy once."""
    import ctypes
    b = Builder("jit_ln_param_grads")
    dy = b.arg(shape, "bf16")
    xh = b.arg(shape, "f32")
    dyf = b.convert(dy, "f32")
    s1 = b.sum(dyf, dims)
    s2 = b.sum(dyf * xh, dims)
    m3 = b.max(xh, dims)
    text = b.text([s1, s2, m3])
    lib = ctypes.CDLL(lib_path)
    buf = ctypes.create_string_buffer(1 << 16)
    t = text.encode()
    assert lib.b200_compile_report(t, len(t), 1, 0, buf, len(buf)) == 0
    assert "reduce x3" in buf.value.decode(), buf.value.decode()
    rng = np.random.default_rng(len(shape))
    ins = [rng.standard_normal(shape).astype(ml_dtypes.bfloat16), rng.standard_normal(shape).astype(np.float32)]
    outs = client.run(text, ins)
    refs = oracle_run(text, ins)
    for o, r in zip(outs, refs):
        assert_close(o, r, RTOL_F32 * 10, "column reductions")


@pytest.mark.parametrize("V", [1000, 50257])
def test_one_hot_pick_is_a_gather(client, lib_path, V):
    """sum_j (label == j ? z[j] : 0) inside a row group (the cross-entropy's picked logit) is read
    as z[label] -- exact, and 0 for labels outside the row."""
    rows = 64
    b = Builder("jit_pick")
    lg = b.arg((rows, V), "f32")
    lab = b.arg((rows,), "i32")
    mx = b.max(lg, 1, keepdims=True)
    z = lg - b.broadcast_to(mx, lg.shape)
    onehot = b.compare(b.broadcast_in_dim(lab, (rows, V), [0]), b.iota((rows, V), 1), "EQ")
    picked = b.sum(b.select(onehot, z, b.const(0.0, "f32", (rows, V))), 1)
    lse = b.log(b.sum(b.exp(z), 1))
    text = b.text([picked, lse - picked])
    rng = np.random.default_rng(V)
    x = rng.standard_normal((rows, V)).astype(np.float32)
    labels = rng.integers(0, V, rows).astype(np.int32)
    labels[:4] = [-1, V, 0, V - 1]
    outs = client.run(text, [x, labels])
    refs = oracle_run(text, [x, labels])
    np.testing.assert_array_equal(outs[0], refs[0])
    assert_close(outs[1], refs[1], RTOL_F32, "loss")


def test_split_k_dot_read_by_a_fused_kernel(client):
    """A bf16 dot computed split-K whose readers are generated kernels keeps its f32 sums and the
    readers round them to bf16 (no separate rounding pass): same values as rounding first."""
    b = Builder("jit_dw_update")
    x = b.arg((4096, 384), "bf16")
    dy = b.arg((4096, 512), "bf16")
    p = b.arg((384, 512), "f32")
    dw = b.dot_general(x, dy, contract=([0], [0]), out_dtype="bf16")
    upd = p - 0.5 * b.convert(dw, "f32")
    text = b.text([upd, b.sum(b.convert(dw, "f32"), [0])])
    rng = np.random.default_rng(13)
    ins = [(rng.standard_normal((4096, 384)) * 0.1).astype(ml_dtypes.bfloat16),
           (rng.standard_normal((4096, 512)) * 0.1).astype(ml_dtypes.bfloat16),
           rng.standard_normal((384, 512)).astype(np.float32)]
    outs = client.run(text, ins)
    refs = oracle_run(text, ins)
    assert_close(outs[0], refs[0], 1e-2, "update")
    assert_close(outs[1], refs[1], 1e-2, "column sum")


def test_memory_spaces_and_placement(client):
    """Each device has HBM ("device", default) and page-locked host memory ("pinned_host"): a buffer
    placed in pinned_host lives in host memory (IsOnCpu), copies between the spaces keep the bytes,
    and an executable refuses a pinned_host argument instead of reading host memory as if it were HBM."""
    mems = client.memories()
    kinds = [client.memory_kind(m) for m in mems]
    assert kinds == ["device", "pinned_host"]
    hbm, host = mems
    assert client.memory_id(hbm) != client.memory_id(host)
    x = (np.arange(4 * 257) % 13 - 6).astype(np.float32).reshape(4, 257)
    hb = client.buffer_from_host(x, memory=host)
    assert hb.is_on_cpu() and hb.memory() == host
    np.testing.assert_array_equal(hb.to_numpy(), x)
    db = hb.copy_to_memory(hbm)
    assert not db.is_on_cpu() and db.memory() == hbm
    np.testing.assert_array_equal(db.to_numpy(), x)
    back = db.copy_to_memory(host)
    assert back.is_on_cpu()
    np.testing.assert_array_equal(back.to_numpy(), x)
    b = Builder("jit_neg")
    y = b.arg((4, 257), "f32")
    exe = client.compile(b.text([-y]))
    np.testing.assert_array_equal(exe.execute([db])[0].to_numpy(), -x)
    with pytest.raises(pjrt.PjrtError) as e:
        exe.execute([hb])
    assert e.value.code_name == "INVALID_ARGUMENT" and "pinned_host" in e.value.message
    for buf in (hb, db, back):
        buf.delete()
    exe.destroy()


def test_external_references_defer_the_free(client):
    x = np.arange(64, dtype=np.int32)
    b = client.buffer_from_host(x)
    b.add_external_ref(+1)
    b.mark_deleted()
    assert b.is_deleted()
    b.add_external_ref(-1)                      # the last reference releases the storage
    with pytest.raises(pjrt.PjrtError):
        b.add_external_ref(-1)                  # no references left
    b.delete()


def test_device_lookup_and_default_assignment(client):
    devs = client.devices()
    assert client.lookup_device(0) == devs[0]
    with pytest.raises(pjrt.PjrtError):
        client.lookup_device(len(devs))
    assert client.default_device_assignment(1, 1) == [0]


@pytest.mark.parametrize("rows,cols", [(8192, 768), (300, 72)])
def test_rounded_sibling_column_sums(client, lib_path, rows, cols):
    """Two column sums over the same rows, each rounded to bf16 as a program output (a LayerNorm's
    parameter gradients as the all_reduce receives them): one merged reduction kernel and one launch
    for both roundings, results against the oracle at the bf16 bar."""
    import ctypes
    b = Builder("jit_rounded_sums")
    dy = b.arg((rows, cols), "f32")
    xh = b.arg((rows, cols), "f32")
    g = b.convert(b.reduce(dy * xh, [0]), "bf16")
    s = b.convert(b.reduce(dy, [0]), "bf16")
    text = b.text([g, s])
    lib = ctypes.CDLL(lib_path)
    buf = ctypes.create_string_buffer(1 << 16)
    assert lib.b200_compile_report(text.encode(), len(text), 1, 0, buf, len(buf)) == 0
    rep = buf.value.decode()
    assert "reduce x2" in rep and f"loop tensor<{cols}xbf16> x2" in rep, rep
    rng = np.random.default_rng(rows + cols)
    ins = [rng.standard_normal((rows, cols)).astype(np.float32), rng.standard_normal((rows, cols)).astype(np.float32)]
    outs = client.run(text, ins)
    refs = oracle_run(text, ins)
    for o, r, name in zip(outs, refs, ("dgamma", "dbeta")):
        assert_close(np.asarray(o, np.float32), np.asarray(r, np.float32), RTOL_BF16, name)
