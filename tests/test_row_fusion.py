"""Row groups: a reduction over the trailing axis and the values of the same rows that follow it
(LayerNorm, softmax, logsumexp) compile to one kernel in which a warp or a block owns a row.

Plan-level checks run without a GPU (b200_compile_report); the `gpu` cases compare the fused kernels
with the numpy oracle on the same seeded inputs, including the fallbacks (a read of another row's
reduction, rows too short to fuse) and reductions whose init value is not the identity."""
import ml_dtypes
import numpy as np
import pytest

from conftest import RTOL_BF16, RTOL_F32, assert_close
from oracle.interp import run as oracle_run
from pjrt_b200.shlo import Builder
from test_compiler import report

BF16 = ml_dtypes.bfloat16


def layernorm(rows, d, dtype="bf16", extra_outputs=False):
    b = Builder("jit_layernorm")
    x, g, bt = b.arg((rows, d), dtype), b.arg((d,), dtype), b.arg((d,), dtype)
    xf = b.convert(x, "f32")
    mu = b.mean(xf, -1, keepdims=True)
    xc = xf - b.broadcast_to(mu, xf.shape)
    var = b.mean(xc * xc, -1, keepdims=True)
    y = xc * b.broadcast_to(b.rsqrt(var + 1e-5), xf.shape) * b.broadcast_to(b.convert(g, "f32"), xf.shape) \
        + b.broadcast_to(b.convert(bt, "f32"), xf.shape)
    outs = [b.convert(y, dtype)]
    if extra_outputs:
        outs += [b.reshape(mu, (rows,)), xc]
    return b.text(outs)


def softmax(shape):
    b = Builder("jit_softmax")
    x = b.arg(shape, "f32")
    m = b.max(x, -1, keepdims=True)
    e = b.exp(x - b.broadcast_to(m, shape))
    s = b.sum(e, -1, keepdims=True)
    return b.text([e / b.broadcast_to(s, shape)])


def logsumexp(rows, n):
    b = Builder("jit_lse")
    x = b.arg((rows, n), "f32")
    m = b.max(x, 1, keepdims=True)
    lse = b.log(b.sum(b.exp(x - b.broadcast_to(m, x.shape)), 1)) + b.reshape(m, (rows,))
    return b.text([lse])


def steps(rep):
    return [l.strip() for l in rep.splitlines() if l.startswith("  [")]


def test_layernorm_is_one_row_kernel(lib_path):
    rc, rep = report(lib_path, layernorm(256, 768))
    assert rc == 0, rep
    st = steps(rep)
    assert len(st) == 1 and st[0].startswith("[0] row tensor<256x768xf32>"), rep


@pytest.mark.parametrize("shape", [(2, 4, 128, 128), (64, 1000), (32, 5003)])
def test_softmax_is_one_row_kernel(lib_path, shape):
    rc, rep = report(lib_path, softmax(shape))
    assert rc == 0, rep
    st = steps(rep)
    assert len(st) == 1 and st[0].startswith("[0] row"), rep


def test_logsumexp_is_one_row_kernel(lib_path):
    rc, rep = report(lib_path, logsumexp(1024, 50257))
    assert rc == 0, rep
    assert len(steps(rep)) == 1, rep


def test_row_group_ends_at_a_read_of_another_row(lib_path):
    b = Builder("jit_shift")
    x = b.arg((64, 256), "f32")
    mu = b.sum(x, 1)
    shifted = b.concatenate([b.slice(mu, [1], [64]), b.slice(mu, [0], [1])], 0)
    y = x - b.broadcast_in_dim(shifted, (64, 256), [0])
    rc, rep = report(lib_path, b.text([y]))
    assert rc == 0, rep
    st = steps(rep)
    assert len(st) == 2 and st[0].startswith("[0] row") and "loop" in st[1], rep


def test_row_fusion_can_be_disabled(lib_path, monkeypatch):
    monkeypatch.setenv("B200_NO_ROWFUSE", "1")
    rc, rep = report(lib_path, layernorm(256, 768))
    assert rc == 0 and "row" not in rep and rep.count("reduce") == 2, rep


# ------------------------------------------------------------------------------------------ GPU
def _ln_inputs(rows, d, dt, seed=0):
    rng = np.random.default_rng(seed)
    return [(rng.standard_normal((rows, d)) * 3 + 1).astype(dt), rng.standard_normal(d).astype(dt),
            rng.standard_normal(d).astype(dt)]


@pytest.mark.gpu
@pytest.mark.parametrize("rows,d,dtype", [(1024, 768, "bf16"), (300, 96, "f32"), (77, 2056, "f32"), (40, 33, "f32"),
                                        (37, 770, "bf16"), (9, 9001, "f32")])
def test_layernorm_vs_oracle(client, rows, d, dtype):
    text = layernorm(rows, d, dtype)
    ins = _ln_inputs(rows, d, BF16 if dtype == "bf16" else np.float32)
    out, = client.run(text, ins)
    ref, = oracle_run(text, ins)
    assert_close(out.astype(np.float32), ref.astype(np.float32), RTOL_BF16 if dtype == "bf16" else RTOL_F32, "layernorm")


@pytest.mark.gpu
def test_layernorm_intermediates_are_stored_when_read_outside(client):
    text = layernorm(512, 768, "f32", extra_outputs=True)
    ins = _ln_inputs(512, 768, np.float32, seed=3)
    outs = client.run(text, ins)
    refs = oracle_run(text, ins)
    assert [o.shape for o in outs] == [(512, 768), (512,), (512, 768)]
    for o, r, w in zip(outs, refs, ("y", "mean", "centered")):
        assert_close(o, r, RTOL_F32, w)


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(2, 4, 128, 128), (64, 1000), (32, 5003), (16, 8192), (3, 5, 2051)])
def test_softmax_vs_oracle(client, shape):
    text = softmax(shape)
    x = (np.random.default_rng(5).standard_normal(shape) * 4).astype(np.float32)
    out, = client.run(text, [x])
    ref, = oracle_run(text, [x])
    assert_close(out, ref, RTOL_F32, "softmax")
    np.testing.assert_allclose(out.sum(-1), 1.0, rtol=1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("rows,n", [(600, 50257), (600, 1000), (64, 50257)])
def test_logsumexp_vs_oracle(client, rows, n):
    text = logsumexp(rows, n)
    x = (np.random.default_rng(7).standard_normal((rows, n)) * 2).astype(np.float32)
    out, = client.run(text, [x])
    ref, = oracle_run(text, [x])
    assert_close(out, ref, RTOL_F32, "logsumexp")


@pytest.mark.gpu
def test_read_of_another_row_falls_back_and_stays_correct(client):
    b = Builder("jit_shift")
    x = b.arg((64, 256), "f32")
    mu = b.sum(x, 1)
    shifted = b.concatenate([b.slice(mu, [1], [64]), b.slice(mu, [0], [1])], 0)
    text = b.text([x - b.broadcast_in_dim(shifted, (64, 256), [0])])
    xv = np.random.default_rng(2).standard_normal((64, 256)).astype(np.float32)
    out, = client.run(text, [xv])
    ref, = oracle_run(text, [xv])
    assert_close(out, ref, RTOL_F32, "shifted")


@pytest.mark.gpu
@pytest.mark.parametrize("rowfuse", [True, False])
@pytest.mark.parametrize("shape,axis", [((256, 640), 1), ((16, 9000), 1), ((640, 48), 0)])
def test_reduce_with_non_identity_init(client, monkeypatch, rowfuse, shape, axis):
    """StableHLO applies the init value once per output; a kernel that starts every thread's
    partial at the init value would add it once per thread."""
    if not rowfuse:
        monkeypatch.setenv("B200_NO_ROWFUSE", "1")
    b = Builder("jit_init")
    x = b.arg(shape, "f32")
    s = b.reduce(x, [axis], "add", init=1.5)
    m = b.reduce(x, [axis], "max", init=2.0)
    text = b.text([s, m])
    xv = np.random.default_rng(4).standard_normal(shape).astype(np.float32)
    outs = client.run(text, [xv])
    np.testing.assert_allclose(outs[0], xv.sum(axis) + 1.5, rtol=1e-4, atol=1e-3)
    np.testing.assert_array_equal(outs[1], np.maximum(xv.max(axis), 2.0))


@pytest.mark.gpu
def test_integer_row_max_is_bit_exact(client):
    b = Builder("jit_imax")
    x = b.arg((512, 300), "i32")
    m = b.max(x, 1, keepdims=True)
    y = x - b.broadcast_to(m, (512, 300))
    text = b.text([y, b.reshape(m, (512,))])
    xv = np.random.default_rng(9).integers(-1 << 30, 1 << 30, (512, 300), dtype=np.int32)
    outs = client.run(text, [xv])
    refs = oracle_run(text, [xv])
    for o, r in zip(outs, refs):
        np.testing.assert_array_equal(o, r)


@pytest.mark.gpu
@pytest.mark.parametrize("n", [1000, 5003])
def test_online_max_sum_edge_rows_match_two_pass(client, n):
    """max and sum(exp(x - max)) share one walk of the row; rows holding -inf (masked), all -inf,
    +inf or NaN must come out as the two-pass definition gives them."""
    b = Builder("jit_lse_edge")
    x = b.arg((8, n), "f32")
    m = b.max(x, 1, keepdims=True)
    s = b.sum(b.exp(x - b.broadcast_to(m, x.shape)), 1)
    text = b.text([s, b.reshape(m, (8,))])
    xv = np.random.default_rng(11).standard_normal((8, n)).astype(np.float32)
    xv[1, n // 2:] = -np.inf          # causal-style mask
    xv[2, :7] = -np.inf               # masked head of the row
    xv[3, :] = -np.inf                # fully masked
    xv[4, 17] = np.inf
    xv[5, 3] = np.nan
    xv[6] *= 30.0                     # large spread: many rescales
    outs = client.run(text, [xv])
    refs = oracle_run(text, [xv])
    for o, r in zip(outs, refs):
        np.testing.assert_array_equal(np.isnan(o), np.isnan(r))
        ok = ~np.isnan(r)
        np.testing.assert_allclose(o[ok], r[ok], rtol=RTOL_F32)
