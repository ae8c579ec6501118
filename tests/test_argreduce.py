"""argmax / argmin: the two-operand reduce (values, iota) that jnp.argmax / argmin lower to
(reference: DetectArgReduce, src/jam/ops/reduce.mm:29-43).  Index results are held bit-exact
against the oracle, which folds the reducer body in index order; the oracle itself is pinned to
numpy's argmax / argmin (first index of the extreme; a NaN counts as the extreme)."""
import ml_dtypes
import numpy as np
import pytest

from oracle.interp import run as oracle_run
from pjrt_b200.shlo import Builder
from test_compiler import report


def program(shape, axis, kind, dtype):
    b = Builder("jit_argreduce")
    x = b.arg(shape, dtype)
    v, i = b.argreduce(x, axis, kind)
    return b.text([v, i])


def inputs(shape, dtype, seed):
    rng = np.random.default_rng(seed)
    if dtype == "i32":
        return rng.integers(-50, 50, shape, dtype=np.int32)      # many ties
    x = rng.standard_normal(shape).astype(np.float32)
    if x.ndim == 2 and x.shape[0] > 4 and x.shape[1] > 8:
        x[1, 3] = x[1, 7] = 40.0           # tie on the max: the first index
        x[2, :] = -np.inf                  # all -inf: index 0
        x[3, 5] = np.nan                   # a NaN is the extreme
        x[4, 2] = -40.0
        x[4, 6] = -40.0                    # tie on the min
    return x.astype(ml_dtypes.bfloat16) if dtype == "bf16" else x


@pytest.mark.parametrize("kind", ["max", "min"])
def test_oracle_argreduce_matches_numpy(kind):
    x = inputs((9, 33), "f32", 1)
    text = program((9, 33), 1, kind, "f32")
    v, i = oracle_run(text, [x])
    ref_i = np.argmax(x, 1) if kind == "max" else np.argmin(x, 1)
    np.testing.assert_array_equal(i, ref_i)
    ref_v = np.take_along_axis(x, ref_i[:, None], 1)[:, 0]
    np.testing.assert_array_equal(np.isnan(v), np.isnan(ref_v))
    np.testing.assert_array_equal(v[~np.isnan(v)], ref_v[~np.isnan(ref_v)])


def test_argreduce_compiles_to_one_kernel(lib_path):
    rc, rep = report(lib_path, program((64, 1000), 1, "max", "f32"))
    steps = [l for l in rep.splitlines() if l.startswith("  [")]
    assert rc == 0 and len(steps) == 1 and "argmax tensor<64x1000xf32>" in steps[0], rep
    rc, rep = report(lib_path, program((300, 12), 0, "min", "bf16"))
    assert rc == 0 and "argmin" in rep, rep


@pytest.mark.gpu
@pytest.mark.parametrize("shape,axis", [((64, 1000), 1), ((9, 33), 1), ((300, 12), 0), ((4, 5, 6), 1)])
@pytest.mark.parametrize("kind", ["max", "min"])
@pytest.mark.parametrize("dtype", ["f32", "bf16", "i32"])
def test_argreduce_bit_exact(client, shape, axis, kind, dtype):
    text = program(shape, axis, kind, dtype)
    x = inputs(shape, dtype, sum(shape) + axis)
    outs = client.run(text, [x])
    refs = oracle_run(text, [x])
    np.testing.assert_array_equal(outs[1], refs[1])
    a, r = np.asarray(outs[0], np.float64), np.asarray(refs[0], np.float64)
    np.testing.assert_array_equal(np.isnan(a), np.isnan(r))
    np.testing.assert_array_equal(a[~np.isnan(a)], r[~np.isnan(r)])
