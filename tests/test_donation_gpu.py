"""Buffer donation through the PJRT C API on a B200 (jax.jit's donate_argnums: `tf.aliasing_output`
and `jax.buffer_donor` on @main's arguments).

A donated argument is deleted by Execute; a result aliased to it is written into its memory when
the plan can do that safely (a loop kernel reading the argument only at the element it writes),
else into a fresh buffer while the argument's memory goes back to the pool.  Listing an argument
in PJRT_ExecuteOptions.non_donatable_input_indices keeps it.  Results are the same either way."""
import numpy as np
import pytest

from conftest import RTOL_BF16, RTOL_F32, assert_close
from oracle.interp import run as oracle_run
from pjrt_b200 import configs, pjrt
from pjrt_b200.shlo import Builder

pytestmark = pytest.mark.gpu


def _update_program(n=4096, d=256):
    """p, g, m -> (p - 0.01 (0.9 m + g), 0.9 m + g): results aliased to p and m, g a buffer donor."""
    b = Builder("jit_donated_update")
    p, g, m = b.arg((n, d), "f32"), b.arg((n, d), "f32"), b.arg((n, d), "f32")
    m1 = m * 0.9 + g
    return b.text([p - m1 * 0.01, m1], aliases={0: 0, 2: 1}, donors=(1,))


def _inputs(seed, n=4096, d=256):
    rng = np.random.default_rng(seed)
    return [rng.standard_normal((n, d), dtype=np.float32) for _ in range(3)]


def test_donated_arguments_are_updated_in_place(client):
    text = _update_program()
    exe = client.compile(text)
    host = _inputs(0)
    bufs = [client.buffer_from_host(x) for x in host]
    addr = [b.device_pointer() for b in bufs]
    p_out, m_out = exe.execute(bufs)
    assert all(b.is_deleted() for b in bufs)
    assert p_out.device_pointer() == addr[0] and m_out.device_pointer() == addr[2]
    ref = oracle_run(text, host)
    assert_close(p_out.to_numpy(), ref[0], RTOL_F32, "p")
    assert_close(m_out.to_numpy(), ref[1], RTOL_F32, "m")
    with pytest.raises(pjrt.PjrtError):
        exe.execute(bufs)                               # a donated buffer cannot be used again
    exe.destroy()


def test_repeated_in_place_steps_match_the_copying_steps(client):
    """Ten steps feeding each result back as the next argument, donated (in place, CUDA-graph
    replays at fixed addresses) and not donated: bit-identical results."""
    text = _update_program()
    exe = client.compile(text)
    host = _inputs(1)

    def run(donate):
        p, m = client.buffer_from_host(host[0]), client.buffer_from_host(host[2])
        for step in range(10):
            g = client.buffer_from_host(host[1] * (1.0 + 0.1 * step))
            p, m = exe.execute([p, g, m], non_donatable=() if donate else (0, 1, 2))
        return p.to_numpy(), m.to_numpy()

    a, b = run(True), run(False)
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_array_equal(a[1], b[1])
    exe.destroy()


def test_non_donatable_arguments_stay_live(client):
    text = _update_program()
    exe = client.compile(text)
    host = _inputs(2)
    bufs = [client.buffer_from_host(x) for x in host]
    addr = [b.device_pointer() for b in bufs]
    p_out, m_out = exe.execute(bufs, non_donatable=(0, 1, 2))
    assert not any(b.is_deleted() for b in bufs)
    assert p_out.device_pointer() not in addr and m_out.device_pointer() not in addr
    np.testing.assert_array_equal(bufs[0].to_numpy(), host[0])
    ref = oracle_run(text, host)
    assert_close(p_out.to_numpy(), ref[0], RTOL_F32, "p")
    exe.destroy()


def test_result_that_cannot_be_in_place_gets_a_fresh_buffer(client):
    """The donated argument is read transposed: the result is written to a fresh buffer and the
    argument is still deleted (its memory released after the execution)."""
    b = Builder("jit_alias_t")
    x, y = b.arg((512, 512), "f32"), b.arg((512, 512), "f32")
    text = b.text([b.transpose(x, (1, 0)) + y], aliases={0: 0})
    exe = client.compile(text)
    host = _inputs(3, 512, 512)[:2]
    bufs = [client.buffer_from_host(v) for v in host]
    addr = bufs[0].device_pointer()
    out, = exe.execute(bufs)
    assert bufs[0].is_deleted() and not bufs[1].is_deleted()
    assert out.device_pointer() != addr
    np.testing.assert_array_equal(out.to_numpy(), host[0].T + host[1])
    exe.destroy()


def test_donating_a_buffer_with_external_references_fails(client):
    exe = client.compile(_update_program(64, 64))
    bufs = [client.buffer_from_host(x) for x in _inputs(4, 64, 64)]
    bufs[0].add_external_ref(1)
    with pytest.raises(pjrt.PjrtError, match="external references"):
        exe.execute(bufs)
    bufs[0].add_external_ref(-1)
    assert not bufs[0].is_deleted()
    exe.destroy()


def test_donating_a_buffer_passed_twice_fails(client):
    exe = client.compile(_update_program(64, 64))
    x = client.buffer_from_host(_inputs(5, 64, 64)[0])
    with pytest.raises(pjrt.PjrtError, match="also passed as argument"):
        exe.execute([x, x, x])
    assert not x.is_deleted()
    exe.destroy()


def test_donated_gpt_step_matches_the_copying_step(client):
    """Two GPT-2 train steps with params and moments donated (AdamW in place) against the same
    program without donation (equal within the bf16 bar: gradient sums that go through atomics may
    differ in their last bits from run to run), and the first step's loss against the oracle."""
    kw = dict(batch=2, layers=2, d=128, heads=2, mlp=512, vocab=512, seq=256)
    plain = configs.gpt2_program(**kw)
    don = configs.gpt2_program(**kw, donate=True, with_inputs=False)
    n_state = 3 * plain.meta["n_tensors"]

    def steps(text, donate):
        exe = client.compile(text)
        state = [client.buffer_from_host(x) for x in plain.inputs[:n_state]]
        rest = [client.buffer_from_host(x) for x in plain.inputs[n_state:]]
        losses = []
        for _ in range(2):
            outs = exe.execute(state + rest)
            state, loss = outs[:n_state], outs[n_state]
            losses.append(float(loss.to_numpy()))
        res = [s.to_numpy() for s in state]
        exe.destroy()
        return losses, res

    la, ra = steps(don.text, True)
    lb, rb = steps(plain.text, False)
    for x, y in zip(la, lb):
        assert abs(x - y) <= 1e-3 * abs(y)
    for k, (x, y) in enumerate(zip(ra, rb)):
        assert_close(np.asarray(x, np.float32), np.asarray(y, np.float32), RTOL_BF16, f"state {k}")
    ref_loss = float(oracle_run(plain.text, plain.inputs)[-1])
    assert abs(la[0] - ref_loss) <= RTOL_BF16 * abs(ref_loss)
