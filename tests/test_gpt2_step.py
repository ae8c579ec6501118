"""The data-parallel decoder train step at a reduced size: forward, autodiff'd
backward, psum of gradients and AdamW, through the plugin vs the CPU oracle on the same text."""
import ml_dtypes
import numpy as np
import pytest

from conftest import RTOL_BF16, RTOL_F32, assert_close, rel_err
from oracle.interp import run as oracle_run, run_spmd
from pjrt_b200 import configs

TINY = dict(layers=2, d=64, heads=2, mlp=128, vocab=96, seq=64)


def tiny(batch=2, world=1, rank=0, with_inputs=True):
    return configs.gpt2_program(batch=batch, world=world, rank=rank, with_inputs=with_inputs, **TINY)


def test_tiny_gpt_step_oracle_dp_equivalence():
    """pmean over 2 ranks with half batches == one rank on the whole batch (CPU oracle)."""
    full = tiny(batch=4)
    p2 = tiny(batch=2, world=2, with_inputs=False)
    ids, tgt = full.inputs[-4], full.inputs[-3]
    shards = []
    for r in range(2):
        ins = list(full.inputs)
        ins[-4], ins[-3] = ids[2 * r:2 * r + 2], tgt[2 * r:2 * r + 2]
        shards.append(ins)
    ref = oracle_run(full.text, full.inputs)
    res = run_spmd(p2.text, shards)
    # gradients are bf16 (params are bf16), so a sum of two half-batch gradients differs from the
    # whole-batch gradient by bf16 rounding: every output is held to the bf16 bar
    for r in range(2):
        for i, (a, b) in enumerate(zip(res[r], ref)):
            assert_close(np.asarray(a, np.float32), np.asarray(b, np.float32), RTOL_BF16, f"rank {r} out {i}")


def test_tiny_gpt_loss_is_cross_entropy_of_a_near_uniform_model():
    p = tiny()
    loss = oracle_run(p.text, p.inputs)[-1]
    assert abs(float(loss) - np.log(TINY["vocab"])) < 0.1, float(loss)


@pytest.mark.gpu
def test_tiny_gpt_step_vs_oracle(client):
    p = tiny()
    outs = client.run(p.text, p.inputs)
    refs = oracle_run(p.text, p.inputs)
    n = len(configs.gpt2_param_shapes(**TINY))
    assert len(outs) == 3 * n + 1
    assert_close(outs[-1], refs[-1], 1e-3, "loss")
    lr = 3e-4
    for i, (o, r) in enumerate(zip(outs[:-1], refs[:-1])):
        o32, r32 = np.asarray(o, np.float32), np.asarray(r, np.float32)
        if i < n:
            # Adam's first step moves each weight by lr * sign(g) (+ decay): a gradient that rounds to
            # the other sign under bf16 moves it the other way, so bound the difference by 2 lr plus
            # one bf16 ulp of the weight rather than comparing updates normwise
            ulp = np.abs(r32) * 2.0 ** -7 + 1e-30
            assert np.all(np.abs(o32 - r32) <= 2.2 * lr + ulp), (i, float(np.max(np.abs(o32 - r32))))
        else:
            # first and second moments carry the (bf16) gradients: the bf16 bar, normwise
            assert_close(o32, r32, 5e-2, f"moment {i}")


@pytest.mark.gpu
def test_tiny_gpt_two_steps_loss_decreases(client):
    p = tiny(batch=4)
    exe = client.compile(p.text)
    bufs = [client.buffer_from_host(x) for x in p.inputs]
    n = len(configs.gpt2_param_shapes(**TINY))
    losses = []
    state = bufs[:3 * n]
    for step in range(1, 6):
        bc1 = np.array(1 - 0.9 ** step, np.float32)
        bc2 = np.array(1 - 0.95 ** step, np.float32)
        scal = [client.buffer_from_host(bc1), client.buffer_from_host(bc2)]
        outs = exe.execute(state + bufs[3 * n:3 * n + 2] + scal)
        losses.append(float(outs[-1].to_numpy()))
        state = outs[:3 * n]
    assert all(np.isfinite(losses)) and losses[-1] < losses[0], losses
    exe.destroy()
