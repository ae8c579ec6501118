"""The data-parallel decoder train step at a reduced size: forward, autodiff'd
backward, psum of gradients and AdamW, through the plugin vs the CPU oracle on the same text."""
import ml_dtypes
import numpy as np
import pytest

from conftest import RTOL_BF16, RTOL_F32, assert_close, rel_err
from oracle import torch_ref
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


HP = dict(lr=3e-4, b1=0.9, b2=0.95, eps=1e-8, wd=0.1)


def torch_gpt_step(inputs, layers, d, heads, mlp, vocab, seq, lr, b1, b2, eps, wd, gelu_c=0.044715):
    """The same train step written independently with torch autograd in float64 (oracle/torch_ref.py):
    pre-LN decoder, causal softmax attention, GELU(tanh) MLP, tied LM head, mean cross-entropy, AdamW
    with decay on the 2-D parameters."""
    return torch_ref.gpt2_step(inputs, layers, d, heads, mlp, vocab, seq, lr, b1, b2, eps, wd, gelu_c=gelu_c, dtype="f64")


def _scaled_f32_inputs(batch, scale, world=1):
    """Inputs of the f32 program with the weight matrices scaled up, so the attention softmax, GELU
    and LayerNorm work away from their near-linear regime and a wrong term in any of them shows."""
    p = configs.gpt2_program(batch=batch * world, dtype="f32", **TINY, **HP)
    ins = list(p.inputs)
    for i, (_, shp) in enumerate(configs.gpt2_param_shapes(**TINY)):
        if len(shp) == 2:
            ins[i] = ins[i] * np.float32(scale)
    return ins


def _normwise(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def _check_against_torch(outs, ref, ins, tol_grad):
    n = len(configs.gpt2_param_shapes(**TINY))
    assert abs(float(outs[-1]) - float(ref[-1])) <= 1e-6 * abs(float(ref[-1]))
    for i in range(n):          # the moments carry the gradients: m1 = 0.1 g, v1 = 0.05 g^2
        assert _normwise(outs[n + i], ref[n + i]) <= tol_grad, ("m", i)
        assert _normwise(outs[2 * n + i], ref[2 * n + i]) <= 2 * tol_grad, ("v", i)
    # the parameter update is AdamW applied to the program's own moments (elements whose gradient
    # is near eps make a comparison with the torch parameters themselves noisy)
    bc1, bc2 = float(ins[3 * n + 2]), float(ins[3 * n + 3])
    for i, (_, shp) in enumerate(configs.gpt2_param_shapes(**TINY)):
        p0 = np.asarray(ins[i], np.float64)
        m1, v1 = np.asarray(outs[n + i], np.float64), np.asarray(outs[2 * n + i], np.float64)
        decay = HP["wd"] if len(shp) == 2 else 0.0
        exp = p0 - HP["lr"] * ((m1 / bc1) / (np.sqrt(v1 / bc2) + HP["eps"]) + decay * p0)
        assert np.abs(np.asarray(outs[i], np.float64) - exp).max() <= 1e-6 * max(np.abs(p0).max(), 1.0), ("p", i)


def test_tiny_gpt_f32_step_matches_independent_torch_autograd():
    """The program the plugin runs (here its f32 form) is the GPT-2 train step: the oracle's loss,
    gradients (through the AdamW moments) and update agree with a float64 torch autograd step."""
    ins = _scaled_f32_inputs(batch=2, scale=10.0)
    text = configs.gpt2_program(batch=2, dtype="f32", with_inputs=False, **TINY, **HP).text
    _check_against_torch(oracle_run(text, ins), torch_gpt_step(ins, **TINY, **HP), ins, tol_grad=2e-5)


def test_tiny_gpt_f32_dp_step_is_pmean_of_the_whole_batch():
    """Two ranks with half batches each (shard_map + psum / 2) give the whole batch's torch step."""
    ins = _scaled_f32_inputs(batch=2, scale=10.0, world=2)
    text = configs.gpt2_program(batch=2, world=2, dtype="f32", with_inputs=False, **TINY, **HP).text
    ref = torch_gpt_step(ins, **TINY, **HP)
    ids, tgt = ins[-4], ins[-3]
    shards = []
    for r in range(2):
        part = list(ins)
        part[-4], part[-3] = ids[2 * r:2 * r + 2], tgt[2 * r:2 * r + 2]
        shards.append(part)
    for outs in run_spmd(text, shards):
        _check_against_torch(outs, ref, ins, tol_grad=2e-5)


def test_planted_mistake_in_the_torch_step_is_detected():
    """Sensitivity of the check above: the same comparison against a torch step whose GELU lacks
    its cubic term fails by orders of magnitude (the mistake is planted in the CPU reference)."""
    ins = _scaled_f32_inputs(batch=2, scale=10.0)
    text = configs.gpt2_program(batch=2, dtype="f32", with_inputs=False, **TINY, **HP).text
    outs = oracle_run(text, ins)
    bad = torch_gpt_step(ins, **TINY, **HP, gelu_c=0.0)
    n = len(configs.gpt2_param_shapes(**TINY))
    assert max(_normwise(outs[n + i], bad[n + i]) for i in range(n)) > 100 * 2e-5


def test_tiny_gpt_bf16_step_near_torch_autograd():
    """The config's own bf16 program: its gradients stay within bf16 pipeline error of float64."""
    p = tiny()
    outs = oracle_run(p.text, p.inputs)
    ref = torch_gpt_step(p.inputs, **TINY, **HP)
    n = len(configs.gpt2_param_shapes(**TINY))
    assert abs(float(outs[-1]) - float(ref[-1])) <= 1e-3 * abs(float(ref[-1]))
    for i in range(n):
        assert _normwise(outs[n + i], ref[n + i]) <= 3e-2, i


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
