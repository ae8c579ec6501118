"""Attention inside a differentiated program: the forward chain and its VJP (dQ, dK, dV dots and the
softmax cotangent between them) become one flash forward (+lse2) and one flash-backward step.

The matcher accepts the cotangent only when it evaluates, on sample rows, to
scale * mask * P * (dP - rowsum(P * dP)); a program whose "backward" computes something else keeps
the unfused path.  GPU cases compare the gradients with the numpy oracle on the same text."""
import math

import ml_dtypes
import numpy as np
import pytest

from conftest import RTOL_BF16, assert_close
from oracle.interp import run as oracle_run
from pjrt_b200 import configs
from pjrt_b200.shlo import Builder, grad
from test_compiler import report

BF16 = ml_dtypes.bfloat16


def attention_grad_program(B=2, H=2, S=256, D=64, causal=True, broken=False):
    """loss = sum(attention(Q, K, V) * W); outputs dQ, dK, dV (and the loss).  With `broken`, the
    backward is written by hand with the row-sum term left out (not a softmax VJP)."""
    b = Builder("jit_attn_grad")
    q, k, v, w = (b.arg((B, H, S, D), "bf16") for _ in range(4))
    s = b.dot_general(q, k, batch=([0, 1], [0, 1]), contract=([3], [3]), out_dtype="f32") * (1.0 / math.sqrt(D))
    if causal:
        mask = b.broadcast_in_dim(b.compare(b.iota((S, S), 0), b.iota((S, S), 1), "GE"), (B, H, S, S), [2, 3])
        s = b.select(mask, s, b.const(-np.inf, "f32", s.shape))
    m = b.stop_gradient(b.max(s, 3, keepdims=True))
    e = b.exp(s - m)
    p = e / b.sum(e, 3, keepdims=True)
    p16 = b.convert(p, "bf16")
    o = b.dot_general(p16, v, batch=([0, 1], [0, 1]), contract=([3], [2]), out_dtype="bf16")
    loss = b.sum(b.convert(o, "f32") * b.convert(w, "f32"), [0, 1, 2, 3])
    if not broken:
        dq, dk, dv = grad(b, loss, [q, k, v])
        return b.text([dq, dk, dv, loss])
    g = w                                                         # d loss / d O
    dv = b.dot_general(p16, g, batch=([0, 1], [0, 1]), contract=([2], [2]), out_dtype="bf16")
    dp = b.convert(b.dot_general(g, v, batch=([0, 1], [0, 1]), contract=([3], [3]), out_dtype="bf16"), "f32")
    t = p * dp * (1.0 / math.sqrt(D))                             # missing "- rowsum(p * dp)"
    dq = b.dot_general(t, k, batch=([0, 1], [0, 1]), contract=([3], [2]), out_dtype="bf16")
    dk = b.dot_general(t, q, batch=([0, 1], [0, 1]), contract=([2], [2]), out_dtype="bf16")
    return b.text([dq, dk, dv, loss])


def _inputs(B, H, S, D, seed):
    rng = np.random.default_rng(seed)
    return [rng.standard_normal((B, H, S, D), dtype=np.float32).astype(BF16) for _ in range(4)]


@pytest.mark.parametrize("causal", [True, False])
def test_attention_vjp_becomes_flash_backward(lib_path, causal):
    rc, rep = report(lib_path, attention_grad_program(causal=causal))
    assert rc == 0, rep
    assert "attention_bwd" in rep and "+lse" in rep and "256x256" not in rep, rep


def test_a_wrong_cotangent_is_not_taken_for_a_softmax_vjp(lib_path):
    rc, rep = report(lib_path, attention_grad_program(broken=True))
    assert rc == 0, rep
    assert "attention_bwd" not in rep, rep


def test_gpt2_step_attention_runs_as_flash_forward_and_backward(lib_path):
    p = configs.gpt2_program(layers=1, d=128, heads=2, mlp=256, vocab=96, seq=256, batch=2, with_inputs=False)
    rc, rep = report(lib_path, p.text)
    assert rc == 0, rep
    assert "attention_bwd causal" in rep and "attention causal +lse" in rep and "256x256" not in rep, rep


@pytest.mark.gpu
@pytest.mark.parametrize("causal,S", [(True, 256), (False, 256), (True, 512)])
def test_attention_gradients_vs_oracle(client, causal, S):
    text = attention_grad_program(S=S, causal=causal)
    ins = _inputs(2, 2, S, 64, S + causal)
    outs = client.run(text, ins)
    refs = oracle_run(text, ins)
    for o, r, name in zip(outs[:3], refs[:3], ("dq", "dk", "dv")):
        assert_close(np.asarray(o, np.float32), np.asarray(r, np.float32), RTOL_BF16, name)
    assert_close(np.float32(outs[3]), np.float32(refs[3]), 1e-2, "loss")


@pytest.mark.gpu
def test_unmatched_backward_stays_correct(client):
    text = attention_grad_program(broken=True)
    ins = _inputs(2, 2, 256, 64, 7)
    outs = client.run(text, ins)
    refs = oracle_run(text, ins)
    for o, r, name in zip(outs[:3], refs[:3], ("dq", "dk", "dv")):
        assert_close(np.asarray(o, np.float32), np.asarray(r, np.float32), RTOL_BF16, name)


@pytest.mark.gpu
def test_gpt_step_with_flash_attention_vs_oracle(client):
    """One layer, head dim 64, seq 256: the decoder step whose attention runs as flash forward and
    backward, against the oracle (parameters bounded as in the tiny-step test; moments normwise)."""
    cfg = dict(layers=1, d=128, heads=2, mlp=256, vocab=96, seq=256)
    p = configs.gpt2_program(batch=2, **cfg)
    outs = client.run(p.text, p.inputs)
    refs = oracle_run(p.text, p.inputs)
    n = len(configs.gpt2_param_shapes(**cfg))
    assert_close(outs[-1], refs[-1], 1e-3, "loss")
    lr = 3e-4
    for i, (o, r) in enumerate(zip(outs[:-1], refs[:-1])):
        o32, r32 = np.asarray(o, np.float32), np.asarray(r, np.float32)
        if i < n:
            ulp = np.abs(r32) * 2.0 ** -7 + 1e-30
            assert np.all(np.abs(o32 - r32) <= 2.2 * lr + ulp), (i, float(np.max(np.abs(o32 - r32))))
        else:
            assert_close(o32, r32, 5e-2, f"moment {i}")
