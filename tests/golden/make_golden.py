"""Generates the golden fixtures that pin the numpy oracle (oracle/interp.py) to an independent
implementation.

The reference ships no golden vectors for its compute ops (its 125-case jax-CPU oracle was never
committed, docs/ops.md:7-10 of the reference) and jax is not installed here, so the expected outputs
come from PyTorch's CPU kernels, computed from the same seeded inputs the StableHLO programs take:
  attention  : torch.nn.functional.scaled_dot_product_attention in fp32 on the bf16 inputs
  MLP step   : torch autograd of the same 2-layer ReLU / softmax-CE model, one SGD step
  GEMM       : fp64 matmul of the bf16 / f32 operands

    python tests/golden/make_golden.py      # rewrites tests/golden/*.npz
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "mccl-jax_b200"))

from pjrt_b200 import configs  # noqa: E402


def f32(a):
    return torch.tensor(np.asarray(a, dtype=np.float32))


def attention(causal):
    p = configs.attention_program(B=1, H=2, S=256, D=64, causal=causal, seed=3)
    q, k, v = (f32(x) for x in p.inputs)
    o = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=causal).numpy()
    return dict(q=p.inputs[0].view(np.uint16), k=p.inputs[1].view(np.uint16), v=p.inputs[2].view(np.uint16), out=o)


def mlp():
    p = configs.mlp_program(batch=32, din=64, hidden=48, classes=10, lr=0.01, seed=5)
    W1, b1, W2, b2, x, y = (torch.tensor(a) for a in p.inputs)
    for t in (W1, b1, W2, b2):
        t.requires_grad_(True)
    logits = torch.relu(x @ W1 + b1) @ W2 + b2
    loss = torch.nn.functional.cross_entropy(logits, y.long())
    loss.backward()
    outs = [loss.detach().numpy()] + [(w - 0.01 * w.grad).detach().numpy() for w in (W1, b1, W2, b2)]
    d = {f"in{i}": a for i, a in enumerate(p.inputs)}
    d.update({f"out{i}": o for i, o in enumerate(outs)})
    return d


def gemm(dtype):
    p = configs.gemm_program(M=96, N=80, K=64, dtype=dtype, seed=7)
    a, b = (np.asarray(x, dtype=np.float64) for x in p.inputs)
    store = (lambda x: x.view(np.uint16)) if dtype == "bf16" else (lambda x: x)
    return dict(a=store(p.inputs[0]), b=store(p.inputs[1]), out=(a @ b).astype(np.float32))


def main():
    np.savez_compressed(os.path.join(HERE, "attention_causal.npz"), **attention(True))
    np.savez_compressed(os.path.join(HERE, "attention_full.npz"), **attention(False))
    np.savez_compressed(os.path.join(HERE, "mlp_step.npz"), **mlp())
    np.savez_compressed(os.path.join(HERE, "gemm_bf16.npz"), **gemm("bf16"))
    np.savez_compressed(os.path.join(HERE, "gemm_f32.npz"), **gemm("f32"))
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
