"""The five benchmark configurations as StableHLO programs plus their seeded synthetic inputs.

Each `*_program(...)` returns `Program(text, inputs, ...)`: `text` is the MLIR module the plugin
compiles, `inputs` a list of numpy arrays (bf16 arrays use ml_dtypes.bfloat16) in argument order.
Shapes and distributions follow the reference's configs: the MLP train step of temp/dp_train.py's
style (here the 784-512-10 classifier), the attention sweep of assets/benchmark_1.png at
[B=4,H=16,S,64], the dot_general sweep, the GPT-2-small data-parallel step and the psum sweep.
"""
from __future__ import annotations

import dataclasses
import math
from typing import List, Optional

import ml_dtypes
import numpy as np

from .shlo import Builder, grad

BF16 = ml_dtypes.bfloat16


@dataclasses.dataclass
class Program:
    name: str
    text: str
    inputs: List[np.ndarray]
    flops: float = 0.0          # algorithmic FLOPs of one execution
    bytes: float = 0.0          # algorithmic HBM bytes of one execution
    meta: dict = dataclasses.field(default_factory=dict)


def np_dtype(dt):
    return {"f32": np.float32, "bf16": BF16, "f16": np.float16, "i32": np.int32, "pred": np.bool_,
            "f64": np.float64, "i64": np.int64, "u32": np.uint32, "i8": np.int8, "u8": np.uint8}[dt]


# ----------------------------------------------------------------------------- C2 attention
def attention_program(B=4, H=16, S=512, D=64, causal=False, seed=0, dtype="bf16", with_inputs=True):
    """softmax(Q K^T / sqrt(d)) V with fp32 scores and softmax, as jax lowers a hand-written attention."""
    b = Builder(f"jit_attention_{'causal' if causal else 'full'}")
    q, k, v = (b.arg((B, H, S, D), dtype) for _ in range(3))
    s = b.dot_general(q, k, batch=([0, 1], [0, 1]), contract=([3], [3]), out_dtype="f32")
    s = s * (1.0 / math.sqrt(D))
    if causal:
        row = b.iota((S, S), 0)
        col = b.iota((S, S), 1)
        mask = b.broadcast_in_dim(b.compare(row, col, "GE"), (B, H, S, S), [2, 3])
        s = b.select(mask, s, b.const(-np.inf, "f32", s.shape))
    m = b.max(s, 3, keepdims=True)
    e = b.exp(s - m)
    p = e / b.sum(e, 3, keepdims=True)
    o = b.dot_general(b.convert(p, dtype), v, batch=([0, 1], [0, 1]), contract=([3], [2]), out_dtype=dtype)
    inputs = []
    if with_inputs:
        rng = np.random.default_rng(seed)
        inputs = [rng.standard_normal((B, H, S, D), dtype=np.float32).astype(np_dtype(dtype)) for _ in range(3)]
    flops = 4.0 * B * H * S * S * D * (0.5 if causal else 1.0)
    return Program(b.name, b.text([o]), inputs, flops=flops, bytes=4.0 * B * H * S * D * 2,
                   meta=dict(B=B, H=H, S=S, D=D, causal=causal))


# ----------------------------------------------------------------------------- C3 GEMM
def gemm_program(M=1024, N=1024, K=1024, batch=0, dtype="bf16", seed=0, with_inputs=True):
    """A[M,K] . B[K,N] with fp32 result (bf16 or fp32 inputs), optionally batched."""
    b = Builder(f"jit_gemm_{dtype}")
    if batch:
        a = b.arg((batch, M, K), dtype)
        c = b.arg((batch, K, N), dtype)
        o = b.dot_general(a, c, batch=([0], [0]), contract=([2], [1]), out_dtype="f32")
    else:
        a = b.arg((M, K), dtype)
        c = b.arg((K, N), dtype)
        o = b.dot_general(a, c, contract=([1], [0]), out_dtype="f32")
    inputs = []
    if with_inputs:
        rng = np.random.default_rng(seed)
        sh_a = (batch, M, K) if batch else (M, K)
        sh_b = (batch, K, N) if batch else (K, N)
        sc = 1.0 / math.sqrt(K)
        inputs = [(rng.standard_normal(sh_a, dtype=np.float32) * sc).astype(np_dtype(dtype)),
                  (rng.standard_normal(sh_b, dtype=np.float32) * sc).astype(np_dtype(dtype))]
    nb = max(batch, 1)
    return Program(b.name, b.text([o]), inputs, flops=2.0 * nb * M * N * K,
                   meta=dict(M=M, N=N, K=K, batch=batch, dtype=dtype))


# ----------------------------------------------------------------------------- C1 MLP train step
def glorot(rng, fan_in, fan_out):
    lim = math.sqrt(6.0 / (fan_in + fan_out))
    return rng.uniform(-lim, lim, (fan_in, fan_out)).astype(np.float32)


def mlp_program(batch=128, din=784, hidden=512, classes=10, lr=0.01, seed=0, with_inputs=True):
    """One SGD step of a 2-layer ReLU MLP with softmax cross-entropy: returns (loss, W1', b1', W2', b2')."""
    b = Builder("jit_mlp_step")
    W1 = b.arg((din, hidden)); b1 = b.arg((hidden,)); W2 = b.arg((hidden, classes)); b2 = b.arg((classes,))
    x = b.arg((batch, din)); y = b.arg((batch,), "i32")
    h = b.maximum(x @ W1 + b1, 0.0)
    logits = h @ W2 + b2
    m = b.max(logits, 1, keepdims=True)
    z = logits - m
    lse = b.log(b.sum(b.exp(z), 1, keepdims=True))
    logp = z - lse
    onehot = b.convert(b.compare(b.broadcast_in_dim(y, (batch, classes), [0]), b.iota((batch, classes), 1), "EQ"), "f32")
    loss = -b.mean(b.sum(logp * onehot, 1), 0)
    gW1, gb1, gW2, gb2 = grad(b, loss, [W1, b1, W2, b2])
    outs = [loss, W1 - lr * gW1, b1 - lr * gb1, W2 - lr * gW2, b2 - lr * gb2]
    inputs = []
    if with_inputs:
        rng = np.random.default_rng(seed)
        inputs = [glorot(rng, din, hidden), np.zeros(hidden, np.float32), glorot(rng, hidden, classes),
                  np.zeros(classes, np.float32), rng.standard_normal((batch, din), dtype=np.float32),
                  rng.integers(0, classes, batch).astype(np.int32)]
    fwd = 2.0 * batch * (din * hidden + hidden * classes)
    return Program(b.name, b.text(outs), inputs, flops=3 * fwd, meta=dict(batch=batch))


# ----------------------------------------------------------------------------- C5 psum sweep
def psum_program(n_elems, world, seed_rank=0, with_inputs=True):
    """shard_map(lambda x: psum(x, 'i')) over a [world*n] f32 array, one shard per device."""
    b = Builder("jit_psum", num_partitions=world)
    x = b.arg((world * n_elems,), "f32")
    xs = b.shard(x, (n_elems,))
    r = b.all_reduce(xs, world)
    o = b.unshard(r, (world * n_elems,))
    inputs = []
    if with_inputs:
        rng = np.random.default_rng(1000 + seed_rank)
        inputs = [rng.standard_normal(n_elems, dtype=np.float32)]
    return Program(b.name, b.text([o]), inputs, bytes=4.0 * n_elems, meta=dict(n=n_elems, world=world))
