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


# ----------------------------------------------------------------------------- C4 GPT-2 DP train step
GPT2_SMALL = dict(layers=12, d=768, heads=12, mlp=3072, vocab=50257, seq=1024)


def gpt2_param_shapes(layers, d, heads, mlp, vocab, seq):
    shapes = [("wte", (vocab, d)), ("wpe", (seq, d))]
    for l in range(layers):
        shapes += [(f"h{l}.ln1_g", (d,)), (f"h{l}.ln1_b", (d,)), (f"h{l}.w_qkv", (d, 3 * d)), (f"h{l}.b_qkv", (3 * d,)),
                   (f"h{l}.w_proj", (d, d)), (f"h{l}.b_proj", (d,)), (f"h{l}.ln2_g", (d,)), (f"h{l}.ln2_b", (d,)),
                   (f"h{l}.w_fc", (d, mlp)), (f"h{l}.b_fc", (mlp,)), (f"h{l}.w_fc2", (mlp, d)), (f"h{l}.b_fc2", (d,))]
    shapes += [("lnf_g", (d,)), ("lnf_b", (d,))]
    return shapes


def gpt2_program(layers=12, d=768, heads=12, mlp=3072, vocab=50257, seq=1024, batch=8, world=1,
                 lr=3e-4, b1=0.9, b2=0.95, eps=1e-8, wd=0.1, seed=0, rank=0, with_inputs=True, dtype="bf16",
                 donate=False):
    """One data-parallel AdamW step of a GPT-2-style decoder (pre-LN, GELU(tanh) MLP, tied LM head).

    Params bf16 (replicated), AdamW moments f32; the batch [world*batch, seq] of token ids is sharded
    over ranks with shard_map (SPMDFullToShardShape); gradients are psum'd (all_reduce) and divided by
    the world size (pmean), as temp/dp_train.py:80-83 does.  Adam bias corrections come in as host
    scalars (dp_train.py:74-76).  Returns (new params..., new m..., new v..., pmean loss).
    `dtype` is the parameter / activation type (bf16, the config's; "f32" gives the same program
    without the 16-bit roundings, which tests compare with an independent autograd implementation).
    `donate`: params and moments are donated, each aliased to its updated value (what
    jax.jit(step, donate_argnums=(params, opt_state)) emits), so the update runs in place.
    """
    b = Builder("jit_gpt2_dp_step", num_partitions=world)
    shapes = gpt2_param_shapes(layers, d, heads, mlp, vocab, seq)
    P = {n: b.arg(s, dtype) for n, s in shapes}
    M = {n: b.arg(s, "f32") for n, s in shapes}
    V = {n: b.arg(s, "f32") for n, s in shapes}
    ids_full = b.arg((world * batch, seq), "i32")
    tgt_full = b.arg((world * batch, seq), "i32")
    bc1 = b.arg((), "f32")
    bc2 = b.arg((), "f32")
    ids = b.shard(ids_full, (batch, seq)) if world > 1 else ids_full
    tgt = b.shard(tgt_full, (batch, seq)) if world > 1 else tgt_full
    Dh = d // heads
    ntok = batch * seq

    def layernorm(x, g, bias):
        xf = b.convert(x, "f32")
        mu = b.mean(xf, -1, keepdims=True)
        xc = xf - b.broadcast_to(mu, xf.shape)
        var = b.mean(xc * xc, -1, keepdims=True)
        inv = b.rsqrt(var + 1e-5)
        y = xc * b.broadcast_to(inv, xf.shape) * b.broadcast_to(b.convert(g, "f32"), xf.shape) \
            + b.broadcast_to(b.convert(bias, "f32"), xf.shape)
        return b.convert(y, dtype)

    def linear(x2, w, bias):                       # x2 [ntok, din] bf16 -> [ntok, dout] bf16
        y = b.dot_general(x2, w, contract=([1], [0]), out_dtype=dtype)
        return y + b.broadcast_to(bias, y.shape)

    def gelu(x):                                   # tanh approximation, in f32
        xf = b.convert(x, "f32")
        inner = (xf + 0.044715 * (xf * xf * xf)) * math.sqrt(2.0 / math.pi)
        return b.convert(0.5 * xf * (1.0 + b.tanh(inner)), dtype)

    x = b.take(P["wte"], ids) + b.broadcast_to(P["wpe"], (batch, seq, d))   # [B, S, d] bf16
    x = b.reshape(x, (ntok, d))
    for l in range(layers):
        p = lambda n: P[f"h{l}.{n}"]
        h = layernorm(x, p("ln1_g"), p("ln1_b"))
        qkv = linear(h, p("w_qkv"), p("b_qkv"))                             # [ntok, 3d]
        heads_of = []
        for i in range(3):
            part = b.slice(qkv, [0, i * d], [ntok, (i + 1) * d])
            heads_of.append(b.transpose(b.reshape(part, (batch, seq, heads, Dh)), (0, 2, 1, 3)))   # [B,H,S,Dh]
        q, k, v = heads_of
        s = b.dot_general(q, k, batch=([0, 1], [0, 1]), contract=([3], [3]), out_dtype="f32")
        s = s * (1.0 / math.sqrt(Dh))
        mask = b.broadcast_in_dim(b.compare(b.iota((seq, seq), 0), b.iota((seq, seq), 1), "GE"), s.shape, [2, 3])
        s = b.select(mask, s, b.const(-np.inf, "f32", s.shape))
        m = b.stop_gradient(b.max(s, 3, keepdims=True))
        e = b.exp(s - b.broadcast_to(m, s.shape))
        pr = e / b.broadcast_to(b.sum(e, 3, keepdims=True), s.shape)
        o = b.dot_general(b.convert(pr, dtype), v, batch=([0, 1], [0, 1]), contract=([3], [2]), out_dtype=dtype)
        o = b.reshape(b.transpose(o, (0, 2, 1, 3)), (ntok, d))
        x = x + linear(o, p("w_proj"), p("b_proj"))
        h = layernorm(x, p("ln2_g"), p("ln2_b"))
        x = x + linear(gelu(linear(h, p("w_fc"), p("b_fc"))), p("w_fc2"), p("b_fc2"))
    x = layernorm(x, P["lnf_g"], P["lnf_b"])
    logits = b.dot_general(x, P["wte"], contract=([1], [1]), out_dtype="f32")      # tied head [ntok, V]
    mx = b.stop_gradient(b.max(logits, 1, keepdims=True))
    z = logits - b.broadcast_to(mx, logits.shape)
    lse = b.log(b.sum(b.exp(z), 1, keepdims=True))
    t2 = b.reshape(tgt, (ntok,))
    onehot = b.compare(b.broadcast_in_dim(t2, (ntok, vocab), [0]), b.iota((ntok, vocab), 1), "EQ")
    picked = b.sum(b.select(onehot, z, b.const(0.0, "f32", z.shape)), 1, keepdims=True)
    loss = b.mean(lse - picked, [0, 1])
    names = [n for n, _ in shapes]
    grads = grad(b, loss, [P[n] for n in names])
    outs_p, outs_m, outs_v = [], [], []
    inv_world = 1.0 / world
    for n, g in zip(names, grads):
        if world > 1:
            g = b.all_reduce(g, world)
        gf = b.convert(g, "f32") * inv_world
        m1 = b1 * M[n] + (1.0 - b1) * gf
        v1 = b2 * V[n] + (1.0 - b2) * (gf * gf)
        pf = b.convert(P[n], "f32")
        mhat = m1 / b.broadcast_to(bc1, m1.shape)
        vhat = v1 / b.broadcast_to(bc2, v1.shape)
        decay = wd if P[n].ndim == 2 else 0.0
        upd = mhat / (b.sqrt(vhat) + eps) + (decay * pf if decay else 0.0)
        outs_p.append(b.convert(pf - lr * upd, dtype))
        outs_m.append(m1)
        outs_v.append(v1)
    lo = b.all_reduce(loss, world) * inv_world if world > 1 else loss
    n_state = 3 * len(shapes)
    text = b.text(outs_p + outs_m + outs_v + [lo], aliases={k: k for k in range(n_state)} if donate else None)
    inputs = []
    if with_inputs:
        inputs = gpt2_inputs(shapes, batch, seq, vocab, seed=seed, rank=rank, dtype=dtype)
    n_params = sum(int(np.prod(s)) for _, s in shapes)
    flops_per_token = 6 * (12 * layers * d * d + d * vocab) + 12 * layers * seq * d
    return Program(b.name, text, inputs, flops=float(flops_per_token) * ntok,
                   meta=dict(n_params=n_params, tokens=ntok, n_tensors=len(shapes), layers=layers, d=d,
                             vocab=vocab, seq=seq, batch=batch, world=world))


def gpt2_inputs(shapes, batch, seq, vocab, seed=0, rank=0, step=1, b1=0.9, b2=0.95, dtype="bf16"):
    """Params ~N(0, 0.02) bf16 (LN gains 1, biases 0) from `seed` (same on every rank); zero moments;
    token ids / targets uniform in [0, vocab) from seed 1000 + rank (dp_train.py:50)."""
    rng = np.random.default_rng(seed)
    params, ms, vs = [], [], []
    for n, s in shapes:
        if n.endswith("_g"):
            a = np.ones(s, np.float32)
        elif len(s) == 1:
            a = np.zeros(s, np.float32)
        else:
            a = rng.standard_normal(s, dtype=np.float32) * 0.02
        params.append(a.astype(np_dtype(dtype)))
        ms.append(np.zeros(s, np.float32))
        vs.append(np.zeros(s, np.float32))
    brng = np.random.default_rng(1000 + rank)
    ids = brng.integers(0, vocab, (batch, seq)).astype(np.int32)
    tgt = brng.integers(0, vocab, (batch, seq)).astype(np.int32)
    bc1 = np.array(1 - b1 ** step, np.float32)
    bc2 = np.array(1 - b2 ** step, np.float32)
    return params + ms + vs + [ids, tgt, bc1, bc2]
