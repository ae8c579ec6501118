"""ORACLE (test infrastructure only): the benchmark workloads restated in torch on the host CPU.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs may import this
module; the plugin never routes through it.  The north star times jaxlib's CPU PJRT backend (XLA:CPU,
compiled f32 code on all host cores) as the reported CPU baseline; jax is not installed on this image,
so the same computations are written here with torch's CPU kernels (f32, all host threads), and in
float64 as an independent check of the programs the plugin compiles:

  * `gpt2_step`: the GPT-2 data-parallel AdamW train step of BASELINE config 4 -- pre-LN decoder,
    causal softmax attention, GELU(tanh) MLP, tied LM head, mean cross-entropy, AdamW with decay on
    the 2-D parameters -- over the same argument list the StableHLO program takes
    (mccl-jax_b200/pjrt_b200/configs.py `gpt2_program` / `gpt2_inputs`).  It mirrors the
    reference's DP driver loop (temp/dp_train.py:77-108: forward, grad, pmean, optimizer update).
  * `attention`: softmax(Q K^T * scale [causal]) V in f32, the dot_general ->
    softmax -> dot_general chain the reference lowers (src/jam/ops/linalg.mm:47-105,
    src/jam/ops/elementwise.mm:71-89).
"""
from __future__ import annotations

import os

import numpy as np


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def gpt2_param_shapes(layers, d, heads, mlp, vocab, seq):
    """Parameter names and shapes in the program's argument order (the same list configs.py
    builds; restated so this module does not import the package under test)."""
    shapes = [("wte", (vocab, d)), ("wpe", (seq, d))]
    for l in range(layers):
        shapes += [(f"h{l}.ln1_g", (d,)), (f"h{l}.ln1_b", (d,)), (f"h{l}.w_qkv", (d, 3 * d)), (f"h{l}.b_qkv", (3 * d,)),
                   (f"h{l}.w_proj", (d, d)), (f"h{l}.b_proj", (d,)), (f"h{l}.ln2_g", (d,)), (f"h{l}.ln2_b", (d,)),
                   (f"h{l}.w_fc", (d, mlp)), (f"h{l}.b_fc", (mlp,)), (f"h{l}.w_fc2", (mlp, d)), (f"h{l}.b_fc2", (d,))]
    shapes += [("lnf_g", (d,)), ("lnf_b", (d,))]
    return shapes


def gpt2_step(inputs, layers, d, heads, mlp, vocab, seq, lr, b1, b2, eps, wd, gelu_c=0.044715, dtype="f64"):
    """One train step on `inputs` (params..., m..., v..., ids, targets, bc1, bc2) with torch autograd in
    `dtype` ("f64" or "f32").  Returns (new params..., new m..., new v..., loss) as numpy arrays, like
    the program.  (A pmean over data-parallel shards of the batch equals this step on the whole
    batch, so it is also the reference for the multi-rank program.)"""
    import torch
    tdt = torch.float64 if dtype == "f64" else torch.float32
    shapes = gpt2_param_shapes(layers, d, heads, mlp, vocab, seq)
    n = len(shapes)
    ndt = np.float64 if dtype == "f64" else np.float32
    P = {nm: torch.tensor(np.asarray(inputs[i], ndt), dtype=tdt, requires_grad=True) for i, (nm, _) in enumerate(shapes)}
    ids = torch.tensor(np.asarray(inputs[3 * n], np.int64))
    tgt = torch.tensor(np.asarray(inputs[3 * n + 1], np.int64))
    bc1, bc2 = float(inputs[3 * n + 2]), float(inputs[3 * n + 3])
    B, S = ids.shape
    H, Dh = heads, d // heads

    def ln(x, g, bias):
        xc = x - x.mean(-1, keepdim=True)
        return xc * torch.rsqrt((xc * xc).mean(-1, keepdim=True) + 1e-5) * g + bias

    x = (P["wte"][ids] + P["wpe"][None]).reshape(B * S, d)
    causal = torch.tril(torch.ones(S, S, dtype=torch.bool))
    for l in range(layers):
        w = lambda k: P[f"h{l}.{k}"]
        qkv = ln(x, w("ln1_g"), w("ln1_b")) @ w("w_qkv") + w("b_qkv")
        q, k, v = [qkv[:, i * d:(i + 1) * d].reshape(B, S, H, Dh).transpose(1, 2) for i in range(3)]
        s = ((q @ k.transpose(-1, -2)) / np.sqrt(Dh)).masked_fill(~causal, float("-inf"))
        o = (torch.softmax(s, -1) @ v).transpose(1, 2).reshape(B * S, d)
        x = x + o @ w("w_proj") + w("b_proj")
        f = ln(x, w("ln2_g"), w("ln2_b")) @ w("w_fc") + w("b_fc")
        x = x + (0.5 * f * (1 + torch.tanh(np.sqrt(2 / np.pi) * (f + gelu_c * f ** 3)))) @ w("w_fc2") + w("b_fc2")
    logits = ln(x, P["lnf_g"], P["lnf_b"]) @ P["wte"].T
    loss = torch.nn.functional.cross_entropy(logits, tgt.reshape(-1))
    loss.backward()
    newp, newm, newv = [], [], []
    with torch.no_grad():
        for i, (nm, shp) in enumerate(shapes):
            g, pv = P[nm].grad, P[nm].detach()
            m1 = b1 * torch.tensor(np.asarray(inputs[n + i], ndt), dtype=tdt) + (1 - b1) * g
            v1 = b2 * torch.tensor(np.asarray(inputs[2 * n + i], ndt), dtype=tdt) + (1 - b2) * g * g
            decay = wd if len(shp) == 2 else 0.0
            newp.append((pv - lr * ((m1 / bc1) / (torch.sqrt(v1 / bc2) + eps) + decay * pv)).numpy())
            newm.append(m1.numpy())
            newv.append(v1.numpy())
    return newp + newm + newv + [loss.detach().numpy()]


def attention(q, k, v, causal, scale=None):
    """softmax(q k^T * scale [causal]) v in f32 on the CPU for numpy or torch q, k, v [..., S, d]."""
    import torch
    q, k, v = (torch.as_tensor(np.asarray(x, np.float32)) if not isinstance(x, torch.Tensor) else x.float()
               for x in (q, k, v))
    scale = 1.0 / np.sqrt(q.shape[-1]) if scale is None else scale
    return torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=bool(causal), scale=scale)
