"""The non-headline workloads of bench.py (`--workload dp | gemm | psum`), each printing one JSON line.

  dp    GPT-2-small data-parallel AdamW step through the PJRT C API: params,
        moments and the token batch stay on the device, step outputs feed the next step; device
        time from CUDA events the executor records (b200_exec_timer), max over ranks; tokens/s for
        the whole job, MFU against the measured dense bf16 peak (854.4 MFLOP/token, PaLM counting).
  gemm  dot_general sweep (config 3) through b200_gemm on HBM-resident operands.
  psum  all_reduce sweep (config 5) through the PJRT plugin, bus GB/s = bytes * 2(n-1)/n / time.
"""
from __future__ import annotations

import ctypes
import datetime
import json
import math
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "lib", "libpjrt_b200.so")


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def _client(world, rank, local):
    from pjrt_b200 import pjrt
    api = pjrt.Api(LIB)
    if world == 1:
        return pjrt.Client(api, device_ordinal=local), None
    import torch.distributed as dist
    port = int(os.environ.get("MASTER_PORT", "29500")) + 17
    store = dist.TCPStore(os.environ.get("MASTER_ADDR", "127.0.0.1"), port, world, rank == 0,
                          timeout=datetime.timedelta(seconds=120))

    def put(k, v):
        store.set(k, v)

    def get(k, ms):
        store.wait([k], datetime.timedelta(milliseconds=max(ms, 1)))
        return store.get(k)
    return pjrt.Client(api, node_id=rank, num_nodes=world, device_ordinal=local, kv_put=put, kv_get=get), store


def _max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_dp(a, world, rank, local):
    import torch
    from pjrt_b200 import configs
    lib = ctypes.CDLL(LIB)
    lib.b200_exec_timer.restype = ctypes.c_double
    cfg = dict(configs.GPT2_SMALL, layers=a.layers)
    batch = 8
    t0 = time.time()
    prog = configs.gpt2_program(batch=batch, world=world, rank=rank, **cfg)
    client, store = _client(world, rank, local)
    exe = client.compile(prog.text)
    compile_s = time.time() - t0
    n = prog.meta["n_tensors"]
    bufs = [client.buffer_from_host(x) for x in prog.inputs[:3 * n + 2]]
    state, data = bufs[:3 * n], bufs[3 * n:]

    def step(s):
        # the bias-correction scalars and last step's buffers are released once this step is
        # enqueued (stream-ordered frees), so steady-state steps reuse the same addresses
        bc = [client.buffer_from_host(np.array(1 - 0.9 ** s, np.float32)),
              client.buffer_from_host(np.array(1 - 0.95 ** s, np.float32))]
        outs = exe.execute(state + data + bc, wait=False)
        for b in bc + state:
            b.delete()
        state[:] = outs[:3 * n]
        return outs[-1]

    lib.b200_graph_stats.restype = ctypes.c_longlong
    losses = []
    s = 1
    for _ in range(a.warmup):
        loss = step(s)
        s += 1
        losses.append(float(loss.to_numpy()))
        loss.delete()
    if world > 1:
        torch.distributed.barrier()
    replays0 = lib.b200_graph_stats(1)
    lib.b200_exec_timer(0)
    t_wall = time.perf_counter()
    loss = None
    for _ in range(a.steps):
        if loss is not None:
            loss.delete()
        loss = step(s)
        s += 1
    last_loss = float(loss.to_numpy())
    loss.delete()
    replays = lib.b200_graph_stats(1) - replays0
    dev_ms = lib.b200_exec_timer(1)
    wall_ms = (time.perf_counter() - t_wall) * 1e3
    ms = _max_over_ranks(dev_ms / a.steps, world)
    tokens = batch * cfg["seq"] * world
    pk, src = _peaks()
    fl_tok = prog.flops / (batch * cfg["seq"])
    tps = tokens / (ms * 1e-3)
    mfu = fl_tok * tps / world / (pk["bf16_tflops"] * 1e12)
    if rank == 0:
        print(json.dumps({
            "metric": "DP train-step tokens/s (GPT-2 small, per-GPU batch 8 x 1024, AdamW)", "value": tps,
            "unit": "tokens/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded ids, N(0,0.02) params)",
            "config": {"workload": "gpt2-small DP step", "layers": cfg["layers"], "d_model": cfg["d"],
                       "heads": cfg["heads"], "vocab": cfg["vocab"], "seq_len": cfg["seq"], "per_gpu_batch": batch,
                       "global_batch": batch * world, "parallelism": f"dp{world}", "params": prog.meta["n_params"]},
            "roofline": {"bound": "tensor", "achieved": fl_tok * tps / world / 1e12, "peak": pk["bf16_tflops"],
                         "unit": "TFLOP/s", "frac": mfu, "peak_source": src + " dense bf16 (burst)",
                         "flops_per_token": fl_tok},
            "wall_ms_per_step": wall_ms / a.steps, "compile_s": compile_s, "graph_replays": replays,
            "loss_first": losses[0], "loss_last": last_loss}))
    for b in state + data:
        b.delete()
    exe.destroy()
    client.close()
    return 0


def run_gemm(a, world, rank, local):
    import torch
    lib = ctypes.CDLL(LIB)
    lib.b200_gemm.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int64] * 4 + [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    torch.cuda.set_device(local)
    st = torch.cuda.current_stream()
    flush = torch.empty(64 * 1024 * 1024, device="cuda")
    pk, src = _peaks()
    rows = []
    shapes = [(1, 1024, 13), (1, 4096, 13), (1, 8192, 13), (16, 2048, 13), (1, 1024, 11), (1, 4096, 11), (1, 8192, 11)]
    only = getattr(a, "only", "")
    custom = None
    if only.startswith("m"):                      # e.g. m8192n3072k768: one rectangular bf16 shape
        import re
        mm = re.fullmatch(r"m(\d+)n(\d+)k(\d+)", only)
        custom = tuple(int(x) for x in mm.groups())
        shapes = [(1, custom, 13)]
    for batch, n, ab in shapes:
        if only and custom is None and only != f"b{batch}-{n}-{'bf16' if ab == 13 else 'f32'}":
            continue
        M, N, K = n if custom else (n, n, n)
        dt = torch.bfloat16 if ab == 13 else torch.float32
        A = (torch.randn(batch, M, K, device="cuda") / math.sqrt(K)).to(dt)
        B = (torch.randn(batch, N, K, device="cuda") / math.sqrt(K)).to(dt)
        C = torch.empty(batch, M, N, device="cuda")
        f = lambda: lib.b200_gemm(A.data_ptr(), B.data_ptr(), C.data_ptr(), batch, M, N, K, ab, 11,
                                  ctypes.c_void_p(st.cuda_stream))
        for _ in range(a.warmup):
            f()
        ts = []
        for _ in range(a.steps if ab == 13 else max(2, a.steps // 4)):
            flush.zero_()
            e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
            e0.record(st)
            f()
            e1.record(st)
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        ms = sorted(ts)[len(ts) // 2]
        tf = 2.0 * batch * M * N * K / (ms * 1e-3) / 1e12
        rows.append({"batch": batch, "M=N=K": n if not custom else f"{M}x{N}x{K}", "inputs": "bf16" if ab == 13 else "f32",
                     "ms": round(ms, 4), "tflops": round(tf, 1), "frac_of_peak": round(tf / pk["bf16_tflops"], 3)})
        del A, B, C
    heads = [r for r in rows if r["M=N=K"] == 8192 and r["inputs"] == "bf16"]
    head = heads[0] if heads else rows[0]
    print(json.dumps({"metric": "dot_general TFLOP/s (bf16 -> f32, 8192^3)", "value": head["tflops"], "unit": "TFLOP/s",
                      "n_gpus": 1, "higher_is_better": True, "dtype": "bf16", "data": "synthetic N(0,1)/sqrt(K)",
                      "config": {"workload": "gemm sweep", "l2": "flushed before every timed call"},
                      "roofline": {"bound": "tensor", "achieved": head["tflops"], "peak": pk["bf16_tflops"],
                                   "frac": head["frac_of_peak"], "peak_source": src + " dense bf16 (burst)"},
                      "sweep": rows}))
    return 0


def _pipelined(exe, bufs, steps):
    """Execute `steps` times back to back: each step's outputs are released (stream-ordered, back to
    the pool) after the next step has been enqueued, and the last step is read back.  Warm-up and
    timed loops both use this, so the allocator pool holds two steps' outputs before timing starts."""
    prev = []
    for _ in range(steps):
        outs = exe.execute(bufs, wait=False)
        for o in prev:
            o.delete()
        prev = outs
    if prev:
        prev[-1].to_numpy()
    for o in prev:
        o.delete()


def run_psum(a, world, rank, local):
    import torch
    from pjrt_b200 import configs
    lib = ctypes.CDLL(LIB)
    lib.b200_exec_timer.restype = ctypes.c_double
    client, store = _client(world, rank, local)
    rows = []
    for kb in (4, 16, 64, 256, 1024, 4096, 16384, 65536, 262144, 1048576):
        n = kb * 1024 // 4
        p = configs.psum_program(n, world, seed_rank=rank)
        exe = client.compile(p.text)
        buf = client.buffer_from_host(p.inputs[0])
        _pipelined(exe, [buf], a.warmup)
        if world > 1:
            torch.distributed.barrier()
        lib.b200_exec_timer(0)
        _pipelined(exe, [buf], a.steps)
        ms = _max_over_ranks(lib.b200_exec_timer(1) / a.steps, world)
        buf.delete()
        exe.destroy()
        algbw = n * 4 / (ms * 1e-3) / 1e9
        row = {"bytes": n * 4, "ms": round(ms, 5), "algbw_GBs": round(algbw, 2),
               "busbw_GBs": round(algbw * 2 * (world - 1) / world, 2)}
        if world > 1:
            # the same all_reduce through torch.distributed (NCCL) for comparison
            t = torch.randn(n, device="cuda")
            for _ in range(a.warmup):
                torch.distributed.all_reduce(t)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
            e0.record()
            for _ in range(a.steps):
                torch.distributed.all_reduce(t)
            e1.record()
            e1.synchronize()
            tms = _max_over_ranks(e0.elapsed_time(e1) / a.steps, world)
            row["torch_nccl_busbw_GBs"] = round(n * 4 / (tms * 1e-3) / 1e9 * 2 * (world - 1) / world, 2)
            del t
        rows.append(row)
    client.close()
    if rank == 0:
        big = rows[-1]
        print(json.dumps({"metric": "all_reduce (psum) bus GB/s at 1 GiB f32", "value": big["busbw_GBs"], "unit": "GB/s",
                          "n_gpus": world, "higher_is_better": True, "dtype": "f32", "data": "synthetic N(0,1) per rank",
                          "config": {"workload": "psum sweep 4 KiB .. 1 GiB through PJRT (NCCL)",
                                     "nvlink_peak_GBs_per_direction": 900},
                          "sweep": rows}))
    return 0


def fused_programs():
    """Memory-bound chains of the train step as standalone programs, with their algorithmic bytes
    (unique inputs read + outputs written once)."""
    from pjrt_b200.shlo import Builder
    progs = []
    rng = np.random.default_rng(0)
    import ml_dtypes
    bf = ml_dtypes.bfloat16
    # AdamW over the flattened GPT-2-small parameters: bf16 p, g; f32 m, v
    n = 124_439_808
    b = Builder("jit_adamw")
    p, g = b.arg((n,), "bf16"), b.arg((n,), "bf16")
    m, v = b.arg((n,), "f32"), b.arg((n,), "f32")
    gf, pf = b.convert(g, "f32"), b.convert(p, "f32")
    m1 = 0.9 * m + 0.1 * gf
    v1 = 0.95 * v + 0.05 * (gf * gf)
    upd = (m1 / 0.1) / (b.sqrt(v1 / 0.05) + 1e-8) + 0.1 * pf
    p1 = b.convert(pf - 3e-4 * upd, "bf16")
    ins = [(rng.standard_normal(n, dtype=np.float32) * 0.02).astype(bf), rng.standard_normal(n, dtype=np.float32).astype(bf),
           np.zeros(n, np.float32), np.zeros(n, np.float32)]
    progs.append(("adamw 124.4M params", b.text([p1, m1, v1]), ins, n * (2 + 2 + 4 + 4 + 2 + 4 + 4)))
    # LayerNorm forward, bf16 [65536, 768]
    rows, d = 65536, 768
    b = Builder("jit_layernorm")
    x, gm, bt = b.arg((rows, d), "bf16"), b.arg((d,), "bf16"), b.arg((d,), "bf16")
    xf = b.convert(x, "f32")
    mu = b.mean(xf, -1, keepdims=True)
    xc = xf - b.broadcast_to(mu, xf.shape)
    var = b.mean(xc * xc, -1, keepdims=True)
    y = xc * b.broadcast_to(b.rsqrt(var + 1e-5), xf.shape) * b.broadcast_to(b.convert(gm, "f32"), xf.shape) \
        + b.broadcast_to(b.convert(bt, "f32"), xf.shape)
    ins = [rng.standard_normal((rows, d), dtype=np.float32).astype(bf), np.ones(d, bf), np.zeros(d, bf)]
    progs.append(("layernorm bf16 [65536,768]", b.text([b.convert(y, "bf16")]), ins, rows * d * 4))
    # GELU (tanh) + bias, bf16 [65536, 3072]
    rows, d = 65536, 3072
    b = Builder("jit_gelu")
    x, bias = b.arg((rows, d), "bf16"), b.arg((d,), "bf16")
    h = b.convert(x + b.broadcast_to(bias, x.shape), "f32")
    inner = (h + 0.044715 * (h * h * h)) * 0.7978845608028654
    out = b.convert(0.5 * h * (1.0 + b.tanh(inner)), "bf16")
    ins = [rng.standard_normal((rows, d), dtype=np.float32).astype(bf), np.zeros(d, bf)]
    progs.append(("bias+gelu bf16 [65536,3072]", b.text([out]), ins, rows * d * 4))
    # softmax cross-entropy row logsumexp over f32 logits [8192, 50257]
    rows, vocab = 8192, 50257
    b = Builder("jit_ce")
    lg = b.arg((rows, vocab), "f32")
    mx = b.max(lg, 1, keepdims=True)
    lse = b.log(b.sum(b.exp(lg - b.broadcast_to(mx, lg.shape)), 1)) + b.reshape(mx, (rows,))
    ins = [rng.standard_normal((rows, vocab), dtype=np.float32)]
    progs.append(("logsumexp f32 [8192,50257]", b.text([lse]), ins, rows * vocab * 4 + rows * 4))
    return progs


def run_fused(a, world, rank, local):
    lib = ctypes.CDLL(LIB)
    lib.b200_exec_timer.restype = ctypes.c_double
    client, _ = _client(1, 0, local)
    pk, src = _peaks()
    rows = []
    for name, text, ins, nbytes in fused_programs():
        if getattr(a, "only", "") and a.only not in name:
            continue
        exe = client.compile(text)
        bufs = [client.buffer_from_host(x) for x in ins]
        _pipelined(exe, bufs, a.warmup)
        lib.b200_exec_timer(2)          # each execution's own device span: host enqueue gaps left out
        _pipelined(exe, bufs, a.steps)
        ms = lib.b200_exec_timer(1) / a.steps
        for o in bufs:
            o.delete()
        exe.destroy()
        gbs = nbytes / (ms * 1e-3) / 1e9
        rows.append({"kernel": name, "ms": round(ms, 4), "bytes": nbytes, "GBs": round(gbs, 1),
                     "frac_of_hbm": round(gbs / pk["hbm_gbs"], 3)})
    client.close()
    worst = min(r["frac_of_hbm"] for r in rows)
    print(json.dumps({"metric": "fused elementwise/reduce kernels, fraction of HBM bandwidth (min over the set)",
                      "value": worst, "unit": "fraction", "n_gpus": 1, "higher_is_better": True, "dtype": "bf16/f32",
                      "data": "synthetic", "config": {"workload": "fused chains through PJRT, device time",
                                                       "timing": "sum of per-execution CUDA-event spans; inputs > L2",
                                                       "hbm_peak_GBs": pk["hbm_gbs"], "peak_source": src},
                      "kernels": rows}))
    return 0


def run_attn_bwd(a, world, rank, local):
    """Flash-attention training kernels through the C ABI: forward with lse2, then the backward
    (delta, dQ/dK/dV, dQ rounding), device time with CUDA events, L2 flushed before each step."""
    import torch
    lib = ctypes.CDLL(LIB)
    lib.b200_attention_fwd_lse.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_void_p]
    lib.b200_attention_bwd.argtypes = [ctypes.c_void_p] * 11 + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_void_p]
    torch.cuda.set_device(local)
    st = torch.cuda.current_stream()
    sp = ctypes.c_void_p(st.cuda_stream)
    flush = torch.empty(64 * 1024 * 1024, device="cuda")
    pk, src = _peaks()
    rows = []
    for B, H, S, causal in [(8, 12, 1024, True), (4, 16, 4096, True), (4, 16, 4096, False)]:
        name = f"{B}x{H}x{S}-{'causal' if causal else 'full'}"
        if getattr(a, "only", "") and a.only != name:
            continue
        g = torch.Generator(device="cuda").manual_seed(S)
        q, k, v, do = (torch.randn(B, H, S, 64, device="cuda", generator=g).to(torch.bfloat16) for _ in range(4))
        o, dq, dk, dv = (torch.empty_like(q) for _ in range(4))
        lse = torch.empty(B, H, S, device="cuda")
        dq_acc = torch.empty(B, H, S, 64, device="cuda")
        delta = torch.empty(B, H, S, device="cuda")
        fwd = lambda: lib.b200_attention_fwd_lse(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(),
                                                 B, H, S, 64, int(causal), 0.125, sp)
        bwd = lambda: lib.b200_attention_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(),
                                             lse.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dq_acc.data_ptr(),
                                             delta.data_ptr(), B, H, S, 64, int(causal), 0.125, sp)
        for _ in range(a.warmup):
            assert fwd() == 0 and bwd() == 0
        tf, tb = [], []
        for _ in range(a.steps):
            flush.zero_()
            e = [torch.cuda.Event(True) for _ in range(3)]
            e[0].record(st)
            fwd()
            e[1].record(st)
            bwd()
            e[2].record(st)
            e[2].synchronize()
            tf.append(e[0].elapsed_time(e[1]))
            tb.append(e[1].elapsed_time(e[2]))
        mf, mb = sorted(tf)[len(tf) // 2], sorted(tb)[len(tb) // 2]
        fl = 4.0 * B * H * S * S * 64 * (0.5 if causal else 1.0)      # forward; the backward is 2.5x
        rows.append({"shape": name, "fwd_ms": round(mf, 4), "fwd_tflops": round(fl / mf / 1e9, 1),
                     "bwd_ms": round(mb, 4), "bwd_tflops": round(2.5 * fl / mb / 1e9, 1)})
    head = rows[0]
    print(json.dumps({"metric": "attention backward TFLOP/s (bf16 [8,12,1024,64] causal, GPT-2 training shape)",
                      "value": head["bwd_tflops"], "unit": "TFLOP/s", "n_gpus": 1, "higher_is_better": True,
                      "dtype": "bf16", "data": "synthetic N(0,1)",
                      "config": {"workload": "flash attention fwd(+lse2) and bwd", "l2": "flushed before every step",
                                 "flops": "bwd = 2.5 x fwd = 10 B H S^2 d (half causal)"},
                      "roofline": {"bound": "tensor", "achieved": head["bwd_tflops"], "peak": pk["bf16_tflops"],
                                   "frac": round(head["bwd_tflops"] / pk["bf16_tflops"], 3), "peak_source": src},
                      "sweep": rows}))
    return 0


def run(a, world, rank, local):
    import torch
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    try:
        return {"dp": run_dp, "gemm": run_gemm, "psum": run_psum, "fused": run_fused,
                "attn_bwd": run_attn_bwd}[a.workload](a, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
