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
        bc = [client.buffer_from_host(np.array(1 - 0.9 ** s, np.float32)),
              client.buffer_from_host(np.array(1 - 0.95 ** s, np.float32))]
        outs = exe.execute(state + data + bc, wait=False)
        return outs

    losses = []
    s = 1
    for _ in range(a.warmup):
        outs = step(s)
        s += 1
        for b in state:
            b.delete()
        state[:] = outs[:3 * n]
        losses.append(float(outs[-1].to_numpy()))
    if world > 1:
        torch.distributed.barrier()
    lib.b200_exec_timer(0)
    t_wall = time.perf_counter()
    for _ in range(a.steps):
        outs = step(s)
        s += 1
        for b in state:
            b.delete()
        state[:] = outs[:3 * n]
    last_loss = float(outs[-1].to_numpy())
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
            "wall_ms_per_step": wall_ms / a.steps, "compile_s": compile_s,
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
    for batch, n, ab in [(1, 1024, 13), (1, 4096, 13), (1, 8192, 13), (16, 2048, 13), (1, 1024, 11), (1, 4096, 11),
                         (1, 8192, 11)]:
        dt = torch.bfloat16 if ab == 13 else torch.float32
        A = (torch.randn(batch, n, n, device="cuda") / math.sqrt(n)).to(dt)
        B = (torch.randn(batch, n, n, device="cuda") / math.sqrt(n)).to(dt)
        C = torch.empty(batch, n, n, device="cuda")
        f = lambda: lib.b200_gemm(A.data_ptr(), B.data_ptr(), C.data_ptr(), batch, n, n, n, ab, 11,
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
        tf = 2.0 * batch * n ** 3 / (ms * 1e-3) / 1e12
        rows.append({"batch": batch, "M=N=K": n, "inputs": "bf16" if ab == 13 else "f32", "ms": round(ms, 4),
                     "tflops": round(tf, 1), "frac_of_peak": round(tf / pk["bf16_tflops"], 3)})
        del A, B, C
    head = [r for r in rows if r["M=N=K"] == 8192 and r["inputs"] == "bf16"][0]
    print(json.dumps({"metric": "dot_general TFLOP/s (bf16 -> f32, 8192^3)", "value": head["tflops"], "unit": "TFLOP/s",
                      "n_gpus": 1, "higher_is_better": True, "dtype": "bf16", "data": "synthetic N(0,1)/sqrt(K)",
                      "config": {"workload": "gemm sweep", "l2": "flushed before every timed call"},
                      "roofline": {"bound": "tensor", "achieved": head["tflops"], "peak": pk["bf16_tflops"],
                                   "frac": head["frac_of_peak"], "peak_source": src + " dense bf16 (burst)"},
                      "sweep": rows}))
    return 0


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
        for _ in range(a.warmup):
            for o in exe.execute([buf]):
                o.delete()
        if world > 1:
            torch.distributed.barrier()
        lib.b200_exec_timer(0)
        outs = []
        for _ in range(a.steps):
            outs += exe.execute([buf], wait=False)
        outs[-1].to_numpy()
        ms = _max_over_ranks(lib.b200_exec_timer(1) / a.steps, world)
        for o in outs:
            o.delete()
        buf.delete()
        exe.destroy()
        algbw = n * 4 / (ms * 1e-3) / 1e9
        rows.append({"bytes": n * 4, "ms": round(ms, 5), "algbw_GBs": round(algbw, 2),
                     "busbw_GBs": round(algbw * 2 * (world - 1) / world, 2)})
    client.close()
    if rank == 0:
        big = rows[-1]
        print(json.dumps({"metric": "all_reduce (psum) bus GB/s at 1 GiB f32", "value": big["busbw_GBs"], "unit": "GB/s",
                          "n_gpus": world, "higher_is_better": True, "dtype": "f32", "data": "synthetic N(0,1) per rank",
                          "config": {"workload": "psum sweep 4 KiB .. 1 GiB through PJRT (NCCL)",
                                     "nvlink_peak_GBs_per_direction": 900},
                          "sweep": rows}))
    return 0


def run(a, world, rank, local):
    import torch
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    try:
        return {"dp": run_dp, "gemm": run_gemm, "psum": run_psum}[a.workload](a, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
