#!/usr/bin/env python3
"""Benchmark of the B200 PJRT plugin's hot path: fused attention TFLOP/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference] [--no-sweep]

One JSON line on rank 0.  The headline workload is attention softmax(Q K^T / sqrt(d)) V with
Q, K, V bf16 [B=4, H=16, S=4096, d=64], non-causal; `sweep` adds S in 512..16384, causal and not.
  value      TFLOP/s of the fused kernel call (b200_attention_fwd, one launch) on
             HBM-resident inputs, CUDA events on the launching stream, L2 flushed (256 MiB write)
             before every timed step; FLOPs = 4 B H S^2 d (half of that causal).
  e2e        the same metric through the PJRT C API with host buffers: BufferFromHostBuffer(Q,K,V)
             + Execute + ToHostBuffer(O) per step, host wall clock around the synchronous calls.
  roofline   achieved / measured dense bf16 peak (MEASURED_PEAKS.json), traffic from the committed
             ncu summary when present.
  cpu_baseline  the numpy oracle (oracle/interp.py) on the host cores over a head subset.
Multi-GPU (`torchrun --nproc-per-node N bench.py --gpus N`): attention does not shard across GPUs
(replicas only); every rank runs the full workload on its own GPU, value = all ranks' FLOPs / max
rank time.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "mccl-jax_b200"))
sys.path.insert(0, ROOT)

LIB = os.path.join(ROOT, "mccl-jax_b200", "lib", "libpjrt_b200.so")
METRIC = "attention TFLOP/s (bf16 [4,16,S,64], fp32 softmax) at S=4096, non-causal"
HEAD = dict(B=4, H=16, S=4096, D=64, causal=False)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p, "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def ncu_traffic(name):
    """dram read+write bytes per launch from the committed ncu summary (profiles/<name>.md)."""
    path = os.path.join(ROOT, "profiles", name + ".md")
    if not os.path.exists(path):
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", open(path).read())
    return float(m.group(1)) if m else None


def attn_flops(B, H, S, D, causal):
    return 4.0 * B * H * S * S * D * (0.5 if causal else 1.0)


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, index):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={index}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for n, v in zip(names, r[5:9]):
                    if v.strip() == "Active":
                        reasons.add(n)
            except Exception:
                pass
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def load_lib():
    l = ctypes.CDLL(LIB)
    l.b200_attention_fwd.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_void_p]
    l.b200_attention_fwd.restype = ctypes.c_int
    return l


def time_kernel(torch, lib, cfg, steps, warmup, flush):
    B, H, S, D, causal = cfg["B"], cfg["H"], cfg["S"], cfg["D"], cfg["causal"]
    g = torch.Generator(device="cuda").manual_seed(0)
    q, k, v = (torch.randn(B, H, S, D, device="cuda", generator=g).to(torch.bfloat16) for _ in range(3))
    o = torch.empty_like(q)
    st = torch.cuda.current_stream()
    sp = ctypes.c_void_p(st.cuda_stream)
    scale = 1.0 / math.sqrt(D)

    def call():
        rc = lib.b200_attention_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), B, H, S, D, int(causal),
                                    scale, sp)
        if rc != 0:
            raise RuntimeError(f"b200_attention_fwd failed ({rc})")

    for _ in range(warmup):
        flush.zero_()
        call()
    torch.cuda.synchronize()
    times = []
    for _ in range(steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        call()
        e1.record(st)
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    torch.cuda.synchronize()
    if lib.b200_take_device_error() != 0:
        raise RuntimeError("tensor-core kernel reported a timed-out wait")
    del q, k, v, o
    return times


def e2e_pjrt(cfg, steps, warmup):
    """Same metric through the PJRT C API with host buffers (pinned host memory via torch)."""
    import torch
    from pjrt_b200 import configs, pjrt
    p = configs.attention_program(with_inputs=True, **{k: cfg[k] for k in ("B", "H", "S", "D", "causal")})
    pinned = [torch.from_numpy(x.view("uint16")).pin_memory() for x in p.inputs]
    import ml_dtypes
    hosts = [t.numpy().view(ml_dtypes.bfloat16) for t in pinned]
    out_host = torch.empty(tuple(p.inputs[0].shape), dtype=torch.int16).pin_memory().numpy().view(ml_dtypes.bfloat16)
    client = pjrt.Client(pjrt.Api(LIB), device_ordinal=torch.cuda.current_device())
    exe = client.compile(p.text)

    def step():
        bufs = [client.buffer_from_host(x) for x in hosts]
        outs = exe.execute(bufs)
        outs[0].to_numpy(out_host)
        for b in bufs + outs:
            b.delete()

    for _ in range(warmup):
        step()
    t = []
    for _ in range(steps):
        t0 = time.perf_counter()
        step()
        t.append((time.perf_counter() - t0) * 1e3)
    exe.destroy()
    client.close()
    h2d = sum(x.nbytes for x in hosts)
    return t, h2d, out_host.nbytes


def cpu_oracle(cfg, runs=2):
    """The numpy oracle on a head subset of the workload; returns (TFLOP/s, sample description)."""
    from oracle.interp import run
    from pjrt_b200 import configs
    heads = 1
    p = configs.attention_program(B=1, H=heads, S=cfg["S"], D=cfg["D"], causal=cfg["causal"], seed=1)
    t0 = time.perf_counter()
    n = 0
    for n in range(1, runs + 1):
        run(p.text, p.inputs)
    dt = (time.perf_counter() - t0) / n
    fl = attn_flops(1, heads, cfg["S"], cfg["D"], cfg["causal"])
    return fl / dt / 1e12, f"{heads} of {cfg['B'] * cfg['H']} (batch, head) pairs at S={cfg['S']}, {n} run(s)"


def cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--kernel-only", action="store_true", help="headline kernel timing only (profiling runs)")
    ap.add_argument("--B", type=int, default=HEAD["B"])
    ap.add_argument("--H", type=int, default=HEAD["H"])
    ap.add_argument("--S", type=int, default=HEAD["S"])
    ap.add_argument("--causal", action="store_true")
    ap.add_argument("--workload", default="attention", choices=["attention", "dp", "gemm", "psum", "fused", "attn_bwd"],
                    help="attention (headline); dp = GPT-2 DP train step; gemm = dot_general sweep; fused = HBM-bound chains; "
                         "psum = all_reduce bandwidth sweep")
    ap.add_argument("--layers", type=int, default=12, help="dp: decoder layers")
    ap.add_argument("--only", default="", help="fused: run only the chains whose name contains this text; "
                                               "gemm: run only one size, e.g. b1-8192-bf16")
    a = ap.parse_args()
    HEAD.update(B=a.B, H=a.H, S=a.S, causal=a.causal)
    a.warmup = max(a.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if a.impl == "b200" and a.workload != "attention":
        import workloads  # mccl-jax_b200/workloads.py
        return workloads.run(a, world, rank, local)

    if a.impl == "reference":
        if rank != 0:
            return 0
        # the reference's CPU implementation of this path is the oracle restatement (the Metal
        # plugin itself cannot run here): numpy on all host cores, a bounded sample per step
        import numpy as np
        per = []
        sample = ""
        for _ in range(a.steps):
            v, sample = cpu_oracle(HEAD, runs=1)
            per.append(v)
        val = statistics.median(per)
        line = {"metric": METRIC, "value": val, "unit": "TFLOP/s", "n_gpus": a.gpus, "steps": a.steps,
                "warmup": a.warmup, "ms_per_step": None, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f64", "data": "synthetic (seeded N(0,1))", "impl": "reference",
                "config": {"workload": "attention B=4 H=16 S=4096 d=64 non-causal (head-subset sample)"},
                "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": cores(), "kind": "port", "sample": sample},
                "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return 0

    import torch
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    lib = load_lib()
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")

    # ---- headline, timed region with clock sampling
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clk = Clocks(local)   # sampled over the headline and the sweep (both timed regions)
    times = time_kernel(torch, lib, HEAD, a.steps, a.warmup, flush)
    ms = sum(times) / len(times)
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    fl = attn_flops(**HEAD)
    value = fl * world / (ms * 1e-3) / 1e12

    result = None
    if rank == 0:
        pk, src = peaks()
        peak = pk["bf16_tflops"]
        per_gpu = fl / (ms * 1e-3) / 1e12
        result = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": a.steps,
                  "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                  "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1))",
                  "config": {"workload": "attention B=4 H=16 S=4096 d=64 non-causal", "B": 4, "H": 16, "S": 4096,
                             "d": 64, "causal": False, "l2": "flushed (256 MiB write) before every timed step",
                             "parallelism": f"replicas x{world}"},
                  "gpu_launches": a.steps,
                  "roofline": {"bound": "tensor", "achieved": per_gpu, "peak": peak, "unit": "TFLOP/s",
                               "frac": per_gpu / peak, "peak_source": src + " dense bf16 (burst)",
                               "traffic": ncu_traffic("attention_fwd_s4096")},
                  "clocks": None}
    if a.kernel_only:
        clk.stop()
        if rank == 0:
            print(json.dumps({"kernel_only": True, "config": dict(HEAD), "ms_per_step": ms, "value": value}))
        if dist:
            dist.destroy_process_group()
        return 0
    # ---- sweep (rank 0 only; not part of the headline)
    if rank == 0 and not a.no_sweep:
        sweep = []
        for S in (512, 1024, 2048, 4096, 8192, 16384):
            for causal in (False, True):
                cfg = dict(B=4, H=16, S=S, D=64, causal=causal)
                t = time_kernel(torch, lib, cfg, max(3, a.steps // 2), 3, flush)
                m = sum(t) / len(t)
                sweep.append({"S": S, "causal": causal, "ms": round(m, 4),
                              "tflops": round(attn_flops(**cfg) / (m * 1e-3) / 1e12, 2)})
        result["sweep"] = sweep
    clocks = clk.stop()
    if rank == 0:
        result["clocks"] = clocks
    # ---- end to end through the PJRT C API with host buffers (every rank, max over ranks)
    if dist:
        dist.barrier()
    t, h2d, d2h = e2e_pjrt(HEAD, max(3, a.steps // 2), 2)
    e2e_ms = sum(t) / len(t)
    if dist:
        tt = torch.tensor([e2e_ms], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_ms = float(tt.item())
    if rank == 0:
        result["e2e"] = {"value": fl / (e2e_ms * 1e-3) / 1e12 * world, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
                         "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                         "path": "PJRT C API: BufferFromHostBuffer x3 + Execute + ToHostBuffer (pinned host)"}
        v, sample = cpu_oracle(HEAD)
        result["cpu_baseline"] = {"value": v, "unit": "TFLOP/s", "cores": cores(), "kind": "port", "sample": sample}
        print(json.dumps(result))
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
