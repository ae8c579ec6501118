#!/usr/bin/env python3
"""Benchmark of the B200 PJRT plugin: data-parallel train-step tokens/s as the
headline, with the attention, dot_general and fused-kernel targets (configs 2, 3) as sub-objects.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
    torchrun --nproc-per-node N bench.py --gpus N ...            (one process per GPU, NCCL)

One JSON line on rank 0:
  value         whole-job tokens/s of the GPT-2-small DP AdamW step (12 layers, d 768, vocab 50257,
                seq 1024, per-GPU batch 8) through the PJRT C API: forward, backward, all_reduce of
                every gradient over NCCL, AdamW; params / moments / token batch resident in HBM; device
                time from CUDA events on the executor's stream over K steps, max over ranks.
  e2e           the same step with each step's token batch uploaded from pinned host memory and the
                loss read back (host wall clock, max over ranks).
  roofline      model FLOPs utilisation against the measured sustained dense bf16 peak.
  cpu_baseline  the same step in torch on the host CPU (f32, all cores; oracle/torch_ref.py), one
                sequence per step (rank 0, N = 1).
  attention / gemm / fused / attn_bwd   (N = 1) config 2's fused attention at [4,16,4096,64] with
                the sequence-length sweep and its own roofline / e2e / torch-CPU baseline; config 3's
                GEMMs; the HBM-bound chains; the flash backward.
  psum          (N > 1) config 5's all_reduce sweep through PJRT.
`--workload attention|gemm|fused|attn_bwd|psum|dp` prints one of those alone (profiling runs).
`--impl reference` times the reference path's CPU implementation (the torch-CPU step) on rank 0.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import re
import statistics
import sys

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "mccl-jax_b200"))
sys.path.insert(0, ROOT)

import workloads as W  # noqa: E402  (mccl-jax_b200/workloads.py)

METRIC = "DP train-step tokens/s (GPT-2 small, per-GPU batch 8 x 1024, AdamW)"


def ncu_traffic(name):
    """DRAM read + write bytes per launch from a committed ncu summary (profiles/<name>.md)."""
    path = os.path.join(ROOT, "profiles", name + ".md")
    if not os.path.exists(path):
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", open(path).read())
    return float(m.group(1)) if m else None


def config_of(dp, world):
    c = dp["cfg"]
    return {"workload": "gpt2-small DP train step (forward, backward, all_reduce of gradients, AdamW)",
            "model": "gpt2-small (random init N(0,0.02))", "layers": c["layers"], "d_model": c["d"], "heads": c["heads"],
            "mlp": c["mlp"], "vocab": c["vocab"], "seq_len": c["seq"], "per_gpu_batch": dp["batch"],
            "global_batch": dp["batch"] * world, "parallelism": f"dp{world}", "params": dp["n_params"],
            "l2": "working set (249 MB params + 1 GB moments + activations) far larger than L2",
            "donation": "params and AdamW moments donated, updated in place" if dp.get("donate") else "none"}


def reference_arm(a, world, rank):
    """The reference path's CPU implementation on the host cores: the torch-CPU f32 GPT-2 step
    (the reference's own code is Metal / MPSGraph and cannot run here), one sequence per step."""
    if rank != 0:
        return 0
    per = []
    dt = threads = None
    for _ in range(a.warmup):
        W.cpu_gpt2_step(a.layers, steps=1)
    for _ in range(a.steps):
        v, dt, threads = W.cpu_gpt2_step(a.layers, steps=1)
        per.append(v)
    val = statistics.median(per)
    sample = f"1 x 1024 tokens per step (of 8 x 1024 per GPU), {a.layers} layers, torch f32 on {threads} threads"
    print(json.dumps({
        "metric": METRIC, "value": val, "unit": "tokens/s", "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": 1e3 * 1024 / val, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded ids, N(0,0.02) params)", "impl": "reference",
        "config": {"workload": "gpt2-small DP train step, torch-CPU (oracle/torch_ref.py)", "layers": a.layers,
                   "seq_len": 1024, "sample": "one sequence per step"},
        "cpu_baseline": {"value": val, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="dp", choices=["dp", "attention", "gemm", "fused", "attn_bwd", "psum"],
                    help="dp (default): the full line; the others print one sub-benchmark alone")
    ap.add_argument("--layers", type=int, default=12, help="decoder layers of the DP step")
    ap.add_argument("--nccl-max-ctas", type=int, default=0,
                    help="DP step: cap on the SMs one NCCL collective occupies (client option nccl_max_ctas; 0 = NCCL's choice)")
    ap.add_argument("--no-donate", action="store_true", help="DP step: params and moments not donated (fresh buffers)")
    ap.add_argument("--no-sub", action="store_true", help="headline only (no sub-benchmarks, no CPU baseline)")
    ap.add_argument("--no-sweep", action="store_true", help="attention: no sequence-length sweep")
    ap.add_argument("--only", default="", help="gemm / fused / attn_bwd: one case by name")
    ap.add_argument("--B", type=int, default=4)
    ap.add_argument("--H", type=int, default=16)
    ap.add_argument("--S", type=int, default=4096)
    ap.add_argument("--causal", action="store_true")
    a = ap.parse_args()
    a.warmup = max(a.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if a.impl == "reference":
        return reference_arm(a, world, rank)

    import torch
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    try:
        if a.workload != "dp":
            fn = {"attention": lambda: W.run_attention(a, local, sweep=not a.no_sweep, e2e=False, cpu=False,
                                                       traffic=ncu_traffic("attention_fwd_s4096")),
                  "gemm": lambda: W.run_gemm(a, local, a.only), "fused": lambda: W.run_fused(a, local, a.only),
                  "attn_bwd": lambda: W.run_attn_bwd(a, local, a.only),
                  "psum": lambda: W.run_psum(a, world, rank, local)}[a.workload]
            r = fn()
            if rank == 0:
                print(json.dumps(dict(r, workload=a.workload, n_gpus=world)))
            return 0

        dp = W.run_dp(a, world, rank, local)
        pk, src = W.peaks()
        line = None
        if rank == 0:
            line = {"metric": METRIC, "value": dp["tokens_per_s"], "unit": "tokens/s", "n_gpus": world, "steps": a.steps,
                    "warmup": a.warmup, "ms_per_step": dp["ms"], "higher_is_better": True, "scaling": "weak",
                    "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded token ids, N(0,0.02) params)",
                    "config": config_of(dp, world), "gpu_launches": dp["launches"], "roofline": dp["roofline"],
                    "e2e": dp["e2e"], "clocks": dp["clocks"],
                    "train": {"compile_s": round(dp["compile_s"], 2), "graph_replays": dp["graph_replays"],
                              "loss_first": dp["loss_first"], "loss_last": dp["loss_last"],
                              "flops_per_token": dp["flops_per_token"]}}
        if world > 1 and not a.no_sub:
            ps = W.run_psum(a, world, rank, local)
            if rank == 0:
                line["psum"] = ps
        if world == 1 and not a.no_sub:
            clk = W.Clocks(local)
            line["attention"] = W.run_attention(a, local, sweep=not a.no_sweep, traffic=ncu_traffic("attention_fwd_s4096"))
            line["gemm"] = W.run_gemm(a, local)
            line["fused"] = W.run_fused(a, local)
            line["attn_bwd"] = W.run_attn_bwd(a, local)
            line["sub_clocks"] = clk.stop()
            v, dt, threads = W.cpu_gpt2_step(a.layers, steps=1)
            line["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
                                    "sample": f"torch-CPU f32 GPT-2 step (oracle/torch_ref.py), one sequence of 1024 "
                                              f"tokens, {a.layers} layers, one timed step after one untimed ({dt:.2f} s)"}
        if rank == 0:
            print(json.dumps(line))
        return 0
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
