"""The measured workloads behind bench.py, one function per BASELINE configuration, each returning a
dict (bench.py assembles them into its JSON line).

  run_dp        config 4: the GPT-2-small data-parallel AdamW train step through the PJRT C API (one
                process per GPU, gradients all-reduced over NCCL).  Params, moments and the token
                batch stay on the device and each step's outputs feed the next; device time from the
                CUDA events the executor records (b200_exec_timer), max over ranks.  The end-to-end
                loop uploads each step's token batch from pinned host memory and reads the loss back.
  run_attention config 2: the fused attention kernel (b200_attention_fwd) on HBM-resident inputs,
                the sequence-length sweep, and the same metric through PJRT with host buffers.
  run_gemm      config 3: dot_general through b200_gemm (bf16) and b200_gemm_split (f32 inputs).
  run_fused     the HBM-bound chains of the train step (AdamW, LayerNorm, bias+GELU, logsumexp)
                through PJRT, GB/s against the measured copy bandwidth.
  run_attn_bwd  the flash backward through the C ABI.
  run_psum      config 5: the all_reduce sweep through PJRT (NCCL), bus GB/s.
  cpu_*         the CPU baselines (oracle/torch_ref.py: torch on all host cores, f32), rank 0 only.
Device time is measured with CUDA events on the stream the kernels run on; L2 is flushed (a
256 MiB write) before timed kernel calls whose inputs fit in L2.
"""
from __future__ import annotations

import ctypes
import datetime
import json
import math
import os
import statistics
import subprocess
import tempfile
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "lib", "libpjrt_b200.so")

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks():
    """(peaks, "measured" | "fallback"): the pool's measured HBM copy and dense bf16 GEMM rates."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback"


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count()


def lib():
    l = ctypes.CDLL(LIB)
    l.b200_exec_timer.restype = ctypes.c_double
    l.b200_graph_stats.restype = ctypes.c_longlong
    l.b200_kernel_launches.restype = ctypes.c_longlong
    l.b200_gemm.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int64] * 4 + [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    l.b200_gemm_split_scratch_bytes.argtypes = [ctypes.c_int64] * 4 + [ctypes.c_int, ctypes.c_int]
    l.b200_gemm_split_scratch_bytes.restype = ctypes.c_size_t
    l.b200_gemm_split.argtypes = ([ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p] +
                                  [ctypes.c_int64] * 4 + [ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p])
    l.b200_attention_fwd.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_void_p]
    l.b200_attention_fwd_lse.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_void_p]
    l.b200_attention_bwd.argtypes = [ctypes.c_void_p] * 11 + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_void_p]
    return l


class Clocks:
    """nvidia-smi samples (SM clock, throttle reasons) while a timed region runs."""

    def __init__(self, index):
        # nvidia-smi numbers the physical GPUs: map this process's device through CUDA_VISIBLE_DEVICES
        vis = [v.strip() for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
        if index < len(vis):
            index = vis[index]
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={index}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None
        # nvidia-smi takes a moment to start: the timed region begins once it is sampling
        t0 = time.time()
        while self.p is not None and time.time() - t0 < 5:
            if os.path.getsize(self.f.name) > 0:
                break
            time.sleep(0.02)

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


def make_client(world, rank, local, nccl_max_ctas=0, port_offset=17):
    """A PJRT client for this rank; with world > 1 the NCCL unique id travels through a TCP store
    (the kv_put / kv_get callbacks of PJRT_Client_Create)."""
    from pjrt_b200 import pjrt
    api = pjrt.Api(LIB)
    if world == 1:
        return pjrt.Client(api, device_ordinal=local), None
    import torch.distributed as dist
    port = int(os.environ.get("MASTER_PORT", "29500")) + port_offset
    store = dist.TCPStore(os.environ.get("MASTER_ADDR", "127.0.0.1"), port, world, rank == 0,
                          timeout=datetime.timedelta(seconds=120))

    def put(k, v):
        store.set(k, v)

    def get(k, ms):
        store.wait([k], datetime.timedelta(milliseconds=max(ms, 1)))
        return store.get(k)
    return pjrt.Client(api, node_id=rank, num_nodes=world, device_ordinal=local, kv_put=put, kv_get=get,
                       nccl_max_ctas=nccl_max_ctas), store


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    import torch
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def pinned(x):
    """A copy of numpy array `x` in page-locked host memory (torch's pinned allocator)."""
    import torch
    t = torch.empty(x.nbytes, dtype=torch.uint8).pin_memory()
    a = t.numpy().view(x.dtype).reshape(x.shape)     # the view's base keeps `t` alive
    a[...] = x
    return a


# ============================================================================ config 4: DP step
def run_dp(a, world, rank, local):
    import torch
    from pjrt_b200 import configs
    L = lib()
    cfg = dict(configs.GPT2_SMALL, layers=a.layers)
    batch = 8
    t0 = time.time()
    # params and moments donated (jax.jit(step, donate_argnums=...)): AdamW updates them in place
    donate = not getattr(a, "no_donate", False)
    prog = configs.gpt2_program(batch=batch, world=world, rank=rank, donate=donate, **cfg)
    client, store = make_client(world, rank, local, nccl_max_ctas=getattr(a, "nccl_max_ctas", 0))
    exe = client.compile(prog.text)
    compile_s = time.time() - t0
    n = prog.meta["n_tensors"]
    state = [client.buffer_from_host(x) for x in prog.inputs[:3 * n]]
    # token batches (this rank's shard [batch, seq]; shard_map retypes the argument): a few distinct
    # ones, seeded per rank, in pinned host memory; the device-resident loop reuses uploaded copies
    brng = np.random.default_rng(1000 + rank)
    host_batches = [[pinned(brng.integers(0, cfg["vocab"], (batch, cfg["seq"])).astype(np.int32)) for _ in range(2)]
                    for _ in range(4)]
    dev_batches = [[client.buffer_from_host(x) for x in hb] for hb in host_batches]
    bc_host = [pinned(np.zeros((), np.float32)), pinned(np.zeros((), np.float32))]

    def step(s, upload):
        """One train step s >= 1.  `upload`: the token batch comes from pinned host memory now (else
        from its device copy).  Argument buffers are released once the step is enqueued (the frees
        are stream-ordered); the step's new state replaces the old."""
        bc_host[0][...] = 1 - 0.9 ** s          # Adam bias corrections, host scalars per step
        bc_host[1][...] = 1 - 0.95 ** s
        bc = [client.buffer_from_host(x) for x in bc_host]     # returns once the host copy is read
        # the device-resident loop keeps one token batch at fixed addresses, so its executions replay
        # a captured CUDA graph (the cache is keyed by argument / output addresses)
        toks = [client.buffer_from_host(x) for x in host_batches[s % 4]] if upload else dev_batches[0]
        outs = exe.execute(state + toks + bc, wait=False)
        for b in bc + state + (toks if upload else []):
            b.delete()
        state[:] = outs[:3 * n]
        return outs[-1]

    s = 1
    losses = []
    for _ in range(a.warmup):
        loss = step(s, False)
        s += 1
        losses.append(float(loss.to_numpy()))
        loss.delete()
    barrier(world)
    clk = Clocks(local) if rank == 0 else None
    replays0 = L.b200_graph_stats(1)
    launches0 = L.b200_kernel_launches()
    L.b200_exec_timer(0)
    loss = None
    for _ in range(a.steps):
        if loss is not None:
            loss.delete()
        loss = step(s, False)
        s += 1
    dev_ms = L.b200_exec_timer(1)            # waits for the last execution
    barrier(world)
    clocks = clk.stop() if clk else None
    launches = L.b200_kernel_launches() - launches0
    replays = L.b200_graph_stats(1) - replays0
    last_loss = float(loss.to_numpy())
    loss.delete()
    ms = max_over_ranks(dev_ms / a.steps, world)
    # ---- end to end: per step, token batch + scalars H2D from pinned memory, loss D2H
    e2e_steps = max(3, a.steps // 2)
    loss_host = pinned(np.zeros((), np.float32))
    for k in range(2 + e2e_steps):
        if k == 2:
            barrier(world)
            t_e = time.perf_counter()
        lb = step(s, True)
        lb.to_numpy(loss_host)
        lb.delete()
        s += 1
    e2e_ms = max_over_ranks((time.perf_counter() - t_e) * 1e3 / e2e_steps, world)
    h2d = sum(x.nbytes for x in host_batches[0]) + 8
    for b in state + [x for db in dev_batches for x in db]:
        b.delete()
    exe.destroy()
    client.close()
    tokens = batch * cfg["seq"] * world
    pk, src = peaks()
    fl_tok = prog.flops / (batch * cfg["seq"])
    tps = tokens / (ms * 1e-3)
    per_gpu_tflops = fl_tok * tps / world / 1e12
    return {
        "ms": ms, "tokens_per_s": tps, "tokens_per_step": tokens, "compile_s": compile_s, "graph_replays": replays,
        "donate": donate,
        "launches": launches, "loss_first": losses[0] if losses else None, "loss_last": last_loss, "clocks": clocks,
        "flops_per_token": fl_tok, "n_params": prog.meta["n_params"], "cfg": cfg, "batch": batch,
        "roofline": {"bound": "tensor", "achieved": per_gpu_tflops, "peak": pk["bf16_tflops_sustained"], "unit": "TFLOP/s",
                     "frac": per_gpu_tflops / pk["bf16_tflops_sustained"], "traffic": None,
                     "kernel": "whole train step (model FLOPs utilisation: 854.4 MFLOP/token, PaLM counting with "
                               "attention as non-causal)",
                     "peak_source": f"{src} dense bf16, sustained (a kernel mix timed inside a long step)"},
        "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": "tokens/s", "ms_per_step": e2e_ms, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": 4,
                "path": "PJRT C API per step: BufferFromHostBuffer(ids, targets, 2 scalars; pinned host) + Execute + "
                        "ToHostBuffer(loss), host wall clock, max over ranks"},
    }


# ============================================================================ config 2: attention
def attn_flops(B, H, S, D, causal):
    return 4.0 * B * H * S * S * D * (0.5 if causal else 1.0)


def time_attention(torch, L, cfg, steps, warmup, flush):
    """Device ms per b200_attention_fwd call (CUDA events on the launching stream, L2 flushed)."""
    B, H, S, D, causal = cfg["B"], cfg["H"], cfg["S"], cfg["D"], cfg["causal"]
    g = torch.Generator(device="cuda").manual_seed(0)
    q, k, v = (torch.randn(B, H, S, D, device="cuda", generator=g).to(torch.bfloat16) for _ in range(3))
    o = torch.empty_like(q)
    st = torch.cuda.current_stream()
    sp = ctypes.c_void_p(st.cuda_stream)

    def call():
        rc = L.b200_attention_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), B, H, S, D, int(causal),
                                  1.0 / math.sqrt(D), sp)
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
    if L.b200_take_device_error() != 0:
        raise RuntimeError("attention kernel reported a timed-out wait")
    return sum(times) / len(times)


def attention_e2e(cfg, steps, warmup, device):
    """The attention metric through the PJRT C API with host buffers (pinned): 3 H2D + Execute +
    1 D2H per step, host wall clock around the synchronous calls."""
    import ml_dtypes
    from pjrt_b200 import configs, pjrt
    p = configs.attention_program(with_inputs=True, **{k: cfg[k] for k in ("B", "H", "S", "D", "causal")})
    hosts = [pinned(x) for x in p.inputs]
    out_host = pinned(np.zeros(p.inputs[0].shape, ml_dtypes.bfloat16))
    client = pjrt.Client(pjrt.Api(LIB), device_ordinal=device)
    exe = client.compile(p.text)

    def step():
        bufs = [client.buffer_from_host(x) for x in hosts]
        outs = exe.execute(bufs)
        outs[0].to_numpy(out_host)
        for b in bufs + outs:
            b.delete()

    for _ in range(warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    ms = (time.perf_counter() - t0) * 1e3 / steps
    exe.destroy()
    client.close()
    return ms, sum(x.nbytes for x in hosts), out_host.nbytes


def run_attention(a, local, sweep=True, e2e=True, cpu=True, traffic=None):
    import torch
    L = lib()
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
    pk, src = peaks()
    head = dict(B=a.B, H=a.H, S=a.S, D=64, causal=a.causal)
    ms = time_attention(torch, L, head, a.steps, a.warmup, flush)
    fl = attn_flops(**head)
    tf = fl / (ms * 1e-3) / 1e12
    r = {"value": tf, "unit": "TFLOP/s", "ms_per_call": ms,
         "config": {"workload": f"attention B={a.B} H={a.H} S={a.S} d=64 {'causal' if a.causal else 'non-causal'}",
                    "dtype": "bf16 in/out, fp32 softmax", "l2": "flushed (256 MiB write) before every timed call"},
         "roofline": {"bound": "tensor", "achieved": tf, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                      "frac": tf / pk["bf16_tflops"], "traffic": traffic,
                      "peak_source": f"{src} dense bf16 (burst: one kernel timed alone)",
                      "algorithmic_flops_per_call": fl, "algorithmic_bytes_per_call": 4.0 * a.B * a.H * a.S * 64 * 2}}
    if sweep:
        rows = []
        for S in (512, 1024, 2048, 4096, 8192, 16384):
            for causal in (False, True):
                cfg = dict(B=4, H=16, S=S, D=64, causal=causal)
                m = time_attention(torch, L, cfg, max(3, a.steps // 2), 3, flush)
                rows.append({"S": S, "causal": causal, "ms": round(m, 4),
                             "tflops": round(attn_flops(**cfg) / (m * 1e-3) / 1e12, 1)})
        r["sweep"] = rows
    del flush
    torch.cuda.empty_cache()
    if e2e:
        e_ms, h2d, d2h = attention_e2e(head, max(3, a.steps // 2), 2, local)
        r["e2e"] = {"value": fl / (e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e_ms, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "path": "PJRT C API: BufferFromHostBuffer x3 + Execute + ToHostBuffer (pinned)"}
    if cpu:
        r["cpu_baseline"] = cpu_attention(head)
    return r


def cpu_attention(cfg):
    """torch-CPU scaled_dot_product_attention in f32 on all host cores, on the whole input."""
    import torch
    from oracle import torch_ref
    torch.set_num_threads(torch_ref.host_threads())
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(cfg["B"], cfg["H"], cfg["S"], cfg["D"], generator=g).to(torch.bfloat16).float() for _ in range(3))
    torch_ref.attention(q[:1, :1], k[:1, :1], v[:1, :1], cfg["causal"])          # warm-up
    t0 = time.perf_counter()
    torch_ref.attention(q, k, v, cfg["causal"])
    dt = time.perf_counter() - t0
    return {"value": attn_flops(**cfg) / dt / 1e12, "unit": "TFLOP/s", "cores": torch_ref.host_threads(), "kind": "port",
            "sample": f"torch-CPU f32 scaled_dot_product_attention on the whole [{cfg['B']},{cfg['H']},{cfg['S']},64] "
                      f"input, one call ({dt:.2f} s)"}


# ============================================================================ config 3: GEMM
def run_gemm(a, local, only=""):
    import torch
    L = lib()
    st = torch.cuda.current_stream()
    sp = ctypes.c_void_p(st.cuda_stream)
    flush = torch.empty(64 * 1024 * 1024, device="cuda")
    pk, src = peaks()
    rows = []
    # (name, batch, M, N, K, operand type, result type): config 3's square sweep, then the GPT-2
    # train step's forward products (tokens x d_model -> qkv / proj / fc1 / fc2, bf16 results)
    shapes = [(f"b{b}-{n}-{dt}", b, n, n, n, dt, "f32") for b, n, dt in
              [(1, 1024, "bf16"), (1, 4096, "bf16"), (1, 8192, "bf16"), (16, 2048, "bf16"), (1, 1024, "f32"),
               (1, 4096, "f32"), (1, 8192, "f32")]]
    shapes += [("gpt2-qkv", 1, 8192, 2304, 768, "bf16", "bf16"), ("gpt2-proj", 1, 8192, 768, 768, "bf16", "bf16"),
               ("gpt2-fc1", 1, 8192, 3072, 768, "bf16", "bf16"), ("gpt2-fc2", 1, 8192, 768, 3072, "bf16", "bf16")]
    for name, batch, m, n, k, dt, odt in shapes:
        if only and only != name:
            continue
        tdt = torch.bfloat16 if dt == "bf16" else torch.float32
        A = (torch.randn(batch, m, k, device="cuda") / math.sqrt(k)).to(tdt)
        B = (torch.randn(batch, n, k, device="cuda") / math.sqrt(k)).to(tdt)
        C = torch.empty(batch, m, n, device="cuda", dtype=torch.bfloat16 if odt == "bf16" else torch.float32)
        oc = 13 if odt == "bf16" else 11
        if dt == "bf16":
            f = lambda: L.b200_gemm(A.data_ptr(), B.data_ptr(), C.data_ptr(), batch, m, n, k, 13, oc, sp)
            path = f"b200_gemm (tcgen05, bf16 x bf16 -> {odt})"
        else:
            nb = L.b200_gemm_split_scratch_bytes(batch, m, n, k, 11, 11)
            scratch = torch.empty(nb, dtype=torch.uint8, device="cuda")
            f = lambda: L.b200_gemm_split(A.data_ptr(), 11, B.data_ptr(), 11, C.data_ptr(), batch, m, n, k, oc,
                                          scratch.data_ptr(), nb, sp)
            path = "b200_gemm_split (f32 operands as 3 bf16 pieces, 6 tcgen05 products, f32 accumulation)"
        for _ in range(a.warmup):
            assert f() == 0
        ts = []
        for _ in range(a.steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
            e0.record(st)
            f()
            e1.record(st)
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        ms = sorted(ts)[len(ts) // 2]
        tf = 2.0 * batch * m * n * k / (ms * 1e-3) / 1e12
        rows.append({"shape": name, "path": path, "ms": round(ms, 4), "tflops": round(tf, 1),
                     "frac_of_bf16_peak": round(tf / pk["bf16_tflops"], 3)})
        del A, B, C
    if L.b200_take_device_error() != 0:
        raise RuntimeError("GEMM kernel reported a timed-out wait")
    del flush
    torch.cuda.empty_cache()
    head = next((r for r in rows if r["shape"] == "b1-8192-bf16"), rows[0])
    return {"value": head["tflops"], "unit": "TFLOP/s", "shape": head["shape"],
            "roofline": {"bound": "tensor", "achieved": head["tflops"], "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": head["frac_of_bf16_peak"], "peak_source": f"{src} dense bf16 (burst)"},
            "config": {"workload": "dot_general sweep, A[M,K] B[N,K] ~ N(0,1)/sqrt(K), f32 result (gpt2-*: bf16)",
                       "l2": "flushed before every timed call", "timing": "median of CUDA-event spans"},
            "sweep": rows}


# ============================================================================ fused HBM-bound chains
def fused_programs():
    """Memory-bound chains of the train step as standalone programs, with their algorithmic bytes
    (unique inputs read + outputs written once)."""
    from pjrt_b200.shlo import Builder
    import ml_dtypes
    progs = []
    rng = np.random.default_rng(0)
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


def _pipelined(exe, bufs, steps):
    """Execute `steps` times back to back: each step's outputs are released (stream-ordered, back to
    the pool) after the next step has been enqueued, and the last step is read back."""
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


def run_fused(a, local, only=""):
    L = lib()
    client, _ = make_client(1, 0, local)
    pk, src = peaks()
    rows = []
    for name, text, ins, nbytes in fused_programs():
        if only and only not in name:
            continue
        exe = client.compile(text)
        bufs = [client.buffer_from_host(x) for x in ins]
        _pipelined(exe, bufs, a.warmup)
        L.b200_exec_timer(2)          # each execution's own device span: host enqueue gaps left out
        _pipelined(exe, bufs, a.steps)
        ms = L.b200_exec_timer(1) / a.steps
        for o in bufs:
            o.delete()
        exe.destroy()
        gbs = nbytes / (ms * 1e-3) / 1e9
        rows.append({"kernel": name, "ms": round(ms, 4), "bytes": nbytes, "GBs": round(gbs, 1),
                     "frac_of_hbm": round(gbs / pk["hbm_gbs"], 3)})
    client.close()
    worst = min(r["frac_of_hbm"] for r in rows)
    return {"value": worst, "unit": "fraction of measured HBM copy bandwidth (min over the set)",
            "config": {"workload": "fused chains through PJRT, device time (per-execution CUDA-event spans)",
                       "l2": "inputs larger than L2", "hbm_peak_GBs": pk["hbm_gbs"], "peak_source": src},
            "kernels": rows}


# ============================================================================ attention backward
def run_attn_bwd(a, local, only=""):
    """Flash-attention training kernels through the C ABI: forward with lse2, then the backward
    (delta, dQ/dK/dV, dQ rounding), device time with CUDA events, L2 flushed before each step."""
    import torch
    L = lib()
    st = torch.cuda.current_stream()
    sp = ctypes.c_void_p(st.cuda_stream)
    flush = torch.empty(64 * 1024 * 1024, device="cuda")
    pk, src = peaks()
    rows = []
    for B, H, S, causal in [(8, 12, 1024, True), (4, 16, 4096, True), (4, 16, 4096, False)]:
        name = f"{B}x{H}x{S}-{'causal' if causal else 'full'}"
        if only and only != name:
            continue
        g = torch.Generator(device="cuda").manual_seed(S)
        q, k, v, do = (torch.randn(B, H, S, 64, device="cuda", generator=g).to(torch.bfloat16) for _ in range(4))
        o, dq, dk, dv = (torch.empty_like(q) for _ in range(4))
        lse = torch.empty(B, H, S, device="cuda")
        dq_acc = torch.empty(B, H, S, 64, device="cuda")
        delta = torch.empty(B, H, S, device="cuda")
        fwd = lambda: L.b200_attention_fwd_lse(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(),
                                               B, H, S, 64, int(causal), 0.125, sp)
        bwd = lambda: L.b200_attention_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(),
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
        fl = attn_flops(B, H, S, 64, causal)     # forward; the backward is 2.5x
        rows.append({"shape": name, "fwd_ms": round(mf, 4), "fwd_tflops": round(fl / mf / 1e9, 1),
                     "bwd_ms": round(mb, 4), "bwd_tflops": round(2.5 * fl / mb / 1e9, 1)})
    if L.b200_take_device_error() != 0:
        raise RuntimeError("attention backward reported a timed-out wait")
    del flush
    torch.cuda.empty_cache()
    head = rows[0]
    return {"value": head["bwd_tflops"], "unit": "TFLOP/s", "shape": head["shape"],
            "roofline": {"bound": "tensor", "achieved": head["bwd_tflops"], "peak": pk["bf16_tflops"],
                         "frac": round(head["bwd_tflops"] / pk["bf16_tflops"], 3), "peak_source": src},
            "config": {"workload": "flash attention fwd(+lse2) and bwd through the C ABI", "l2": "flushed before every step",
                       "flops": "bwd = 2.5 x fwd = 10 B H S^2 d (half causal)"},
            "sweep": rows}


# ============================================================================ config 5: psum
def run_psum(a, world, rank, local):
    import torch
    from pjrt_b200 import configs
    L = lib()
    client, store = make_client(world, rank, local, port_offset=23)
    rows = []
    for kb in (4, 16, 64, 256, 1024, 4096, 16384, 65536, 262144, 1048576):
        n = kb * 1024 // 4
        p = configs.psum_program(n, world, seed_rank=rank)
        exe = client.compile(p.text)
        buf = client.buffer_from_host(p.inputs[0])
        _pipelined(exe, [buf], a.warmup)
        barrier(world)
        L.b200_exec_timer(0)
        _pipelined(exe, [buf], a.steps)
        ms = max_over_ranks(L.b200_exec_timer(1) / a.steps, world)
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
            tms = max_over_ranks(e0.elapsed_time(e1) / a.steps, world)
            row["torch_nccl_busbw_GBs"] = round(n * 4 / (tms * 1e-3) / 1e9 * 2 * (world - 1) / world, 2)
            del t
        rows.append(row)
    client.close()
    big = rows[-1]
    return {"value": big["busbw_GBs"], "unit": "GB/s", "metric": "all_reduce (psum) bus GB/s at 1 GiB f32",
            "config": {"workload": "psum sweep 4 KiB .. 1 GiB through PJRT (NCCL)", "nvlink_peak_GBs_per_direction": 900,
                       "nvlink_measured_peer_copy_GBs": 770},
            "sweep": rows}


# ============================================================================ CPU baselines
def cpu_gpt2_step(layers, steps=1, batch=1, seed=0):
    """torch-CPU f32 GPT-2 train step (oracle/torch_ref.py) on all host cores: `batch` sequences of
    1024 tokens per step, timed over `steps` steps after one untimed step.  Returns (tokens/s,
    seconds per step, threads)."""
    import torch
    from oracle import torch_ref
    from pjrt_b200 import configs
    threads = torch_ref.host_threads()
    torch.set_num_threads(threads)
    cfg = dict(configs.GPT2_SMALL, layers=layers)
    shapes = torch_ref.gpt2_param_shapes(**{k: cfg[k] for k in ("layers", "d", "heads", "mlp", "vocab", "seq")})
    ins = configs.gpt2_inputs(shapes, batch, cfg["seq"], cfg["vocab"], seed=seed, dtype="f32")
    hp = dict(lr=3e-4, b1=0.9, b2=0.95, eps=1e-8, wd=0.1)
    kw = dict(layers=cfg["layers"], d=cfg["d"], heads=cfg["heads"], mlp=cfg["mlp"], vocab=cfg["vocab"], seq=cfg["seq"], **hp)
    torch_ref.gpt2_step(ins, dtype="f32", **kw)
    t0 = time.perf_counter()
    for _ in range(steps):
        torch_ref.gpt2_step(ins, dtype="f32", **kw)
    dt = (time.perf_counter() - t0) / steps
    return batch * cfg["seq"] / dt, dt, threads
