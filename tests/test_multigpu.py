"""Multi-process paths: NCCL collectives through the PJRT plugin on 2+ GPUs (one process per GPU,
as the reference runs one device per process), and the failure path where a rank never joins.
The CPU part checks the oracle's collective semantics against real torch.distributed (gloo) ranks."""
import json
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def run_ranks(case, world, env_extra=None, timeout=180):
    port = free_port()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", **(env_extra or {}))
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "mp_worker.py"), case, str(r), str(world), str(port)],
                              stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True, env=env)
             for r in range(world)]
    outs = []
    for p in procs:
        try:
            o, e = p.communicate(timeout=timeout)
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
        outs.append((p.returncode, o, e))
    return outs


def gpu_count():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_nccl_collectives_through_pjrt(lib_path, world):
    if gpu_count() < world:
        pytest.skip(f"needs {world} GPUs")
    for rc, o, e in run_ranks("collectives", world):
        assert rc == 0, (o, e[-2000:])
        res = json.loads(o.strip().splitlines()[-1])
        assert res["ok"] and res["psum_known_answer"], res


@pytest.mark.gpu
def test_dp_step_on_two_ranks_matches_the_oracle(lib_path):
    """The tiny GPT-2 DP step (shard_map + psum of ~40 gradients, small ones as NCCL groups) on two
    GPUs against the oracle's two-rank run."""
    if gpu_count() < 2:
        pytest.skip("needs 2 GPUs")
    for rc, o, e in run_ranks("dp_step", 2):
        assert rc == 0, (o, e[-2000:])
        assert json.loads(o.strip().splitlines()[-1])["ok"]


@pytest.mark.gpu
def test_rank_that_leaves_between_steps_gives_deadline_error(lib_path):
    """A rank that leaves between executions: the survivor's next execution fails with
    DEADLINE_EXCEEDED from the host-side execution handshake -- no collective is enqueued, so nothing
    waits on the GPU for the missing rank -- and its client still closes."""
    if gpu_count() < 2:
        pytest.skip("needs 2 GPUs")
    outs = run_ranks("peer_leaves", 2, {"B200_EXEC_HANDSHAKE_MS": "3000"}, timeout=120)
    for rc, o, e in outs:
        assert rc == 0, (o, e[-2000:])
    res = json.loads(outs[0][1].strip().splitlines()[-1])
    assert res["code"] == "DEADLINE_EXCEEDED" and res["s"] < 30 and res["close_s"] < 30, res


@pytest.mark.gpu
def test_rank_that_never_joins_gives_deadline_error(lib_path):
    if gpu_count() < 2:
        pytest.skip("needs 2 GPUs")
    outs = run_ranks("never_joins", 2, {"B200_COMM_TIMEOUT_MS": "4000"})
    rc, o, e = outs[0]
    assert rc == 0, (o, e[-2000:])
    res = json.loads(o.strip().splitlines()[-1])
    assert res["code"] == "DEADLINE_EXCEEDED" and res["s"] < 60, res


def _gloo_rank(rank, world, port, q):
    import torch
    import torch.distributed as dist
    sys.path[:0] = [os.path.dirname(HERE), os.path.join(os.path.dirname(HERE), "mccl-jax_b200")]
    from pjrt_b200 import configs
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    x = configs.psum_program(4096, world, seed_rank=rank).inputs[0]
    t = torch.from_numpy(x.copy())
    dist.all_reduce(t)
    q.put((rank, t.numpy()))
    dist.destroy_process_group()


def test_oracle_psum_matches_gloo_allreduce():
    """The oracle's all_reduce (run_spmd) agrees with torch.distributed gloo across 2 CPU ranks."""
    import torch.multiprocessing as mp
    from oracle.interp import run_spmd
    from pjrt_b200 import configs
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=_gloo_rank, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in ps:
        p.join(timeout=60)
    prog = configs.psum_program(4096, world, with_inputs=False)
    ref = run_spmd(prog.text, [configs.psum_program(4096, world, seed_rank=r).inputs for r in range(world)])
    for r in range(world):
        np.testing.assert_allclose(got[r], ref[r][0], rtol=1e-6, atol=1e-6)
