"""One rank of the multi-process PJRT tests (tests/test_multigpu.py): a PJRT client with
node_id = rank of num_nodes = world, the NCCL unique id exchanged through a TCPStore passed as the
client's kv_put / kv_get callbacks — the same process model as the reference's
temp/dp_train.py:27-32 and src/mccl/collective/smoke_multi.cc.

    python tests/mp_worker.py <case> <rank> <world> <port>

Prints one JSON line with the case's result; exit code 0 = pass.
"""
import datetime
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path[:0] = [ROOT, os.path.join(ROOT, "mccl-jax_b200")]

import numpy as np  # noqa: E402


def kv_client(rank, world, port):
    import torch.distributed as dist
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=60))

    def put(k, v):
        store.set(k, v)

    def get(k, timeout_ms):
        store.wait([k], datetime.timedelta(milliseconds=max(timeout_ms, 1)))
        return store.get(k)
    return store, put, get


def main():
    case, rank, world, port = sys.argv[1], int(sys.argv[2]), int(sys.argv[3]), int(sys.argv[4])
    from pjrt_b200 import configs, pjrt
    from pjrt_b200.shlo import Builder
    store, put, get = kv_client(rank, world, port)
    api = pjrt.Api(os.path.join(ROOT, "mccl-jax_b200", "lib", "libpjrt_b200.so"))
    if case == "never_joins":
        # rank 1 exits before creating its client: rank 0 must get a deadline error, not hang
        if rank == 1:
            print(json.dumps({"rank": rank, "skipped": True}))
            return 0
        t0 = time.time()
        try:
            pjrt.Client(api, node_id=rank, num_nodes=world, device_ordinal=rank, kv_put=put, kv_get=get)
        except pjrt.PjrtError as e:
            print(json.dumps({"rank": rank, "code": e.code_name, "msg": e.message[:200], "s": time.time() - t0}))
            return 0 if e.code_name == "DEADLINE_EXCEEDED" else 1
        print(json.dumps({"rank": rank, "error": "client created without its peer"}))
        return 1
    client = pjrt.Client(api, node_id=rank, num_nodes=world, device_ordinal=rank, kv_put=put, kv_get=get)
    out = {"rank": rank}
    ok = True
    if case == "peer_leaves":
        # both ranks run one psum; rank 1 then leaves (client closed, process gone) between executions;
        # rank 0's next execution must end in DEADLINE_EXCEEDED from the execution handshake (run with
        # B200_EXEC_HANDSHAKE_MS set) before any collective is enqueued, and its client must close
        p = configs.psum_program(1024, world, with_inputs=False)
        exe = client.compile(p.text)
        r = client.run(exe, [np.full(1024, rank + 1, np.float32)])[0]
        ok &= bool(np.all(r == world * (world + 1) / 2))
        store.set(f"step1_done/{rank}", b"1")
        store.wait([f"step1_done/{q}" for q in range(world)], datetime.timedelta(seconds=60))
        if rank == 1:
            exe.destroy()
            client.close()
            out.update(ok=bool(ok), left=True)
            print(json.dumps(out))
            return 0 if ok else 1
        time.sleep(1.0)
        t0 = time.time()
        try:
            client.run(exe, [np.full(1024, 1.0, np.float32)])
            out["error"] = "the execution ran without its peer"
            ok = False
        except pjrt.PjrtError as e:
            out.update(code=e.code_name, msg=e.message[:300], s=time.time() - t0)
            ok &= e.code_name == "DEADLINE_EXCEEDED"
        # the communicator is gone: a further execution fails at once with the same cause
        try:
            client.run(exe, [np.full(1024, 1.0, np.float32)])
            ok = False
        except pjrt.PjrtError as e:
            out["again"] = e.message[:200]
        exe.destroy()
        t1 = time.time()
        client.close()
        out["close_s"] = time.time() - t1
        out["ok"] = bool(ok)
        print(json.dumps(out))
        return 0 if ok else 1
    if case == "dp_step":
        # the GPT-2 DP train step (tiny widths, with its ~40 gradient all-reduces, small ones grouped)
        # on `world` ranks against the oracle's run of all ranks
        from oracle.interp import run_spmd
        tiny = dict(layers=2, d=64, heads=2, mlp=128, vocab=96, seq=64)
        progs = [configs.gpt2_program(batch=2, world=world, rank=q, **tiny) for q in range(world)]
        outs = client.run(progs[rank].text, progs[rank].inputs)
        refs = run_spmd(progs[0].text, [pq.inputs for pq in progs])[rank]
        n = progs[0].meta["n_tensors"]
        errs = []
        for i, (o, r) in enumerate(zip(outs, refs)):
            o32, r32 = np.asarray(o, np.float32), np.asarray(r, np.float32)
            if i < n:
                ok &= bool(np.all(np.abs(o32 - r32) <= 2.2 * 3e-4 + np.abs(r32) * 2.0 ** -7 + 1e-30))
            else:
                e = float(np.max(np.abs(o32 - r32)) / max(float(np.max(np.abs(r32))), 1e-30))
                errs.append(e)
                ok &= e <= (1e-3 if i == len(outs) - 1 else 5e-2)
        out["max_moment_err"] = max(errs)
    if case == "collectives":
        # smoke_multi.cc:32-48 known answer: rank r contributes r+1 in 1024 floats -> n(n+1)/2
        p = configs.psum_program(1024, world, with_inputs=False)
        r = client.run(p.text, [np.full(1024, rank + 1, np.float32)])[0]
        ok &= bool(np.all(r == world * (world + 1) / 2))
        out["psum_known_answer"] = bool(np.all(r == world * (world + 1) / 2))
        # random psum against the sum of every rank's seeded input (the oracle's all_reduce)
        n = 1 << 16
        mine = configs.psum_program(n, world, seed_rank=rank).inputs[0]
        expect = sum(configs.psum_program(n, world, seed_rank=q).inputs[0].astype(np.float64) for q in range(world))
        r = client.run(configs.psum_program(n, world, with_inputs=False).text, [mine])[0]
        e = float(np.max(np.abs(r - expect)) / np.max(np.abs(expect)))
        out["psum_rel_err"] = e
        ok &= e <= 1e-6
        # all_gather / reduce_scatter along dim 0
        b = Builder("jit_ag_rs", num_partitions=world)
        x = b.arg((8 * world, 5), "f32")
        g = b.all_gather(x, world)
        s = b.reduce_scatter(x, world)
        xv = (np.arange(8 * world * 5, dtype=np.float32).reshape(8 * world, 5) + 100 * rank)
        gv, sv = client.run(b.text([g, s]), [xv])
        allx = [np.arange(8 * world * 5, dtype=np.float32).reshape(8 * world, 5) + 100 * q for q in range(world)]
        ok &= np.array_equal(gv, np.concatenate(allx, 0))
        ok &= np.array_equal(sv, np.split(sum(allx), world, 0)[rank])
        out["gather_scatter"] = bool(np.array_equal(gv, np.concatenate(allx, 0)))
    client.close()
    out["ok"] = bool(ok)
    print(json.dumps(out))
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
