"""bench.py's reference arm on the CPU: one JSON line with the contract's keys, at one process and
under torchrun with two ranks (rank 0 alone prints; the other rank exits 0 without work)."""
import json
import os
import socket
import subprocess
import sys

from conftest import ROOT

KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better", "scaling", "vs_baseline",
        "dtype", "data", "impl", "config", "cpu_baseline", "e2e"}


def _lines(out):
    return [json.loads(l) for l in out.decode().splitlines() if l.startswith("{")]


def _check(line, n_gpus):
    assert KEYS <= set(line), KEYS - set(line)
    assert line["impl"] == "reference" and line["n_gpus"] == n_gpus
    assert line["value"] > 0 and line["higher_is_better"] is True
    assert "workload" in line["config"]
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["unit"] == line["unit"] and cb["cores"] >= 1
    assert cb["kind"] in ("port", "reference") and cb["sample"]
    e = line["e2e"]
    assert e["value"] == line["value"] and e["unit"] == line["unit"]
    assert e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0", "--layers", "1"],
                       cwd=ROOT, capture_output=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _lines(r.stdout)
    assert len(lines) == 1
    _check(lines[0], 1)


def test_reference_arm_under_torchrun_two_ranks():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, OMP_NUM_THREADS="1")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", str(port), "bench.py", "--impl", "reference",
                        "--gpus", "2", "--steps", "1", "--warmup", "0", "--layers", "1"],
                       cwd=ROOT, capture_output=True, timeout=600, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _lines(r.stdout)
    assert len(lines) == 1
    _check(lines[0], 2)
