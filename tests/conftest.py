"""Shared test setup: import paths, the `gpu` marker, and tolerance helpers.

Tolerances follow the north-star parity bar: bit-exact for integer / index / compare work, and for
floating point a normwise relative error  max|got - ref| / max(|ref|, tiny)  of at most 1e-5 for f32
results and 2e-2 for bf16 results (f32 results computed from bf16 operands are held to the bf16 bar).
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "mccl-jax_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

LIB = os.path.join(PKG, "lib", "libpjrt_b200.so")

RTOL_F32 = 1e-5
RTOL_BF16 = 2e-2


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (run with -m gpu on the GPU box)")


def rel_err(got, ref):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    scale = max(float(np.max(np.abs(ref))) if ref.size else 0.0, 1e-30)
    return float(np.max(np.abs(got - ref))) / scale if ref.size else 0.0


def assert_close(got, ref, rtol, what=""):
    assert np.asarray(got).shape == np.asarray(ref).shape, (what, np.asarray(got).shape, np.asarray(ref).shape)
    assert np.all(np.isfinite(np.asarray(got, dtype=np.float64)) == np.isfinite(np.asarray(ref, dtype=np.float64))), what
    e = rel_err(got, ref)
    assert e <= rtol, f"{what}: normwise relative error {e:.3e} > {rtol:.1e}"


@pytest.fixture(scope="session")
def lib_path():
    if not os.path.exists(LIB):
        import build  # mccl-jax_b200/build.py
        build.build()
    return LIB


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.fixture(scope="session")
def client(lib_path, cuda):
    from pjrt_b200 import pjrt
    c = pjrt.Client(pjrt.Api(lib_path))
    yield c
    c.close()
