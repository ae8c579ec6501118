"""Hand-written sm_100a kernels through their C-ABI entry points (include/b200_kernels.h) on
HBM-resident inputs, against fp32 PyTorch references of the same op."""
import ctypes

import numpy as np
import pytest

from conftest import RTOL_BF16, RTOL_F32, rel_err

pytestmark = pytest.mark.gpu

BF16, F16, F32, S32, S64 = 13, 10, 11, 4, 5


@pytest.fixture(scope="module")
def lib(lib_path, cuda):
    l = ctypes.CDLL(lib_path)
    l.b200_gemm.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int64] * 4 + [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    l.b200_attention_fwd.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_void_p]
    l.b200_scatter_add_rows.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int64] * 3 + [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    return l


def stream(torch):
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def check_device_error(lib):
    assert lib.b200_take_device_error() == 0


@pytest.mark.parametrize("batch,M,N,K", [(1, 128, 256, 64), (1, 1024, 1024, 1024), (1, 200, 300, 136),
                                         (3, 256, 128, 512), (1, 77, 50, 8), (2, 1000, 520, 1000)])
@pytest.mark.parametrize("out", [F32, BF16])
def test_gemm_bf16_tensor_cores(lib, cuda, batch, M, N, K, out):
    torch = cuda
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K)
    a = (torch.randn(batch, M, K, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
    b = (torch.randn(batch, N, K, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
    c = torch.empty(batch, M, N, device="cuda", dtype=torch.float32 if out == F32 else torch.bfloat16)
    rc = lib.b200_gemm(a.data_ptr(), b.data_ptr(), c.data_ptr(), batch, M, N, K, BF16, out, stream(torch))
    assert rc == 0
    torch.cuda.synchronize()
    check_device_error(lib)
    ref = torch.bmm(a.float(), b.float().transpose(1, 2))
    e = rel_err(c.float().cpu().numpy(), ref.cpu().numpy())
    assert e <= (RTOL_F32 * 10 if out == F32 else RTOL_BF16), e


@pytest.mark.parametrize("bn", ["256", "192", "128"])
@pytest.mark.parametrize("batch,M,N,K", [(1, 8192, 768, 768), (2, 300, 1000, 200), (1, 130, 200, 4096)])
@pytest.mark.parametrize("out", [F32, BF16])
def test_gemm_every_tile_width(lib, cuda, monkeypatch, bn, batch, M, N, K, out):
    """The 256-, 192- and 128-column tile kernels (the launcher picks one per shape by a wave
    model) on full and ragged shapes, B200_GEMM_BN forcing each."""
    torch = cuda
    monkeypatch.setenv("B200_GEMM_BN", bn)
    g = torch.Generator(device="cuda").manual_seed(M + 3 * N + K)
    a = (torch.randn(batch, M, K, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
    b = (torch.randn(batch, N, K, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
    c = torch.empty(batch, M, N, device="cuda", dtype=torch.float32 if out == F32 else torch.bfloat16)
    assert lib.b200_gemm(a.data_ptr(), b.data_ptr(), c.data_ptr(), batch, M, N, K, BF16, out, stream(torch)) == 0
    torch.cuda.synchronize()
    check_device_error(lib)
    ref = torch.bmm(a.float(), b.float().transpose(1, 2))
    e = rel_err(c.float().cpu().numpy(), ref.cpu().numpy())
    assert e <= (RTOL_F32 * 10 if out == F32 else RTOL_BF16), e


@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (300, 200, 100), (64, 10, 784)])
def test_gemm_f32_simt(lib, cuda, M, N, K):
    torch = cuda
    a = torch.randn(1, M, K, device="cuda", dtype=torch.float64).float()
    b = torch.randn(1, N, K, device="cuda", dtype=torch.float64).float()
    c = torch.empty(1, M, N, device="cuda")
    assert lib.b200_gemm(a.data_ptr(), b.data_ptr(), c.data_ptr(), 1, M, N, K, F32, F32, stream(torch)) == 0
    ref = (a.double() @ b.double().transpose(1, 2)).cpu().numpy()
    assert rel_err(c.cpu().numpy(), ref) <= RTOL_F32


@pytest.mark.parametrize("B,H,S", [(1, 1, 256), (2, 3, 512), (1, 2, 1024)])
@pytest.mark.parametrize("causal", [False, True])
def test_attention_fwd(lib, cuda, B, H, S, causal):
    torch = cuda
    D = 64
    g = torch.Generator(device="cuda").manual_seed(S + H + causal)
    q, k, v = (torch.randn(B, H, S, D, device="cuda", generator=g).to(torch.bfloat16) for _ in range(3))
    o = torch.empty_like(q)
    rc = lib.b200_attention_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), B, H, S, D, int(causal),
                                1.0 / 8.0, stream(torch))
    assert rc == 0
    torch.cuda.synchronize()
    check_device_error(lib)
    ref = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(), is_causal=causal)
    assert rel_err(o.float().cpu().numpy(), ref.cpu().numpy()) <= RTOL_BF16


@pytest.mark.parametrize("causal", [False, True])
def test_attention_vt_variant_agrees(lib, cuda, causal):
    """V read MN-major in place vs V transposed first and read K-major: two operand layouts."""
    torch = cuda
    B, H, S, D = 2, 2, 512, 64
    g = torch.Generator(device="cuda").manual_seed(99)
    q, k, v = (torch.randn(B, H, S, D, device="cuda", generator=g).to(torch.bfloat16) for _ in range(3))
    o1, o2, vt = torch.empty_like(q), torch.empty_like(q), torch.empty_like(q)
    lib.b200_attention_fwd_vt.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_void_p]
    assert lib.b200_attention_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o1.data_ptr(), B, H, S, D, int(causal),
                                  0.125, stream(torch)) == 0
    assert lib.b200_attention_fwd_vt(q.data_ptr(), k.data_ptr(), v.data_ptr(), vt.data_ptr(), o2.data_ptr(), B, H, S, D,
                                     int(causal), 0.125, stream(torch)) == 0
    torch.cuda.synchronize()
    check_device_error(lib)
    assert rel_err(o1.float().cpu().numpy(), o2.float().cpu().numpy()) <= 1e-2
    ref = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(), is_causal=causal)
    assert rel_err(o2.float().cpu().numpy(), ref.cpu().numpy()) <= RTOL_BF16


def test_attention_large_logits_rescale(lib, cuda):
    """Scores spread over hundreds of units exercise the lazy O rescaling (max moves by > 2^8)."""
    torch = cuda
    B, H, S, D = 1, 2, 1024, 64
    g = torch.Generator(device="cuda").manual_seed(5)
    q = (torch.randn(B, H, S, D, device="cuda", generator=g) * 4).to(torch.bfloat16)
    k = (torch.randn(B, H, S, D, device="cuda", generator=g) * 4).to(torch.bfloat16)
    ramp = torch.linspace(0, 3, S, device="cuda").view(1, 1, S, 1)
    k = (k.float() * (1 + ramp)).to(torch.bfloat16)            # later keys dominate: the max keeps rising
    v = torch.randn(B, H, S, D, device="cuda", generator=g).to(torch.bfloat16)
    o = torch.empty_like(q)
    assert lib.b200_attention_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), B, H, S, D, 0, 0.125,
                                  stream(torch)) == 0
    torch.cuda.synchronize()
    check_device_error(lib)
    ref = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(), scale=0.125)
    assert rel_err(o.float().cpu().numpy(), ref.cpu().numpy()) <= RTOL_BF16


def test_attention_rejects_unsupported_shapes(lib, cuda):
    torch = cuda
    q = torch.zeros(1, 1, 200, 64, device="cuda", dtype=torch.bfloat16)
    assert lib.b200_attention_fwd(q.data_ptr(), q.data_ptr(), q.data_ptr(), q.data_ptr(), 1, 1, 200, 64, 0, 1.0,
                                  stream(torch)) != 0


@pytest.mark.parametrize("dtype", [F32, BF16])
def test_scatter_add_rows(lib, cuda, dtype):
    torch = cuda
    tdt = torch.float32 if dtype == F32 else torch.bfloat16
    rows, L, n = 50, 24, 300
    idx = torch.randint(-3, rows + 3, (n,), device="cuda", dtype=torch.int32)
    upd = torch.randn(n, L, device="cuda").to(tdt)
    out = torch.zeros(rows, L, device="cuda", dtype=tdt)
    assert lib.b200_scatter_add_rows(idx.data_ptr(), upd.data_ptr(), out.data_ptr(), n, L, rows, dtype, S32,
                                     stream(torch)) == 0
    ref = torch.zeros(rows, L, device="cuda", dtype=torch.float64)
    keep = (idx >= 0) & (idx < rows)
    ref.index_add_(0, idx[keep].long(), upd[keep].double())
    assert rel_err(out.float().cpu().numpy(), ref.cpu().numpy()) <= (RTOL_F32 * 10 if dtype == F32 else RTOL_BF16)


def _attention_ref(torch, q, k, v, do, causal, scale):
    """fp32 autograd reference: O, log2-sum-exp of the scaled scores, dQ, dK, dV."""
    qf, kf, vf = (t.float().requires_grad_(True) for t in (q, k, v))
    s = (qf @ kf.transpose(-1, -2)) * scale
    if causal:
        S = q.shape[2]
        mask = torch.ones(S, S, device="cuda", dtype=torch.bool).tril()
        s = s.masked_fill(~mask, float("-inf"))
    lse2 = torch.logsumexp(s, -1) / np.log(2.0)
    o = torch.softmax(s, -1) @ vf
    o.backward(do.float())
    return o.detach(), lse2.detach(), qf.grad, kf.grad, vf.grad


@pytest.mark.parametrize("B,H,S,causal", [(1, 2, 256, True), (2, 3, 512, False), (2, 2, 1024, True), (1, 1, 256, False)])
def test_attention_backward_vs_autograd(lib, cuda, B, H, S, causal):
    """Forward with lse2 output, then dQ, dK, dV from the backward kernel (recomputed scores, atomics
    into an f32 dQ accumulator), against fp32 autograd of the same attention."""
    torch = cuda
    lib.b200_attention_fwd_lse.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_void_p]
    lib.b200_attention_bwd.argtypes = [ctypes.c_void_p] * 11 + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_void_p]
    g = torch.Generator(device="cuda").manual_seed(S + B + H + causal)
    q, k, v, do = (torch.randn(B, H, S, 64, device="cuda", generator=g).to(torch.bfloat16) for _ in range(4))
    scale = 0.125
    o = torch.empty_like(q)
    lse2 = torch.empty(B, H, S, device="cuda")
    assert lib.b200_attention_fwd_lse(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse2.data_ptr(),
                                      B, H, S, 64, int(causal), scale, stream(torch)) == 0
    dq, dk, dv = torch.empty_like(q), torch.empty_like(q), torch.empty_like(q)
    dq_acc = torch.empty(B, H, S, 64, device="cuda")
    delta = torch.empty(B, H, S, device="cuda")
    assert lib.b200_attention_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(), lse2.data_ptr(),
                                  dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dq_acc.data_ptr(), delta.data_ptr(),
                                  B, H, S, 64, int(causal), scale, stream(torch)) == 0
    torch.cuda.synchronize()
    check_device_error(lib)
    ro, rl, rdq, rdk, rdv = _attention_ref(torch, q, k, v, do, causal, scale)
    assert rel_err(o.float().cpu().numpy(), ro.cpu().numpy()) <= RTOL_BF16
    np.testing.assert_allclose(lse2.cpu().numpy(), rl.cpu().numpy(), rtol=1e-4, atol=1e-3)
    for got, ref, name in ((dq, rdq, "dq"), (dk, rdk, "dk"), (dv, rdv, "dv")):
        e = rel_err(got.float().cpu().numpy(), ref.cpu().numpy())
        assert e <= RTOL_BF16, (name, e)


@pytest.mark.parametrize("batch,M,N,K", [(1, 256, 384, 8192), (2, 640, 768, 4096), (1, 768, 768, 8192)])
def test_gemm_split_k_f32(lib, cuda, batch, M, N, K):
    """Few output tiles and a long K: the K range is split across CTAs and the f32 partials are added
    into C (zeroed first) with atomics."""
    torch = cuda
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    a = (torch.randn(batch, M, K, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
    b = torch.randn(batch, N, K, device="cuda", generator=g).to(torch.bfloat16)
    c = torch.full((batch, M, N), 7.0, device="cuda")
    assert lib.b200_gemm(a.data_ptr(), b.data_ptr(), c.data_ptr(), batch, M, N, K, BF16, F32, stream(torch)) == 0
    torch.cuda.synchronize()
    check_device_error(lib)
    ref = torch.bmm(a.float(), b.float().transpose(1, 2))
    assert rel_err(c.cpu().numpy(), ref.cpu().numpy()) <= RTOL_F32 * 10


def _split_lib(lib):
    lib.b200_gemm_split_scratch_bytes.argtypes = [ctypes.c_int64] * 4 + [ctypes.c_int, ctypes.c_int]
    lib.b200_gemm_split_scratch_bytes.restype = ctypes.c_size_t
    lib.b200_gemm_split.argtypes = ([ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p] +
                                    [ctypes.c_int64] * 4 + [ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p])
    return lib


def run_split_gemm(lib, torch, a, b, out_dt):
    """C = A . B^T through b200_gemm_split for torch operands [batch, M, K] / [batch, N, K]."""
    code = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}
    batch, M, K = a.shape
    N = b.shape[1]
    _split_lib(lib)
    nbytes = lib.b200_gemm_split_scratch_bytes(batch, M, N, K, code[a.dtype], code[b.dtype])
    scratch = torch.empty(max(nbytes, 1), dtype=torch.uint8, device="cuda")
    c = torch.empty(batch, M, N, device="cuda", dtype=out_dt)
    rc = lib.b200_gemm_split(a.data_ptr(), code[a.dtype], b.data_ptr(), code[b.dtype], c.data_ptr(), batch, M, N, K,
                             code[out_dt], scratch.data_ptr(), nbytes, stream(torch))
    assert rc == 0, rc
    torch.cuda.synchronize()
    check_device_error(lib)
    return c


@pytest.mark.parametrize("ta,tb", [("f32", "f32"), ("bf16", "f32"), ("f32", "bf16"), ("f16", "f32")])
@pytest.mark.parametrize("batch,M,N,K", [(1, 128, 256, 64), (1, 300, 200, 100), (2, 1000, 520, 1000), (1, 77, 50, 8),
                                         (1, 1024, 1024, 1024), (3, 256, 136, 4100)])
def test_gemm_split_is_f32_accurate(lib, cuda, ta, tb, batch, M, N, K):
    """f32 (and mixed f32 x 16-bit) products on the bf16 tensor cores through three-piece splits hold
    the f32 bar against float64, including ragged M / N / K and K % 64 != 0."""
    torch = cuda
    dt = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}
    g = torch.Generator(device="cuda").manual_seed(M + 3 * N + 7 * K + batch)
    a = (torch.randn(batch, M, K, device="cuda", generator=g, dtype=torch.float64) / K ** 0.5).to(dt[ta])
    b = torch.randn(batch, N, K, device="cuda", generator=g, dtype=torch.float64).to(dt[tb])
    c = run_split_gemm(lib, torch, a, b, torch.float32)
    ref = torch.bmm(a.double(), b.double().transpose(1, 2))
    assert rel_err(c.cpu().numpy(), ref.cpu().numpy()) <= RTOL_F32


def test_gemm_split_bf16_result_and_wide_range(lib, cuda):
    """A bf16 result rounds once from the f32-accurate product; operands spanning 2^-30 .. 2^30 keep
    their small terms (each piece is a bf16 of its own remainder, with f32's exponent range)."""
    torch = cuda
    g = torch.Generator(device="cuda").manual_seed(5)
    a = torch.randn(1, 256, 512, device="cuda", generator=g) * torch.exp2(torch.randint(-30, 30, (1, 256, 512), device="cuda",
                                                                                      generator=g).float())
    b = torch.randn(1, 192, 512, device="cuda", generator=g)
    c32 = run_split_gemm(lib, torch, a, b, torch.float32)
    ref = torch.bmm(a.double(), b.double().transpose(1, 2))
    assert rel_err(c32.cpu().numpy(), ref.cpu().numpy()) <= RTOL_F32
    c16 = run_split_gemm(lib, torch, a, b, torch.bfloat16)
    assert torch.equal(c16, ref.float().to(torch.bfloat16)) or rel_err(c16.float().cpu().numpy(), ref.cpu().numpy()) <= 2 ** -8


def test_bounded_wait_runs_out_and_reports_without_faulting(lib, cuda):
    """The pipelines' bounded mbarrier wait, on a barrier nobody arrives at with a ~1 ms budget, gives
    up, records its error code and returns: the host reads the code once, and the context keeps
    working (a GEMM afterwards is correct)."""
    torch = cuda
    lib.b200_selftest_wait_timeout.argtypes = [ctypes.c_longlong, ctypes.c_void_p, ctypes.c_void_p]
    check_device_error(lib)
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert lib.b200_selftest_wait_timeout(2_000_000, flag.data_ptr(), stream(torch)) == 0
    torch.cuda.synchronize()
    assert int(flag.item()) == 1
    assert lib.b200_take_device_error() == 1            # a timed-out pipeline wait
    assert lib.b200_take_device_error() == 0            # read once, then cleared
    a = torch.randn(1, 256, 128, device="cuda").to(torch.bfloat16)
    b = torch.randn(1, 128, 128, device="cuda").to(torch.bfloat16)
    c = torch.empty(1, 256, 128, device="cuda")
    assert lib.b200_gemm(a.data_ptr(), b.data_ptr(), c.data_ptr(), 1, 256, 128, 128, BF16, F32, stream(torch)) == 0
    torch.cuda.synchronize()
    check_device_error(lib)
    assert rel_err(c.cpu().numpy(), torch.bmm(a.float(), b.float().transpose(1, 2)).cpu().numpy()) <= RTOL_F32 * 10


def test_kernel_launch_counter_counts_this_librarys_launches(lib, cuda):
    torch = cuda
    lib.b200_kernel_launches.restype = ctypes.c_longlong
    a = torch.randn(1, 256, 64, device="cuda").to(torch.bfloat16)
    c = torch.empty(1, 256, 256, device="cuda")
    n0 = lib.b200_kernel_launches()
    for _ in range(3):
        assert lib.b200_gemm(a.data_ptr(), a.data_ptr(), c.data_ptr(), 1, 256, 256, 64, BF16, F32, stream(torch)) == 0
    assert lib.b200_kernel_launches() - n0 == 3
