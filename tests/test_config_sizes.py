"""Parity at the benchmark configurations' own sizes, on a B200.

The kernels the bench times are checked here on exactly the shapes it times:
  * attention forward [4,16,S,64] bf16, S = 512 .. 4096 on the whole tensor and S = 8192 / 16384 on
    sampled (batch, head) pairs, causal and not, against fp32 softmax(QK^T/8)V;
  * the same through the PJRT C API (compiled StableHLO text) at S = 4096;
  * the flash backward at [4,16,4096] (causal and full) and the GPT-2 shape [8,12,1024] causal,
    against fp32 autograd;
  * dot_general 4096^3 / 8192^3 bf16 -> f32, batched 16 x 2048^3, and the f32-input variant at
    1024^3 / 4096^3, against float64 on sampled rows;
  * one GPT-2 train step at full width (d 768, 12 heads, vocab 50257, seq 1024; 2 layers, batch 2)
    against the CPU oracle on the same program text.
Bars: 2e-2 normwise for bf16 results, 1e-4 for f32 results of bf16 products, 1e-5 for f32 inputs.
"""
import ctypes
import math

import numpy as np
import pytest

from conftest import RTOL_BF16, RTOL_F32, assert_close, rel_err
from pjrt_b200 import configs

pytestmark = pytest.mark.gpu

BF16, F32 = 13, 11


@pytest.fixture(scope="module")
def lib(lib_path, cuda):
    l = ctypes.CDLL(lib_path)
    l.b200_gemm.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int64] * 4 + [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    l.b200_attention_fwd.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_void_p]
    l.b200_attention_fwd_lse.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_void_p]
    l.b200_attention_bwd.argtypes = [ctypes.c_void_p] * 11 + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_void_p]
    return l


def _stream(torch):
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _attention_ref(torch, q, k, v, causal):
    """fp32 softmax(q k^T / sqrt(d)) v for q, k, v [n, S, d] (one (batch, head) slab per row)."""
    s = torch.matmul(q.float(), k.float().transpose(-1, -2)) / math.sqrt(q.shape[-1])
    if causal:
        S = q.shape[-2]
        s.masked_fill_(~torch.ones(S, S, dtype=torch.bool, device=s.device).tril(), float("-inf"))
    return torch.matmul(torch.softmax(s, -1), v.float())


def _qkv(torch, B, H, S, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(B, H, S, 64, device="cuda", generator=g).to(torch.bfloat16) for _ in range(3)]


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("S", [512, 1024, 2048, 4096])
def test_attention_forward_config_shape_whole_tensor(lib, cuda, S, causal):
    torch = cuda
    B, H = 4, 16
    q, k, v = _qkv(torch, B, H, S, seed=S + causal)
    o = torch.empty_like(q)
    assert lib.b200_attention_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), B, H, S, 64, int(causal),
                                  0.125, _stream(torch)) == 0
    torch.cuda.synchronize()
    assert lib.b200_take_device_error() == 0
    worst = 0.0
    for b in range(B):                    # one batch at a time: [16, S, S] fp32 scores at most 1 GiB
        ref = _attention_ref(torch, q[b], k[b], v[b], causal)
        worst = max(worst, rel_err(o[b].float().cpu().numpy(), ref.cpu().numpy()))
    assert worst <= RTOL_BF16, worst


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("S", [8192, 16384])
def test_attention_forward_long_sequences_on_sampled_heads(lib, cuda, S, causal):
    """The kernel runs on the whole [4,16,S,64] problem; the fp32 reference on 4 (batch, head)
    pairs spread over the grid (first, last, and two inside)."""
    torch = cuda
    B, H = 4, 16
    q, k, v = _qkv(torch, B, H, S, seed=3 * S + causal)
    o = torch.empty_like(q)
    assert lib.b200_attention_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), B, H, S, 64, int(causal),
                                  0.125, _stream(torch)) == 0
    torch.cuda.synchronize()
    assert lib.b200_take_device_error() == 0
    for b, h in [(0, 0), (1, 7), (2, 12), (3, 15)]:
        ref = _attention_ref(torch, q[b, h:h + 1], k[b, h:h + 1], v[b, h:h + 1], causal)
        e = rel_err(o[b, h:h + 1].float().cpu().numpy(), ref.cpu().numpy())
        assert e <= RTOL_BF16, (b, h, e)


@pytest.mark.parametrize("causal", [False, True])
def test_attention_config_through_pjrt(client, cuda, causal):
    """BASELINE config 2 at S = 4096 as a compiled StableHLO program (the attention chain matched
    into the fused kernel) against fp32 torch on the same seeded inputs."""
    torch = cuda
    p = configs.attention_program(B=4, H=16, S=4096, D=64, causal=causal, seed=41)
    out = client.run(p.text, p.inputs)[0]
    q, k, v = (torch.from_numpy(x.astype(np.float32)).cuda() for x in p.inputs)
    worst = 0.0
    for b in range(4):
        ref = _attention_ref(torch, q[b], k[b], v[b], causal)
        worst = max(worst, rel_err(out[b].astype(np.float32), ref.cpu().numpy()))
    assert worst <= RTOL_BF16, worst


@pytest.mark.parametrize("B,H,S,causal", [(8, 12, 1024, True), (4, 16, 4096, True), (4, 16, 4096, False)])
def test_attention_backward_config_shapes(lib, cuda, B, H, S, causal):
    """Flash forward (+lse2) and backward at the bench's shapes against fp32 autograd of the same
    attention, batch by batch."""
    torch = cuda
    q, k, v = _qkv(torch, B, H, S, seed=7 * S + causal)
    g = torch.Generator(device="cuda").manual_seed(99)
    do = torch.randn(B, H, S, 64, device="cuda", generator=g).to(torch.bfloat16)
    o, dq, dk, dv = (torch.empty_like(q) for _ in range(4))
    lse = torch.empty(B, H, S, device="cuda")
    dq_acc = torch.empty(B, H, S, 64, device="cuda")
    delta = torch.empty(B, H, S, device="cuda")
    st = _stream(torch)
    assert lib.b200_attention_fwd_lse(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), B, H, S, 64,
                                      int(causal), 0.125, st) == 0
    assert lib.b200_attention_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(), lse.data_ptr(),
                                  dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dq_acc.data_ptr(), delta.data_ptr(),
                                  B, H, S, 64, int(causal), 0.125, st) == 0
    torch.cuda.synchronize()
    assert lib.b200_take_device_error() == 0
    worst = {"o": 0.0, "dq": 0.0, "dk": 0.0, "dv": 0.0}
    for b in range(B):
        qf, kf, vf = (x[b].float().requires_grad_(True) for x in (q, k, v))
        ref = _attention_ref(torch, qf, kf, vf, causal)
        ref.backward(do[b].float())
        for name, got, exp in (("o", o[b], ref.detach()), ("dq", dq[b], qf.grad), ("dk", dk[b], kf.grad),
                               ("dv", dv[b], vf.grad)):
            worst[name] = max(worst[name], rel_err(got.float().cpu().numpy(), exp.cpu().numpy()))
        del qf, kf, vf, ref
    assert all(e <= RTOL_BF16 for e in worst.values()), worst


def _sampled_rows(torch, M, n, seed):
    g = torch.Generator().manual_seed(seed)
    rows = torch.randperm(M, generator=g)[:n].sort().values
    rows[0], rows[-1] = 0, M - 1          # the first and last row blocks always
    return rows.cuda()


@pytest.mark.parametrize("batch,n", [(1, 4096), (1, 8192), (16, 2048)])
def test_gemm_bf16_config_sizes(lib, cuda, batch, n):
    """A[M,K] . B[K,N] bf16 ~ N(0,1)/sqrt(K), fp32 result, against float64 on
    256 sampled rows of every batch."""
    torch = cuda
    g = torch.Generator(device="cuda").manual_seed(n + batch)
    a = (torch.randn(batch, n, n, device="cuda", generator=g) / math.sqrt(n)).to(torch.bfloat16)
    b = (torch.randn(batch, n, n, device="cuda", generator=g) / math.sqrt(n)).to(torch.bfloat16)   # [N, K]
    c = torch.empty(batch, n, n, device="cuda")
    assert lib.b200_gemm(a.data_ptr(), b.data_ptr(), c.data_ptr(), batch, n, n, n, BF16, F32, _stream(torch)) == 0
    torch.cuda.synchronize()
    assert lib.b200_take_device_error() == 0
    rows = _sampled_rows(torch, n, 256, seed=n)
    for i in range(batch):
        ref = a[i, rows].double() @ b[i].double().t()
        e = rel_err(c[i, rows].cpu().numpy(), ref.cpu().numpy())
        assert e <= RTOL_F32 * 10, (i, e)


@pytest.mark.parametrize("path", ["split", "simt"])
@pytest.mark.parametrize("n", [1024, 4096])
def test_gemm_f32_config_sizes(lib, cuda, n, path):
    """The f32-input variant of config 3 at the f32 bar (1e-5), against float64 on sampled rows: the
    tensor-core split product (b200_gemm_split) and the SIMT kernel (b200_gemm with f32 inputs)."""
    torch = cuda
    g = torch.Generator(device="cuda").manual_seed(n + 5)
    a = torch.randn(1, n, n, device="cuda", generator=g) / math.sqrt(n)
    b = torch.randn(1, n, n, device="cuda", generator=g) / math.sqrt(n)
    c = torch.empty(1, n, n, device="cuda")
    if path == "simt":
        assert lib.b200_gemm(a.data_ptr(), b.data_ptr(), c.data_ptr(), 1, n, n, n, F32, F32, _stream(torch)) == 0
    else:
        lib.b200_gemm_split_scratch_bytes.argtypes = [ctypes.c_int64] * 4 + [ctypes.c_int, ctypes.c_int]
        lib.b200_gemm_split_scratch_bytes.restype = ctypes.c_size_t
        lib.b200_gemm_split.argtypes = ([ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p] +
                                        [ctypes.c_int64] * 4 + [ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p])
        nbytes = lib.b200_gemm_split_scratch_bytes(1, n, n, n, F32, F32)
        scratch = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        assert lib.b200_gemm_split(a.data_ptr(), F32, b.data_ptr(), F32, c.data_ptr(), 1, n, n, n, F32, scratch.data_ptr(),
                                   nbytes, _stream(torch)) == 0
    torch.cuda.synchronize()
    assert lib.b200_take_device_error() == 0
    rows = _sampled_rows(torch, n, 256, seed=n + 1)
    ref = a[0, rows].double() @ b[0].double().t()
    assert rel_err(c[0, rows].cpu().numpy(), ref.cpu().numpy()) <= RTOL_F32


@pytest.mark.parametrize("dtype,n,batch", [("bf16", 4096, 0), ("f32", 4096, 0), ("bf16", 2048, 16)])
def test_gemm_config_through_pjrt(client, cuda, dtype, n, batch):
    """Config 3 programs compiled from StableHLO (dot_general with [K, N] right operands, read
    MN-major in place) against float64 on sampled rows."""
    torch = cuda
    p = configs.gemm_program(n, n, n, batch=batch, dtype=dtype, seed=n + batch)
    out = client.run(p.text, p.inputs)[0]
    a, b = (torch.from_numpy(np.asarray(x, np.float64)).cuda() for x in p.inputs)
    rows = _sampled_rows(torch, n, 128, seed=3).cpu().numpy()
    bar = RTOL_F32 if dtype == "f32" else RTOL_F32 * 10
    if batch:
        for i in (0, batch - 1):
            ref = (a[i, rows] @ b[i]).cpu().numpy()
            assert rel_err(out[i, rows], ref) <= bar
    else:
        ref = (a[rows] @ b).cpu().numpy()
        assert rel_err(out[rows], ref) <= bar


def test_gpt2_full_width_step_vs_oracle(client):
    """One GPT-2 train step at the config's full width -- d 768, 12 heads, MLP 3072, vocab 50257
    (the padded-pitch logits path), seq 1024 -- with 2 layers and batch 2, through PJRT against the
    CPU oracle on the same text: loss to 1e-3, moments (the gradients) to the bf16 bar, weights to
    Adam's first-step bound."""
    from oracle.interp import run as oracle_run
    p = configs.gpt2_program(layers=2, batch=2)
    outs = client.run(p.text, p.inputs)
    refs = oracle_run(p.text, p.inputs)
    n = p.meta["n_tensors"]
    assert len(outs) == len(refs) == 3 * n + 1
    assert_close(outs[-1], refs[-1], 1e-3, "loss")
    lr = 3e-4
    for i, (o, r) in enumerate(zip(outs[:-1], refs[:-1])):
        o32, r32 = np.asarray(o, np.float32), np.asarray(r, np.float32)
        if i < n:
            ulp = np.abs(r32) * 2.0 ** -7 + 1e-30
            assert np.all(np.abs(o32 - r32) <= 2.2 * lr + ulp), (i, float(np.max(np.abs(o32 - r32))))
        else:
            assert_close(o32, r32, 5e-2, f"moment {i}")
