"""The allocation-free attention entry point, b200_attention_fwd_noalloc.

Some callers cannot allocate device memory at the point where they run attention: a host framework
whose caching allocator already owns the device's memory budget, or a latency-critical path where
cudaMalloc / cudaFree (which may synchronize the device) are not allowed.  For them the library keeps
the attention's scratch (V transposed) in a fixed 32 MiB device array of its own, and this entry point
allocates nothing.  These tests call it through the C ABI, twice in a row (the array keeps the
previous call's contents, which must not leak into the next result), and compare it with
b200_attention_fwd, the regular entry point, at the tolerance used for the two attention operand
layouts elsewhere in the suite (1e-2 normwise).  The file is named to be collected last, and it
creates its inputs itself, so it passes alone in a fresh process and after the rest of the suite.
"""
import ctypes

import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

LAYOUT_RTOL = 1e-2


@pytest.fixture(scope="module")
def lib(lib_path, cuda):
    l = ctypes.CDLL(lib_path)
    sig = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_void_p]
    l.b200_attention_fwd.argtypes = sig
    l.b200_attention_fwd_noalloc.argtypes = sig
    return l


@pytest.mark.parametrize("causal", [False, True])
def test_noalloc_matches_regular_entry_point_on_two_calls(lib, cuda, causal):
    torch = cuda
    B, H, S, D = 2, 4, 1024, 64
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    ref = None
    for call in range(2):
        g = torch.Generator(device="cuda").manual_seed(100 + call + 10 * causal)
        q, k, v = (torch.randn(B, H, S, D, device="cuda", generator=g).to(torch.bfloat16) for _ in range(3))
        out = torch.empty_like(q)
        ref = torch.empty_like(q)
        assert lib.b200_attention_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), ref.data_ptr(), B, H, S, D,
                                      int(causal), 0.125, st) == 0
        assert lib.b200_attention_fwd_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), B, H, S, D,
                                              int(causal), 0.125, st) == 0
        torch.cuda.synchronize()
        assert lib.b200_take_device_error() == 0
        e = rel_err(out.float().cpu().numpy(), ref.float().cpu().numpy())
        assert e <= LAYOUT_RTOL, (call, e)


def test_noalloc_rejects_problems_larger_than_its_scratch(lib, cuda):
    torch = cuda
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # [8, 16, 4096, 64] bf16 needs 64 MiB of scratch: refused with -5, nothing launched
    assert lib.b200_attention_fwd_noalloc(None, None, None, None, 8, 16, 4096, 64, 0, 0.125, st) == -5
