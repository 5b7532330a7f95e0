"""The no-allocation GEMM entry point, called through its exported C symbol.

Some callers cannot allocate GPU memory (allocator callbacks, plugin hosts
that forbid cudaMalloc after start-up, real-time loops).  For them the library
exports ``osb_gemm_bf16_noalloc``, which keeps its split-K scratch in a fixed
device array and needs only inputs and outputs.  This test checks it against
the regular entry point (which uses a caller-side workspace) on two calls in a
row, and that problems too large for the fixed scratch are refused.  The file
is named so that pytest collects it last.
"""

import ctypes

import pytest
import torch

from online_speculation_b200.ops import kernels as ops

pytestmark = pytest.mark.gpu

TOLERANCE = 1e-2  # relative Frobenius error, as in the other GEMM tests


def _entry():
    import online_speculation_b200._C as ext

    lib = ctypes.CDLL(ext.__file__)
    fn = lib.osb_gemm_bf16_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int,
                   ctypes.c_int, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_longlong, ctypes.c_int, ctypes.c_void_p]
    lib.osb_gemm_noalloc_last_error.restype = ctypes.c_char_p
    lib.osb_gemm_noalloc_scratch_floats.restype = ctypes.c_longlong
    return fn, lib


def _call(fn, w, x, out, *, swiglu=False, bias=None, residual=None):
    stream = torch.cuda.current_stream().cuda_stream
    M, K = w.shape
    N = x.shape[0]
    return fn(w.data_ptr(), w.stride(0), x.data_ptr(), x.stride(0), M, N, K, out.data_ptr(), out.stride(0),
              int(out.dtype == torch.float32), None if bias is None else bias.data_ptr(),
              None if residual is None else residual.data_ptr(), 0 if residual is None else residual.stride(0),
              int(swiglu), stream)


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


@pytest.mark.parametrize("M,N,K,swiglu,bias", [
    (4608, 64, 3584, False, True),    # decode shape: split-K through the static scratch
    (1024, 16, 4096, False, False),
    (2560, 64, 1536, True, False),    # fused SwiGLU epilogue with split-K
    (37888, 64, 512, False, False),   # enough tiles: no split-K, no scratch
])
def test_noalloc_matches_regular_entry_point(M, N, K, swiglu, bias):
    fn, lib = _entry()
    torch.manual_seed(M + N + K)
    dev = torch.device("cuda", 0)
    w = (torch.randn(M, K, device=dev) * 0.05).bfloat16()
    x = torch.randn(N, K, device=dev).bfloat16()
    b = torch.randn(M, device=dev).bfloat16() if bias else None
    expected = ops.linear(x, w, bias=b, swiglu=swiglu)
    torch.cuda.synchronize()
    for _ in range(2):  # two calls in a row share (and reuse) the static scratch
        out = torch.full_like(expected, float("nan"))
        rc = _call(fn, w, x, out, swiglu=swiglu, bias=b)
        assert rc == 0, lib.osb_gemm_noalloc_last_error().decode()
        torch.cuda.synchronize()
        assert _rel(out, expected) < TOLERANCE


def test_noalloc_rejects_problems_beyond_its_scratch():
    fn, lib = _entry()
    dev = torch.device("cuda", 0)
    w = torch.zeros(512, 4096, device=dev, dtype=torch.bfloat16)
    x = torch.zeros(200, 4096, device=dev, dtype=torch.bfloat16)
    out = torch.zeros(200, 512, device=dev, dtype=torch.bfloat16)
    rc = _call(fn, w, x, out)
    assert rc == 2
    message = lib.osb_gemm_noalloc_last_error().decode()
    assert "at most" in message and str(lib.osb_gemm_noalloc_scratch_floats()) in message
