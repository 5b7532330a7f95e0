"""The no-allocation GEMM entry point, called through its exported C symbol.

Some callers cannot allocate GPU memory (allocator callbacks, plugin hosts
that forbid cudaMalloc after start-up, real-time loops).  For them the library
exports ``osb_gemm_bf16_noalloc``, which keeps its split-K scratch in a fixed
device array and needs only inputs and outputs.  These tests check it against
an fp32 oracle and against the regular entry point (which uses a caller-side
workspace) over consecutive calls of different split-K shapes, read its status
word after every call, and check that problems too large for the fixed scratch
and malformed arguments are refused.  The file is named so that pytest collects
it last.
"""

import ctypes
import os

import pytest
import torch

from online_speculation_b200.ops import kernels as ops

TOLERANCE = 1e-2  # relative Frobenius error, as in the other GEMM tests


def _library():
    import online_speculation_b200._C as ext

    lib = ctypes.CDLL(ext.__file__)
    fn = lib.osb_gemm_bf16_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int,
                   ctypes.c_int, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_longlong, ctypes.c_int, ctypes.c_void_p]
    lib.osb_gemm_noalloc_last_error.restype = ctypes.c_char_p
    lib.osb_gemm_noalloc_scratch_floats.restype = ctypes.c_longlong
    lib.osb_gemm_noalloc_status.restype = ctypes.c_int
    lib.osb_gemm_noalloc_status.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]
    return fn, lib


def _call(fn, w, x, out, *, swiglu=False, bias=None, residual=None):
    stream = torch.cuda.current_stream().cuda_stream
    M, K = w.shape
    N = x.shape[0]
    return fn(w.data_ptr(), w.stride(0), x.data_ptr(), x.stride(0), M, N, K, out.data_ptr(), out.stride(0),
              int(out.dtype == torch.float32), None if bias is None else bias.data_ptr(),
              None if residual is None else residual.data_ptr(), 0 if residual is None else residual.stride(0),
              int(swiglu), stream)


def _status(lib) -> int:
    code = ctypes.c_int(-1)
    rc = lib.osb_gemm_noalloc_status(torch.cuda.current_stream().cuda_stream, ctypes.byref(code))
    assert rc == 0, lib.osb_gemm_noalloc_last_error().decode()
    return code.value


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


def _problem(M, N, K, swiglu, bias, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    dev = torch.device("cuda", 0)
    w = (torch.randn(M, K, device=dev, generator=g) * 0.05).bfloat16()
    x = torch.randn(N, K, device=dev, generator=g).bfloat16()
    b = torch.randn(M, device=dev, generator=g).bfloat16() if bias else None
    return w, x, b


# (M, N, K, swiglu, bias).  Split-K plans of the regular launcher on 148 SMs:
#   4608 x 64 x 3584   -> 64-token tiles, 36 tiles x 4 splits (1.18 M partial floats)
#   1024 x 16 x 4096   -> 32-token tiles, 8 tiles x 16 splits (0.52 M partial floats)
#   2560 x 64 x 1536   -> SwiGLU epilogue, 20 tiles x 6 splits
#   37888 x 64 x 512   -> 296 tiles: no split-K, no scratch
SHAPES = [(4608, 64, 3584, False, True), (1024, 16, 4096, False, False), (2560, 64, 1536, True, False),
          (37888, 64, 512, False, False)]


@pytest.mark.gpu
@pytest.mark.parametrize("first,second", [(0, 1), (1, 2), (2, 0), (3, 1)])
def test_noalloc_matches_oracle_and_regular_entry_point(first, second):
    """Two consecutive calls of different split-K shapes share the static scratch: leftover
    counters or partial tiles of one call would show up in the other's result."""
    fn, lib = _library()
    problems = [_problem(*SHAPES[i], seed=100 + i) for i in (first, second)]
    for (M, N, K, swiglu, _), (w, x, b) in zip((SHAPES[first], SHAPES[second]), problems):
        oracle = ops.linear_reference(x, w, bias=b, swiglu=swiglu)
        regular = ops.linear(x, w, bias=b, swiglu=swiglu)
        out = torch.full_like(regular, float("nan"))
        rc = _call(fn, w, x, out, swiglu=swiglu, bias=b)
        assert rc == 0, lib.osb_gemm_noalloc_last_error().decode()
        assert _status(lib) == 0
        assert _rel(out, oracle) < TOLERANCE, (M, N, K)
        assert _rel(out, regular) < TOLERANCE, (M, N, K)


@pytest.mark.gpu
def test_noalloc_rejects_problems_beyond_its_scratch():
    """128 x 4096 x 12288: 16 tiles of 256 tokens split 9 ways need 4.72 M partial floats,
    more than the 2.62 M the static scratch holds, so the call is refused and nothing runs."""
    fn, lib = _library()
    dev = torch.device("cuda", 0)
    w = torch.zeros(128, 12288, device=dev, dtype=torch.bfloat16)
    x = torch.zeros(4096, 12288, device=dev, dtype=torch.bfloat16)
    out = torch.full((4096, 128), 7.0, device=dev, dtype=torch.bfloat16)
    rc = _call(fn, w, x, out)
    assert rc == 2
    message = lib.osb_gemm_noalloc_last_error().decode()
    assert "4718592" in message and str(lib.osb_gemm_noalloc_scratch_floats()) in message
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())


def test_noalloc_refuses_malformed_arguments():
    """Argument checks run before any device work, so this needs only the built library."""
    try:
        fn, lib = _library()
    except (ImportError, OSError) as error:
        pytest.skip(f"extension not built: {error}")
    fake = 1 << 20   # never dereferenced: every case below is refused first
    M, N, K = 256, 32, 512
    cases = [
        dict(w=fake + 8, ldw=K, ldx=K, ldo=M),          # w not on a 16-byte boundary
        dict(w=fake, ldw=K + 4, ldx=K, ldo=M),          # weight row stride not a multiple of 8
        dict(w=fake, ldw=K, ldx=K, ldo=M - 1),          # output stride below the output width
    ]
    for c in cases:
        rc = fn(c["w"], c["ldw"], fake, c["ldx"], M, N, K, fake, c["ldo"], 0, None, None, 0, 0, None)
        assert rc == 1, (c, lib.osb_gemm_noalloc_last_error().decode())
    rc = fn(fake, K, fake, K, M, N, K, fake, M, 0, None, fake, M // 2, 0, None)   # residual stride too small
    assert rc == 1
    assert b"residual" in lib.osb_gemm_noalloc_last_error()


if __name__ == "__main__":   # pragma: no cover
    raise SystemExit(pytest.main([os.path.abspath(__file__), "-q"]))
