"""The allocation-free GEMM entry point, called through its exported C symbol.

`lf_gemm_bf16_noalloc` serves callers that cannot allocate device memory
(host applications that own every device allocation, processes under a strict
memory cap, plugins that may not allocate after start-up): its split-K
scratch is a fixed array inside the library.  This test checks it against
the fp32 product of the same operands and against the allocating entry point
(`_C.gemm`), on two calls in a row through the shared scratch, with the
tolerance of the other GEMM tests; it also checks that an oversized split-K
plan and bad arguments are rejected without touching the output.  The file
is named to be collected last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

OK, BAD_ARGUMENT, TOO_LARGE = 0, 1, 2
SCRATCH_FLOATS = 4 * 1024 * 1024


@pytest.fixture(scope="module")
def lib():
    from lunaflux_b200.ops import _ext
    C = _ext.load()  # loads torch's libraries and the extension
    so = ctypes.CDLL(C.__file__)
    fn = so.lf_gemm_bf16_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p]
    return C, fn


def call(fn, A, B, D, epi):
    stream = torch.cuda.current_stream().cuda_stream
    return fn(A.data_ptr(), B.data_ptr(), D.data_ptr(), A.shape[0], B.shape[0], A.shape[1], A.stride(0),
              B.stride(0), D.stride(0), epi, stream)


def _close(a, b, atol, rtol, what):
    err = (a.float() - b.float()).abs()
    tol = atol + rtol * b.float().abs()
    bad = (err > tol).sum().item()
    assert bad == 0, f"{what}: {bad} / {err.numel()} elements off, max err {err.max().item():.4g}"


def _fp32_reference(A, B, epi):
    ref = A.float() @ B.float().t()
    if epi == 2:
        M, N = ref.shape
        v = ref.view(M, N // 64, 2, 32)
        ref = (torch.nn.functional.silu(v[:, :, 0]) * v[:, :, 1]).reshape(M, N // 2)
    return ref


# Skinny shapes take the split-K path (scratch in use); the large one does not.
@pytest.mark.parametrize("M,N,K,epi", [(1, 4096, 14336, 0), (64, 4096, 4096, 0), (128, 1792, 4096, 2),
                                       (3, 512, 4096, 1), (2048, 2048, 512, 0)])
def test_noalloc_matches_fp32_product(lib, M, N, K, epi):
    C, fn = lib
    torch.manual_seed(M + N + K)
    A = torch.randn(M, K, device="cuda").bfloat16()
    B = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    cols = N // 2 if epi == 2 else N
    dt = torch.float32 if epi == 1 else torch.bfloat16
    ref = _fp32_reference(A, B, epi)
    alloc = torch.empty(M, cols, device="cuda", dtype=dt)
    C.gemm(A, B, alloc, epi, 0, None)
    for _ in range(2):  # two calls in a row through the shared scratch
        D = torch.full((M, cols), float("nan"), device="cuda", dtype=dt)
        assert call(fn, A, B, D, epi) == OK
        torch.cuda.synchronize()
        _close(D, ref, 3e-2, 3e-2, f"noalloc vs fp32 {M}x{N}x{K} epi={epi}")
        _close(D, alloc, 3e-2, 3e-2, f"noalloc vs _C.gemm {M}x{N}x{K} epi={epi}")
    assert C.read_error(True)[0] == 0


def test_noalloc_rejects_oversized_plans_and_bad_arguments(lib):
    C, fn = lib
    # the smallest 256-row shape whose split-K plan needs more scratch than
    # the array holds, on this device's SM count
    M, K = 256, 16384
    shape = None
    for N in range(256, 8192, 256):
        splits = C.gemm_plan_splitk(M, N, K)
        if splits > 1 and splits * M * N > SCRATCH_FLOATS:
            shape = (M, N, K)
            break
    if shape is None:
        pytest.skip("no 256-row shape splits beyond the scratch on this device")
    M, N, K = shape
    A = torch.zeros(M, K, device="cuda", dtype=torch.bfloat16)
    B = torch.zeros(N, K, device="cuda", dtype=torch.bfloat16)
    D = torch.full((M, N), 7.0, device="cuda", dtype=torch.bfloat16)
    assert call(fn, A, B, D, 0) == TOO_LARGE
    assert call(fn, A[:, :7], B[:, :7], D, 0) == BAD_ARGUMENT  # K not a multiple of 8
    assert call(fn, A, B, D, 9) == BAD_ARGUMENT                # unknown epilogue
    torch.cuda.synchronize()
    assert bool((D == 7.0).all()), "a rejected call wrote its output"
