"""The allocation-free GEMM entry point, called through its exported C symbol.

`lf_gemm_bf16_noalloc` serves callers that cannot allocate device memory
(host applications that own every device allocation, processes under a strict
memory cap, plugins that may not allocate after start-up): its split-K
scratch is a fixed array inside the library.  This test checks it against
the allocating entry point (`_C.gemm` with a caller workspace) on two calls in
a row, with the same tolerance as the other GEMM tests, and checks that an
oversized split-K plan is rejected.  The file is named to be collected last.
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


# Skinny shapes take the split-K path (scratch in use); the large one does not.
@pytest.mark.parametrize("M,N,K,epi", [(1, 4096, 14336, 0), (64, 4096, 4096, 0), (128, 1792, 4096, 2),
                                       (3, 512, 4096, 1), (2048, 2048, 512, 0)])
def test_noalloc_matches_allocating_entry_point(lib, M, N, K, epi):
    C, fn = lib
    torch.manual_seed(M + N + K)
    A = torch.randn(M, K, device="cuda").bfloat16()
    B = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    cols = N // 2 if epi == 2 else N
    dt = torch.float32 if epi == 1 else torch.bfloat16
    ws = torch.zeros(512 * 32768, device="cuda")
    ref = torch.empty(M, cols, device="cuda", dtype=dt)
    C.gemm(A, B, ref, epi, 0, ws)
    for _ in range(2):  # two calls in a row through the shared scratch
        D = torch.full((M, cols), float("nan"), device="cuda", dtype=dt)
        assert call(fn, A, B, D, epi) == OK
        torch.cuda.synchronize()
        _close(D, ref, 3e-2, 3e-2, f"noalloc {M}x{N}x{K} epi={epi}")
    assert C.read_error(True)[0] == 0


def test_noalloc_rejects_oversized_plans_and_bad_arguments(lib):
    C, fn = lib
    # 256 x 2560 splits K 7 ways: 7 x 655360 floats of scratch, more than the 4M-float array.
    M, N, K = 256, 2560, 16384
    splits = C.gemm_plan_splitk(M, N, K)
    assert splits * M * N > SCRATCH_FLOATS
    A = torch.zeros(M, K, device="cuda", dtype=torch.bfloat16)
    B = torch.zeros(N, K, device="cuda", dtype=torch.bfloat16)
    D = torch.zeros(M, N, device="cuda", dtype=torch.bfloat16)
    assert call(fn, A, B, D, 0) == TOO_LARGE
    assert call(fn, A[:, :7], B[:, :7], D, 0) == BAD_ARGUMENT  # K not a multiple of 8
    assert call(fn, A, B, D, 9) == BAD_ARGUMENT
