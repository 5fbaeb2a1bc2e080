"""Block-scaled fp8 GEMM and activation quantisation against fp32 references."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def C():
    from lunaflux_b200.ops import _ext
    return _ext.load()


def _close(a, b, atol, rtol, what):
    err = (a.float() - b.float()).abs()
    tol = atol + rtol * b.float().abs()
    bad = (err > tol).sum().item()
    assert bad == 0, f"{what}: {bad} / {err.numel()} elements off, max err {err.max().item():.4g}"


def test_act_quant_matches_reference(C):
    from lunaflux_b200.models.fp8 import quantize_act
    x = (torch.randn(77, 1024, device="cuda") * 3).bfloat16()
    q = torch.empty(77, 1024, device="cuda", dtype=torch.float8_e4m3fn)
    s = torch.empty(77, 8, device="cuda")
    C.act_quant(x, q, s)
    rq, rs = quantize_act(x)
    _close(s, rs, 0, 1e-6, "act scales")
    deq = q.float().view(77, 8, 128) * s[..., None]
    _close(deq.view(77, 1024), x.float(), 1e-3, 0.07, "act dequant")


@pytest.mark.parametrize("M,N,K,epi", [(1, 1024, 8192, 0), (128, 3584, 8192, 0), (300, 8192, 1024, 0),
                                       (2048, 1024, 2048, 1), (256, 7168, 8192, 2), (5, 256, 128, 0)])
def test_gemm_fp8_block_scaled(C, M, N, K, epi):
    from lunaflux_b200.models.fp8 import dequantize_weight, quantize_weight
    torch.manual_seed(M + N)
    x = torch.randn(M, K, device="cuda").bfloat16()
    w = torch.randn(N, K, device="cuda") * 0.02
    w8, sw = quantize_weight(w)
    q = torch.empty(M, K, device="cuda", dtype=torch.float8_e4m3fn)
    s = torch.empty(M, K // 128, device="cuda")
    C.act_quant(x, q, s)
    a = q.float() * s.repeat_interleave(128, 1)
    ref = a @ dequantize_weight(w8, sw).t()
    if epi == 2:
        v = ref.view(M, N // 64, 2, 32)
        ref = (torch.nn.functional.silu(v[:, :, 0]) * v[:, :, 1]).reshape(M, N // 2)
    out = torch.empty(ref.shape, device="cuda", dtype=torch.float32 if epi == 1 else torch.bfloat16)
    C.gemm_fp8(q, s, w8, sw, out, epi)
    _close(out, ref, 2e-2, 2e-2, f"fp8 gemm {M}x{N}x{K} epi={epi}")
    assert C.read_error(True)[0] == 0


@pytest.mark.parametrize("M,N,K,epi", [(128, 1280, 8192, 0), (5, 1024, 8192, 1), (256, 2048, 4096, 2),
                                       (100, 1280, 4096, 0)])
def test_gemm_fp8_split_k(C, M, N, K, epi):
    """Decode shapes split K over the idle SMs (atomic fp32 partials into the
    workspace, then the finalize kernel): same values as the fp32 reference,
    and the workspace is all-zero again afterwards."""
    from lunaflux_b200.models.fp8 import dequantize_weight, quantize_weight
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    splits, _ = C.fp8_plan_splits(-(-M // 128) * (N // 128), K // 128, sms)
    assert splits > 1, "the case must exercise the split path"
    torch.manual_seed(M * 7 + N)
    x = torch.randn(M, K, device="cuda").bfloat16()
    w = torch.randn(N, K, device="cuda") * 0.02
    w8, sw = quantize_weight(w)
    q = torch.empty(M, K, device="cuda", dtype=torch.float8_e4m3fn)
    s = torch.empty(M, K // 128, device="cuda")
    C.act_quant(x, q, s)
    ref = (q.float() * s.repeat_interleave(128, 1)) @ dequantize_weight(w8, sw).t()
    if epi == 2:
        v = ref.view(M, N // 64, 2, 32)
        ref = (torch.nn.functional.silu(v[:, :, 0]) * v[:, :, 1]).reshape(M, N // 2)
    ws = torch.zeros(M * N + 64, device="cuda")
    out = torch.full(ref.shape, 7.0, device="cuda", dtype=torch.float32 if epi == 1 else torch.bfloat16)
    for _ in range(2):                                  # the second call relies on the workspace re-zeroed
        C.gemm_fp8(q, s, w8, sw, out, epi, ws)
        torch.cuda.synchronize()
        _close(out, ref, 2e-2, 2e-2, f"fp8 split gemm {M}x{N}x{K} epi={epi}")
        assert ws.abs().max().item() == 0
    assert C.read_error(True)[0] == 0
