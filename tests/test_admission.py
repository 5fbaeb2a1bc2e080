"""Model admission: kernel constraints, parallel plan, memory plan."""
from lunaflux_b200.models import spec as specs
from lunaflux_b200.models.admission import Rejection, admit, memory_plan

GIB = 1 << 30
B200 = 183359 * (1 << 20)


def test_llama3_8b_fits_and_tp_plans():
    s = specs.llama3_8b()
    for tp in (1, 2, 4, 8):
        a = admit(s, tp=tp, max_context=1296, max_batch=256, device_bytes=B200)
        assert a.ok, a.details
    m1 = memory_plan(s, 1, 1, 1296, 256, 8192)
    m8 = memory_plan(s, 8, 1, 1296, 256, 8192)
    assert 14 * GIB < m1.weight_bytes < 17 * GIB          # ~8B parameters in bf16
    assert m8.weight_bytes < m1.weight_bytes / 6 and m8.kv_bytes == m1.kv_bytes / 8


def test_llama3_70b_needs_tp_in_bf16_but_fits_fp8_at_tp8():
    bf16 = specs.LlamaSpec(**{**specs.llama3_70b(fp8=False).__dict__})
    a = admit(bf16, tp=1, max_context=2576, max_batch=128, device_bytes=B200)
    assert not a.ok and Rejection.MEMORY in a.reasons
    assert admit(specs.llama3_70b(fp8=True), tp=8, max_context=2576, max_batch=128, device_bytes=B200).ok


def test_rejections_are_typed_and_complete():
    bad = specs.LlamaSpec(hidden=320, layers=2, heads=34, kv_heads=2, head_dim=64, ffn=102, vocab=1001,
                          max_position=512)
    a = admit(bad, tp=4, max_context=1024)
    assert not a.ok
    want = {Rejection.HEAD_DIM, Rejection.GQA_GROUP, Rejection.TP_HEADS, Rejection.TP_FFN, Rejection.TP_VOCAB,
            Rejection.GEMM_ALIGN, Rejection.CONTEXT}
    assert want <= set(a.reasons) and len(a.details) == len(a.reasons)
    assert Rejection.TP_WORLD in admit(specs.llama3_8b(), tp=16).reasons
    assert Rejection.EP_EXPERTS in admit(specs.llama3_8b(), ep=2).reasons
    assert admit(specs.mixtral_8x7b(), tp=8, ep=8, max_context=640, max_batch=512, device_bytes=B200).ok
