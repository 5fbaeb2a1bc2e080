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
    # every projection and the LM head split 8 ways; the 1 GiB embedding table is replicated
    emb = s.vocab * s.hidden * 2
    assert m8.weight_bytes - emb < (m1.weight_bytes - emb) / 7.9 and m8.kv_bytes == m1.kv_bytes / 8


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


def _runtime_bytes(spec, tp, ep=1):
    from lunaflux_b200.models.weights import build_runtime, random_checkpoint
    from lunaflux_b200.parallel.tp import TPShard
    ck = random_checkpoint(spec, 0)
    return build_runtime(spec, ck.__getitem__, TPShard(0, tp, spec), ep_rank=0, ep_size=ep).nbytes()


def test_memory_plan_weights_equal_the_runtime_layout():
    """The plan's weight term is the bytes build_runtime really holds on a
    rank: replicated embedding, vocabulary-sharded LM head, FFN shards padded
    to the interleave group, fp32 router, fp8 block scales."""
    import pytest
    dense = specs.tiny_llama()                                   # ffn 172: padded per shard
    gqa = specs.LlamaSpec(hidden=64, layers=2, heads=4, kv_heads=1, head_dim=16, ffn=96, vocab=256,
                          max_position=512)                       # KV heads replicated past tp 1
    moe = specs.LlamaSpec(hidden=64, layers=2, heads=4, kv_heads=2, head_dim=16, ffn=96, vocab=256,
                          max_position=512, experts=4, experts_per_token=2)
    fp8 = specs.LlamaSpec(hidden=256, layers=1, heads=2, kv_heads=1, head_dim=128, ffn=512, vocab=256,
                          max_position=512, fp8_block=128)
    cases = [(dense, 1, 1), (dense, 2, 1), (dense, 4, 1), (gqa, 2, 1), (gqa, 4, 1),
             (moe, 1, 1), (moe, 2, 1), (moe, 1, 2), (fp8, 1, 1), (fp8, 2, 1)]
    for spec, tp, ep in cases:
        try:
            want = _runtime_bytes(spec, tp, ep)
        except Exception as e:                                    # a layout this CPU build cannot make
            pytest.fail(f"{spec} tp={tp} ep={ep}: {e}")
        assert memory_plan(spec, tp, ep, 64, 4, 64).weight_bytes == want, (spec, tp, ep)


def test_plan_arguments_out_of_range_are_rejections():
    import pytest
    s = specs.llama3_8b()
    assert Rejection.CONTEXT in admit(s, max_context=0).reasons
    assert Rejection.CONTEXT in admit(s, max_context=s.max_position + 1).reasons
    assert Rejection.BATCH in admit(s, max_batch=0).reasons
    assert Rejection.BATCH in admit(s, step_tokens=-1).reasons
    assert Rejection.TP_WORLD in admit(s, tp=0).reasons
    for ep in (0, 16):
        assert Rejection.EP_EXPERTS in admit(specs.mixtral_8x7b(), ep=ep).reasons
    with pytest.raises(ValueError):
        admit(s, reserve_fraction=1.0)
    # the memory check uses the reserve: a plan that fits only without it is refused
    need = admit(s, max_context=1296, max_batch=256).memory.total
    assert admit(s, max_context=1296, max_batch=256, device_bytes=need, reserve_fraction=0.0).ok
    a = admit(s, max_context=1296, max_batch=256, device_bytes=need, reserve_fraction=0.05)
    assert a.reasons == [Rejection.MEMORY] and len(a.details) == 1


def test_memory_plan_kv_equals_the_runner_arena():
    """The KV term is the runner's arena: every sequence's pages plus the
    reserved all-zero page that padded rows read."""
    from lunaflux_b200.config import CacheConfig, SchedulerConfig
    from lunaflux_b200.engine.engine import EngineOptions, LLMEngine
    from lunaflux_b200.models.weights import build_runtime, random_checkpoint
    from lunaflux_b200.ops import TorchOps
    spec = specs.tiny_llama()
    ck = random_checkpoint(spec, 0)
    eng = LLMEngine(build_runtime(spec, ck.__getitem__), TorchOps(), "cpu",
                    SchedulerConfig(step_token_budget=64, max_active_requests=4, prefill_chunk_tokens=64),
                    CacheConfig(), EngineOptions(max_context=256, num_pages=4 * 256 // 16, graph_sizes=()))
    assert memory_plan(spec, 1, 1, 256, 4, 64).kv_bytes == eng.runner.kv.nbytes
