"""Launch contracts (CPU): operand admission for the step's entry points and
paged admission of packed steps against the KV arena.

Reference behaviour: kernels/launch_contract (typed rejections of launch
metadata: dimensions, operand roles, alignment; admit_paged_kv bounds step
counts, positions, lengths and page indices by the KV layout)."""
import numpy as np
import pytest
import torch

from lunaflux_b200.ops import launch_contract as lc
from lunaflux_b200.ops.launch_contract import CONTRACTS, Issue, LaunchContractError, PagedIssue, PagedStepError, admit

bf, f32, i32 = torch.bfloat16, torch.float32, torch.int32


def z(*shape, dtype=bf):
    return torch.zeros(*shape, dtype=dtype)


def test_gemm_admits_and_binds_dims():
    a = admit(CONTRACTS["linear"], (z(256, 4096), z(6144, 4096), z(256, 6144)), {"epi": 0})
    assert a.dim("M") == 256 and a.dim("N") == 6144 and a.dim("K") == 4096
    assert dict(a.operand_bytes)["A"] == 256 * 4096 * 2
    # SwiGLU output is half as wide
    admit(CONTRACTS["linear"], (z(8, 64), z(128, 64), z(8, 64)), {"epi": 2})
    # fp32 logits
    admit(CONTRACTS["linear"], (z(8, 64), z(128, 64), z(8, 128, dtype=f32)), {"epi": 1})


@pytest.mark.parametrize("case,issue", [
    ("dtype", Issue.DTYPE), ("rank", Issue.RANK), ("k_mismatch", Issue.SHAPE),
    ("out_cols", Issue.RULE), ("n_tile", Issue.RULE), ("stride", Issue.LAYOUT), ("noncontig", Issue.LAYOUT),
    ("base", Issue.ALIGNMENT), ("missing", Issue.MISSING),
])
def test_gemm_rejections_are_typed(case, issue):
    A, B, D = z(16, 64), z(128, 64), z(16, 128)
    if case == "dtype":
        A = A.half()
    elif case == "rank":
        A = z(2, 8, 64)
    elif case == "k_mismatch":
        B = z(128, 72)
    elif case == "out_cols":
        D = z(16, 64)
    elif case == "n_tile":
        B, D = z(104, 64), z(16, 104)
    elif case == "stride":
        A = z(16, 68)[:, :64]          # 136-byte rows
    elif case == "noncontig":
        A = z(64, 16).t()
    elif case == "base":
        A = z(16 * 64 + 1)[1:].view(16, 64)
    elif case == "missing":
        A = None
    with pytest.raises(LaunchContractError) as e:
        admit(CONTRACTS["linear"], (A, B, D), {"epi": 0})
    assert e.value.issue is issue and e.value.op == "linear"


def test_attention_contracts():
    kc = z(9, 8, 16, 128)
    q, out = z(32, 6144), z(32, 4096)
    bt = torch.zeros(4, 8, dtype=i32)
    admit(CONTRACTS["attn_decode"], (q, out, z(4, dtype=i32), z(4, dtype=i32), bt, kc, kc), {"Hq": 32, "Hkv": 8})
    admit(CONTRACTS["attn_prefill"], (q, out, z(5, dtype=i32), z(4, dtype=i32), bt, kc, kc), {"Hq": 32, "Hkv": 8})
    with pytest.raises(LaunchContractError) as e:   # GQA ratio
        admit(CONTRACTS["attn_decode"], (q, out, z(4, dtype=i32), z(4, dtype=i32), bt, kc, kc), {"Hq": 36, "Hkv": 8})
    assert e.value.issue is Issue.RULE
    with pytest.raises(LaunchContractError) as e:   # KV head count disagrees with the cache
        admit(CONTRACTS["attn_decode"], (q, out, z(4, dtype=i32), z(4, dtype=i32), bt, kc, kc), {"Hq": 32, "Hkv": 4})
    assert e.value.issue is Issue.SHAPE
    with pytest.raises(LaunchContractError) as e:   # page of 32 tokens
        admit(CONTRACTS["attn_decode"], (q, out, z(4, dtype=i32), z(4, dtype=i32), bt, z(9, 8, 32, 128),
                                         z(9, 8, 32, 128)), {"Hq": 32, "Hkv": 8})
    assert e.value.issue is Issue.SHAPE


def test_qkv_rope_and_sampler_contracts():
    kc = z(9, 8, 16, 128)
    args = (z(4, 4096), z(6144, 4096), z(4, 6144), z(4, dtype=i32), z(4, dtype=i32), z(2048 * 64 * 2, dtype=f32), kc, kc)
    admit(CONTRACTS["linear_qkv_rope"], args, {"Hq": 32, "Hkv": 8, "page": 16})
    with pytest.raises(LaunchContractError):
        admit(CONTRACTS["linear_qkv_rope"], args, {"Hq": 24, "Hkv": 8, "page": 16})
    admit(CONTRACTS["sample"], (z(4, 1000, dtype=f32), z(32, dtype=i32), z(4, dtype=i32)))
    with pytest.raises(LaunchContractError) as e:
        admit(CONTRACTS["sample"], (z(4, 1000, dtype=f32), z(31, dtype=i32), z(4, dtype=i32)))
    assert e.value.issue is Issue.RULE


def test_moe_and_fp8_contracts():
    admit(CONTRACTS["moe_grouped_linear"], (z(512, 256), z(8, 1024, 256), z(512, 512), z(9, dtype=i32)),
          {"epi": 2, "align": 256, "num_groups": 8})
    with pytest.raises(LaunchContractError):   # 384 rows are not whole 256-row segments
        admit(CONTRACTS["moe_grouped_linear"], (z(384, 256), z(8, 1024, 256), z(384, 512), z(9, dtype=i32)),
              {"epi": 2, "align": 256, "num_groups": 8})
    admit(CONTRACTS["moe_route"], (z(4, 256), z(8, 256, dtype=f32), None, z(4, 2, dtype=i32), z(4, 2, dtype=f32)),
          {"topk": 2})
    with pytest.raises(LaunchContractError):   # 6 experts
        admit(CONTRACTS["moe_route"], (z(4, 256), z(6, 256, dtype=f32), None, z(4, 2, dtype=i32), z(4, 2, dtype=f32)),
              {"topk": 2})
    e4 = torch.float8_e4m3fn
    admit(CONTRACTS["linear_fp8"], (z(4, 256, dtype=e4), z(4, 2, dtype=f32), z(512, 256, dtype=e4),
                                    z(4, 2, dtype=f32), z(4, 512)), {"epi": 0})
    with pytest.raises(LaunchContractError):   # missing weight scales
        admit(CONTRACTS["linear_fp8"], (z(4, 256, dtype=e4), z(4, 2, dtype=f32), z(512, 256, dtype=e4),
                                        z(2, 2, dtype=f32), z(4, 512)), {"epi": 0})
    admit(CONTRACTS["act_quant"], (z(4, 256), z(4, 256, dtype=e4), z(4, 2, dtype=f32)))


def test_install_admits_before_the_call():
    calls = []

    class Fake:
        def gemm(self, A, B, out, epi=0, ws=None):
            calls.append("gemm")

        def rmsnorm(self, x, residual, w, out, eps):
            calls.append("rmsnorm")

    ops = Fake()
    lc.install(ops)
    ops.gemm(z(8, 64), z(128, 64), z(8, 128))
    ops.rmsnorm(z(8, 64), None, z(64), z(8, 64), 1e-5)
    assert calls == ["gemm", "rmsnorm"] and ops.admitted == 2
    with pytest.raises(LaunchContractError):
        ops.gemm(z(8, 64), z(128, 64), z(8, 96))
    assert calls == ["gemm", "rmsnorm"]        # the rejected call never reached the launch


# ------------------------------------------------------------------ paged admission
def _step(rows_prefill, rows_decode, W=4, P=16):
    """A packed step from hand-made rows: prefill (pages, start, n), decode (pages, position)."""
    from lunaflux_b200.engine.step_inputs import make_layout
    Tp = sum(n for _, _, n in rows_prefill)
    Rp, Rd = len(rows_prefill), len(rows_decode)
    T = Tp + Rd
    L = make_layout(T, Rp, Rd, 1, W)
    buf = np.zeros(L.total, dtype=np.int32)

    def put(name, arr):
        o, n = L.field(name)
        buf[o:o + n] = arr

    pos, slots, qs, sl, pbt = [], [], [0], [], []
    for pages, s, n in rows_prefill:
        for p in range(s, s + n):
            pos.append(p)
            slots.append(pages[p // P] * P + p % P)
        qs.append(qs[-1] + n)
        sl.append(s + n)
        pbt += pages + [0] * (W - len(pages))
    dbt, dsl = [], []
    for pages, p in rows_decode:
        pos.append(p)
        slots.append(pages[p // P] * P + p % P)
        dsl.append(p + 1)
        dbt += pages + [0] * (W - len(pages))
    put("tokens", np.arange(T) % 50)
    put("positions", pos)
    put("slots", slots)
    if Rp:
        put("p_qstart", qs)
        put("p_seqlen", sl)
        put("p_bt", pbt)
    if Rd:
        put("d_tok", np.arange(Tp, T))
        put("d_seqlen", dsl)
        put("d_bt", dbt)
    put("s_idx", [T - 1])
    return L, buf


def test_paged_step_admits_a_consistent_step():
    L, buf = _step([([1, 2], 0, 20), ([3], 4, 6)], [([4, 5], 17), ([6], 0)])
    lc.check_paged_step(L, buf, num_pages=8, page_size=16, vocab=64)


@pytest.mark.parametrize("mutate,issue", [
    (lambda L, b: _set(L, b, "p_bt", 0, 99), PagedIssue.PAGE),
    (lambda L, b: _set(L, b, "d_bt", 1, -1), PagedIssue.PAGE),
    (lambda L, b: _set(L, b, "d_seqlen", 0, 4 * 16 + 1), PagedIssue.SEQ_LEN),
    (lambda L, b: _set(L, b, "slots", 3, 5 * 16), PagedIssue.SLOT),
    (lambda L, b: _set(L, b, "slots", 0, 10 ** 6), PagedIssue.SLOT),
    (lambda L, b: _set(L, b, "p_qstart", 1, 30), PagedIssue.Q_START),
    (lambda L, b: _set(L, b, "positions", 2, 25), PagedIssue.POSITION),
    (lambda L, b: _set(L, b, "tokens", 0, 64), PagedIssue.TOKEN),
    (lambda L, b: _set(L, b, "s_idx", 0, 1000), PagedIssue.SAMPLE),
])
def test_paged_step_rejections(mutate, issue):
    L, buf = _step([([1, 2], 0, 20), ([3], 4, 6)], [([4, 5], 17), ([6], 0)])
    mutate(L, buf)
    with pytest.raises(PagedStepError) as e:
        lc.check_paged_step(L, buf, num_pages=8, page_size=16, vocab=64)
    assert e.value.issue is issue


def _set(L, buf, name, i, v):
    o, n = L.field(name)
    assert i < n
    buf[o + i] = v


def test_engine_steps_pass_paged_admission(monkeypatch):
    """Every step the CPU engine packs for a real workload is admitted."""
    monkeypatch.setenv("LUNAFLUX_CHECK_LAUNCHES", "1")
    from lunaflux_b200.config import CacheConfig, SchedulerConfig
    from lunaflux_b200.engine.engine import EngineOptions, LLMEngine
    from lunaflux_b200.models.spec import tiny_llama
    from lunaflux_b200.models.weights import build_runtime, random_checkpoint
    from lunaflux_b200.ops.torch_ops import TorchOps

    spec = tiny_llama()
    ck = random_checkpoint(spec, 0)
    w = build_runtime(spec, lambda n: ck[n])
    sched = SchedulerConfig(step_token_budget=32, max_active_requests=4, prefill_chunk_tokens=16,
                            emergency_decode_page_reserve=1, waiting_age_threshold_steps=8)
    eng = LLMEngine(w, TorchOps(), "cpu", sched, CacheConfig(prefix_enabled=True),
                    EngineOptions(max_context=128, num_pages=32, graph_sizes=()))
    assert eng.runner.check_steps
    calls = []
    real = lc.check_paged_step

    def spy(*a, **k):
        calls.append(1)
        return real(*a, **k)

    monkeypatch.setattr("lunaflux_b200.engine.runner.check_paged_step", spy)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, spec.vocab, (n,), generator=g).tolist() for n in (5, 19, 33, 40)]
    outs = eng.generate(prompts, 8)
    assert all(len(o) == 8 for o in outs) and len(calls) >= 8


def test_fp8_split_plan_covers_k_exactly():
    """The fp8 split-K plan (host code of the extension): every split gets at
    least 4 K blocks, the splits cover K exactly, and shapes with many tiles
    or short K are not split."""
    from lunaflux_b200.ops import _ext
    try:
        C = _ext.load()
    except Exception as e:   # pragma: no cover - the extension is built by build()
        pytest.skip(f"extension not loadable here: {e}")
    for tiles in (1, 8, 10, 20, 56, 64, 74, 75, 148, 300):
        for num_kb in (1, 8, 28, 31, 32, 64, 112):
            splits, per = C.fp8_plan_splits(tiles, num_kb, 148)
            assert splits >= 1 and per >= 1
            assert (splits - 1) * per < num_kb <= splits * per
            if splits > 1:
                assert per >= 4 and tiles * 2 <= 148 and num_kb >= 32 and tiles * splits <= 148
            if tiles * 2 > 148 or num_kb < 32:
                assert splits == 1
