"""Kernel micro-benchmarks: each hot sm_100a kernel against its library baseline.

    python -m lunaflux_b200.bench.kernels [--only gemm|attn|norm|sample|fp8|moe] [--json out.json] [--variants]

Timing: CUDA events on the launching stream, warm-up first, an L2 flush (a
256 MB write) before every timed launch, median of the timed launches.  The
roofline denominators come from MEASURED_PEAKS.json when present.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics

import torch

from lunaflux_b200.ops import _ext

_FLUSH = None


def _flush():
    global _FLUSH
    if _FLUSH is None:
        _FLUSH = torch.empty(256 * 1024 * 1024 // 4, device="cuda", dtype=torch.float32)
    _FLUSH.fill_(1.0)


def time_fn(fn, iters=10, warmup=3, flush=True):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        if flush:
            _flush()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    return statistics.median(ts)


def peaks():
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                     "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def bench_gemm(C, results, only_case="", variants=False):
    hbm, tflops_peak, src = peaks()
    shapes = [
        ("prefill qkv", 8192, 6144, 4096, 0), ("prefill o", 8192, 4096, 4096, 0),
        ("prefill gate_up+swiglu", 8192, 28672, 4096, 2), ("prefill down", 8192, 4096, 14336, 0),
        ("decode256 qkv", 256, 6144, 4096, 0), ("decode256 o", 256, 4096, 4096, 0),
        ("decode256 gate_up+swiglu", 256, 28672, 4096, 2), ("decode256 down", 256, 4096, 14336, 0),
        ("decode256 lm_head", 256, 128256, 4096, 1), ("decode64 qkv", 64, 6144, 4096, 0),
        ("decode1 down", 1, 4096, 14336, 0), ("tp8 decode256 gate_up", 256, 3584, 4096, 2),
        ("square 8192", 8192, 8192, 8192, 0),
    ]
    for name, M, N, K, epi in shapes:
        if only_case and name != only_case:
            continue
        A = torch.randn(M, K, device="cuda").bfloat16()
        B = (torch.randn(N, K, device="cuda") * 0.02).bfloat16()
        if epi == 2:
            D = torch.empty(M, N // 2, device="cuda", dtype=torch.bfloat16)
        elif epi == 1:
            D = torch.empty(M, N, device="cuda", dtype=torch.float32)
        else:
            D = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        ws = torch.zeros(512 * 32768, device="cuda")
        ours = time_fn(lambda: C.gemm(A, B, D, epi, 0, ws))
        if epi == 2:
            def base():
                gu = A @ B.t()
                torch.nn.functional.silu(gu[:, : N // 2]) * gu[:, N // 2:]
        elif epi == 1:
            def base():
                torch.matmul(A, B.t(), out=None).float()
        else:
            def base():
                A @ B.t()
        ref = time_fn(base)
        extra = {}
        if variants:
            # opt-in kernel variants of the same call, timed the same way
            # (the CTA-pair kernel is on by default: time the single-CTA kernel)
            pair_was = C.gemm_get_pair()
            for key, setter, on in (("single_cta_ms", C.gemm_set_pair, False),
                                    ("cluster_256_rows_ms", C.gemm_set_cluster_mb2, True)):
                setter(on)
                try:
                    extra[key] = time_fn(lambda: C.gemm(A, B, D, epi, 0, ws))
                finally:
                    setter(pair_was if setter is C.gemm_set_pair else False)
        flops = 2.0 * M * N * K
        bytes_ = 2.0 * (M * K + N * K) + D.numel() * D.element_size()
        t_roof = max(flops / (tflops_peak * 1e12), bytes_ / (hbm * 1e9)) * 1e3
        c, cbn, _, cmb = C.gemm_plan_cluster(M, N, K, epi)
        r = dict(kernel="gemm_bf16", case=name, M=M, N=N, K=K, bn=cbn if c else C.gemm_choose_bn(M, N, epi),
                 cluster_splitk=c, cluster_rows=128 * cmb if c else None, ours_ms=ours,
                 torch_ms=ref, speedup=ref / ours, tflops=flops / ours / 1e9, roofline_ms=t_roof,
                 frac_of_roofline=t_roof / ours, peaks=src, **extra)
        results.append(r)
        print(json.dumps(r))
        del A, B, D


def bench_qkv_rope(C, results):
    """QKV projection followed by RoPE + paged KV write, against the single
    kernel with both in its epilogue (Llama-3-8B heads at TP 1)."""
    Hq, Hkv, D, P = 32, 8, 128, 16
    K, N = 4096, (32 + 16) * 128
    pages = 4096
    table = torch.randn(8192, D // 2, 2, device="cuda")
    kc = torch.zeros(pages, Hkv, P, D, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    B = (torch.randn(N, K, device="cuda") * 0.02).bfloat16()
    for M in (256, 8192):
        A = torch.randn(M, K, device="cuda").bfloat16()
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        pos = torch.randint(0, 8192, (M,), device="cuda", dtype=torch.int32)
        slots = torch.randperm(pages * P, device="cuda")[:M].int()

        def two():
            C.gemm(A, B, out, 0, 0, None)
            C.rope_kv_write(out, pos, slots, table, kc, vc, Hq, Hkv, P)

        def one():
            C.gemm_qkv_rope(A, B, out, pos, slots, table, kc, vc, Hq, Hkv, P)

        r = dict(kernel="qkv_rope", M=M, N=N, K=K, gemm_then_rope_ms=time_fn(two), fused_ms=time_fn(one))
        results.append(r)
        print(json.dumps(r))


def bench_attn(C, results):
    hbm, _, src = peaks()
    D, P = 128, 16
    for rows, L, Hq, Hkv in [(256, 1152, 32, 8), (64, 2048, 32, 8), (1, 4096, 32, 8), (128, 2304, 8, 1)]:
        pages_per = math.ceil(L / P)
        n_pages = rows * pages_per + 1
        kc = torch.randn(n_pages, Hkv, P, D, device="cuda").bfloat16()
        vc = torch.randn_like(kc)
        bt = (torch.randperm(n_pages - 1, device="cuda")[: rows * pages_per] + 1).int().view(rows, pages_per)
        q = torch.randn(rows, (Hq + 2 * Hkv) * D, device="cuda").bfloat16()
        out = torch.empty(rows, Hq * D, device="cuda", dtype=torch.bfloat16)
        tok = torch.arange(rows, device="cuda", dtype=torch.int32)
        sl = torch.full((rows,), L, device="cuda", dtype=torch.int32)
        splits = C.attn_decode_splits(rows, Hkv, L, torch.cuda.get_device_properties(0).multi_processor_count)
        po = torch.empty(rows * Hq * splits * D, device="cuda")
        pl = torch.empty(rows * Hq * splits, device="cuda")
        ms = time_fn(lambda: C.attn_decode(q, out, tok, sl, bt, kc, vc, Hq, Hkv, splits, po, pl))
        kv_bytes = rows * L * Hkv * D * 2 * 2
        # every split count the model could pick, timed the same way (checks the cost model)
        sweep = {}
        for s_ in (1, 2, 3, 4, 6, 8):
            if s_ > 1 and math.ceil(L / P) // s_ < 8:
                break
            po_ = torch.empty(rows * Hq * s_ * D, device="cuda")
            pl_ = torch.empty(rows * Hq * s_, device="cuda")
            sweep[s_] = time_fn(lambda: C.attn_decode(q, out, tok, sl, bt, kc, vc, Hq, Hkv, s_, po_, pl_))
        lib_ms = None
        try:   # vLLM's paged flash-attention on the same cache (the library baseline's kernel)
            from lunaflux_b200.ops.library_ops import LibraryOps
            lib = LibraryOps("cuda")
            lib_ms = time_fn(lambda: lib.attn_decode(q, out, tok, sl, bt, kc, vc, Hq, Hkv, 1, po, pl))
        except Exception:
            pass
        r = dict(kernel="attn_decode", rows=rows, seq=L, Hq=Hq, Hkv=Hkv, splits=splits, ours_ms=ms,
                 gbs=kv_bytes / ms / 1e6, frac_of_hbm=kv_bytes / ms / 1e6 / hbm, peaks=src,
                 split_sweep_ms=sweep, library_ms=lib_ms)
        results.append(r)
        print(json.dumps(r))
    # prefill: 8 prompts x 1024 tokens, causal
    for nreq, L, Hq, Hkv in [(8, 1024, 32, 8), (2, 4096, 32, 8)]:
        pages_per = math.ceil(L / P)
        n_pages = nreq * pages_per + 1
        kc = torch.randn(n_pages, Hkv, P, D, device="cuda").bfloat16()
        vc = torch.randn_like(kc)
        bt = (torch.randperm(n_pages - 1, device="cuda")[: nreq * pages_per] + 1).int().view(nreq, pages_per)
        T = nreq * L
        q = torch.randn(T, (Hq + 2 * Hkv) * D, device="cuda").bfloat16()
        out = torch.empty(T, Hq * D, device="cuda", dtype=torch.bfloat16)
        qs = torch.arange(0, T + 1, L, device="cuda", dtype=torch.int32)
        sl = torch.full((nreq,), L, device="cuda", dtype=torch.int32)
        ms = time_fn(lambda: C.attn_prefill(q, out, qs, sl, bt, kc, vc, Hq, Hkv, L))
        os.environ["LUNAFLUX_PREFILL_MMA_SYNC"] = "1"     # the mma.sync kernel, for comparison
        try:
            ms_sync = time_fn(lambda: C.attn_prefill(q, out, qs, sl, bt, kc, vc, Hq, Hkv, L))
        finally:
            del os.environ["LUNAFLUX_PREFILL_MMA_SYNC"]
        flops = nreq * Hq * 4.0 * D * L * L / 2
        qf = q[:, : Hq * D].view(nreq, L, Hq, D).transpose(1, 2)
        kf = torch.randn(nreq, Hkv, L, D, device="cuda").bfloat16().repeat_interleave(Hq // Hkv, 1)
        vf = torch.randn_like(kf)
        from torch.nn.attention import SDPBackend, sdpa_kernel
        dense = {}
        for name_, be in (("flash", SDPBackend.FLASH_ATTENTION), ("cudnn", SDPBackend.CUDNN_ATTENTION)):
            try:
                with sdpa_kernel([be]):
                    dense[name_] = time_fn(lambda: torch.nn.functional.scaled_dot_product_attention(
                        qf, kf, vf, is_causal=True))
            except Exception:
                dense[name_] = None
        lib_ms = None
        try:   # vLLM's paged flash-attention on the same paged cache (the library baseline's kernel)
            from lunaflux_b200.ops.library_ops import LibraryOps
            lib = LibraryOps("cuda")
            host = {"seq_lens": sl.cpu().numpy()}
            lib_ms = time_fn(lambda: lib.attn_prefill(q, out, qs, sl, bt, kc, vc, Hq, Hkv, L, host=host))
        except Exception:
            pass
        r = dict(kernel="attn_prefill", nreq=nreq, seq=L, ours_ms=ms, mma_sync_ms=ms_sync,
                 sdpa_dense_ms=dense, library_paged_ms=lib_ms, tflops=flops / ms / 1e9, peaks=src)
        results.append(r)
        print(json.dumps(r))


def bench_norm(C, results):
    hbm, _, src = peaks()
    for T, H in [(8192, 4096), (256, 4096), (8192, 8192)]:
        x = torch.randn(T, H, device="cuda").bfloat16()
        res = torch.randn_like(x)
        w = torch.ones(H, device="cuda", dtype=torch.bfloat16)
        out = torch.empty_like(x)
        ms = time_fn(lambda: C.rmsnorm(x, res, w, out, 1e-5))
        byts = 4 * T * H * 2
        r = dict(kernel="rmsnorm_residual", T=T, H=H, ours_ms=ms, gbs=byts / ms / 1e6, frac_of_hbm=byts / ms / 1e6 / hbm,
                 peaks=src)
        results.append(r)
        print(json.dumps(r))


def bench_sample(C, results):
    """Greedy argmax and the top-k / top-p sampler over a Llama-3 logits row
    block, against torch.argmax and torch.topk + softmax + multinomial."""
    from lunaflux_b200.sampling.host import pack_params
    hbm, _, src = peaks()
    for R, V in [(256, 128256), (1, 128256), (256, 16032)]:
        logits = torch.randn(R, V, device="cuda") * 3
        out = torch.empty(R, dtype=torch.int32, device="cuda")
        ms_arg = time_fn(lambda: C.argmax(logits, out, None))
        base_arg = time_fn(lambda: torch.argmax(logits, -1))
        rows = [(1, 40, 0.7, 0.9, 1000 + i, i) for i in range(R)]
        params = torch.from_numpy(pack_params(rows).view("u1").copy()).cuda()
        ms_s = time_fn(lambda: C.sample(logits, params, out, None))

        def torch_sample():
            v, i = torch.topk(logits / 0.7, 40, dim=-1)
            p = torch.softmax(v, -1)
            c = torch.cumsum(p, -1)
            p = torch.where(c - p > 0.9, torch.zeros_like(p), p)
            return i.gather(1, torch.multinomial(p, 1))

        base_s = time_fn(torch_sample)
        byts = R * V * 4
        r = dict(kernel="sample", rows=R, vocab=V, argmax_ms=ms_arg, torch_argmax_ms=base_arg, topk_topp_ms=ms_s,
                 torch_topk_topp_ms=base_s, argmax_frac_of_hbm=byts / ms_arg / 1e6 / hbm, peaks=src)
        results.append(r)
        print(json.dumps(r))


def bench_fp8(C, results):
    """Block-scaled e4m3 GEMM (128 x 128 weight blocks, 1 x 128 activation
    groups) on the Llama-3-70B TP 8 shard shapes, against cuBLAS bf16 and
    torch._scaled_mm (row-wise fp8 scales, the library's fp8 path)."""
    from lunaflux_b200.models.fp8 import quantize_act, quantize_weight
    _, tflops_peak, src = peaks()
    shapes = [("tp8 qkv", 1280, 8192), ("tp8 o", 8192, 1024), ("tp8 gate_up", 7168, 8192), ("tp8 down", 8192, 3584)]
    for M in (128, 8192):
        for name, N, K in shapes:
            x = torch.randn(M, K, device="cuda").bfloat16()
            w = (torch.randn(N, K, device="cuda") * 0.02)
            w8, sw = quantize_weight(w)
            q, s_ = quantize_act(x)
            q, s_ = q.cuda().contiguous(), s_.cuda().contiguous()
            out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
            w8c, swc = w8.cuda(), sw.cuda()
            ms_nosplit = time_fn(lambda: C.gemm_fp8(q, s_, w8c, swc, out, 0))
            ws = torch.zeros(M * N, device="cuda") if M <= 256 else None
            ms = time_fn(lambda: C.gemm_fp8(q, s_, w8c, swc, out, 0, ws)) if ws is not None else ms_nosplit
            wb = w.bfloat16()
            base_bf16 = time_fn(lambda: x @ wb.t())
            scaled = None
            try:
                a8 = x.to(torch.float8_e4m3fn)
                b8 = w.to(torch.float8_e4m3fn)
                sa = torch.ones(M, 1, device="cuda")
                sb = torch.ones(1, N, device="cuda")
                scaled = time_fn(lambda: torch._scaled_mm(a8, b8.t(), sa, sb, out_dtype=torch.bfloat16))
            except Exception:
                pass
            flops = 2.0 * M * N * K
            r = dict(kernel="gemm_fp8_block", case=f"M{M} {name}", M=M, N=N, K=K, ours_ms=ms, ours_no_split_ms=ms_nosplit,
                     cublas_bf16_ms=base_bf16,
                     scaled_mm_rowwise_ms=scaled, tflops=flops / ms / 1e9, peaks=src)
            results.append(r)
            print(json.dumps(r))


def bench_moe(C, results):
    """Mixtral-8x7B MoE layer pieces at one GPU (8 experts, top 2): routing,
    alignment, gather, grouped gate/up + SwiGLU, grouped down, combine; the
    library baseline loops over experts with index_select + cuBLAS."""
    from ..engine.runner import ModelRunner
    _, _, src = peaks()
    E, topk, H, F = 8, 2, 4096, 14336
    for T in (512, 8192):
        al = 256 if T >= ModelRunner.MOE_PAIR_TOKENS else 128      # the runner's segment alignment
        h = torch.randn(T, H, device="cuda").bfloat16()
        router = torch.randn(E, H, device="cuda") * 0.02
        wgu = (torch.randn(E, 2 * F, H, device="cuda") * 0.02).bfloat16()
        wd = (torch.randn(E, H, F, device="cuda") * 0.02).bfloat16()
        ids = torch.empty(T, topk, dtype=torch.int32, device="cuda")
        wts = torch.empty(T, topk, dtype=torch.float32, device="cuda")
        cap = -(-(T * topk + E * (al - 1)) // al) * al
        groups = torch.empty(E + 1, dtype=torch.int32, device="cuda")
        perm = torch.empty(cap, dtype=torch.int32, device="cuda")
        slot = torch.empty(T * topk, dtype=torch.int32, device="cuda")
        xg = torch.empty(cap, H, device="cuda", dtype=torch.bfloat16)
        act = torch.empty(cap, F, device="cuda", dtype=torch.bfloat16)
        y = torch.empty(cap, H, device="cuda", dtype=torch.bfloat16)
        out = torch.empty(T, H, device="cuda", dtype=torch.bfloat16)

        def ours():
            C.moe_route(h, router, None, topk, ids, wts)
            C.moe_align(ids, T, topk, 0, E, groups, perm, slot, al)
            C.moe_gather(h, perm, groups, E, topk, xg)
            C.gemm_grouped(xg, wgu, act, groups, E, 2, al)
            C.gemm_grouped(act, wd, y, groups, E, 0, al)
            C.moe_combine(y, slot, wts, T, topk, out)

        pieces = {}
        ours()
        for key, fn in (("route", lambda: C.moe_route(h, router, None, topk, ids, wts)),
                        ("align", lambda: C.moe_align(ids, T, topk, 0, E, groups, perm, slot, al)),
                        ("gather", lambda: C.moe_gather(h, perm, groups, E, topk, xg)),
                        ("grouped_gate_up", lambda: C.gemm_grouped(xg, wgu, act, groups, E, 2, al)),
                        ("grouped_down", lambda: C.gemm_grouped(act, wd, y, groups, E, 0, al)),
                        ("combine", lambda: C.moe_combine(y, slot, wts, T, topk, out))):
            pieces[key] = time_fn(fn)
        total = time_fn(ours)

        def library():
            logits = h.float() @ router.t()
            w_, i_ = torch.softmax(logits, -1).topk(topk, -1)
            w_ = w_ / w_.sum(-1, keepdim=True)
            acc = torch.zeros(T, H, device="cuda", dtype=torch.float32)
            for e in range(E):
                rows, k = (i_ == e).nonzero(as_tuple=True)
                if rows.numel() == 0:
                    continue
                xe = h.index_select(0, rows)
                gu = xe @ wgu[e].t()
                v = gu.view(-1, 2 * F // 64, 2, 32)
                a = (torch.nn.functional.silu(v[:, :, 0]) * v[:, :, 1]).reshape(-1, F)
                acc.index_add_(0, rows, (a @ wd[e].t()).float() * w_[rows, k, None])
            return acc

        base = time_fn(library)
        flops = 2.0 * T * topk * (2 * F * H + F * H)
        r = dict(kernel="moe_layer", tokens=T, experts=E, topk=topk, align=al, ours_ms=total, pieces_ms=pieces,
                 expert_tflops=flops / (pieces["grouped_gate_up"] + pieces["grouped_down"]) / 1e9,
                 library_ms=base, speedup=base / total, peaks=src)
        results.append(r)
        print(json.dumps(r))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="")
    ap.add_argument("--json", default="")
    ap.add_argument("--case", default="", help="run only this GEMM case (for profiler captures)")
    ap.add_argument("--variants", action="store_true",
                    help="also time the opt-in GEMM variants (CTA pair, 256-row cluster tiles) and the fused QKV")
    args = ap.parse_args()
    C = _ext.load()
    results = []
    if args.only in ("", "gemm"):
        bench_gemm(C, results, args.case, args.variants)
    if args.variants and args.only in ("", "gemm"):
        bench_qkv_rope(C, results)
    if args.only in ("", "attn"):
        bench_attn(C, results)
    if args.only in ("", "norm"):
        bench_norm(C, results)
    if args.only in ("", "sample"):
        bench_sample(C, results)
    if args.only in ("", "fp8"):
        bench_fp8(C, results)
    if args.only in ("", "moe"):
        bench_moe(C, results)
    if args.json:
        with open(args.json, "w") as f:
            json.dump(results, f, indent=1)


if __name__ == "__main__":
    main()
