"""Numerics of every sm_100a kernel against a plain PyTorch fp32 reference."""
import math

import os

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


@pytest.mark.parametrize("M,N,K", [(1, 256, 64), (7, 512, 128), (128, 1024, 4096), (300, 6144, 4096),
                                   (1024, 4096, 1024), (129, 32, 8), (256, 14336 * 2 // 8, 4096)])
@pytest.mark.parametrize("bn", [0, 32, 64, 128, 256])
def test_gemm_bf16(C, M, N, K, bn):
    if bn and N % bn:
        pytest.skip("N not a multiple of BN")
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    B = (torch.randn(N, K, device="cuda", generator=g) * 0.05).bfloat16()
    D = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    C.gemm(A, B, D, 0, bn)
    ref = A.float() @ B.float().t()
    _close(D, ref, 2e-2, 2e-2, f"gemm {M}x{N}x{K} bn={bn}")
    D32 = torch.empty(M, N, device="cuda", dtype=torch.float32)
    C.gemm(A, B, D32, 1, bn)
    _close(D32, ref, 1e-3, 1e-3, f"gemm fp32 {M}x{N}x{K} bn={bn}")


@pytest.mark.parametrize("M,N,K,epi", [(1, 4096, 14336, 0), (256, 4096, 4096, 0), (100, 6144, 4096, 0),
                                       (256, 3584, 4096, 2), (3, 512, 4096, 1), (256, 4096, 14336, 2)])
def test_gemm_splitk(C, M, N, K, epi):
    A = torch.randn(M, K, device="cuda").bfloat16()
    B = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    ws = torch.zeros(512 * 32768, device="cuda")
    out_cols = N // 2 if epi == 2 else N
    D = torch.empty(M, out_cols, device="cuda", dtype=torch.float32 if epi == 1 else torch.bfloat16)
    prev = None
    for _ in range(2):  # two calls: the result must be bitwise reproducible
        C.gemm(A, B, D, epi, 0, ws)
        ref = A.float() @ B.float().t()
        if epi == 2:
            Fh = N // 2
            v = ref.view(M, Fh // 32, 2, 32)
            ref = (torch.nn.functional.silu(v[:, :, 0]) * v[:, :, 1]).reshape(M, Fh)
        _close(D, ref, 3e-2, 3e-2, f"split-K gemm {M}x{N}x{K} epi={epi}")
        if prev is not None:
            assert torch.equal(prev, D)
        prev = D.clone()
    assert C.gemm_plan_splitk(M, N, K) >= 1


@pytest.mark.parametrize("M,N,K,epi", [(256, 6144, 4096, 0), (256, 4096, 14336, 0), (256, 768, 4096, 0),
                                       (256, 4096, 512, 1), (64, 3584, 4096, 2), (1, 4096, 1792, 1),
                                       (129, 1024, 4096, 2), (256, 1536, 1024, 0), (250, 1536, 1024, 2)])
def test_gemm_cluster_splitk(C, M, N, K, epi):
    """Decode shapes that take the cluster split-K path: values against the fp32
    reference, bitwise reproducibility, and the plan itself."""
    c, bn, kb, mb = C.gemm_plan_cluster(M, N, K, epi)
    assert c >= 2 and mb == 1, (c, bn, kb, mb)
    assert (c - 1) * kb < (K + 63) // 64 <= c * kb
    _check_cluster_gemm(C, M, N, K, epi)


def _check_cluster_gemm(C, M, N, K, epi):
    A = torch.randn(M, K, device="cuda").bfloat16()
    B = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    out_cols = N // 2 if epi == 2 else N
    D = torch.empty(M, out_cols, device="cuda", dtype=torch.float32 if epi == 1 else torch.bfloat16)
    ref = A.float() @ B.float().t()
    if epi == 2:
        v = ref.view(M, N // 64, 2, 32)
        ref = (torch.nn.functional.silu(v[:, :, 0]) * v[:, :, 1]).reshape(M, N // 2)
    C.gemm(A, B, D, epi, 0, None)
    first = D.clone()
    C.gemm(A, B, D, epi, 0, None)
    assert torch.equal(first, D)
    _close(D, ref, 3e-2, 3e-2, f"cluster split-K {M}x{N}x{K} epi={epi}")
    assert C.read_error(True)[0] == 0


@pytest.mark.parametrize("M,N,K,epi", [(256, 6144, 4096, 0), (256, 4096, 14336, 0), (256, 4096, 4096, 1),
                                       (129, 1024, 4096, 2), (250, 1536, 1024, 2), (200, 6144, 4096, 1)])
def test_gemm_cluster_splitk_256_row_tiles(C, M, N, K, epi):
    """Cluster split-K with 256-row tiles (two MMAs per staged weight slab,
    the two partial M-blocks reduced in turn): values, reproducibility, plan."""
    C.gemm_set_cluster_mb2(True)
    try:
        c, bn, kb, mb = C.gemm_plan_cluster(M, N, K, epi)
        assert c >= 2 and mb == 2 and bn == 256, (c, bn, kb, mb)
        assert (c - 1) * kb < (K + 63) // 64 <= c * kb
        _check_cluster_gemm(C, M, N, K, epi)
    finally:
        C.gemm_set_cluster_mb2(False)


@pytest.mark.parametrize("M,N,K,epi", [(200, 10240, 512, 0), (256, 28672, 4096, 2), (129, 32768, 256, 1),
                                       (256, 9728, 1024, 0)])
def test_gemm_256_row_tiles(C, M, N, K, epi):
    """129..256 rows with enough 256-wide tiles: one 256-row tile per CTA (two
    M=128 MMAs sharing each staged weight slab, a single TMEM accumulator)."""
    assert C.gemm_plan_cluster(M, N, K, epi)[0] == 0
    A = torch.randn(M, K, device="cuda").bfloat16()
    B = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    out_cols = N // 2 if epi == 2 else N
    D = torch.empty(M, out_cols, device="cuda", dtype=torch.float32 if epi == 1 else torch.bfloat16)
    C.gemm(A, B, D, epi, 0, None)
    ref = A.float() @ B.float().t()
    if epi == 2:
        v = ref.view(M, N // 64, 2, 32)
        ref = (torch.nn.functional.silu(v[:, :, 0]) * v[:, :, 1]).reshape(M, N // 2)
    _close(D, ref, 3e-2, 3e-2, f"256-row tiles {M}x{N}x{K} epi={epi}")
    assert C.read_error(True)[0] == 0


def test_gemm_strided_a(C):
    A_full = torch.randn(64, 3 * 256, device="cuda").bfloat16()
    A = A_full[:, 256:512]
    B = torch.randn(128, 256, device="cuda").bfloat16() * 0.1
    D = torch.empty(64, 128, device="cuda", dtype=torch.bfloat16)
    C.gemm(A, B, D, 0, 0)
    _close(D, A.float() @ B.float().t(), 2e-2, 2e-2, "strided gemm")


@pytest.mark.parametrize("M,F,K", [(5, 256, 128), (200, 1792, 4096), (1024, 512, 512)])
@pytest.mark.parametrize("bn", [0, 64, 128, 256])
def test_gemm_swiglu(C, M, F, K, bn):
    if bn and (2 * F) % bn:
        pytest.skip("shape")
    Wg = torch.randn(F, K, device="cuda") * 0.05
    Wu = torch.randn(F, K, device="cuda") * 0.05
    # interleave in groups of 32 rows: [g0..g31, u0..u31, g32..]
    W = torch.stack([Wg.view(F // 32, 32, K), Wu.view(F // 32, 32, K)], 1).reshape(2 * F, K).bfloat16()
    x = torch.randn(M, K, device="cuda").bfloat16()
    out = torch.empty(M, F, device="cuda", dtype=torch.bfloat16)
    C.gemm(x, W, out, 2, bn)
    g = x.float() @ Wg.bfloat16().float().t()
    u = x.float() @ Wu.bfloat16().float().t()
    ref = torch.nn.functional.silu(g) * u
    _close(out, ref, 3e-2, 3e-2, "swiglu gemm")


@pytest.mark.parametrize("H", [64, 4096, 8192])
def test_rmsnorm(C, H):
    T = 37
    x = torch.randn(T, H, device="cuda").bfloat16()
    r = torch.randn(T, H, device="cuda").bfloat16()
    w = (1 + 0.1 * torch.randn(H, device="cuda")).bfloat16()
    out = torch.empty_like(x)
    C.rmsnorm(x, None, w, out, 1e-5)
    xf = x.float()
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5) * w.float()
    _close(out, ref, 2e-2, 2e-2, "rmsnorm")
    r2 = r.clone()
    C.rmsnorm(x, r2, w, out, 1e-5)
    s = (x.float() + r.float()).bfloat16().float()
    _close(r2, s, 1e-6, 0, "residual")
    ref = s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + 1e-5) * w.float()
    _close(out, ref, 2e-2, 2e-2, "rmsnorm+residual")


def test_embed(C):
    E = torch.randn(1000, 256, device="cuda").bfloat16()
    ids = torch.randint(0, 1000, (33,), device="cuda", dtype=torch.int32)
    out = torch.empty(33, 256, device="cuda", dtype=torch.bfloat16)
    C.embed(ids, E, out)
    assert torch.equal(out, E[ids.long()])


@pytest.mark.parametrize("H", [64, 4096])
def test_rmsnorm_gathered_rows(C, H):
    """Output row i normalises input row rows[i] (residual added, not written
    back): bitwise what the full norm gives on that row."""
    T = 29
    x = torch.randn(T, H, device="cuda").bfloat16()
    r = torch.randn(T, H, device="cuda").bfloat16()
    w = (1 + 0.1 * torch.randn(H, device="cuda")).bfloat16()
    rows = torch.tensor([28, 0, 5, 5, 17], device="cuda", dtype=torch.int32)
    out = torch.zeros(rows.numel(), H, device="cuda", dtype=torch.bfloat16)
    r_keep = r.clone()
    C.rmsnorm(x, r, w, out, 1e-5, rows)
    torch.cuda.synchronize()
    assert torch.equal(r, r_keep)
    s = (x.float() + r.float()).bfloat16().float()[rows.long()]
    ref = s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + 1e-5) * w.float()
    _close(out, ref, 2e-2, 2e-2, "gathered rmsnorm")
    full = torch.empty_like(x)
    C.rmsnorm(x, r.clone(), w, full, 1e-5)
    assert torch.equal(out, full[rows.long()])
    # an index outside the input is a bad index: the row is zeroed and the error word set
    C.read_error(True)
    bad = torch.tensor([3, T], device="cuda", dtype=torch.int32)
    out2 = torch.ones(2, H, device="cuda", dtype=torch.bfloat16)
    C.rmsnorm(x, r, w, out2, 1e-5, bad)
    torch.cuda.synchronize()
    assert C.read_error(True)[0] != 0 and out2[1].abs().sum().item() == 0
    assert torch.equal(out2[0], full[3])


def test_embed_forwarded_tokens(C):
    """Rows from `first` with a slot >= 0 take prev[slot] (and store it in ids)."""
    E = torch.randn(1000, 256, device="cuda").bfloat16()
    ids = torch.randint(0, 1000, (12,), device="cuda", dtype=torch.int32)
    prev = torch.tensor([7, 999, 42, 3], device="cuda", dtype=torch.int32)
    fwd = torch.tensor([2, -1, 0, 1, -1], device="cuda", dtype=torch.int32)
    first = 6
    want = ids.clone()
    for i, f in enumerate(fwd.tolist()):
        if f >= 0:
            want[first + i] = prev[f]
    out = torch.empty(12, 256, device="cuda", dtype=torch.bfloat16)
    C.embed(ids, E, out, fwd, first, prev)
    torch.cuda.synchronize()
    assert torch.equal(ids, want)
    assert torch.equal(out, E[want.long()])


def rope_table(max_pos, D, theta):
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.float64) / D))
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None]
    return torch.stack([ang.cos(), ang.sin()], -1).float()


def ref_rope(x, pos, table):
    D = x.shape[-1]
    cs = table[pos.long()]
    c, s = cs[..., 0][:, None, :], cs[..., 1][:, None, :]
    x1, x2 = x[..., : D // 2], x[..., D // 2:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1)


def test_rope_kv_write(C):
    T, Hq, Hkv, D, P = 20, 8, 2, 128, 16
    pages = 10
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device="cuda").bfloat16()
    pos = torch.randint(0, 500, (T,), device="cuda", dtype=torch.int32)
    slots = torch.randperm(pages * P, device="cuda")[:T].int()
    table = rope_table(1024, D, 500000.0).cuda()
    kc = torch.zeros(pages, Hkv, P, D, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    q0 = qkv.clone()
    C.rope_kv_write(qkv, pos, slots, table, kc, vc, Hq, Hkv, P)
    q = q0[:, : Hq * D].float().view(T, Hq, D)
    k = q0[:, Hq * D:(Hq + Hkv) * D].float().view(T, Hkv, D)
    v = q0[:, (Hq + Hkv) * D:].view(T, Hkv, D)
    _close(qkv[:, : Hq * D].view(T, Hq, D), ref_rope(q, pos, table.cuda()), 2e-2, 2e-2, "rope q")
    kr = ref_rope(k, pos, table.cuda())
    pg, off = (slots // P).long(), (slots % P).long()
    _close(kc[pg, :, off], kr, 2e-2, 2e-2, "k cache")
    assert torch.equal(vc[pg, :, off], v)


def make_paged(rows_lens, Hkv, D, P, extra_pages=7, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    n_pages = [math.ceil(L / P) for L in rows_lens]
    total = sum(n_pages) + extra_pages + 1
    perm = torch.randperm(total - 1, generator=g) + 1  # page 0 is the reserved zero page
    kc = torch.randn(total, Hkv, P, D, generator=g).bfloat16()
    vc = torch.randn(total, Hkv, P, D, generator=g).bfloat16()
    kc[0] = 0
    vc[0] = 0
    maxp = max(n_pages)
    bt = torch.zeros(len(rows_lens), maxp + 3, dtype=torch.int32)
    i = 0
    for r, n in enumerate(n_pages):
        bt[r, :n] = perm[i:i + n].int()
        i += n
    return kc.cuda(), vc.cuda(), bt.cuda()


def ref_attention(q, kc, vc, bt, L, qpos, Hq, Hkv):
    """q [nq, Hq, D] for one row at absolute positions qpos; full causal softmax in fp32."""
    D, P = kc.shape[-1], kc.shape[2]
    n = math.ceil(L / P)
    pages = bt[:n].long()
    K = kc[pages].float().permute(1, 0, 2, 3).reshape(Hkv, n * P, D)[:, :L]
    V = vc[pages].float().permute(1, 0, 2, 3).reshape(Hkv, n * P, D)[:, :L]
    G = Hq // Hkv
    K = K.repeat_interleave(G, 0)
    V = V.repeat_interleave(G, 0)
    s = torch.einsum("qhd,hkd->hqk", q.float(), K) / math.sqrt(D)
    mask = torch.arange(L, device=q.device)[None, :] > qpos[:, None]
    s = s.masked_fill(mask[None], float("-inf"))
    p = s.softmax(-1)
    return torch.einsum("hqk,hkd->qhd", p, V)


@pytest.mark.parametrize("Hq,Hkv", [(32, 8), (8, 8), (64, 8), (4, 1)])
@pytest.mark.parametrize("splits", [1, 2, 5])
def test_attn_decode(C, Hq, Hkv, splits):
    D, P = 128, 16
    lens = [1, 15, 16, 17, 100, 1025, 333]
    kc, vc, bt = make_paged(lens, Hkv, D, P)
    R = len(lens)
    T = R + 3
    q = torch.randn(T, (Hq + 2 * Hkv) * D, device="cuda").bfloat16()
    tok = torch.tensor([3, 0, 1, 2, 4, 5, 6], device="cuda", dtype=torch.int32)[:R]
    out = torch.zeros(T, Hq * D, device="cuda", dtype=torch.bfloat16)
    sl = torch.tensor(lens, device="cuda", dtype=torch.int32)
    po = torch.empty(R * Hq * splits * D, device="cuda")
    pl = torch.empty(R * Hq * splits, device="cuda")
    C.attn_decode(q, out, tok, sl, bt, kc, vc, Hq, Hkv, splits, po, pl)
    assert C.read_error(True)[0] == 0
    for r, L in enumerate(lens):
        t = tok[r].item()
        qq = q[t, : Hq * D].view(1, Hq, D)
        ref = ref_attention(qq, kc, vc, bt[r], L, torch.tensor([L - 1], device="cuda"), Hq, Hkv)
        _close(out[t].view(Hq, D), ref[0], 2e-2, 2e-2, f"decode row {r} L={L}")


@pytest.mark.parametrize("Hq,Hkv", [(32, 8), (16, 16), (8, 1)])
def test_attn_prefill(C, Hq, Hkv):
    D, P = 128, 16
    # (query chunk length, total kv length) per row: fresh prompts and later chunks
    rows = [(5, 5), (64, 64), (65, 200), (130, 130), (1, 17), (200, 1000)]
    lens = [L for _, L in rows]
    kc, vc, bt = make_paged(lens, Hkv, D, P, seed=1)
    qls = [ql for ql, _ in rows]
    qs = torch.tensor([0] + list(torch.tensor(qls).cumsum(0)), dtype=torch.int32, device="cuda")
    T = sum(qls)
    q = torch.randn(T, (Hq + 2 * Hkv) * D, device="cuda").bfloat16()
    out = torch.zeros(T, Hq * D, device="cuda", dtype=torch.bfloat16)
    sl = torch.tensor(lens, device="cuda", dtype=torch.int32)
    C.attn_prefill(q, out, qs, sl, bt, kc, vc, Hq, Hkv, max(qls))
    assert C.read_error(True)[0] == 0
    for r, (ql, L) in enumerate(rows):
        s0 = qs[r].item()
        qq = q[s0:s0 + ql, : Hq * D].view(ql, Hq, D)
        qpos = torch.arange(L - ql, L, device="cuda")
        ref = ref_attention(qq, kc, vc, bt[r], L, qpos, Hq, Hkv)
        _close(out[s0:s0 + ql].view(ql, Hq, D), ref, 2e-2, 2e-2, f"prefill row {r}")


def test_argmax(C):
    R, V = 9, 128256
    logits = torch.randn(R, V, device="cuda")
    logits[3, 77] = 50.0
    logits[3, 99] = 50.0  # tie: lowest id wins
    out = torch.empty(R, device="cuda", dtype=torch.int32)
    st = torch.empty(R, device="cuda", dtype=torch.int32)
    C.argmax(logits, out, st)
    exp = logits.argmax(-1)
    exp[3] = 77
    assert torch.equal(out.long(), exp)
    assert int(st.abs().sum()) == 0
    # a non-finite logit: status -1 for its row, or (no status array, as the
    # engine calls it) error code 6 with the row, so the step fails closed
    logits[5, 10] = float("nan")
    logits[5, 11] = 60.0
    C.read_error(True)
    C.argmax(logits, out, st)
    torch.cuda.synchronize()
    assert int(out[5]) == 11 and int(st[5]) == -1 and C.read_error(True)[0] == 0
    C.argmax(logits, out, None)
    torch.cuda.synchronize()
    assert C.read_error(True) == (6, 5)


def _params(rows):
    import numpy as np
    dt = np.dtype([("mode", "<i4"), ("top_k", "<i4"), ("temperature", "<f4"), ("top_p", "<f4"),
                   ("seed", "<u8"), ("sample_index", "<i8")])
    a = np.zeros(len(rows), dtype=dt)
    for i, r in enumerate(rows):
        a[i] = r
    return torch.from_numpy(a.view(np.uint8).copy()).cuda()


def _host_sample(logits, temperature, top_k, top_p, u):
    """fp64 restatement of the reference sampler (sampling/stochastic.mbt)."""
    l = logits.double().cpu()
    order = sorted(range(l.numel()), key=lambda i: (-l[i].item(), i))
    if top_k > 0:
        order = order[:top_k]
    mx = l[order[0]].item()
    w = [math.exp((l[i].item() - mx) / temperature) for i in order]
    total = sum(w)
    cnt = len(order)
    if 0 < top_p < 1:
        thr, cum, cnt = top_p * total, 0.0, 0
        while cnt < len(order) and cum < thr:
            cum += w[cnt]
            cnt += 1
        cnt = max(cnt, 1)
    ret = sum(w[:cnt])
    target, cum = u * ret, 0.0
    for j in range(cnt):
        cum += w[j]
        if cum > target:
            return order[j]
    return order[cnt - 1]


def test_sample_matches_host_replay(C):
    V = 3000
    g = torch.Generator(device="cpu").manual_seed(3)
    logits = (torch.randn(6, V, generator=g) * 3).cuda()
    rows = [(1, 0, 0.7, 0.9, 11, 0), (1, 50, 1.0, 1.0, 12, 5), (1, 0, 1.3, 0.5, 13, 9),
            (0, 0, 1.0, 1.0, 14, 0), (1, 1, 0.5, 1.0, 15, 2), (1, 200, 0.8, 0.95, 16, 100)]
    out = torch.empty(6, device="cuda", dtype=torch.int32)
    C.sample(logits, _params(rows), out, None)
    for i, (mode, k, t, p, seed, idx) in enumerate(rows):
        if mode == 0:
            assert out[i].item() == logits[i].argmax().item()
            continue
        u = C.counter_unit(seed, idx)
        assert out[i].item() == _host_sample(logits[i], t, k, p, u), f"row {i}"


def test_error_word_roundtrip(C):
    assert C.read_error(True)[0] == 0
    C.inject_error(5)
    assert C.read_error(True)[0] == 5
    assert C.read_error(True)[0] == 0


def test_moe_kernels_match_torch(C):
    T, H, E, k, F = 300, 1024, 8, 2, 512
    torch.manual_seed(0)
    h = torch.randn(T, H, device="cuda").bfloat16()
    wr = torch.randn(E, H, device="cuda") * 0.05
    ids = torch.empty(T, k, device="cuda", dtype=torch.int32)
    w = torch.empty(T, k, device="cuda")
    C.moe_route(h, wr, None, k, ids, w)
    p = (h.float() @ wr.t()).softmax(-1)
    pv, pi = p.topk(k, -1)
    assert (ids.long() == pi).float().mean().item() > 0.99
    _close(w, pv / pv.sum(-1, keepdim=True), 1e-4, 1e-4, "route weights")
    rows = -(-(T * k + E * 127) // 128) * 128
    groups = torch.empty(E + 1, device="cuda", dtype=torch.int32)
    perm = torch.empty(rows, device="cuda", dtype=torch.int32)
    slot = torch.empty(T * k, device="cuda", dtype=torch.int32)
    C.moe_align(ids, T, k, 0, E, groups, perm, slot)
    g = groups.tolist()
    assert all(x % 128 == 0 for x in g) and g[0] == 0
    flat = ids.view(-1).long()
    for e in range(E):
        seg = perm[g[e]:g[e + 1]]
        real = seg[seg >= 0].long()
        assert torch.equal(torch.sort(real).values, (flat == e).nonzero().flatten())
    x = torch.empty(rows, H, device="cuda", dtype=torch.bfloat16)
    C.moe_gather(h, perm, groups, E, k, x)
    Wg = torch.randn(E, F, H, device="cuda") * 0.03
    Wu = torch.randn(E, F, H, device="cuda") * 0.03
    Wd = (torch.randn(E, H, F, device="cuda") * 0.03).bfloat16()
    Wgu = torch.stack([Wg.view(E, F // 32, 32, H), Wu.view(E, F // 32, 32, H)], 2).reshape(E, 2 * F, H).bfloat16()
    act = torch.empty(rows, F, device="cuda", dtype=torch.bfloat16)
    y = torch.empty(rows, H, device="cuda", dtype=torch.bfloat16)
    C.gemm_grouped(x, Wgu, act, groups, E, 2)
    C.gemm_grouped(act, Wd, y, groups, E, 0)
    out = torch.empty(T, H, device="cuda", dtype=torch.bfloat16)
    C.moe_combine(y, slot, w, T, k, out)
    ref = torch.zeros(T, H, device="cuda")
    hf = h.float()
    for e in range(E):
        sel = (ids.long() == e)
        rows_e = sel.any(-1).nonzero().flatten()
        if rows_e.numel() == 0:
            continue
        a = torch.nn.functional.silu(hf[rows_e] @ Wg[e].bfloat16().float().t()) * (hf[rows_e] @ Wu[e].bfloat16().float().t())
        ye = a.bfloat16().float() @ Wd[e].float().t()
        ref[rows_e] += (w * sel).sum(-1)[rows_e, None] * ye
    _close(out, ref, 3e-2, 5e-2, "moe forward")
    assert C.read_error(True)[0] == 0


@pytest.mark.parametrize("M,Hq,Hkv,K", [(1, 32, 8, 4096), (37, 32, 8, 4096), (256, 32, 8, 4096),
                                        (200, 64, 8, 1024), (1000, 32, 8, 4096), (5000, 3, 1, 512),
                                        (256, 4, 1, 4096)])
def test_gemm_qkv_rope_matches_gemm_then_rope(C, M, Hq, Hkv, K):
    """The fused QKV epilogue (cluster split-K, 256-row tiles and persistent
    tiles, BN 256 and 128) against the GEMM followed by rope_kv_write: Q
    columns and the K / V cache pages, within bf16 rounding."""
    D, P, pages = 128, 16, 512
    N = (Hq + 2 * Hkv) * D
    g = torch.Generator(device="cuda").manual_seed(M + Hq)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    B = (torch.randn(N, K, device="cuda", generator=g) * 0.05).bfloat16()
    pos = torch.randint(0, 1000, (M,), device="cuda", generator=g, dtype=torch.int32)
    slots = torch.randperm(pages * P, device="cuda", generator=g)[:M].int()
    slots[::7] = -1                       # padding rows: no KV write
    table = rope_table(1024, D, 500000.0).cuda()
    kc = torch.zeros(pages, Hkv, P, D, device="cuda").bfloat16()
    vc = torch.zeros_like(kc)
    kc_ref, vc_ref = kc.clone(), vc.clone()
    ref = torch.empty(M, N, device="cuda").bfloat16()
    C.gemm(A, B, ref, 0, 0, None)
    C.rope_kv_write(ref, pos, slots, table, kc_ref, vc_ref, Hq, Hkv, P)
    out = torch.zeros(M, N, device="cuda").bfloat16()
    assert C.gemm_qkv_rope(A, B, out, pos, slots, table, kc, vc, Hq, Hkv, P)
    torch.cuda.synchronize()
    assert C.read_error(True)[0] == 0
    _close(out[:, :Hq * D].float(), ref[:, :Hq * D].float(), 3e-2, 3e-2, "fused Q")
    _close(kc.float(), kc_ref.float(), 3e-2, 3e-2, "fused K cache")
    _close(vc.float(), vc_ref.float(), 3e-2, 3e-2, "fused V cache")


@pytest.mark.parametrize("M,N,K,epi", [(2048, 4096, 4096, 0), (8192, 6144, 4096, 0), (4096, 28672, 4096, 2),
                                       (300, 32768, 512, 1), (2048, 4096, 1000, 0),
                                       # one M-tile: 192- and 256-wide tiles, two or more per pair
                                       (256, 28672, 4096, 2), (129, 32768, 256, 1), (200, 28672, 1024, 0)])
def test_gemm_cta_pair(C, M, N, K, epi):
    """256 x 256 tiles on CTA pairs (tcgen05.mma cta_group::2, B split over
    the pair): values against the fp32 reference, including a pair whose
    second CTA's rows are all past M and a K tail."""
    A = torch.randn(M, K, device="cuda").bfloat16()
    B = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    out_cols = N // 2 if epi == 2 else N
    D = torch.empty(M, out_cols, device="cuda", dtype=torch.float32 if epi == 1 else torch.bfloat16)
    was = C.gemm_get_pair()
    C.gemm_set_pair(True)
    try:
        C.gemm(A, B, D, epi, 0, None)
        torch.cuda.synchronize()
    finally:
        C.gemm_set_pair(was)
    assert C.read_error(True)[0] == 0
    ref = A.float() @ B.float().t()
    if epi == 2:
        v = ref.view(M, N // 64, 2, 32)
        ref = (torch.nn.functional.silu(v[:, :, 0]) * v[:, :, 1]).reshape(M, N // 2)
    _close(D, ref, 3e-2, 3e-2, f"cta-pair gemm {M}x{N}x{K} epi={epi}")


@pytest.mark.parametrize("ranks", [2, 8])
def test_sample_from_shard_candidates_equals_full_row(C, ranks):
    """Per-shard top-64 keys, gathered, then the draw: the same tokens as the
    sampler over the whole row, for top_k <= 64 (greedy and stochastic rows)."""
    from lunaflux_b200.sampling.host import pack_params
    R, kc = 37, 64
    V = 16032 * ranks                      # the Llama-3 vocabulary shard at TP 8, times the ranks
    g = torch.Generator(device="cuda").manual_seed(ranks)
    logits = torch.randn(R, V, device="cuda", generator=g) * 3
    rows = [(0 if i % 5 == 0 else 1, 1 + (7 * i) % 64, 0.7 + 0.05 * (i % 9), 0.9 if i % 2 else 1.0, 1000 + i, i)
            for i in range(R)]
    params = torch.from_numpy(pack_params(rows).view("u1").copy()).cuda()
    full = torch.empty(R, dtype=torch.int32, device="cuda")
    C.sample(logits, params, full)
    Vl = V // ranks
    keys = torch.zeros(ranks, R, kc + 1, dtype=torch.int64, device="cuda")
    for k in range(ranks):
        C.topk_keys(logits[:, k * Vl:(k + 1) * Vl].contiguous(), k * Vl, kc, keys[k])
    got = torch.empty(R, dtype=torch.int32, device="cuda")
    C.sample_keys(keys, R, ranks, kc, params, got)
    torch.cuda.synchronize()
    assert torch.equal(got, full)


def test_peer_wait_runs_out_and_the_step_fails(C):
    """A bounded wait on another rank's words that never arrive: the
    low-latency all-reduce is launched as rank 0 of a group of 2 on one GPU,
    with rank 1's inboxes in local memory that nothing writes.  With the wait
    limit shortened to 50 ms the kernel returns on its own, records
    kErrPeerTimeout, the context stays usable and the runner's error check
    raises StepFailed."""
    import time
    import types
    from lunaflux_b200.engine.runner import ModelRunner, StepFailed
    from lunaflux_b200.ops import KernelOps
    M, N = 4, 256
    pairs = M * N // 2
    words = lambda n: torch.zeros(n, 2, dtype=torch.int32, device="cuda")  # noqa: E731 (uint2 words)
    rs = [words(2 * pairs), words(2 * pairs)]
    ag = [words(pairs), words(pairs)]
    state = torch.zeros(4, dtype=torch.int32, device="cuda")
    ws = torch.randn(M * N, device="cuda")
    D = torch.zeros(M, N, dtype=torch.bfloat16, device="cuda")
    C.read_error(True)
    C.set_wait_limit_ns(50_000_000)
    try:
        t0 = time.perf_counter()
        C.partials_allreduce_ll(ws, 1, D, [t.data_ptr() for t in rs], [t.data_ptr() for t in ag], 0, state, 0, pairs)
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
    finally:
        C.set_wait_limit_ns(1_000_000_000)
    assert elapsed < 5.0, elapsed
    runner = types.SimpleNamespace(ops=KernelOps())
    with pytest.raises(StepFailed) as e:
        ModelRunner.check_device_errors(runner)
    assert e.value.code == 2          # kErrPeerTimeout
    # the context is still usable
    x = torch.ones(1024, device="cuda")
    assert float(x.sum()) == 1024.0
    assert C.read_error(True)[0] == 0


@pytest.mark.parametrize("epi", [0, 2])
def test_grouped_gemm_256_row_segments_on_cta_pairs(C, epi):
    """Expert segments padded to 256 rows run on the CTA-pair kernel (one
    expert per 256-row tile, tiles past the last segment skipped): every
    segment's rows against the fp32 product with its expert's weights."""
    E, T, k, H, N = 8, 4096, 2, 1024, 2048
    g = torch.Generator(device="cuda").manual_seed(7 + epi)
    ids = torch.randint(0, E, (T, k), device="cuda", generator=g, dtype=torch.int32)
    ids[:, 1] = (ids[:, 0] + 1 + torch.randint(0, E - 1, (T,), device="cuda", generator=g, dtype=torch.int32)) % E
    rows = -(-(T * k + E * 255) // 256) * 256
    groups = torch.zeros(E + 1, dtype=torch.int32, device="cuda")
    perm = torch.empty(rows, dtype=torch.int32, device="cuda")
    slot = torch.empty(T * k, dtype=torch.int32, device="cuda")
    C.moe_align(ids, T, k, 0, E, groups, perm, slot, 256)
    gh = groups.tolist()
    assert all(x % 256 == 0 for x in gh)
    A = (torch.randn(rows, H, device="cuda", generator=g)).bfloat16()
    B = (torch.randn(E, N, H, device="cuda", generator=g) * 0.05).bfloat16()
    cols = N // 2 if epi == 2 else N
    D = torch.full((rows, cols), 7.0, device="cuda", dtype=torch.bfloat16)
    C.gemm_grouped(A, B, D, groups, E, epi, 256)
    torch.cuda.synchronize()
    assert C.read_error(True)[0] == 0
    for e in range(E):
        a, b = gh[e], gh[e + 1]
        if a == b:
            continue
        ref = A[a:b].float() @ B[e].float().t()
        if epi == 2:
            v = ref.view(b - a, N // 64, 2, 32)
            ref = (torch.nn.functional.silu(v[:, :, 0]) * v[:, :, 1]).reshape(b - a, N // 2)
        _close(D[a:b], ref, 3e-2, 3e-2, f"expert {e} rows {a}..{b} epi={epi}")
    assert bool((D[gh[E]:] == 7.0).all()), "rows past the last segment were written"
