"""PyTorch restatement of the operator contracts (CPU path and baseline).

Same signatures and in-place semantics as ``KernelOps``; attention reads the
same paged KV layout ([page][kv_head][token][dim]) through the block table.
Host-side copies of the row metadata (``host=`` dicts of numpy arrays) are
used so no device->host synchronisation happens inside a step.
"""
from __future__ import annotations

import math
from typing import Optional

import numpy as np
import torch
import torch.nn.functional as F

from ..sampling.host import PARAM_DTYPE, counter_unit, stochastic_sample


ERR_NON_FINITE = 6      # the device error code of csrc/kernels/common.cuh


class TorchOps:
    name = "torch"

    def __init__(self, device="cpu"):
        self.device = torch.device(device)
        self.launches = 0
        self._error = (0, 0)      # (code, info) as the device error word keeps them

    @staticmethod
    def forward_tokens(ids, fwd):
        """Rows fwd[1].. whose slot fwd[0][i] >= 0 take fwd[2][slot] (in place)."""
        f, first, prev = fwd
        tok = ids[first:first + f.shape[0]]
        g = torch.index_select(prev, 0, torch.clamp(f, 0, prev.numel() - 1))
        tok.copy_(torch.where(f >= 0, g, tok))

    def embed(self, ids, table, out, fwd=None):
        if fwd is not None:
            self.forward_tokens(ids, fwd)
        out[: ids.shape[0]] = table[ids.long()]

    def rmsnorm(self, x, residual, w, out, eps, rows=None):
        if rows is not None:
            idx = rows.long()
            src = x.index_select(0, idx)
            if residual is not None:
                src = (src + residual.index_select(0, idx)).to(x.dtype)
            out = out[: idx.shape[0]]
        elif residual is not None:
            residual.copy_(x + residual)
            src = residual
        else:
            src = x
        xf = src.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()
        out.copy_(y.to(out.dtype))

    def gemm(self, A, B, out, epi: int = 0, ws=None):
        if epi == 2:
            gu = (A @ B.t()).float()
            M, N = gu.shape
            v = gu.view(M, N // 64, 2, 32)
            out.copy_((F.silu(v[:, :, 0]) * v[:, :, 1]).reshape(M, N // 2).to(out.dtype))
        elif epi == 1:
            out.copy_((A @ B.t()).float())
        else:
            torch.matmul(A, B.t(), out=out) if A.dtype == out.dtype else out.copy_(A @ B.t())

    def rope_kv_write(self, qkv, positions, slots, cos_sin, kc, vc, Hq, Hkv, page):
        T = qkv.shape[0]
        D = kc.shape[-1]
        h = D // 2
        cs = cos_sin[positions[:T].long()]  # [T, D/2, 2]
        c, s = cs[..., 0][:, None, :], cs[..., 1][:, None, :]
        q = qkv[:, : Hq * D].view(T, Hq, D)
        k = qkv[:, Hq * D:(Hq + Hkv) * D].view(T, Hkv, D)
        v = qkv[:, (Hq + Hkv) * D:(Hq + 2 * Hkv) * D].view(T, Hkv, D)

        def rot(x):
            xf = x.float()
            x1, x2 = xf[..., :h], xf[..., h:]
            return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1).to(x.dtype)

        q.copy_(rot(q))
        kr = rot(k)
        sl = slots[:T].long()
        ok = sl >= 0
        pg, off = (sl // page)[ok], (sl % page)[ok]
        kc[pg, :, off] = kr[ok]
        vc[pg, :, off] = v[ok]

    def _row_kv(self, kc, vc, bt_row, L):
        P = kc.shape[2]
        n = -(-L // P)
        pages = bt_row[:n].long()
        Hkv, D = kc.shape[1], kc.shape[3]
        K = kc[pages].permute(1, 0, 2, 3).reshape(Hkv, n * P, D)[:, :L]
        V = vc[pages].permute(1, 0, 2, 3).reshape(Hkv, n * P, D)[:, :L]
        return K, V

    def attn_prefill(self, q, out, q_start, seq_lens, bt, kc, vc, Hq, Hkv, max_q_len, host=None):
        qs = host["q_start"]
        sl = host["seq_lens"]
        D = kc.shape[-1]
        G = Hq // Hkv
        scale = 1.0 / math.sqrt(D)
        for r in range(len(sl)):
            s0, s1 = int(qs[r]), int(qs[r + 1])
            ql, L = s1 - s0, int(sl[r])
            K, V = self._row_kv(kc, vc, bt[r], L)
            qq = q[s0:s1, : Hq * D].view(ql, Hq, D).float().transpose(0, 1)
            Kf = K.float().repeat_interleave(G, 0)
            Vf = V.float().repeat_interleave(G, 0)
            sc = torch.matmul(qq, Kf.transpose(1, 2)) * scale
            qpos = torch.arange(L - ql, L, device=q.device)
            mask = torch.arange(L, device=q.device)[None, :] > qpos[:, None]
            sc = sc.masked_fill(mask[None], float("-inf"))
            p = sc.softmax(-1)
            o = torch.matmul(p, Vf).transpose(0, 1).reshape(ql, Hq * D)
            out[s0:s1, : Hq * D] = o.to(out.dtype)

    def decode_splits(self, rows, Hkv, max_seq):
        return 1

    def attn_decode(self, q, out, tok, seq_lens, bt, kc, vc, Hq, Hkv, splits, part_o, part_lse, host=None):
        sl = host["seq_lens"]
        tk = host["tok"]
        R = len(sl)
        if R == 0:
            return
        D, P = kc.shape[-1], kc.shape[2]
        G = Hq // Hkv
        Lmax = int(sl.max())
        n = -(-Lmax // P)
        pages = bt[:R, :n].long()                                   # [R, n]
        K = kc[pages].permute(0, 2, 1, 3, 4).reshape(R, Hkv, n * P, D)
        V = vc[pages].permute(0, 2, 1, 3, 4).reshape(R, Hkv, n * P, D)
        tok_t = torch.as_tensor(tk, device=q.device, dtype=torch.long)
        qq = q[tok_t, : Hq * D].view(R, Hkv, G, D).float()
        sc = torch.matmul(qq, K.float().transpose(-1, -2)) / math.sqrt(D)  # [R, Hkv, G, n*P]
        lens = torch.as_tensor(sl, device=q.device, dtype=torch.long)
        mask = torch.arange(n * P, device=q.device)[None, :] >= lens[:, None]
        sc = sc.masked_fill(mask[:, None, None, :], float("-inf"))
        p = sc.softmax(-1)
        o = torch.matmul(p, V.float()).reshape(R, Hq * D)
        out[tok_t, : Hq * D] = o.to(out.dtype)

    def _finite(self, logits):
        """Non-finite logits fail the step (error code 6, info = the first
        bad row), as the device samplers record them; the row is still
        sampled over its finite entries."""
        ok = torch.isfinite(logits)
        if bool(ok.all()):
            return logits
        if not self._error[0]:
            self._error = (ERR_NON_FINITE, int((~ok).any(-1).nonzero()[0]))
        return torch.where(ok, logits, torch.full_like(logits, float("-inf")))

    def argmax(self, logits, out):
        out[: logits.shape[0]] = torch.argmax(self._finite(logits), -1).to(torch.int32)

    def sample(self, logits, params, out):
        logits = self._finite(logits)
        R = logits.shape[0]
        p = params.detach().cpu().numpy().view(PARAM_DTYPE)[:R]
        lg = logits.detach().double().cpu().numpy()
        res = np.zeros(R, dtype=np.int32)
        for i in range(R):
            if p["mode"][i] == 0:
                res[i] = int(np.argmax(lg[i]))
            else:
                tk = int(p["top_k"][i])
                tp = float(p["top_p"][i])
                u = counter_unit(int(p["seed"][i]), int(p["sample_index"][i]))
                res[i] = stochastic_sample(lg[i], float(p["temperature"][i]), tk if tk > 0 else None,
                                           tp if 0 < tp < 1 else None, u)
        out[:R] = torch.from_numpy(res).to(out.device)

    def read_error(self, clear=True):
        e = self._error
        if clear:
            self._error = (0, 0)
        return e

    # vocab-parallel greedy: composite key (logit, lowest global id) per row
    def argmax_keys(self, logits, id_offset, keys):
        R = logits.shape[0]
        idx = torch.argmax(logits, -1)
        val = logits.gather(1, idx[:, None])[:, 0]
        u = val.float().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
        fk = torch.where(u >= 0x80000000, (~u) & 0xFFFFFFFF, u | 0x80000000)
        keys[:R] = (fk << 32) | (0xFFFFFFFF - (idx + id_offset))

    @staticmethod
    def _keys(logits, id_offset):
        """Composite keys (logit, then lowest id) as unsigned-ordered int64:
        the top bit is flipped so that signed comparison keeps the order."""
        R, V = logits.shape
        u = logits.float().contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
        fk = torch.where(u >= 0x80000000, (~u) & 0xFFFFFFFF, u | 0x80000000)
        ids = torch.arange(V, device=logits.device, dtype=torch.int64) + id_offset
        return (fk << 32) | (0xFFFFFFFF - ids)[None, :]

    def topk_keys(self, logits, id_offset, kc, keys):
        R, V = logits.shape
        k = self._keys(logits, id_offset)
        finite = torch.isfinite(logits)
        flip = torch.iinfo(torch.int64).min
        ordered = torch.where(finite, k ^ flip, torch.full_like(k, flip))
        n = min(kc, V)
        top = ordered.topk(n, dim=1).values ^ flip
        out = keys[: R * (kc + 1)].view(R, kc + 1)
        out.zero_()
        cnt = finite.sum(1)
        for r in range(R):
            m = int(min(n, int(cnt[r])))
            out[r, :m] = top[r, :m]
            out[r, kc] = 1 if bool(finite[r].all()) else 2

    def sample_keys(self, keys, rows, ranks, kc, params, out):
        k = keys[: ranks * rows * (kc + 1)].view(ranks, rows, kc + 1).cpu().numpy().astype(np.uint64)
        p = params.detach().cpu().numpy().view(PARAM_DTYPE)[:rows]
        res = np.zeros(rows, dtype=np.int32)
        for r in range(rows):
            c = k[:, r, :kc].reshape(-1)
            c = c[c != 0]
            hi = (c >> np.uint64(32)).astype(np.uint32)
            bits = np.where(hi & 0x80000000, hi & 0x7FFFFFFF, ~hi).astype(np.uint32)
            vals = bits.view(np.float32).astype(np.float64)
            ids = (0xFFFFFFFF - (c & np.uint64(0xFFFFFFFF))).astype(np.int64)
            top = int(ids[np.lexsort((ids, -vals))[0]])
            bad = bool((k[:, r, kc] == 2).any())
            if bad or p["mode"][r] == 0 or not p["temperature"][r] > 0:
                res[r] = top
                continue
            tk = int(p["top_k"][r])
            tp_ = float(p["top_p"][r])
            u = counter_unit(int(p["seed"][r]), int(p["sample_index"][r]))
            res[r] = stochastic_sample(vals, float(p["temperature"][r]), tk if tk > 0 else None,
                                       tp_ if 0 < tp_ < 1 else None, u, ids=ids)
        out[:rows] = torch.from_numpy(res).to(out.device)

    def keys_to_tokens(self, keys, rows, ranks, out):
        k = keys[: rows * ranks].view(ranks, rows)
        # int64 compare is signed; flip the top bit so unsigned order is kept
        kk = k ^ torch.iinfo(torch.int64).min
        best = k.gather(0, kk.argmax(0)[None])[0]
        out[:rows] = (0xFFFFFFFF - (best & 0xFFFFFFFF)).to(torch.int32)

    # ---------------------------------------------------------------- MoE
    def moe_route(self, h, router, bias, topk, ids, weights):
        logits = h.float() @ router.float().t()
        if bias is not None:
            logits = logits + bias
        p = logits.softmax(-1)
        w, i = p.topk(topk, -1)
        T = h.shape[0]
        ids[:T] = i.to(torch.int32)
        weights[:T] = w / w.sum(-1, keepdim=True)

    def moe_align(self, ids, T, topk, e0, El, groups, perm, slot, align: int = 128):
        flat = ids[:T].reshape(-1).long().cpu()
        perm.fill_(-1)
        slot_h = torch.full((T * topk,), -1, dtype=torch.int32)
        off = 0
        offs = []
        for e in range(El):
            offs.append(off)
            sel = (flat == e0 + e).nonzero().flatten()
            for j, a in enumerate(sel.tolist()):
                perm[off + j] = a
                slot_h[a] = off + j
            off += -(-len(sel) // align) * align
        offs.append(off)
        groups[:El + 1] = torch.tensor(offs, dtype=torch.int32)
        slot.view(-1)[:T * topk] = slot_h.to(slot.device)

    def moe_gather(self, h, perm, groups, El, topk, out):
        used = int(groups[El])
        p = perm[:used].long()
        ok = p >= 0
        out[:used] = 0
        out[:used][ok] = h[(p[ok] // topk)]

    def gemm_grouped(self, A, B, out, groups, num_groups, epi, align: int = 128):
        g = groups[:num_groups + 1].tolist()
        for e in range(num_groups):
            if g[e + 1] > g[e]:
                self.gemm(A[g[e]:g[e + 1]], B[e], out[g[e]:g[e + 1]], epi)

    def moe_combine(self, y, slot, w, T, topk, out):
        s = slot.view(-1)[:T * topk].long().view(T, topk)
        acc = torch.zeros(T, y.shape[1], dtype=torch.float32, device=y.device)
        for k in range(topk):
            ok = s[:, k] >= 0
            acc[ok] += w[:T, k][ok, None].float() * y[s[ok, k]].float()
        out[:T] = acc.to(out.dtype)

    # ---------------------------------------------------------------- fp8
    def act_quant(self, x, q, s):
        from ..models.fp8 import quantize_act
        rq, rs = quantize_act(x)
        q.copy_(rq)
        s.copy_(rs)

    def gemm_fp8(self, q, s, w8, sw, out, epi, ws=None):
        from ..models.fp8 import dequantize_weight
        a = (q.float() * s.repeat_interleave(128, 1)).to(torch.bfloat16)
        w = dequantize_weight(w8, sw).to(torch.bfloat16)
        self.gemm(a, w, out, epi)
