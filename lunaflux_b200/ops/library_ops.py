"""The library baseline operator set: what a serving engine builds from vendor
and library kernels alone, on the same engine, scheduler and KV layout.

* projections and the LM head: cuBLAS through ``torch.matmul`` (bf16 in,
  bf16 or fp32 out), SwiGLU as a separate elementwise pass;
* paged attention, prefill and decode: vLLM's flash-attention varlen kernel
  with a block table (the kernel vLLM itself serves with), reading this
  engine's ``[page][kv_head][16][dim]`` cache through a strided view, so no
  gather and no copy of the KV;
* RMSNorm: ``torch.nn.functional.rms_norm`` after an in-place residual add;
* RoPE + KV write: vectorised torch ops with no host synchronisation (padded
  rows write zeros into the reserved zero page), so decode steps are
  captured in CUDA graphs exactly like the product's;
* embedding, argmax: torch.

Tensor-parallel collectives are NCCL (``parallel.comm.TPComm``).  The
reference has no such arm; its benchmarking contract names the best pinned
library stack as the bar (docs/BENCHMARKING.md:82-88).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from .torch_ops import TorchOps


def _load_flash():
    try:
        from vllm.vllm_flash_attn import flash_attn_varlen_func, is_fa_version_supported
    except Exception as e:  # pragma: no cover - needs the GPU wheel's CUDA libraries
        raise RuntimeError(f"library baseline: vLLM flash-attention is not importable ({e})") from e
    version = 2
    for v in (3, 2):
        try:
            if is_fa_version_supported(v):
                version = v
                break
        except Exception:
            continue
    return flash_attn_varlen_func, version


class LibraryOps(TorchOps):
    name = "library"

    def __init__(self, device):
        super().__init__(device)
        self.flash, self.fa_version = _load_flash()
        self._arange = torch.arange(0, 4097, dtype=torch.int32, device=self.device)

    # ------------------------------------------------------------ dense ops
    def embed(self, ids, table, out, fwd=None):
        if fwd is not None:
            self.forward_tokens(ids, fwd)
        torch.index_select(table, 0, ids.long(), out=out[: ids.shape[0]])

    def rmsnorm(self, x, residual, w, out, eps, rows=None):
        if rows is not None:
            return super().rmsnorm(x, residual, w, out, eps, rows)
        if residual is not None:
            residual.add_(x)
            src = residual
        else:
            src = x
        out.copy_(F.rms_norm(src, (src.shape[-1],), w, eps))

    def gemm(self, A, B, out, epi: int = 0, ws=None):
        if A.shape[0] == 0:
            return
        if epi == 2:
            gu = torch.matmul(A, B.t())
            M, N = gu.shape
            v = gu.view(M, N // 64, 2, 32)
            torch.mul(F.silu(v[:, :, 0]), v[:, :, 1], out=out.view(M, N // 64, 32))
        elif epi == 1:
            try:
                torch.mm(A, B.t(), out_dtype=torch.float32, out=out)
            except TypeError:
                out.copy_(torch.matmul(A, B.t()))
        else:
            torch.matmul(A, B.t(), out=out)

    def rope_kv_write(self, qkv, positions, slots, cos_sin, kc, vc, Hq, Hkv, page):
        T = qkv.shape[0]
        if T == 0:
            return
        D = kc.shape[-1]
        h = D // 2
        cs = cos_sin.index_select(0, positions[:T].long())          # [T, D/2, 2]
        c, s = cs[..., 0][:, None, :], cs[..., 1][:, None, :]
        q = qkv[:, : Hq * D].view(T, Hq, D)
        k = qkv[:, Hq * D:(Hq + Hkv) * D].view(T, Hkv, D)
        v = qkv[:, (Hq + Hkv) * D:(Hq + 2 * Hkv) * D].view(T, Hkv, D)

        def rot(x):
            xf = x.float()
            x1, x2 = xf[..., :h], xf[..., h:]
            return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1).to(x.dtype)

        q.copy_(rot(q))
        sl = slots[:T].long()
        ok = (sl >= 0)
        slc = torch.where(ok, sl, torch.zeros_like(sl))              # padded rows: page 0, offset 0
        keep = ok[:, None, None].to(qkv.dtype)
        pg, off = slc // page, slc % page
        kc[pg, :, off] = rot(k) * keep                               # zeros into the zero page
        vc[pg, :, off] = v * keep

    # ------------------------------------------------------------ attention
    def _paged(self, kc, vc):
        # [page][kv_head][tok][dim] -> [page][tok][kv_head][dim] view (no copy)
        return kc.permute(0, 2, 1, 3), vc.permute(0, 2, 1, 3)

    def attn_prefill(self, q, out, q_start, seq_lens, bt, kc, vc, Hq, Hkv, max_q_len, host=None):
        Tp = q.shape[0]
        if Tp == 0:
            return
        D = kc.shape[-1]
        R = seq_lens.shape[0]
        k, v = self._paged(kc, vc)
        sl = host.get("seq_lens") if host else None
        max_k = int(sl.max()) if sl is not None and len(sl) else bt.shape[1] * kc.shape[2]
        qq = q[:, : Hq * D].view(Tp, Hq, D)
        self.flash(qq, k, v, max_seqlen_q=max_q_len, cu_seqlens_q=q_start[: R + 1], max_seqlen_k=max_k,
                   seqused_k=seq_lens, softmax_scale=1.0 / math.sqrt(D), causal=True, block_table=bt[:R],
                   out=out[:, : Hq * D].view(Tp, Hq, D), fa_version=self.fa_version)

    def decode_splits(self, rows, Hkv, max_seq):
        return 1

    def attn_decode(self, q, out, tok, seq_lens, bt, kc, vc, Hq, Hkv, splits, part_o, part_lse, host=None):
        R = seq_lens.shape[0]
        if R == 0:
            return
        D = kc.shape[-1]
        k, v = self._paged(kc, vc)
        idx = tok[:R].long()
        qq = q.index_select(0, idx)[:, : Hq * D].reshape(R, Hq, D)
        o = torch.empty_like(qq)
        self.flash(qq, k, v, max_seqlen_q=1, cu_seqlens_q=self._arange[: R + 1], max_seqlen_k=bt.shape[1] * kc.shape[2],
                   seqused_k=seq_lens, softmax_scale=1.0 / math.sqrt(D), causal=True, block_table=bt[:R],
                   out=o, fa_version=self.fa_version)
        out[:, : Hq * D].index_copy_(0, idx, o.view(R, Hq * D))

    def argmax(self, logits, out):
        out[: logits.shape[0]].copy_(torch.argmax(logits, -1))
