"""Per-rank model runner: weights, paged KV arena, static workspace, the
decoder forward over an operator set, and CUDA-graph capture of decode steps.

Reference counterparts: engine/device_step (PagedGraphExecutor: stage ->
execute -> sample_completion -> finish; paged_executor_prepare.mbt:292),
engine/device_memory (one activation arena reused by every step),
kv/device_arena (one allocation for the whole KV arena, prepare.mbt:66).
Differences by design: no per-launch synchronisation (the reference calls
cuStreamSynchronize after every launch, internal/cuda/launch.c:146-161); the
whole decode step is one CUDA-graph replay per batch bucket; sampling runs on
the device and only the sampled int32 ids come back to the host.
"""
from __future__ import annotations

import math
import os
import time
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch

from ..models.spec import LlamaSpec, rope_inv_freq
from ..models.weights import ModelWeights
from ..scheduler.scheduler import StepPlan
from ..ops.launch_contract import check_paged_step
from .step_inputs import HostStep, build_host_step, device_views, make_layout


class StepFailed(RuntimeError):
    def __init__(self, code: int, info: int):
        super().__init__(f"device error {code} (info {info})")
        self.code = code
        self.info = info


def rope_table(max_pos: int, head_dim: int, theta: float, device=None, scaling: tuple = ()) -> torch.Tensor:
    """[max_pos, head_dim / 2, (cos, sin)] fp32, angles in float64."""
    inv = rope_inv_freq(head_dim, theta, scaling)
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None]
    t = torch.stack([ang.cos(), ang.sin()], -1).float().contiguous()
    return t if device is None else t.to(device)


# Candidates per vocabulary shard for the vocabulary-parallel stochastic sampler.
SAMPLE_KC = 64
# forward()'s sampling mode: greedy, stochastic, stochastic with every
# stochastic row's top_k in (0, SAMPLE_KC].
SAMPLE_GREEDY, SAMPLE_FULL, SAMPLE_TOPK = 0, 1, 2


def sample_mode(rows, candidates: bool) -> int:
    stoch = [r for r in rows if r.sample and r.req.sampling.mode.value == 1]
    if not stoch:
        return SAMPLE_GREEDY
    if candidates and all(0 < (r.req.sampling.top_k or 0) <= SAMPLE_KC for r in stoch):
        return SAMPLE_TOPK
    return SAMPLE_FULL


class ModelRunner:
    def __init__(self, weights: ModelWeights, ops, device, num_pages: int, max_tokens: int, max_rows: int,
                 max_context: int, page: int = 16, graph_sizes: Sequence[int] = (), comm=None,
                 check_errors_every: int = 16, sequence_parallel: bool = False, overlap: bool = False,
                 sample_candidates: bool = False, moe_all_to_all: bool = False):
        self.w = weights
        self.spec: LlamaSpec = weights.spec
        self.shard = weights.shard
        self.ops = ops
        self.device = torch.device(device)
        self.comm = comm
        self.P = page
        self.max_tokens = max_tokens
        self.max_rows = max_rows
        self.max_context = max_context
        self.W = -(-max_context // page)
        self.num_pages = num_pages + 1          # physical page 0 is the reserved zero page
        self.check_every = check_errors_every
        # admit each packed step against the KV arena before its upload
        self.check_steps = os.environ.get("LUNAFLUX_CHECK_LAUNCHES") == "1"
        s, sh = self.spec, self.shard
        dt = weights.embed.dtype
        self.dtype = dt
        self.Hq, self.Hkv, self.D = sh.heads, sh.kv_heads, s.head_dim
        H = s.hidden
        dev = self.device
        # KV arena: [layer][K/V][page][kv_head][16][D]
        self.kv = torch.zeros(s.layers, 2, self.num_pages, self.Hkv, page, self.D, dtype=dt, device=dev)
        self.cos_sin = rope_table(s.max_position, s.head_dim, s.rope_theta, dev, s.rope_scaling)
        T, R = max_tokens, max_rows
        self.resid = torch.empty(T, H, dtype=dt, device=dev)
        self.h = torch.empty(T, H, dtype=dt, device=dev)
        self.delta = torch.empty(T, H, dtype=dt, device=dev)
        # Sequence parallelism (Megatron): between the row-parallel projections
        # and the next column-parallel one the residual stream lives sharded by
        # tokens, so the norms and residual adds run on T / tp rows; the
        # row-parallel partial sums are reduce-scattered instead of all-reduced
        # and the normed rows all-gathered before the next projection.
        self.sp = bool(sequence_parallel) and comm is not None and sh.size > 1
        # expert parallelism over the token-sharded rows (dispatch / combine
        # all-to-all) instead of experts on the gathered rows
        self.moe_a2a = None
        if self.sp and s.is_moe and moe_all_to_all:
            from ..parallel.moe_a2a import ExpertAllToAll, LibraryExpertAllToAll
            if weights.ep_size != sh.size:
                raise ValueError("the expert all-to-all needs experts sharded over every rank (ep_size == tp)")
            if dev.type == "cuda" and os.environ.get("LUNAFLUX_MOE_A2A_LIBRARY") != "1":
                ffn = weights.layers[0].experts_d.shape[-1]
                self.moe_a2a = ExpertAllToAll(s.experts, s.experts_per_token, sh.size, sh.rank, s.hidden, ffn,
                                              -(-T // sh.size), dev, getattr(comm, "group", None))
            else:
                self.moe_a2a = LibraryExpertAllToAll(s.experts, s.experts_per_token, sh.size, sh.rank,
                                                     getattr(comm, "group", None))
                if dev.type == "cuda":
                    graph_sizes = ()     # the library exchange sizes itself on the host: not capturable
        if self.sp:
            tp = sh.size
            Tl = -(-T // tp)
            if getattr(comm, "fused", False) and hasattr(comm, "enable_norm_gather"):
                comm.enable_norm_gather(Tl, dev)   # RMSNorm with the all-gather in its epilogue
            self.sp_full = torch.zeros(Tl * tp, H, dtype=dt, device=dev)    # gathered rows / partial sums
            self.sp_resid = torch.zeros(Tl, H, dtype=dt, device=dev)
            self.sp_h = torch.zeros(Tl, H, dtype=dt, device=dev)
            self.sp_delta = torch.zeros(Tl, H, dtype=dt, device=dev)
        self.qkv = torch.empty(T, sh.qkv_size, dtype=dt, device=dev)
        self.attn = torch.empty(T, self.Hq * self.D, dtype=dt, device=dev)
        self.act = torch.empty(T, sh.ffn_padded, dtype=dt, device=dev)
        self.hs = torch.empty(R, H, dtype=dt, device=dev)
        self.logits = torch.empty(R, sh.vocab, dtype=torch.float32, device=dev)
        self.full_logits = (torch.empty(R, s.vocab, dtype=torch.float32, device=dev)
                            if sh.size > 1 else self.logits)
        self.out_tok = torch.zeros(R, dtype=torch.int32, device=dev)
        # Overlapped steps: the next step is launched before this one's tokens
        # reach the host; its decode rows read them here, on the device.
        self.overlap = bool(overlap)
        self.prev_tok = torch.zeros(R, dtype=torch.int32, device=dev)
        if s.is_moe:
            self._init_moe(T, dev)
        if s.fp8_block:
            kmax = max(H, self.Hq * self.D, sh.ffn_padded)
            self.q8 = torch.zeros(T * kmax, dtype=torch.float8_e4m3fn, device=dev)
            self.q8s = torch.zeros(T * (kmax // 128), dtype=torch.float32, device=dev)
            # split-K workspace of the decode-sized fp8 GEMMs (all-zero between GEMMs)
            nmax = max(H, sh.qkv_size, 2 * sh.ffn_padded)
            self.fp8_ws = (torch.zeros(min(T, 256) * nmax, dtype=torch.float32, device=dev)
                           if dev.type == "cuda" else None)
        self.keys_local = torch.zeros(R, dtype=torch.int64, device=dev)
        self.keys_all = torch.zeros(R * sh.size, dtype=torch.int64, device=dev)
        # Vocabulary-parallel stochastic sampling from per-shard candidates
        # (each shard's SAMPLE_KC largest keys; exact when every stochastic row
        # has 0 < top_k <= SAMPLE_KC) instead of gathering every shard's logits.
        self.sample_candidates = bool(sample_candidates) and sh.size > 1
        if self.sample_candidates:
            self.cand_local = torch.zeros(R * (SAMPLE_KC + 1), dtype=torch.int64, device=dev)
            self.cand_all = torch.zeros(sh.size * R * (SAMPLE_KC + 1), dtype=torch.int64, device=dev)
        # split-K GEMM workspace (kept all-zero between GEMMs) and split-KV decode partials
        ws_elems = 512 * max(32768, sh.qkv_size, 2 * sh.ffn_padded)
        if s.fp8_block and comm is not None and getattr(comm, "fused", False):
            ws_elems = max(ws_elems, T * H)  # fp32 partials of the fp8 row-parallel projections
        self.gemm_ws = torch.zeros(ws_elems, dtype=torch.float32, device=dev) if dev.type == "cuda" else None
        self.max_splits = 32
        self.part_o = torch.empty(R * self.Hq * self.max_splits * self.D, dtype=torch.float32, device=dev)
        self.part_lse = torch.empty(R * self.Hq * self.max_splits, dtype=torch.float32, device=dev)
        # packed step inputs: one device block + two pinned host blocks (double buffer)
        cap = make_layout(T, R, R, R, self.W).total + 64
        self.in_dev = torch.zeros(cap, dtype=torch.int32, device=dev)
        pin = dev.type == "cuda"
        self.in_host = [torch.zeros(cap, dtype=torch.int32, pin_memory=pin) for _ in range(2)]
        self.in_evt = [None, None]
        self.out_host = [torch.zeros(R, dtype=torch.int32, pin_memory=pin) for _ in range(2)]
        self._oflip = 0
        self._flip = 0
        self._embed_fwd = None
        self.graphs: Dict[tuple, torch.cuda.CUDAGraph] = {}
        self.graph_launches: Dict[tuple, int] = {}
        self.graph_sizes = sorted(b for b in graph_sizes if b <= R)
        self.stream = torch.cuda.Stream(device=dev) if dev.type == "cuda" else None
        self.steps = 0
        self.last_bucket: Optional[int] = None      # graph bucket of the last step (None: eager)
        self.capture_times: List[float] = []      # seconds per capture, until taken
        # accounting for the bench
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self.device_ms = 0.0          # sum over steps of device time from first kernel to sampled ids
        if dev.type == "cuda":
            self._ev_begin = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
            self._ev_end = [torch.cuda.Event(enable_timing=True) for _ in range(2)]

    # ------------------------------------------------------------------ forward
    def _layer_kv(self, l):
        return self.kv[l, 0], self.kv[l, 1]

    def forward(self, v: Dict[str, torch.Tensor], T: int, Tp: int, Rp: int, Rd: int, Rs: int, max_q_len: int,
                splits: int, stochastic: bool, host_meta=None, gather: bool = True):
        # decode rows whose input token was sampled by the previous step (not
        # yet on the host) take it from that step's output inside the embedding
        self._embed_fwd = (v["d_fwd"][:Rd], Tp, self.prev_tok) if self.overlap and Rd else None
        if self.sp:
            out = self.forward_sp(v, T, Tp, Rp, Rd, Rs, max_q_len, splits, stochastic, host_meta, gather)
        else:
            out = self._forward_tp(v, T, Tp, Rp, Rd, Rs, max_q_len, splits, stochastic, host_meta, gather)
        if self.overlap:
            self.prev_tok[:Rs].copy_(out)
        return out

    def _forward_tp(self, v, T, Tp, Rp, Rd, Rs, max_q_len, splits, stochastic, host_meta=None, gather=True):
        ops, s, w = self.ops, self.spec, self.w
        eps = s.rms_eps
        resid, h, delta = self.resid[:T], self.h[:T], self.delta[:T]
        act = self.act[:T]
        ws = self.gemm_ws
        hm = host_meta or {}
        if self.comm is not None and getattr(self.comm, "fused", False):
            self.comm.begin_forward()
        ops.embed(v["tokens"], w.embed, resid, self._embed_fwd)
        for l, lw in enumerate(w.layers):
            if l == 0:
                ops.rmsnorm(resid, None, lw.ln1, h, eps)
            else:
                ops.rmsnorm(delta, resid, lw.ln1, h, eps)
            attn = self._attention(l, lw, v, h, T, Tp, Rp, Rd, max_q_len, splits, hm)
            delta = self._row_parallel(attn, lw, "wo", self.delta[:T], ws)
            ops.rmsnorm(delta, resid, lw.ln2, h, eps)
            if s.is_moe:
                delta = self.delta[:T]
                self.moe(h, delta, lw)
            else:
                self._proj(h, lw, "wgu", act, 2)
                delta = self._row_parallel(act, lw, "wd", self.delta[:T], ws)
        if gather:
            # the final norm only for the sampled rows, gathered as it reads them
            hs = self.hs[:Rs]
            ops.rmsnorm(delta, resid, w.norm, hs, eps, v["s_idx"])
            return self._sample(hs, v, Rs, stochastic, False)
        ops.rmsnorm(delta, resid, w.norm, h, eps)
        return self._sample(h, v, Rs, stochastic, gather)

    def _sample(self, h, v, Rs, stochastic, gather):
        """LM head on the sampled rows of h and the on-device sampler (vocab
        shards exchange candidates or logits under tensor parallelism)."""
        ops, w = self.ops, self.w
        if gather:
            hs = self.hs[:Rs]
            torch.index_select(h, 0, v["s_idx"], out=hs)   # int32 ids: no index copy
        else:
            hs = h[:Rs]
        logits = self.logits[:Rs]
        ops.gemm(hs, w.lm_head, logits, 1, self.gemm_ws)
        out = self.out_tok[:Rs]
        tp = self.shard.size
        if self.comm is not None and tp > 1:
            if stochastic == SAMPLE_TOPK and self.sample_candidates:
                # every stochastic row keeps at most SAMPLE_KC tokens: exchange
                # each shard's SAMPLE_KC largest keys, then draw on every rank
                kc = SAMPLE_KC
                cand = self.cand_local[: Rs * (kc + 1)]
                ops.topk_keys(logits, self.shard.rank * self.shard.vocab, kc, cand)
                allc = self.cand_all[: tp * Rs * (kc + 1)]
                self.comm.all_gather_flat(cand, allc)
                ops.sample_keys(allc, Rs, tp, kc, v["s_params"], out)
            elif stochastic:
                # top-k / top-p need the whole distribution: gather the vocab shards
                full = self.full_logits[:Rs]
                self.comm.all_gather_cols(logits, full)
                ops.sample(full, v["s_params"], out)
            else:
                # greedy: exchange one (logit, lowest id) key per row and shard
                keys = self.keys_local[:Rs]
                ops.argmax_keys(logits, self.shard.rank * self.shard.vocab, keys)
                allk = self.keys_all[: tp * Rs]
                self.comm.all_gather_flat(keys, allk)
                ops.keys_to_tokens(allk, Rs, tp, out)
            return out
        if stochastic:
            ops.sample(logits, v["s_params"], out)
        else:
            ops.argmax(logits, out)
        return out

    def _attention(self, l, lw, v, h, T, Tp, Rp, Rd, max_q_len, splits, hm):
        """QKV projection, RoPE + paged KV write, prefill and decode attention
        for the T token rows of h; returns the attention output rows."""
        ops, Hq, Hkv = self.ops, self.Hq, self.Hkv
        kc, vc = self._layer_kv(l)
        qkv, attn = self.qkv[:T], self.attn[:T]
        fused = (self._fp8(lw, "wqkv") is None and hasattr(ops, "qkv_rope")
                 and ops.qkv_rope(h, lw.wqkv, qkv, v["positions"], v["slots"], self.cos_sin, kc, vc, Hq, Hkv, self.P))
        if not fused:
            self._proj(h, lw, "wqkv", qkv, 0)
            ops.rope_kv_write(qkv, v["positions"], v["slots"], self.cos_sin, kc, vc, Hq, Hkv, self.P)
        if Rp:
            ops.attn_prefill(qkv[:Tp], attn[:Tp], v["p_qstart"], v["p_seqlen"], v["p_bt"], kc, vc, Hq, Hkv,
                             max_q_len, host={"q_start": hm.get("q_start"), "seq_lens": hm.get("seq_lens")})
        if Rd:
            ops.attn_decode(qkv, attn, v["d_tok"], v["d_seqlen"], v["d_bt"], kc, vc, Hq, Hkv, splits,
                            self.part_o, self.part_lse,
                            host={"seq_lens": hm.get("d_seq_lens"), "tok": hm.get("d_tok")})
        return attn

    def forward_sp(self, v, T, Tp, Rp, Rd, Rs, max_q_len, splits, stochastic, host_meta=None, gather=True):
        """The forward with the residual stream sharded by tokens: this rank
        owns rows [rank * Tl, (rank + 1) * Tl) of the (padded) step."""
        ops, s, w, comm = self.ops, self.spec, self.w, self.comm
        tp, rank = self.shard.size, self.shard.rank
        eps = s.rms_eps
        hm = host_meta or {}
        Tl = -(-T // tp)
        full = self.sp_full[: Tl * tp]
        resid, h, delta = self.sp_resid[:Tl], self.sp_h[:Tl], self.sp_delta[:Tl]
        act = self.act[:T]
        ws = self.gemm_ws
        # embeddings of every token, then this rank's rows (padding rows are zero)
        emb = self.h[:T]
        ops.embed(v["tokens"], w.embed, emb, self._embed_fwd)
        full[T:].zero_()
        full[:T].copy_(emb)
        resid.copy_(full[rank * Tl:(rank + 1) * Tl])

        def gather_rows(local):
            comm.all_gather_rows(local, full)
            return full[:T]

        fused_gather = getattr(comm, "ng_rows", 0) >= Tl
        if getattr(comm, "fused", False):
            comm.begin_forward()

        def norm_gather(x, residual, weight, final=False):
            """RMSNorm of the local rows (residual added in place), gathered:
            in one kernel with the all-gather in its epilogue when the fused
            comm is set up for it, else the norm and the library all-gather."""
            if fused_gather:
                ops.launches += 2
                return comm.norm_gather(x, residual, weight, eps, final)[:T]
            ops.rmsnorm(x, residual, weight, h, eps)
            return gather_rows(h)

        def scatter_gemm(A, lw, name):
            """delta = this rank's rows of the row-parallel projection: one
            kernel with the reduce-scatter inside when the fused comm takes
            the shape, else the partial GEMM and the library reduce-scatter."""
            if (T == Tl * tp and self._fp8(lw, name) is None
                    and hasattr(comm, "gemm_reduce_scatter")
                    and comm.gemm_reduce_scatter(A, getattr(lw, name), delta)):
                ops.launches += 1
                return
            part = self.delta[:T]
            self._row_parallel_partial(A, lw, name, part, ws)
            scatter_partial(part)

        def scatter_partial(partial_rows):
            # partial_rows: [T, H] this rank's partial sums; padding rows add zero
            if partial_rows.data_ptr() != full.data_ptr():
                full[:T].copy_(partial_rows)
            full[T:].zero_()
            comm.reduce_scatter_rows(full, delta)

        for l, lw in enumerate(w.layers):
            if l == 0:
                hf = norm_gather(resid, None, lw.ln1)
            else:
                hf = norm_gather(delta, resid, lw.ln1)
            attn = self._attention(l, lw, v, hf, T, Tp, Rp, Rd, max_q_len, splits, hm)
            scatter_gemm(attn, lw, "wo")
            if s.is_moe and self.moe_a2a is not None:
                # tokens stay sharded: dispatch to the experts' ranks and back
                ops.rmsnorm(delta, resid, lw.ln2, h, eps)
                delta.copy_(self.moe_a2a.forward(h, lw, ops, self.router_bias))
            elif s.is_moe:
                hf = norm_gather(delta, resid, lw.ln2)
                d_part = self.delta[:T]
                self.moe(hf, d_part, lw, reduce=False)
                scatter_partial(d_part)
            else:
                hf = norm_gather(delta, resid, lw.ln2)
                self._proj(hf, lw, "wgu", act, 2)
                scatter_gemm(act, lw, "wd")
        hf = norm_gather(delta, resid, w.norm, final=True)
        return self._sample(hf, v, Rs, stochastic, gather)

    def _row_parallel_partial(self, A, lw, name, out, ws):
        """This rank's partial sum of a row-parallel projection (no reduction)."""
        f = self._fp8(lw, name)
        if f is not None:
            q, s = self._quant(A)
            self.ops.gemm_fp8(q, s, f[0], f[1], out, 0, self.fp8_ws)
        else:
            self.ops.gemm(A, getattr(lw, name), out, 0, ws)

    def _fp8(self, lw, name):
        return lw.fp8.get(name) if lw.fp8 is not None else None

    def _quant(self, x):
        """Per-token, per-128-channel e4m3 copy of x (static buffers)."""
        T, K = x.shape
        q = self.q8[: T * K].view(T, K)
        s = self.q8s[: T * (K // 128)].view(T, K // 128)
        self.ops.act_quant(x, q, s)
        return q, s

    def _proj(self, x, lw, name, out, epi):
        """Column-parallel projection: block-scaled fp8 when the layer has fp8
        weights, bf16 tcgen05 GEMM otherwise."""
        f = self._fp8(lw, name)
        if f is not None:
            q, s = self._quant(x)
            self.ops.gemm_fp8(q, s, f[0], f[1], out, epi, self.fp8_ws)
        else:
            self.ops.gemm(x, getattr(lw, name), out, epi, self.gemm_ws)

    def _row_parallel(self, A, lw, name, out, ws):
        """Row-parallel projection: partial GEMM then the sum over ranks, either
        as one fused GEMM + all-reduce kernel or as GEMM followed by the
        library all-reduce (the measured baseline).  Returns the tensor holding
        the result: ``out``, or with the fused path a view of the symmetric
        result region."""
        f = self._fp8(lw, name)
        fused = self.comm is not None and getattr(self.comm, "fused", False)
        if f is not None:
            q, s = self._quant(A)
            if fused:
                part = ws[: out.numel()].view(out.shape)
                self.ops.gemm_fp8(q, s, f[0], f[1], part, 1, self.fp8_ws)
                self.ops.launches += 1
                return self.comm.reduce_partials(part)
            self.ops.gemm_fp8(q, s, f[0], f[1], out, 0, self.fp8_ws)
            if self.comm is not None:
                self.comm.all_reduce(out)
            return out
        W = getattr(lw, name)
        if self.comm is None:
            self.ops.gemm(A, W, out, 0, ws)
        elif fused:
            self.ops.launches += 2
            return self.comm.gemm_allreduce(A, W, ws)
        else:
            self.ops.gemm(A, W, out, 0, ws)
            self.comm.all_reduce(out)
        return out

    # Steps of at least this many tokens pad expert segments to 256 rows, so
    # the grouped GEMMs run on CTA pairs (one expert per 256-row tile); smaller
    # steps (decode, captured in graphs) keep 128-row segments.
    MOE_PAIR_TOKENS = 2048

    def _moe_align(self, T: int) -> int:
        return 256 if T >= self.MOE_PAIR_TOKENS and self.device.type == "cuda" else 128

    def _moe_rows(self, T: int, align: Optional[int] = None) -> int:
        """Rows of the expert-ordered activations for T tokens: every
        assignment plus up to align - 1 padding rows per local expert."""
        a = self._moe_align(T) if align is None else align
        return -(-(T * self.spec.experts_per_token + self.moe_El * (a - 1)) // a) * a

    def _init_moe(self, T: int, dev):
        s = self.spec
        k = s.experts_per_token
        self.moe_El = s.experts // self.w.ep_size
        self.moe_e0 = self.w.ep_rank * self.moe_El
        rows = max(self._moe_rows(T, 128), self._moe_rows(T, 256))
        Fp = self.w.layers[0].experts_d.shape[-1]
        self.moe_ids = torch.zeros(T, k, dtype=torch.int32, device=dev)
        self.moe_w = torch.zeros(T, k, dtype=torch.float32, device=dev)
        self.moe_groups = torch.zeros(self.moe_El + 1, dtype=torch.int32, device=dev)
        self.moe_perm = torch.zeros(rows, dtype=torch.int32, device=dev)
        self.moe_slot = torch.zeros(T * k, dtype=torch.int32, device=dev)
        self.moe_x = torch.zeros(rows, s.hidden, dtype=self.dtype, device=dev)
        self.moe_act = torch.zeros(rows, Fp, dtype=self.dtype, device=dev)
        self.moe_y = torch.zeros(rows, s.hidden, dtype=self.dtype, device=dev)
        self.router_bias: Optional[torch.Tensor] = None  # fp32 [E] logit bias (load-skew experiments)

    def moe(self, h, delta, lw, reduce: bool = True):
        """Routed SwiGLU experts: route -> align -> gather -> grouped gate/up
        GEMM (SwiGLU epilogue) -> grouped down GEMM -> weighted combine, then
        the sum over ranks (experts or expert shards live on different ranks)."""
        ops, k, El = self.ops, self.spec.experts_per_token, self.moe_El
        T = h.shape[0]
        al = self._moe_align(T)
        rows = self._moe_rows(T, al)
        ids, w = self.moe_ids[:T], self.moe_w[:T]
        ops.moe_route(h, lw.router, self.router_bias, k, ids, w)
        ops.moe_align(ids, T, k, self.moe_e0, El, self.moe_groups, self.moe_perm[:rows], self.moe_slot[:T * k], al)
        ops.moe_gather(h, self.moe_perm[:rows], self.moe_groups, El, k, self.moe_x[:rows])
        ops.gemm_grouped(self.moe_x[:rows], lw.experts_gu, self.moe_act[:rows], self.moe_groups, El, 2, al)
        ops.gemm_grouped(self.moe_act[:rows], lw.experts_d, self.moe_y[:rows], self.moe_groups, El, 0, al)
        ops.moe_combine(self.moe_y[:rows], self.moe_slot[:T * k], w, T, k, delta)
        if self.comm is not None and reduce:
            self.comm.all_reduce(delta)

    # ------------------------------------------------------------------ one step
    def _upload(self, hs: HostStep, host_buf: torch.Tensor):
        n = hs.layout.total
        if self.device.type == "cuda":
            self.in_dev[:n].copy_(host_buf[:n], non_blocking=True)
        else:
            self.in_dev[:n].copy_(host_buf[:n])
        self.h2d_bytes += n * 4

    def execute(self, plan: StepPlan, table_matrix: np.ndarray) -> np.ndarray:
        """Runs one step and returns the sampled token ids (sampling rows, plan
        order).  On CUDA the step is one NVTX range (visible to Nsight tools),
        named by its kind and size."""
        if self.device.type != "cuda":
            return self._execute(plan, table_matrix)
        kind = "decode" if all(r.decode for r in plan.rows) else "mixed"
        torch.cuda.nvtx.range_push(f"lunaflux.step.{kind} rows={len(plan.rows)} tokens={plan.num_tokens}")
        try:
            return self._execute(plan, table_matrix)
        finally:
            torch.cuda.nvtx.range_pop()

    def _execute(self, plan: StepPlan, table_matrix: np.ndarray) -> np.ndarray:
        return self.wait(self.launch(plan, table_matrix))

    def launch(self, plan: StepPlan, table_matrix: np.ndarray):
        """Packs and uploads the step, launches it (graph replay or eager
        forward) and queues the copy of its sampled ids to pinned host memory.
        Returns a handle for ``wait``; nothing here waits for the device."""
        rows = plan.rows
        decode_only = all(r.decode for r in rows)
        stoch = sample_mode(rows, self.sample_candidates)
        bucket = None
        if decode_only and self.graph_sizes and self.device.type == "cuda":
            nd = len(rows)
            bucket = next((b for b in self.graph_sizes if b >= nd), None)
        self.last_bucket = bucket
        slot = self._flip
        self._flip ^= 1
        if self.in_evt[slot] is not None:
            self.in_evt[slot].synchronize()  # the previous upload from this pinned block has finished
        host_buf = self.in_host[slot]
        hs = build_host_step(plan, table_matrix, self.P, self.W, host_buf.numpy(), bucket=bucket)
        if self.check_steps:
            check_paged_step(hs.layout, hs.buf, self.num_pages, self.P, self.spec.vocab)
        if hs.any_forwarded and not self.overlap:
            raise ValueError("a step forwards device tokens but the runner was built without overlap")
        L = hs.layout
        Rs_real = sum(1 for r in rows if r.sample)
        oslot = self._oflip
        self._oflip ^= 1
        if bucket is not None:
            key = (bucket, stoch)
            g = self.graphs.get(key)
            if g is None:
                g = self.capture(bucket, stoch)
            self._upload(hs, host_buf)
            self._record_upload(slot)
            self._begin_step(oslot)
            g.replay()
            self.ops.launches += self.graph_launches[key]
        else:
            self._upload(hs, host_buf)
            self._record_upload(slot)
            self._begin_step(oslot)
            v = device_views(self.in_dev, L)
            Tp = L.T - L.Rd
            splits = self.ops.decode_splits(L.Rd, self.Hkv, max(hs.max_seq, 1)) if L.Rd else 1
            self.forward(v, L.T, Tp, L.Rp, L.Rd, L.Rs, hs.max_q_len, splits, stoch, hs.host_meta)
        out = self.out_tok[:Rs_real]
        dst = self.out_host[oslot][:Rs_real]
        done = None
        if self.device.type == "cuda":
            self._ev_end[oslot].record()
            dst.copy_(out, non_blocking=True)
            done = torch.cuda.Event()
            done.record()
        else:
            dst.copy_(out)
        self.d2h_bytes += Rs_real * 4
        return (oslot, Rs_real, done)

    def wait(self, handle) -> np.ndarray:
        """Waits for a launched step and returns its sampled ids (sampling
        rows, plan order)."""
        oslot, Rs_real, done = handle
        if done is not None:
            done.synchronize()
            self.device_ms += self._ev_begin[oslot].elapsed_time(self._ev_end[oslot])
        res = self.out_host[oslot][:Rs_real].numpy().copy()
        self.steps += 1
        if self.check_every and self.steps % self.check_every == 0:
            self.check_device_errors()
        return res

    def _begin_step(self, oslot: int):
        if self.device.type == "cuda":
            self._ev_begin[oslot].record()

    def _record_upload(self, slot):
        if self.device.type == "cuda":
            e = torch.cuda.Event()
            e.record()
            self.in_evt[slot] = e

    def check_device_errors(self):
        code, info = self.ops.read_error(True)
        if code:
            raise StepFailed(code, info)

    # ------------------------------------------------------------------ graphs
    def capture(self, bucket: int, stochastic: bool) -> "torch.cuda.CUDAGraph":
        """Captures the decode step for ``bucket`` rows reading its inputs at
        the fixed offsets of ``make_layout(bucket, 0, bucket, bucket, W)``."""
        t_start = time.perf_counter()
        L = make_layout(bucket, 0, bucket, bucket, self.W)
        v = device_views(self.in_dev, L)
        # a capture in the middle of overlapped steps must not lose the
        # in-flight step's tokens (the warm-up passes overwrite them)
        saved_prev = self.prev_tok.clone() if self.overlap else None
        splits = self.ops.decode_splits(bucket, self.Hkv, self.max_context)
        splits = min(splits, self.max_splits)
        # inputs for warm-up: every row a padded row (zero page, no KV write)
        self.in_dev[: L.total].zero_()
        o, n = L.field("slots")
        self.in_dev[o:o + n].fill_(-1)
        o, n = L.field("d_seqlen")
        self.in_dev[o:o + n].fill_(1)
        o, n = L.field("d_tok")
        self.in_dev[o:o + n].copy_(torch.arange(n, dtype=torch.int32, device=self.device))
        o, n = L.field("s_idx")
        self.in_dev[o:o + n].copy_(torch.arange(n, dtype=torch.int32, device=self.device))
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(2):
                self.forward(v, bucket, 0, 0, bucket, bucket, 0, splits, stochastic, gather=False)
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        before = getattr(self.ops, "launches", 0)
        with torch.cuda.graph(g, stream=s):
            self.forward(v, bucket, 0, 0, bucket, bucket, 0, splits, stochastic, gather=False)
        torch.cuda.synchronize(self.device)
        self.graph_launches[(bucket, stochastic)] = getattr(self.ops, "launches", 0) - before
        self.ops.launches = before
        self.graphs[(bucket, stochastic)] = g
        if saved_prev is not None:
            self.prev_tok.copy_(saved_prev)
        self.capture_times.append(time.perf_counter() - t_start)
        return g

    def take_capture_times(self) -> List[float]:
        t, self.capture_times = self.capture_times, []
        return t

    def capture_all(self, stochastic: bool = False):
        for b in self.graph_sizes:
            if (b, stochastic) not in self.graphs:
                self.capture(b, stochastic)
