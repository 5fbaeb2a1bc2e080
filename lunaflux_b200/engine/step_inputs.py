"""Per-step device descriptor: packing a StepPlan into one int32 block.

The reference's paged step descriptor is seven Int32 device operands
(engine/device_step/README.mbt.md:1-110; stage.mbt:166-268): counts, token
ids, absolute positions, CSR query-row offsets, sequence lengths, CSR page
offsets and physical page indices, uploaded with synchronous copies.  Here the
same information (with a dense per-row block table instead of CSR page
offsets, plus KV write slots and the sampling records) is packed on the host
into ONE pinned int32 buffer and uploaded with ONE asynchronous copy per
step.  The field offsets depend only on (T, Rp, Rd, Rs, W); a CUDA graph
captured for a decode bucket therefore always finds its inputs at the same
device addresses.
"""
from __future__ import annotations

import dataclasses
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from ..sampling.host import PARAM_DTYPE
from ..scheduler.scheduler import Row, StepPlan

PARAM_INTS = PARAM_DTYPE.itemsize // 4  # 8 int32 per sampling record


def _al(n: int) -> int:
    return (n + 3) & ~3  # 16-byte aligned regions


@dataclasses.dataclass(frozen=True)
class Layout:
    T: int
    Rp: int
    Rd: int
    Rs: int
    W: int
    offsets: Tuple[Tuple[str, int, int], ...]   # (field, offset, length) in int32 units
    total: int

    def field(self, name: str) -> Tuple[int, int]:
        for n, o, l in self.offsets:
            if n == name:
                return o, l
        raise KeyError(name)


def make_layout(T: int, Rp: int, Rd: int, Rs: int, W: int) -> Layout:
    fields = [("tokens", T), ("positions", T), ("slots", T), ("p_qstart", Rp + 1), ("p_seqlen", Rp),
              ("p_bt", Rp * W), ("d_tok", Rd), ("d_seqlen", Rd), ("d_bt", Rd * W), ("d_fwd", Rd), ("s_idx", Rs),
              ("s_params", Rs * PARAM_INTS)]
    offs = []
    o = 0
    for name, n in fields:
        offs.append((name, o, n))
        o += _al(n)
    return Layout(T, Rp, Rd, Rs, W, tuple(offs), o)


@dataclasses.dataclass
class HostStep:
    layout: Layout
    buf: np.ndarray                 # int32 view of the packed block (len == layout.total)
    max_q_len: int
    max_seq: int
    any_stochastic: bool
    host_meta: Dict[str, np.ndarray]
    graph_bucket: Optional[int]
    any_forwarded: bool = False     # some decode row reads its input token on the device


def row_tokens(r: Row) -> np.ndarray:
    req = r.req
    n_prompt = len(req.prompt)
    s, e = r.start, r.start + r.n
    if e <= n_prompt:
        return np.asarray(req.prompt[s:e], dtype=np.int32)
    parts = []
    if s < n_prompt:
        parts.append(np.asarray(req.prompt[s:], dtype=np.int32))
    parts.append(np.asarray(req.output[max(0, s - n_prompt):e - n_prompt], dtype=np.int32))
    return np.concatenate(parts)


def build_host_step(plan: StepPlan, table_matrix: np.ndarray, P: int, W: int, out: np.ndarray,
                    bucket: Optional[int] = None) -> HostStep:
    """Packs ``plan`` into ``out`` (an int32 array, e.g. a pinned buffer's numpy view).

    ``bucket``: pad a decode-only plan to this many rows (CUDA-graph replay)."""
    pr = [r for r in plan.rows if not r.decode]
    dr = [r for r in plan.rows if r.decode]
    if bucket is not None and pr:
        raise ValueError("graph buckets are decode-only")
    Rp = len(pr)
    Rd = len(dr) if bucket is None else bucket
    Tp = sum(r.n for r in pr)
    T = Tp + Rd
    srows = [r for r in plan.rows if r.sample]
    Rs = len(srows) if bucket is None else bucket
    L = make_layout(T, Rp, Rd, Rs, W)
    buf = out[: L.total]

    def put(name, arr):
        o, n = L.field(name)
        buf[o:o + n] = arr

    def view(name):
        o, n = L.field(name)
        return buf[o:o + n]

    # --- prefill rows
    max_q = 0
    max_seq = 0
    if not Rp:
        put("p_qstart", (0,))      # the field exists (Rp + 1 = 1 word): no stale word from a reused buffer
    if Rp:
        ns = np.fromiter((r.n for r in pr), dtype=np.int64, count=Rp)
        starts = np.fromiter((r.start for r in pr), dtype=np.int64, count=Rp)
        tbl = np.fromiter((r.req.table.index for r in pr), dtype=np.int64, count=Rp)
        qs = np.zeros(Rp + 1, dtype=np.int32)
        np.cumsum(ns, out=qs[1:])
        toks = np.concatenate([row_tokens(r) for r in pr])
        pos = np.concatenate([np.arange(s, s + n, dtype=np.int64) for s, n in zip(starts, ns)])
        rowid = np.repeat(np.arange(Rp), ns)
        slots = table_matrix[tbl[rowid], pos // P].astype(np.int64) * P + pos % P
        view("tokens")[:Tp] = toks
        view("positions")[:Tp] = pos
        view("slots")[:Tp] = slots
        put("p_qstart", qs)
        put("p_seqlen", (starts + ns).astype(np.int32))
        put("p_bt", table_matrix[tbl, :W].reshape(-1))
        max_q = int(ns.max())
        max_seq = int((starts + ns).max())
    # --- decode rows
    nd = len(dr)
    if Rd:
        d_tok = np.arange(Tp, Tp + Rd, dtype=np.int32)
        put("d_tok", d_tok)
        seql = np.ones(Rd, dtype=np.int32)
        bt = view("d_bt").reshape(Rd, W)
        toks = view("tokens")[Tp:]
        pos = view("positions")[Tp:]
        slots = view("slots")[Tp:]
        fwd = view("d_fwd")
        fwd[:] = -1
        if nd:
            fwd[:nd] = np.fromiter((r.fwd for r in dr), dtype=np.int32, count=nd)
            starts = np.fromiter((r.start for r in dr), dtype=np.int64, count=nd)
            tbl = np.fromiter((r.req.table.index for r in dr), dtype=np.int64, count=nd)
            toks[:nd] = np.fromiter((r.req.output[-1] if r.req.output else r.req.prompt[-1] for r in dr),
                                    dtype=np.int32, count=nd)
            pos[:nd] = starts
            slots[:nd] = table_matrix[tbl, starts // P].astype(np.int64) * P + starts % P
            seql[:nd] = starts + 1
            bt[:nd] = table_matrix[tbl, :W]
            max_seq = max(max_seq, int(starts.max()) + 1)
        if Rd > nd:
            toks[nd:] = 0
            pos[nd:] = 0
            slots[nd:] = -1
            bt[nd:] = 0
        put("d_seqlen", seql)
    # --- sampling rows (columns gathered in one pass, written field by field)
    sidx = view("s_idx")
    params = view("s_params").view(PARAM_DTYPE) if Rs else np.zeros(0, dtype=PARAM_DTYPE)
    any_stoch = False
    any_fwd = bool(nd) and any(r.fwd >= 0 for r in dr)
    if Rs:
        params[:] = 0
        qs_arr = view("p_qstart") if Rp else None
        idx, mode, topk, temp, topp, seed, count = [], [], [], [], [], [], []
        p_i = d_i = 0
        for r in plan.rows:
            if r.decode:
                row_last = Tp + d_i
                d_i += 1
            else:
                row_last = int(qs_arr[p_i + 1]) - 1
                p_i += 1
            if not r.sample:
                continue
            sp = r.req.sampling
            idx.append(row_last)
            seed.append(sp.seed)
            count.append(r.sample_index)
            if sp.mode.value == 1:
                any_stoch = True
                mode.append(1)
                topk.append(sp.top_k or 0)
                temp.append(sp.temperature)
                topp.append(sp.top_p if sp.top_p is not None else 1.0)
            else:
                mode.append(0)
                topk.append(0)
                temp.append(1.0)
                topp.append(1.0)
        n = len(idx)
        sidx[:n] = idx
        params["mode"][:n] = mode
        params["top_k"][:n] = topk
        params["temperature"][:n] = temp
        params["top_p"][:n] = topp
        params["seed"][:n] = seed
        params["sample_index"][:n] = count
        if Rs > n:
            sidx[n:] = np.arange(Tp + n, Tp + Rs, dtype=np.int32)
            params["temperature"][n:] = 1.0
            params["top_p"][n:] = 1.0
    host_meta = {}
    if Rp:
        host_meta["q_start"] = view("p_qstart").copy()
        host_meta["seq_lens"] = view("p_seqlen").copy()
    if Rd:
        host_meta["d_seq_lens"] = view("d_seqlen").copy()
        host_meta["d_tok"] = view("d_tok").copy()
    return HostStep(L, buf, max_q, max_seq, any_stoch, host_meta, bucket, any_fwd)


def device_views(dev: torch.Tensor, L: Layout) -> Dict[str, torch.Tensor]:
    """Slices the device copy of a packed block into typed views."""
    v = {}
    for name, o, n in L.offsets:
        v[name] = dev[o:o + n]
    v["p_bt"] = v["p_bt"].view(L.Rp, L.W) if L.Rp else v["p_bt"].view(0, max(L.W, 1))
    v["d_bt"] = v["d_bt"].view(L.Rd, L.W) if L.Rd else v["d_bt"].view(0, max(L.W, 1))
    v["s_params"] = v["s_params"]
    return v
