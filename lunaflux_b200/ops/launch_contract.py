"""Launch contracts: what every compiled entry point accepts, checked before launch.

Reference: kernels/launch_contract (admits bounded launch metadata for each
kernel: exact dimensions, ordered operand roles, byte counts, alignments;
typed rejections; README.mbt.md) and its paged admission (admit_paged_kv:
step counts, positions, sequence lengths and page indices bounded by the KV
layout).  The reference admits contracts for AOT modules loaded at run time;
here the kernels are compiled in, so a contract describes the operands of one
``_C`` entry point and ``admit`` checks real tensors against it.  The design
is this project's own:

* a ``Contract`` lists operand ``Role`` s in call order; each role names its
  dtypes, its shape as a tuple of dimension symbols ("M", "K", ...) or
  literals, and whether it must be row-major with 16-byte rows (what TMA and
  the vectorised epilogues need);
* the first role that uses a symbol binds it; later uses must agree;
* ``rules`` are extra predicates over the bound dimensions (divisibility the
  kernels rely on, output widths that depend on the epilogue);
* ``admit`` returns an inert ``Admitted`` record (op, bound dimensions, bytes
  per operand) or raises ``LaunchContractError`` naming op, role and issue.

``check_paged_step`` is the paged half: a packed step descriptor
(``engine.step_inputs``) is validated against the KV arena it will index
(page ids, sequence lengths against the block-table width, KV write slots,
query offsets), on the host, before the upload.

``KernelOps`` checks every launch against these contracts when
``LUNAFLUX_CHECK_LAUNCHES=1`` (off by default: the bindings keep their own
cheaper checks, and a decode step is captured in a CUDA graph anyway).
"""
from __future__ import annotations

import dataclasses
import enum
from typing import Callable, Dict, Mapping, Optional, Sequence, Tuple, Union

Dim = Union[str, int]


class Issue(enum.Enum):
    MISSING = "missing operand"
    DTYPE = "dtype"
    RANK = "rank"
    SHAPE = "shape"
    LAYOUT = "layout (row-major, 16-byte rows)"
    ALIGNMENT = "alignment (16-byte base)"
    DEVICE = "device"
    RULE = "rule"


class LaunchContractError(ValueError):
    def __init__(self, op: str, role: str, issue: Issue, detail: str = ""):
        super().__init__(f"launch contract {op}: {role}: {issue.value}" + (f" ({detail})" if detail else ""))
        self.op, self.role, self.issue = op, role, issue


@dataclasses.dataclass(frozen=True)
class Role:
    name: str
    dtypes: Tuple[str, ...]            # torch dtype names: "bfloat16", "float32", "int32", ...
    shape: Tuple[Dim, ...]             # dimension symbols or literals; "*" matches anything
    rowmajor: bool = True              # contiguous last dim, 16-byte row stride, 16-byte base
    optional: bool = False


@dataclasses.dataclass(frozen=True)
class Rule:
    text: str                          # what the kernel needs, for the error message
    check: Callable[[Mapping[str, int]], bool]


@dataclasses.dataclass(frozen=True)
class Contract:
    op: str
    symbol: str                        # the _C entry point
    roles: Tuple[Role, ...]
    rules: Tuple[Rule, ...] = ()
    params: Tuple[str, ...] = ()       # integer parameters that bind symbols (e.g. "epi", "Hq")


@dataclasses.dataclass(frozen=True)
class Admitted:
    """Inert launch metadata of one admitted call."""
    op: str
    dims: Tuple[Tuple[str, int], ...]
    operand_bytes: Tuple[Tuple[str, int], ...]

    def dim(self, name: str) -> int:
        return dict(self.dims)[name]


def _dtype_name(t) -> str:
    return str(t.dtype).replace("torch.", "")


def _check_role(c: Contract, role: Role, t, dims: Dict[str, int]):
    if _dtype_name(t) not in role.dtypes:
        raise LaunchContractError(c.op, role.name, Issue.DTYPE, f"{_dtype_name(t)} not in {role.dtypes}")
    if role.shape != ("*",):
        if t.dim() != len(role.shape):
            raise LaunchContractError(c.op, role.name, Issue.RANK, f"{t.dim()} != {len(role.shape)}")
        for i, d in enumerate(role.shape):
            n = int(t.shape[i])
            if d == "*":
                continue
            if isinstance(d, int):
                if n != d:
                    raise LaunchContractError(c.op, role.name, Issue.SHAPE, f"dim {i}: {n} != {d}")
            elif d in dims:
                if dims[d] != n:
                    raise LaunchContractError(c.op, role.name, Issue.SHAPE, f"{d} = {dims[d]} but dim {i} is {n}")
            else:
                dims[d] = n
    if role.rowmajor and t.numel() > 0:
        es = t.element_size()
        if t.dim() >= 1 and t.stride(-1) != 1:
            raise LaunchContractError(c.op, role.name, Issue.LAYOUT, "last dimension not contiguous")
        if t.dim() >= 2 and (t.stride(-2) * es) % 16 != 0:
            raise LaunchContractError(c.op, role.name, Issue.LAYOUT, f"row stride {t.stride(-2) * es} B")
        if t.data_ptr() % 16 != 0:
            raise LaunchContractError(c.op, role.name, Issue.ALIGNMENT, hex(t.data_ptr()))


def admit(c: Contract, operands: Sequence, params: Optional[Mapping[str, int]] = None,
          device_type: Optional[str] = None) -> Admitted:
    """Checks `operands` (in the contract's role order; None for an absent
    optional operand) and `params` against `c`; returns the admitted metadata."""
    dims: Dict[str, int] = dict(params or {})
    if len(operands) != len(c.roles):
        raise LaunchContractError(c.op, "operands", Issue.MISSING, f"{len(operands)} given, {len(c.roles)} roles")
    sizes = []
    for role, t in zip(c.roles, operands):
        if t is None:
            if not role.optional:
                raise LaunchContractError(c.op, role.name, Issue.MISSING)
            continue
        if device_type is not None and t.device.type != device_type:
            raise LaunchContractError(c.op, role.name, Issue.DEVICE, f"{t.device.type} != {device_type}")
        _check_role(c, role, t, dims)
        sizes.append((role.name, int(t.numel() * t.element_size())))
    for r in c.rules:
        try:
            ok = bool(r.check(dims))
        except KeyError as e:
            raise LaunchContractError(c.op, "rules", Issue.RULE, f"{r.text}: {e} unbound") from None
        if not ok:
            raise LaunchContractError(c.op, "rules", Issue.RULE, f"{r.text}; dims {dims}")
    return Admitted(c.op, tuple(sorted(dims.items())), tuple(sizes))


# ---------------------------------------------------------------------------
# The contracts of the step's entry points
# ---------------------------------------------------------------------------
BF16, F32, I32, I64, U8 = ("bfloat16",), ("float32",), ("int32",), ("int64",), ("uint8",)


def _r(text: str, fn: Callable[[Mapping[str, int]], bool]) -> Rule:
    return Rule(text, fn)


def _gemm_out_cols(d) -> bool:
    return d["Dc"] == (d["N"] // 2 if d["epi"] == 2 else d["N"])


CONTRACTS: Dict[str, Contract] = {c.op: c for c in (
    Contract("linear", "gemm",
             (Role("A", BF16, ("M", "K")), Role("B", BF16, ("N", "K")), Role("D", BF16 + F32, ("M", "Dc"))),
             (_r("K % 8 == 0 (16-byte TMA rows)", lambda d: d["K"] % 8 == 0),
              _r("N % 32 == 0 (narrowest tile)", lambda d: d["N"] % 32 == 0),
              _r("SwiGLU needs N % 64 == 0 (32 gate + 32 up rows per group)", lambda d: d["epi"] != 2 or d["N"] % 64 == 0),
              _r("output columns: N, or N / 2 for SwiGLU", _gemm_out_cols)),
             params=("epi",)),
    Contract("linear_qkv_rope", "gemm_qkv_rope",
             (Role("A", BF16, ("M", "K")), Role("B", BF16, ("N", "K")), Role("D", BF16, ("M", "N")),
              Role("positions", I32, ("Tp",), rowmajor=False), Role("slots", I32, ("Ts",), rowmajor=False),
              Role("cos_sin", F32, ("*",), rowmajor=False),
              Role("kcache", BF16, ("pages", "Hkv", "page", 128), rowmajor=False),
              Role("vcache", BF16, ("pages", "Hkv", "page", 128), rowmajor=False)),
             (_r("N == (Hq + 2 Hkv) * 128", lambda d: d["N"] == (d["Hq"] + 2 * d["Hkv"]) * 128),
              _r("positions / slots cover every row", lambda d: d["Tp"] >= d["M"] and d["Ts"] >= d["M"]),
              _r("K % 8 == 0", lambda d: d["K"] % 8 == 0)),
             params=("Hq",)),
    Contract("rmsnorm", "rmsnorm",
             (Role("x", BF16, ("T", "H")), Role("residual", BF16, ("T", "H"), optional=True),
              Role("w", BF16, ("H",), rowmajor=False), Role("out", BF16, ("To", "H")),
              Role("rows", I32, ("R",), rowmajor=False, optional=True)),
             (_r("H % 8 == 0 (16-byte vectors)", lambda d: d["H"] % 8 == 0),
              _r("out holds every output row", lambda d: d["To"] >= d.get("R", d["T"])))),
    Contract("embed", "embed",
             (Role("ids", I32, ("T",), rowmajor=False), Role("table", BF16, ("V", "H")),
              Role("out", BF16, ("To", "H")), Role("fwd", I32, ("F",), rowmajor=False, optional=True),
              Role("prev", I32, ("Pv",), rowmajor=False, optional=True)),
             (_r("out holds every token", lambda d: d["To"] >= d["T"]), _r("H % 8 == 0", lambda d: d["H"] % 8 == 0),
              _r("forwarded rows inside the step", lambda d: d.get("first", 0) + d.get("F", 0) <= d["T"]))),
    Contract("rope_kv_write", "rope_kv_write",
             (Role("qkv", BF16, ("T", "Nq")), Role("positions", I32, ("Tp",), rowmajor=False),
              Role("slots", I32, ("Ts",), rowmajor=False), Role("cos_sin", F32, ("*",), rowmajor=False),
              Role("kcache", BF16, ("pages", "Hkv", "page", "D"), rowmajor=False),
              Role("vcache", BF16, ("pages", "Hkv", "page", "D"), rowmajor=False)),
             (_r("qkv width >= (Hq + 2 Hkv) * D", lambda d: d["Nq"] >= (d["Hq"] + 2 * d["Hkv"]) * d["D"]),
              _r("positions / slots cover every row", lambda d: d["Tp"] >= d["T"] and d["Ts"] >= d["T"])),
             params=("Hq",)),
    Contract("attn_prefill", "attn_prefill",
             (Role("q", BF16, ("Tq", "Nq")), Role("out", BF16, ("To", "No")),
              Role("q_start", I32, ("R1",), rowmajor=False), Role("seq_lens", I32, ("R",), rowmajor=False),
              Role("block_table", I32, ("Rb", "W"), rowmajor=False),
              Role("kcache", BF16, ("pages", "Hkv", 16, 128), rowmajor=False),
              Role("vcache", BF16, ("pages", "Hkv", 16, 128), rowmajor=False)),
             (_r("q_start has rows + 1 entries", lambda d: d["R1"] >= d["R"] + 1),
              _r("a block-table row per sequence", lambda d: d["Rb"] >= d["R"]),
              _r("GQA: Hq a multiple of Hkv", lambda d: d["Hq"] % d["Hkv"] == 0),
              _r("q holds Hq heads, out Hq heads", lambda d: d["Nq"] >= d["Hq"] * 128 and d["No"] >= d["Hq"] * 128)),
             params=("Hq",)),
    Contract("attn_decode", "attn_decode",
             (Role("q", BF16, ("Tq", "Nq")), Role("out", BF16, ("To", "No")),
              Role("tok_index", I32, ("R",), rowmajor=False), Role("seq_lens", I32, ("Rs",), rowmajor=False),
              Role("block_table", I32, ("Rb", "W"), rowmajor=False),
              Role("kcache", BF16, ("pages", "Hkv", 16, 128), rowmajor=False),
              Role("vcache", BF16, ("pages", "Hkv", 16, 128), rowmajor=False)),
             (_r("lengths and block-table rows per decode row", lambda d: d["Rs"] >= d["R"] and d["Rb"] >= d["R"]),
              _r("GQA group of at most 16 heads", lambda d: d["Hq"] % d["Hkv"] == 0 and d["Hq"] // d["Hkv"] <= 16),
              _r("q / out hold Hq heads", lambda d: d["Nq"] >= d["Hq"] * 128 and d["No"] >= d["Hq"] * 128)),
             params=("Hq",)),
    Contract("argmax", "argmax",
             (Role("logits", F32, ("R", "V")), Role("out", I32, ("Ro",), rowmajor=False)),
             (_r("a token per row", lambda d: d["Ro"] >= d["R"]),)),
    Contract("sample", "sample",
             (Role("logits", F32, ("R", "V")), Role("params", I32, ("Pn",), rowmajor=False),
              Role("out", I32, ("Ro",), rowmajor=False)),
             (_r("a token per row", lambda d: d["Ro"] >= d["R"]),
              _r("a 32-byte sampling record (8 int32) per row", lambda d: d["Pn"] >= 8 * d["R"]))),
    Contract("moe_grouped_linear", "gemm_grouped",
             (Role("A", BF16, ("M", "K")), Role("B", BF16, ("Eb", "N", "K")), Role("D", BF16, ("M", "Dc")),
              Role("groups", I32, ("G1",), rowmajor=False)),
             (_r("segments aligned to 128 or 256 rows", lambda d: d["align"] in (128, 256)),
              _r("M a multiple of the segment alignment", lambda d: d["M"] % d["align"] == 0),
              _r("K % 8 == 0 and N % 64 == 0", lambda d: d["K"] % 8 == 0 and d["N"] % 64 == 0),
              _r("a weight slab per group", lambda d: d["Eb"] >= d["num_groups"]),
              _r("groups has num_groups + 1 offsets", lambda d: d["G1"] >= d["num_groups"] + 1),
              _r("output columns: N, or N / 2 for SwiGLU", _gemm_out_cols)),
             params=("epi", "align", "num_groups")),
    Contract("linear_fp8", "gemm_fp8",
             (Role("A", ("float8_e4m3fn",), ("M", "K")), Role("sa", F32, ("Ms", "Kbs"), rowmajor=False),
              Role("B", ("float8_e4m3fn",), ("N", "K")), Role("sb", F32, ("Nb", "Kb"), rowmajor=False),
              Role("D", BF16 + F32, ("M", "Dc"))),
             (_r("K and N multiples of 128 (scale blocks)", lambda d: d["K"] % 128 == 0 and d["N"] % 128 == 0),
              _r("an activation scale per row and per 128 of K", lambda d: d["Ms"] >= d["M"] and d["Kbs"] >= d["K"] // 128),
              _r("a weight scale per 128 x 128 block", lambda d: d["Nb"] * d["Kb"] >= (d["N"] // 128) * (d["K"] // 128)),
              _r("output columns: N, or N / 2 for SwiGLU", _gemm_out_cols)),
             params=("epi",)),
    Contract("act_quant", "act_quant",
             (Role("x", BF16, ("T", "K")), Role("q", ("float8_e4m3fn",), ("Tq", "K")),
              Role("s", F32, ("Ts", "Kb"), rowmajor=False)),
             (_r("K % 128 == 0", lambda d: d["K"] % 128 == 0),
              _r("q and s hold every row", lambda d: d["Tq"] >= d["T"] and d["Ts"] >= d["T"]),
              _r("a scale per 128 of K", lambda d: d["Kb"] >= d["K"] // 128))),
    Contract("moe_route", "moe_route",
             (Role("h", BF16, ("T", "H")), Role("router", F32, ("E", "H")),
              Role("bias", F32, ("Eb",), rowmajor=False, optional=True),
              Role("ids", I32, ("Ti", "k"), rowmajor=False), Role("weights", F32, ("Tw", "kw"), rowmajor=False)),
             (_r("2, 4, 8 or 16 experts", lambda d: d["E"] in (2, 4, 8, 16)),
              _r("1 <= topk <= min(8, E)", lambda d: 1 <= d["topk"] <= min(8, d["E"])),
              _r("H % 256 == 0", lambda d: d["H"] % 256 == 0),
              _r("ids / weights: a row of topk per token",
                 lambda d: d["Ti"] >= d["T"] and d["Tw"] >= d["T"] and d["k"] >= d["topk"] and d["kw"] >= d["topk"])),
             params=("topk",)),
)}


# ---------------------------------------------------------------------------
# Paged admission: a packed step against the KV arena it indexes
# ---------------------------------------------------------------------------
class PagedIssue(enum.Enum):
    PAGE = "page index outside the KV arena"
    SEQ_LEN = "sequence length beyond the block-table width"
    SLOT = "KV write slot outside the arena or not in the row's pages"
    Q_START = "query offsets not monotone or not covering the prefill tokens"
    POSITION = "position not below its row's sequence length"
    TOKEN = "token id outside the vocabulary"
    SAMPLE = "sampled row index outside the step"


class PagedStepError(ValueError):
    def __init__(self, field: str, issue: PagedIssue, detail: str = ""):
        super().__init__(f"paged step: {field}: {issue.value}" + (f" ({detail})" if detail else ""))
        self.field, self.issue = field, issue


def check_paged_step(layout, buf, num_pages: int, page_size: int, vocab: Optional[int] = None) -> None:
    """Validates a packed step block (``step_inputs.build_host_step``) before it
    is uploaded: every page id, slot, position, length and offset it holds
    must stay inside the KV arena of ``num_pages`` pages of ``page_size``
    tokens and inside the step's own token range.  Padded decode rows (slot
    -1, the zero page, length 1) are admitted.  Raises ``PagedStepError``."""
    import numpy as np

    L = layout

    def f(name):
        o, n = L.field(name)
        return np.asarray(buf[o:o + n], dtype=np.int64)

    W, P = L.W, page_size
    cap = W * P
    toks, pos, slots = f("tokens"), f("positions"), f("slots")
    if vocab is not None and L.T and (toks.min() < 0 or toks.max() >= vocab):
        raise PagedStepError("tokens", PagedIssue.TOKEN, f"range [{toks.min()}, {toks.max()}] vocab {vocab}")
    for name in ("p_bt", "d_bt"):
        bt = f(name)
        if bt.size and (bt.min() < 0 or bt.max() >= num_pages):
            raise PagedStepError(name, PagedIssue.PAGE, f"range [{bt.min()}, {bt.max()}] of {num_pages}")
    ok = slots >= 0
    if ok.any() and slots[ok].max() >= num_pages * P:
        raise PagedStepError("slots", PagedIssue.SLOT, f"max {slots[ok].max()} of {num_pages * P}")
    Tp = 0
    if L.Rp:
        qs, sl = f("p_qstart"), f("p_seqlen")
        bt = f("p_bt").reshape(L.Rp, W)
        if qs[0] != 0 or (np.diff(qs) <= 0).any() or qs[-1] > L.T:
            raise PagedStepError("p_qstart", PagedIssue.Q_START, str(qs.tolist()[:8]))
        Tp = int(qs[-1])
        if (sl > cap).any() or (sl < np.diff(qs)).any():
            raise PagedStepError("p_seqlen", PagedIssue.SEQ_LEN, f"max {sl.max()} of {cap}")
        row = np.repeat(np.arange(L.Rp), np.diff(qs))
        p = pos[:Tp]
        if (p < 0).any() or (p >= sl[row]).any():
            raise PagedStepError("positions", PagedIssue.POSITION)
        want = bt[row, p // P] * P + p % P
        if (slots[:Tp] != want).any():
            raise PagedStepError("slots", PagedIssue.SLOT, "prefill slot not at its position's page")
    if L.Rd:
        tok, sl = f("d_tok"), f("d_seqlen")
        bt = f("d_bt").reshape(L.Rd, W)
        if (tok < Tp).any() or (tok >= L.T).any():
            raise PagedStepError("d_tok", PagedIssue.Q_START, "decode row outside the step's tokens")
        if (sl < 1).any() or (sl > cap).any():
            raise PagedStepError("d_seqlen", PagedIssue.SEQ_LEN, f"range [{sl.min()}, {sl.max()}] of {cap}")
        live = slots[tok] >= 0
        p = pos[tok]
        if (p[live] != sl[live] - 1).any():
            raise PagedStepError("positions", PagedIssue.POSITION, "decode position != length - 1")
        want = bt[np.arange(L.Rd), p // P] * P + p % P
        if (slots[tok][live] != want[live]).any():
            raise PagedStepError("slots", PagedIssue.SLOT, "decode slot not at its position's page")
    if L.Rs:
        si = f("s_idx")
        if (si < 0).any() or (si >= L.T).any():
            raise PagedStepError("s_idx", PagedIssue.SAMPLE)


# ---------------------------------------------------------------------------
# KernelOps method -> (contract, operand order, parameter names)
# ---------------------------------------------------------------------------
def launch_checks():
    """Argument adapters: each maps a ``KernelOps`` call's arguments to
    (contract, operands, params) for ``admit``."""
    C = CONTRACTS
    return {
        "gemm": lambda A, B, out, epi=0, ws=None: (C["linear"], (A, B, out), {"epi": epi}),
        "qkv_rope": lambda A, B, qkv, positions, slots, cos_sin, kc, vc, Hq, Hkv, page:
            (C["linear_qkv_rope"], (A, B, qkv, positions, slots, cos_sin, kc, vc), {"Hq": Hq, "Hkv": Hkv, "page": page}),
        "rmsnorm": lambda x, residual, w, out, eps, rows=None: (C["rmsnorm"], (x, residual, w, out, rows), {}),
        "embed": lambda ids, table, out, fwd=None:
            (C["embed"], (ids, table, out) + ((None, None) if fwd is None else (fwd[0], fwd[2])),
             {} if fwd is None else {"first": fwd[1]}),
        "rope_kv_write": lambda qkv, positions, slots, cos_sin, kc, vc, Hq, Hkv, page:
            (C["rope_kv_write"], (qkv, positions, slots, cos_sin, kc, vc), {"Hq": Hq, "Hkv": Hkv, "page": page}),
        "attn_prefill": lambda q, out, q_start, seq_lens, bt, kc, vc, Hq, Hkv, max_q_len, host=None:
            (C["attn_prefill"], (q, out, q_start, seq_lens, bt, kc, vc), {"Hq": Hq, "Hkv": Hkv}),
        "attn_decode": lambda q, out, tok, seq_lens, bt, kc, vc, Hq, Hkv, splits, part_o, part_lse, host=None:
            (C["attn_decode"], (q, out, tok, seq_lens, bt, kc, vc), {"Hq": Hq, "Hkv": Hkv}),
        "argmax": lambda logits, out: (C["argmax"], (logits, out), {}),
        "sample": lambda logits, params, out: (C["sample"], (logits, params, out), {}),
        "gemm_grouped": lambda A, B, out, groups, num_groups, epi, align=128:
            (C["moe_grouped_linear"], (A, B, out, groups), {"epi": epi, "align": align, "num_groups": num_groups}),
        "gemm_fp8": lambda q, s, w8, sw, out, epi, ws=None: (C["linear_fp8"], (q, s, w8, sw, out), {"epi": epi}),
        "act_quant": lambda x, q, s: (C["act_quant"], (x, q, s), {}),
        "moe_route": lambda h, router, bias, topk, ids, weights:
            (C["moe_route"], (h, router, bias, ids, weights), {"topk": topk}),
    }


def install(ops) -> None:
    """Wraps the checked methods of an operator set so each call is admitted
    against its contract before it launches (``LUNAFLUX_CHECK_LAUNCHES=1``)."""
    import functools

    ops.admitted = 0
    for name, adapt in launch_checks().items():
        fn = getattr(ops, name, None)
        if fn is None:
            continue

        def wrapped(*a, _fn=fn, _adapt=adapt, **k):
            c, operands, params = _adapt(*a, **k)
            admit(c, operands, params)
            ops.admitted += 1
            return _fn(*a, **k)

        setattr(ops, name, functools.wraps(fn)(wrapped))
