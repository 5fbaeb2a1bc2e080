"""Host (fp64) samplers and the per-row parameter records for the device sampler."""
from __future__ import annotations

import math
from typing import Optional, Sequence, Tuple

import numpy as np

M64 = (1 << 64) - 1
GOLDEN = 0x9E3779B97F4A7C15


class SamplingError(ValueError):
    pass


def counter_state(seed: int, sample_index: int) -> int:
    """splitmix-style counter-addressed state (sampling/rng.mbt counter_state)."""
    v = (seed + (sample_index + 1) * GOLDEN) & M64
    v = ((v ^ (v >> 30)) * 0xBF58476D1CE4E5B9) & M64
    v = ((v ^ (v >> 27)) * 0x94D049BB133111EB) & M64
    v ^= v >> 31
    return v if v != 0 else GOLDEN


def counter_unit(seed: int, sample_index: int) -> float:
    """Uniform in [0, 1) from the top 53 bits of the counter state."""
    return float(counter_state(seed, sample_index) >> 11) * 1.1102230246251565e-16


class XorShift64:
    """Sequential stream (sampling/rng.mbt SamplingRng)."""

    def __init__(self, seed: int):
        if not (0 < seed <= M64):
            raise SamplingError("seed must be non-zero")
        self.state = seed

    def next_unit(self) -> float:
        v = self.state
        v ^= (v << 13) & M64
        v ^= v >> 7
        v ^= (v << 17) & M64
        self.state = v
        return float(v >> 11) * 1.1102230246251565e-16


def greedy(logits: Sequence[float]) -> int:
    a = np.asarray(logits, dtype=np.float64)
    if a.size == 0:
        raise SamplingError("empty input")
    if not np.isfinite(a).all():
        raise SamplingError("non-finite logit")
    return int(np.argmax(a))  # numpy returns the first (lowest) index on ties


def prepare_distribution(logits, temperature: float, top_k: Optional[int], top_p: Optional[float],
                         ids=None) -> Tuple[np.ndarray, np.ndarray, float]:
    """Returns (token ids in sorted order, weights, retained mass) of the
    nucleus.  ``ids`` gives the token id of each logit (default: its
    position), for a distribution given as a subset of the vocabulary."""
    a = np.asarray(logits, dtype=np.float64)
    tok = np.arange(a.size) if ids is None else np.asarray(ids, dtype=np.int64)
    if a.size == 0:
        raise SamplingError("empty input")
    if not (math.isfinite(temperature) and temperature > 0):
        raise SamplingError("invalid temperature")
    if top_k is not None and top_k <= 0:
        raise SamplingError("invalid top_k")
    if top_p is not None and not (0.0 < top_p <= 1.0):
        raise SamplingError("invalid top_p")
    if not np.isfinite(a).all():
        raise SamplingError("non-finite logit")
    order = np.lexsort((tok, -a))  # logit desc, then id asc
    k = a.size if top_k is None else min(top_k, a.size)
    order = order[:k]
    mx = a[order[0]]
    with np.errstate(over="ignore"):       # the spread of extreme finite logits may overflow to -inf: weight 0
        w = np.exp((a[order] - mx) / temperature)
    total = float(np.sum(w)) if k < 64 else math.fsum(w)
    if not (total > 0 and math.isfinite(total)):
        raise SamplingError("invalid distribution")
    if top_p is not None:
        thr = top_p * total
        # smallest prefix with cumulative >= thr (sequential accumulation)
        cum = 0.0
        cnt = 0
        while cnt < k and cum < thr:
            cum += w[cnt]
            cnt += 1
        cnt = max(cnt, 1)
    else:
        cnt = k
    ret = 0.0
    for x in w[:cnt]:
        ret += x
    return tok[order[:cnt]], w[:cnt], ret


def stochastic_sample(logits, temperature: float, top_k: Optional[int], top_p: Optional[float], u: float,
                      ids=None) -> int:
    ids, w, mass = prepare_distribution(logits, temperature, top_k, top_p, ids)
    target = u * mass
    cum = 0.0
    for i in range(len(ids)):
        cum += w[i]
        if cum > target:
            return int(ids[i])
    return int(ids[-1])


# Device record (csrc/kernels/elementwise.h SampleParams), 32 bytes per row.
PARAM_DTYPE = np.dtype([("mode", "<i4"), ("top_k", "<i4"), ("temperature", "<f4"), ("top_p", "<f4"),
                        ("seed", "<u8"), ("sample_index", "<i8")])


def pack_params(rows) -> np.ndarray:
    """rows: iterable of (mode, top_k, temperature, top_p, seed, sample_index)."""
    rows = list(rows)
    a = np.zeros(len(rows), dtype=PARAM_DTYPE)
    for i, r in enumerate(rows):
        a[i] = r
    return a
