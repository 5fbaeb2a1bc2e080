"""Greedy and stochastic sampling.

Host restatement (fp64, exact reference semantics) used by the CPU path and as
the replay oracle; the device path is the ``sample`` / ``argmax`` kernels.

Reference: sampling/greedy.mbt (max finite logit, lowest id on ties),
sampling/stochastic.mbt (sort by logit desc / id asc, top-k, max-shifted
temperature softmax, smallest nucleus with cumulative >= top_p * total,
renormalise, first index whose inclusive cumulative exceeds u * mass),
sampling/rng.mbt (xorshift64 stream and the counter-addressed draw).
"""
from .host import (  # noqa: F401
    SamplingError, counter_state, counter_unit, XorShift64, greedy, prepare_distribution, stochastic_sample,
    pack_params, PARAM_DTYPE,
)
