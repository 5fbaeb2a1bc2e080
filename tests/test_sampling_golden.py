"""Host sampler against the reference's golden vectors (sampling/
stochastic_test.mbt: "golden seeded selections and replay state are
stable", "golden distribution applies top-k before top-p and orders ties",
"top-p threshold keeps the smallest exact equal-mass nucleus",
"max-shifted softmax handles extreme finite logits and temperature",
"identical seeds reproduce a multi-step stream"; greedy_test.mbt:
"greedy selects boundaries, negatives, and lowest tied token")."""
import math

import pytest

from lunaflux_b200.sampling.host import (SamplingError, XorShift64, counter_unit, greedy, prepare_distribution,
                                         stochastic_sample)


def probs(w, mass):
    return [x / mass for x in w]


def test_golden_seeded_selections_and_rng_state():
    low = XorShift64(1)
    assert stochastic_sample([0.0, 0.0, 0.0], 1.0, None, None, low.next_unit()) == 0
    assert low.state == 1082269761
    high = XorShift64(0x6C576FAC43FD007C)
    assert stochastic_sample([0.0, 0.0, 0.0], 1.0, None, None, high.next_unit()) == 2
    assert high.state == 0xC4992A768ECD657C


def test_top_k_applies_before_top_p_and_ties_order_by_id():
    ids, w, mass = prepare_distribution([math.log(4.0), math.log(2.0), 0.0, -20.0], 1.0, 3, 0.8)
    assert list(ids) == [0, 1]
    p = probs(w, mass)
    assert abs(p[0] - 2 / 3) <= 1e-14 and abs(p[1] - 1 / 3) <= 1e-14
    ids, w, mass = prepare_distribution([4.0, 4.0, 4.0], 1.0, 2, None)
    assert list(ids) == [0, 1] and probs(w, mass) == [0.5, 0.5]


def test_top_p_keeps_the_smallest_equal_mass_nucleus():
    ids, w, mass = prepare_distribution([0.0] * 4, 1.0, None, 0.5)
    assert len(ids) == 2 and probs(w, mass) == [0.5, 0.5]
    ids, w, mass = prepare_distribution([0.0] * 4, 1.0, None, 0.5000000000000001)
    assert len(ids) == 3 and all(abs(x - 1 / 3) <= 1e-15 for x in probs(w, mass))
    ids, w, mass = prepare_distribution([0.0] * 4, 1.0, None, 0.25)
    assert list(ids) == [0] and probs(w, mass) == [1.0]


def test_extreme_finite_logits_and_temperatures():
    big = 1.7976931348623157e308
    ids, w, mass = prepare_distribution([big, -big], 1.0, None, None)
    assert list(ids) == [0, 1] and probs(w, mass) == [1.0, 0.0]
    ids, w, mass = prepare_distribution([1.0, 0.0], 1e-3, None, None)
    assert probs(w, mass)[0] == 1.0
    ids, w, mass = prepare_distribution([1.0, 0.0], 100.0, None, None)
    assert abs(probs(w, mass)[0] - 1 / (1 + math.exp(-0.01))) < 1e-14


@pytest.mark.parametrize("bad", [[], [float("nan")], [0.0, float("inf")], [float("-inf"), 0.0]])
def test_invalid_inputs_are_refused(bad):
    with pytest.raises(SamplingError):
        prepare_distribution(bad, 1.0, None, None)


def test_streams_replay_and_positions_are_distinct():
    a, b = XorShift64(0x123456789ABCDEF0), XorShift64(0x123456789ABCDEF0)
    xs = [a.next_unit() for _ in range(64)]
    assert xs == [b.next_unit() for _ in range(64)] and a.state == b.state
    picks = [stochastic_sample([2.0, 1.5, 1.0, -3.0], 0.75, 3, 0.95, u) for u in xs]
    assert set(picks) <= {0, 1, 2}
    # counter-addressed draws: a function of (seed, index) only, distinct per index
    us = [counter_unit(0x123456789ABCDEF0, i) for i in range(64)]
    assert us == [counter_unit(0x123456789ABCDEF0, i) for i in range(64)]
    assert len(set(us)) == 64 and all(0.0 <= u < 1.0 for u in us)


def test_greedy_boundaries_negatives_and_lowest_tie():
    assert greedy([5.0, 1.0, 2.0]) == 0
    assert greedy([1.0, 2.0, 5.0]) == 2
    assert greedy([-3.0, -1.0, -2.0]) == 1
    assert greedy([7.0, 9.0, 9.0, 1.0]) == 1
