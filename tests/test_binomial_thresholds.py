"""The binomial inversion by integer thresholds (no GPU).

The reference draws Binomial(n, p) by inversion (executor.rs:224-268): with
u = m * 2^-53 from the counter stream, it returns the first x for which the
running remainder u - P(0) - ... - P(x-1), rounded after every subtraction,
is <= P(x); past the bound it restarts with the next draw.  The plan
compiler replaces the walk by per-x thresholds on m (the generated
`b2_bthr_*` tables, compared by `b2_binomial_thr`): the result is the number
of thresholds below m, and all K of them below m is a restart.  Here the
sequential walk, in IEEE doubles, decides every draw again for the tables of
the fixture models, on random m and on every threshold and its neighbours.
"""
from __future__ import annotations

import math
import re

import numpy as np
import pytest

from conftest import MODELS

TABLE = re.compile(r"// inversion thresholds of binomial\(n = (\d+), p = \(?([^)\s]+)\)?\)\n"
                   r"__constant__ u64 (b2_bthr_\d+)\[(\d+)\] = \{([^}]*)\};")


def probabilities(n, p, k):
    """P(X = x), x < k, with the products, division and order of the
    inversion loop (executor.rs:224-268)."""
    reverse = p > 0.5
    prob = 1.0 - p if reverse else p
    q = 1.0 - prob
    tab = [math.exp(float(n) * math.log(q))]
    for x in range(1, k):
        tab.append((float(n - x + 1) * prob * tab[x - 1]) / (float(x) * q))
    return tab


def walk(m, tab):
    """The loop itself on one draw: x, or None for a restart."""
    u = float(m) * 2.0 ** -53
    for x, px in enumerate(tab):
        if u <= px:
            return x
        u -= px
    return None


def tables(src):
    out = []
    for n, p, name, k, body in TABLE.findall(src):
        thr = [int(v.rstrip("ul")) for v in body.split(",")]
        assert len(thr) == int(k)
        out.append((int(n), float.fromhex(p), thr))
    return out


@pytest.mark.parametrize("name", ["cuba_poisson_small", "brunel_small"])
def test_thresholds_decide_every_draw_like_the_walk(pkg, name):
    src = pkg.codegen((MODELS / f"{name}.json").read_bytes())
    found = tables(src)
    assert found, "the model draws no table-driven binomial"
    rng = np.random.default_rng(7)
    for n, p, thr in found:
        k = len(thr)
        tab = probabilities(n, p, k)
        assert all(a <= b for a, b in zip(thr, thr[1:]))
        draws = set(int(v) for v in rng.integers(0, 2 ** 53, size=20000, dtype=np.uint64))
        for t in thr:
            draws.update(v for v in (t - 1, t, t + 1) if 0 <= v < 2 ** 53)
        draws.update((0, 1, 2 ** 53 - 2, 2 ** 53 - 1))
        for m in sorted(draws):
            x = sum(1 for t in thr if m > t)
            assert walk(m, tab) == (x if x < k else None), (n, p, m)


def test_threshold_counts_follow_the_distribution(pkg):
    """Sanity of the tables themselves: the draw fractions below each
    threshold are the binomial CDF (to the 2^-53 resolution of a draw)."""
    src = pkg.codegen((MODELS / "brunel_small.json").read_bytes())
    for n, p, thr in tables(src):
        cdf = 0.0
        for x, t in enumerate(thr[:-1]):
            cdf += math.comb(n, x) * p ** x * (1 - p) ** (n - x)
            assert abs((t + 1) * 2.0 ** -53 - cdf) < 1e-9
