"""CPU: the oracle's discrete adjoint against finite differences of its forward.

The reference has no exact gradient (src/runtime_api/learn/LearnRuntime.cpp:208-210),
so the adjoint restatement is checked against 4th-order central differences of
the forward it differentiates.  Tolerance: 2e-6 relative (the FD noise floor of
a 4000-step spiking trace; the adjoint itself is exact to rounding).
"""
import numpy as np
import pytest

from heliox_b200 import synth
from oracle import oracle as O

T = 1200


def _loss(g, c):
    return float(np.sum(c * O.forward(g, T)[0]))


def _fd4(g, c, tab, field, j, rel=1e-3):
    def with_val(x):
        gg = g.copy()
        if tab == "cm":
            gg.cm[j] = x
        else:
            getattr(gg, tab).fields[field][j] = x
        return _loss(gg, c)

    base = g.cm[j] if tab == "cm" else getattr(g, tab).fields[field][j]
    h = rel * max(abs(base), 1e-2)
    return (-with_val(base + 2 * h) + 8 * with_val(base + h) - 8 * with_val(base - h) + with_val(base - 2 * h)) / (12 * h)


@pytest.fixture(scope="module")
def case():
    g = synth.ball_and_stick()
    rng = np.random.default_rng(3)
    c = rng.standard_normal((T + 1, 1))
    tr, gr = O.adjoint(g, T, c)
    return g, c, tr, gr


@pytest.mark.parametrize(
    "key,tab,field,j",
    [
        ("hh.gnabar", "hh", "gnabar", 0),
        ("hh.gkbar", "hh", "gkbar", 0),
        ("hh.gl", "hh", "gl", 0),
        ("hh.el", "hh", "el", 0),
        ("pas.g", "pas", "g", 0),
        ("pas.e", "pas", "e", 10),
        ("IClamp.amp", "iclamp", "amp", 0),
        ("cm", "cm", None, 0),
        ("cm", "cm", None, 40),
    ],
)
def test_adjoint_matches_fd(case, key, tab, field, j):
    g, c, tr, gr = case
    fd = _fd4(g, c, tab, field, j)
    ad = gr[key][j]
    assert abs(ad - fd) <= 2e-6 * abs(fd) + 1e-12, (key, ad, fd)


def test_adjoint_trace_equals_forward(case):
    g, c, tr, gr = case
    tr2, _ = O.forward(g, T)
    assert np.array_equal(tr, tr2)


def test_directional_derivative_random_tree():
    """All parameters at once: g . u against the FD of L along u."""
    g = synth.random_tree_cell(5, ncomp=120)
    n = 600
    rng = np.random.default_rng(1)
    c = rng.standard_normal((n + 1, 1))
    _, gr = O.adjoint(g, n, c)
    u = {k: rng.standard_normal(g.hh.n) for k in ("gnabar", "gkbar", "gl")}
    up = rng.standard_normal(g.pas.n)

    def L(s):
        gg = g.copy()
        for k in u:
            gg.hh.fields[k] = g.hh.fields[k] * (1 + s * u[k])
        gg.pas.fields["g"] = g.pas.fields["g"] * (1 + s * up)
        return float(np.sum(c * O.forward(gg, n)[0]))

    h = 1e-4
    fd = (-L(2 * h) + 8 * L(h) - 8 * L(-h) + L(-2 * h)) / (12 * h)
    ad = sum(np.dot(gr["hh." + k], g.hh.fields[k] * u[k]) for k in u) + np.dot(gr["pas.g"], g.pas.fields["g"] * up)
    assert abs(ad - fd) <= 1e-6 * abs(fd), (ad, fd)
