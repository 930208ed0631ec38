"""GPU parity of cells larger than one CTA (split into a top part and
subtrees over a cooperative launch) against the CPU oracle."""
import numpy as np
import pytest

from heliox_b200 import synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu

V_TOL = 1e-9
G_TOL = 1e-7
KINDS = ("hh.gnabar", "hh.gkbar", "hh.gl", "hh.el", "pas.g", "pas.e", "cm", "IClamp.amp")


@pytest.fixture(scope="module")
def Sim():
    from heliox_b200.runtime import Sim as S

    return S


def _probes(g, k=40):
    return np.unique(np.linspace(0, g.nnode - 1, k).astype(np.int32))


def _check(s, g, T, tape_budget=0):
    p = _probes(g)
    c = np.random.default_rng(2).standard_normal((T + 1, p.shape[0]))
    tr = s.forward_capture(T, probes=p)
    gg = s.backward(c, keys=KINDS)
    ref, gr = O.adjoint(g, T, c, probe=p)
    assert np.max(np.abs(tr - ref)) / np.max(np.abs(ref)) <= V_TOL
    for k in KINDS:
        scale = np.max(np.abs(gr[k]))
        if scale > 0:
            assert np.max(np.abs(gg[k] - gr[k])) / scale <= G_TOL, k


def test_split_cell_forward_and_adjoint(Sim):
    g = synth.random_tree_cell(7, ncomp=6000, max_levels=40, amp=0.8)
    s = Sim(0)
    s.load_group(g)
    assert s.plan_stats()["nsub"] > 0
    _check(s, g, 600)


def test_split_cell_checkpointed(Sim):
    g = synth.random_tree_cell(8, ncomp=5000, max_levels=40, amp=0.8)
    s = Sim(0, tape_budget_bytes=16 << 20)
    s.load_group(g)
    assert s.plan_stats()["nsub"] > 0
    _check(s, g, 500)


def test_giant_cell_forward(Sim):
    g = synth.giant_cell()
    s = Sim(0)
    s.load_group(g)
    st = s.plan_stats()
    assert st["nsub"] > 0
    p = _probes(g, 64)
    tr = s.simulate(300, probes=p)
    ref, _ = O.forward(g, 300, probe=p)
    assert np.max(np.abs(tr - ref)) / np.max(np.abs(ref)) <= V_TOL


def test_split_barrier_wait_gives_up_and_context_recovers(Sim):
    """A grid-barrier wait of the split kernels bounded to one ~100 ns sleep
    runs out (148 CTAs never arrive within it at every barrier of 200 steps):
    the wait sets the error flag, the remaining barriers return at once, the
    launch finishes and the forward reports the timeout.  With the default
    bound restored the same context runs the same forward to the oracle's
    trace."""
    from heliox_b200.runtime import HxError

    g = synth.random_tree_cell(7, ncomp=6000, max_levels=40, amp=0.8)
    p = _probes(g)
    s = Sim(0)
    s.load_group(g)
    assert s.plan_stats()["nsub"] > 0
    s.set_split_barrier_limit(1)
    with pytest.raises(HxError, match="timed out"):
        s.simulate(200, probes=p)
    s.set_split_barrier_limit(0)
    tr = s.simulate(200, probes=p)
    ref, _ = O.forward(g, 200, probe=p)
    assert np.max(np.abs(tr - ref)) / np.max(np.abs(ref)) <= V_TOL
    s.close()
