"""CPU: the oracle pinned to the reference itself.

Golden fixtures (tests/golden/*.npz, made by tests/golden/make_golden.py) hold
voltage traces produced by the reference's own CPU integrator
(oracle/_ref/hxref_run: src/simulate.cpp + mechanisms + CoreNEURON loader,
compiled from the reference sources).  The oracle must reproduce them bit for
bit.  Where the harness is built (a checkout with the reference sources), more
seeded cases are compared live, and the oracle's adjoint is checked against
finite differences of the reference's own forward.
"""
import glob
import os

import numpy as np
import pytest

from heliox_b200 import synth
from oracle import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = sorted(p for p in glob.glob(os.path.join(HERE, "golden", "*.npz")) if not p.endswith("adam.npz"))

import importlib.util

_spec = importlib.util.spec_from_file_location("make_golden", os.path.join(HERE, "golden", "make_golden.py"))
_mg = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(_mg)


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[:-4] for p in GOLDEN])
def test_oracle_bit_exact_vs_reference_golden(path):
    name = os.path.basename(path)[:-4]
    make, nstep, _ = _mg.CASES[name]
    d = np.load(path)
    g = make()
    tr, _ = O.forward(g, int(d["nstep"]), probe=d["probes"])
    assert tr.shape == d["trace"].shape
    assert np.array_equal(tr, d["trace"]), np.max(np.abs(tr - d["trace"]))


def test_golden_fixtures_present():
    names = {os.path.basename(p)[:-4] for p in GOLDEN}
    assert set(_mg.CASES) <= names


needs_ref = pytest.mark.skipif(not O.ref_available(), reason="reference harness not built (oracle/ref_build.sh)")


@needs_ref
@pytest.mark.parametrize("seed", [1, 2, 3])
def test_oracle_bit_exact_vs_reference_live(seed):
    g = synth.random_tree_batch(2, seed0=1000 * seed)
    teacher = synth.perturb_conductances(g, 0.2, seed=seed)
    for grp in (g, teacher):
        p = np.concatenate([grp.soma_nodes(), np.arange(grp.ncell, grp.nnode, 97)]).astype(np.int32)
        ref, _ = O.ref_forward(grp, 1500, probe=p)
        ora, _ = O.forward(grp, 1500, probe=p)
        assert np.array_equal(ref, ora)


@needs_ref
def test_adjoint_vs_fd_of_reference_forward():
    """dL/dtheta of the oracle adjoint against 4th-order FD of the reference forward."""
    g = synth.ball_and_stick()
    T = 1000
    rng = np.random.default_rng(7)
    c = rng.standard_normal((T + 1, 1))
    _, gr = O.adjoint(g, T, c)

    def L(tab, field, j, x):
        gg = g.copy()
        getattr(gg, tab).fields[field][j] = x
        return float(np.sum(c * O.ref_forward(gg, T)[0]))

    for key, tab, field, j in (("hh.gnabar", "hh", "gnabar", 0), ("hh.gl", "hh", "gl", 0), ("pas.g", "pas", "g", 3)):
        x0 = getattr(g, tab).fields[field][j]
        h = 1e-3 * abs(x0)
        fd = (-L(tab, field, j, x0 + 2 * h) + 8 * L(tab, field, j, x0 + h) - 8 * L(tab, field, j, x0 - h)
              + L(tab, field, j, x0 - 2 * h)) / (12 * h)
        assert abs(gr[key][j] - fd) <= 2e-6 * abs(fd), (key, gr[key][j], fd)


def test_adam_port_bit_exact_vs_reference_golden():
    d = np.load(os.path.join(HERE, "golden", "adam.npz"))
    a = _mg.ADAM
    ws, m, v = O.adam_port(d["w0"], d["grads"], a["lr"], a["inv_record_steps"], a["beta1"], a["beta2"], a["eps"],
                           a["impedance"])
    assert np.array_equal(ws, d["weights"])
    assert np.array_equal(m, d["m"]) and np.array_equal(v, d["v"])
