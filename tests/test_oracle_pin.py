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
GOLDEN = sorted(p for p in glob.glob(os.path.join(HERE, "golden", "*.npz"))
                if not p.endswith("adam.npz") and not p.endswith("_perm3.npz"))
PERM3 = sorted(glob.glob(os.path.join(HERE, "golden", "*_perm3.npz")))

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
    tr, st = O.forward(g, int(d["nstep"]), probe=d["probes"])
    assert tr.shape == d["trace"].shape
    assert np.array_equal(tr, d["trace"]), np.max(np.abs(tr - d["trace"]))
    if g.has_network:
        # spk.dat holds times with 8 significant digits, sorted by (time, gid)
        mine = sorted(st["spikes"])
        ref = [tuple(r) for r in d["spikes"]]
        assert [gid for _, gid in mine] == [int(gid) for _, gid in ref]
        assert np.allclose([t for t, _ in mine], [t for t, _ in ref], rtol=1e-7, atol=1e-9)


def test_golden_fixtures_present():
    names = {os.path.basename(p)[:-4] for p in GOLDEN}
    assert set(_mg.CASES) <= names
    assert {f"{c}_perm3" for c in _mg.PERM3} <= {os.path.basename(p)[:-4] for p in PERM3}


@pytest.mark.parametrize("path", PERM3, ids=[os.path.basename(p)[:-4] for p in PERM3])
def test_oracle_vs_reference_permute3_golden(path):
    """The reference run with its default node permutation (type 3: branches
    split over threads, cpu_solve_permute3) eliminates in another order than
    solve_serial, so it agrees with the serial-order oracle to rounding only:
    within 1e-9 of the trace scale (measured: 0 to 8e-11), spikes identical."""
    name = os.path.basename(path)[: -len("_perm3.npz")]
    make, nstep, _ = _mg.CASES[name]
    d = np.load(path)
    assert int(d["permute_type"]) == 3
    g = make()
    tr, st = O.forward(g, int(d["nstep"]), probe=d["probes"])
    rel = np.max(np.abs(tr - d["trace"])) / np.max(np.abs(d["trace"]))
    assert rel <= 1e-9, rel
    if g.has_network:
        mine = sorted(st["spikes"])
        ref = [tuple(r) for r in d["spikes"]]
        assert [gid for _, gid in mine] == [int(gid) for _, gid in ref]
        assert np.allclose([t for t, _ in mine], [t for t, _ in ref], rtol=1e-7, atol=1e-9)


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


@needs_ref
@pytest.mark.parametrize("seed", [21, 22])
def test_oracle_network_bit_exact_vs_reference_live(seed):
    """Event network (ExpSyn, Exp2Syn, NetStims with noise 1) against the
    reference's CPU mode, whose NetStim stream starts from a zeroed state."""
    g = synth.spiking_network(ncell=6, seed=seed, nstim=5, weight=(0.02, 0.08), stim_noise=1.0, stim_interval=4.0)
    p = np.arange(g.nnode, dtype=np.int32)[::11]
    ref, rs = O.ref_forward(g, 2000, probe=p)
    ora, st = O.forward(g, 2000, probe=p)
    assert np.array_equal(ref, ora)
    assert [gid for _, gid in sorted(st["spikes"])] == [gid for _, gid in rs]


@needs_ref
def test_oracle_coupled_bit_exact_vs_reference_live():
    g = synth.coupled_network(ncell=5, seed=31, ngap=5, ngapj=4, ngraded=12)
    p = np.arange(g.nnode, dtype=np.int32)[::9]
    ref, _ = O.ref_forward(g, 2000, probe=p)
    ora, _ = O.forward(g, 2000, probe=p)
    assert np.array_equal(ref, ora)


@needs_ref
def test_network_adjoint_vs_fd_of_reference_forward():
    """Weight / conductance gradients of the oracle adjoint against 4th-order FD of
    the reference forward (event schedule unchanged by the small steps)."""
    T = 800
    rng = np.random.default_rng(5)
    cases = (
        (synth.spiking_network(ncell=4, seed=3, nstim=2, weight=(0.02, 0.06)),
         (("exp2syn", "weight", "Exp2Syn.weight"), ("expsyn", "weight", "ExpSyn.weight"))),
        (synth.coupled_network(ncell=4, seed=8, ngap=3, ngapj=2, ngraded=5, ngapnp=2),
         (("halfgap", "g", "HalfGap.g"), ("gapjunction", "w", "gapjunction_lr.w"),
          ("graded", "w", "neuron_to_neuron_syn_lr.w"), ("gapnoptr", "weight", "gapjunction_noptr.weight"))),
    )
    for g, checks in cases:
        p = g.soma_nodes()
        c = rng.standard_normal((T + 1, p.shape[0]))
        _, gr = O.adjoint(g, T, c, probe=p)

        def L(gg):
            return float(np.sum(c * O.ref_forward(gg, T, probe=p)[0]))

        for tab, field, key in checks:
            t = getattr(g, tab)
            j = int(np.argmax(np.abs(gr[key])))
            x0 = t.fields[field][j]
            h = 1e-3 * abs(x0)
            vals = []
            for dx in (2 * h, h, -h, -2 * h):
                gg = g.copy()
                getattr(gg, tab).fields[field][j] = x0 + dx
                vals.append(L(gg))
            fd = (-vals[0] + 8 * vals[1] - 8 * vals[2] + vals[3]) / (12 * h)
            assert abs(gr[key][j] - fd) <= 1e-6 * abs(fd), (key, gr[key][j], fd)


@needs_ref
@pytest.mark.parametrize("case", ["trees3", "tree_deep", "net_spiking"])
def test_oracle_vs_reference_permute1_live(case):
    """The reference with permute type 1 (cpu_solve_permute1,
    simulate.cpp:583-629: the node order of permute_order.cpp's type-1 split)
    eliminates in another order than solve_serial: it agrees with the
    serial-order oracle to rounding (measured 1e-13 .. 3e-13 of the trace
    scale), spikes identical."""
    make, nstep, _ = _mg.CASES[case]
    g = make()
    p = g.soma_nodes()
    ref, rs = O.ref_forward(g, nstep, probe=p, permute_type=1)
    ora, st = O.forward(g, nstep, probe=p)
    assert np.max(np.abs(ref - ora)) / np.max(np.abs(ora)) <= 1e-9
    if g.has_network:
        assert [gid for _, gid in sorted(st["spikes"])] == [int(gid) for _, gid in rs]


@needs_ref
@pytest.mark.parametrize("permute_type", [1, 3])
def test_oracle_library_cells_vs_reference_permuted_live(permute_type):
    """Library cells under the reference's permuted node orders: rounding-level
    agreement with the serial-order oracle (measured 1e-11 of the trace scale
    over 1200 steps of spiking library cells)."""
    g = synth.lib_tree_batch(2, seed0=700, nmax=200)
    p = g.soma_nodes()
    ref, _ = O.ref_forward(g, 1200, probe=p, permute_type=permute_type)
    ora, _ = O.forward(g, 1200, probe=p)
    assert np.max(np.abs(ref - ora)) / np.max(np.abs(ora)) <= 1e-9


@needs_ref
@pytest.mark.parametrize("kind", ["event", "coupled"])
def test_oracle_library_networks_bit_exact_vs_reference_live(kind):
    """Library cells in an event network and in a coupled network (HalfGap,
    gapjunction_lr / _noptr, graded synapses): the network currents before
    the library ones on a node, as the reference's mechanism list orders them."""
    if kind == "event":
        g = synth.lib_network("event", ncell=5, seed=43, nstim=3, weight=(0.02, 0.08), stim_noise=1.0,
                              stim_interval=5.0)
    else:
        g = synth.lib_network("coupled", ncell=5, seed=44, ngap=4, ngapj=3, ngraded=8, ngapnp=3)
    p = np.arange(g.nnode, dtype=np.int32)[::7]
    ref, _ = O.ref_forward(g, 1600, probe=p)
    ora, _ = O.forward(g, 1600, probe=p)
    assert np.array_equal(ref, ora)


@needs_ref
@pytest.mark.parametrize("seed,cadyn", [(1, "CaDynamics_E2"), (2, "CaDynamics_E2"), (3, "cainternm_lr")])
def test_oracle_library_cells_bit_exact_vs_reference_live(seed, cadyn):
    """The library channel set, ions and calcium dynamics (CaDynamics_E2 or
    cainternm_lr; library cells and a teacher with perturbed channel
    densities) against the reference."""
    g = synth.lib_tree_batch(2, seed0=3000 + seed, nmax=180, cadyn=cadyn)
    teacher = synth.perturb_lib(g, 0.3, seed=seed)
    for grp in (g, teacher):
        probe = np.array(list(grp.soma_nodes()) + [grp.nnode - 1], dtype=np.int32)
        tr, _ = O.forward(grp, 1600, probe=probe)
        ref, _ = O.ref_forward(grp, 1600, probe=probe)
        assert np.array_equal(tr, ref), np.max(np.abs(tr - ref))
