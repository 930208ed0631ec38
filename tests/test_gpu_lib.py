"""GPU parity of the library mechanisms (ions, CaDynamics_E2 and the
user-mech channel set) against the CPU oracle, through the C ABI.

The oracle's library forward is pinned bit-exact to the reference
(tests/test_oracle_pin.py); the reference has no gradient, so the GPU
adjoint's library gradients are checked against 4th-order central finite
differences of the oracle forward along seeded directions, per parameter
kind.  A finite difference cannot resolve a derivative below the rounding
of the voltages it differences (~1e-14 mV over the trace, divided by the
step, and spike times shift non-smoothly with the step): the gate is
|<grad, u> - FD| <= 1e-6 |FD| + 4 max(|FD(h) - FD(2h)|, |FD(h) - FD(h/2)|),
the second term the measured resolution of the difference quotient itself, and
most kinds must be resolved to 1e-6 so that the comparison is not vacuous
(all to 1e-3).
"""
import numpy as np
import pytest

from heliox_b200 import synth
from heliox_b200.model import LIB_FIELDS, LIB_NTRAIN
from oracle import oracle as O

pytestmark = pytest.mark.gpu

V_TOL = 1e-9
FD_TOL = 1e-6
LIB_KEYS = [f"{nm}.{f}" for nm, fs in LIB_FIELDS.items() for f in fs[: LIB_NTRAIN[nm]]]


@pytest.fixture(scope="module")
def Sim():
    from heliox_b200.runtime import Sim as S

    return S


def _group(cadyn="CaDynamics_E2"):
    return synth.lib_tree_batch(3, seed0=4100, nmax=160, cadyn=cadyn)


def _probes(g):
    return np.array(list(g.soma_nodes()) + [g.nnode - 1, g.nnode // 2], dtype=np.int32)


def test_forward_library_cells(Sim):
    g = _group()
    probes = _probes(g)
    s = Sim(0)
    s.load_group(g)
    tr = s.simulate(2000, probes=probes)
    ref, _ = O.forward(g, 2000, probe=probes)
    err = np.max(np.abs(tr - ref)) / np.max(np.abs(ref))
    assert err <= V_TOL, err
    up = (ref[1:, 0] > 0) & (ref[:-1, 0] <= 0)
    assert up.sum() >= 2  # the soma spikes: the channels are exercised


def test_forward_library_cells_cainternm(Sim):
    """The worm-lr calcium dynamics cainternm_lr in place of CaDynamics_E2."""
    g = _group("cainternm_lr")
    probes = _probes(g)
    s = Sim(0)
    s.load_group(g)
    tr = s.simulate(2000, probes=probes)
    ref, _ = O.forward(g, 2000, probe=probes)
    assert np.max(np.abs(tr - ref)) / np.max(np.abs(ref)) <= V_TOL


def test_forward_mixed_hh_and_library(Sim):
    from heliox_b200.model import concat_groups

    g = concat_groups([synth.lib_tree_cell(11, ncomp=80), synth.random_tree_cell(12, ncomp=90),
                       synth.lib_tree_cell(13, ncomp=120)])
    g.celsius = 20.0
    probes = _probes(g)
    s = Sim(0)
    s.load_group(g)
    tr = s.simulate(1500, probes=probes)
    ref, _ = O.forward(g, 1500, probe=probes)
    assert np.max(np.abs(tr - ref)) / np.max(np.abs(ref)) <= V_TOL


def _loss(g, T, probes, c):
    tr, _ = O.forward(g, T, probe=probes)
    return float(np.sum(c * tr))


def _fd(g, key, u, T, probes, c, h=1e-3):
    """d/de L(p * (1 + e u)) at e = 0, 4th-order central differences."""
    mech, var = key.split(".")
    p0 = g.lib[mech].fields[var].copy()
    vals = []
    for e in (2 * h, h, -h, -2 * h):
        g.lib[mech].fields[var] = p0 * (1.0 + e * u)
        vals.append(_loss(g, T, probes, c))
    g.lib[mech].fields[var] = p0
    return (-vals[0] + 8 * vals[1] - 8 * vals[2] + vals[3]) / (12 * h)


def test_library_gradients_vs_finite_differences(Sim):
    """Spiking (800 steps: the soma fires, calcium enters) and subthreshold
    (190 steps, before the IClamp: every voltage below -60 mV, so the K_Pst
    time constant stays on one branch of its v < -50 switch, K_Pst.cu rates)
    regimes with CaDynamics_E2, and the spiking regime with cainternm_lr as
    the calcium dynamics (the kinds that read or write calcium, and
    kqt3_lr).  Every kind must agree in every run; each kind must be
    resolved by the finite differences to 1e-3 in one of them, and two
    thirds of them to 1e-6 (the calcium-buffer parameters and the small
    densities move the voltages least)."""
    from heliox_b200.model import LIB_IONS

    best = {}
    ca_keys = [k for k in LIB_KEYS if "ca" in LIB_IONS.get(k.split(".")[0], ()) or k.startswith("kqt3_lr.")]
    for T, h, cadyn in ((800, 1e-3, "CaDynamics_E2"), (190, 1e-2, "CaDynamics_E2"), (800, 1e-3, "cainternm_lr")):
        g = _group(cadyn)
        keys = [k for k in (LIB_KEYS if cadyn == "CaDynamics_E2" else ca_keys) if k.split(".")[0] in g.lib]
        probes = _probes(g)
        rng = np.random.default_rng(17)
        c = rng.standard_normal((T + 1, probes.size)) * 1e-2
        c[0] = 0.0
        s = Sim(0)
        s.load_group(g)
        tr = s.forward_capture(T, probes=probes)
        ref, _ = O.forward(g, T, probe=probes)
        assert np.max(np.abs(tr - ref)) / np.max(np.abs(ref)) <= V_TOL
        grads = s.backward(c, keys=keys)
        for key in keys:
            mech, var = key.split(".")
            p = g.lib[mech].fields[var]
            u = rng.standard_normal(p.size)
            fd = _fd(g, key, u, T, probes, c, h=h)
            noise = max(abs(fd - _fd(g, key, u, T, probes, c, h=2 * h)),
                        abs(fd - _fd(g, key, u, T, probes, c, h=0.5 * h)))
            ad = float(np.sum(grads[key] * p * u))
            assert abs(ad - fd) <= FD_TOL * abs(fd) + 4 * noise, (T, key, ad, fd, noise)
            best[key] = min(best.get(key, np.inf), noise / abs(fd))
        s.close()
    assert set(best) == set(LIB_KEYS), set(LIB_KEYS) - set(best)
    assert all(r <= 1e-3 for r in best.values()), best
    assert sum(r <= FD_TOL for r in best.values()) >= (2 * len(LIB_KEYS)) // 3, best


def test_library_checkpointed_backward_equals_full_tape(Sim):
    g = _group()
    T = 600
    probes = _probes(g)
    rng = np.random.default_rng(3)
    full = Sim(0)
    full.load_group(g)
    tr = full.forward_capture(T, probes=probes)
    c = rng.standard_normal(tr.shape)
    g_full = full.backward(c)
    from heliox_b200.model import LIB_STATES

    nst = sum(g.lib[m].n * len(st) for m, st in LIB_STATES.items() if m in g.lib)
    ck = Sim(0, tape_budget_bytes=(4 * g.nnode + nst) * 8 * 60)  # 60 rows: checkpointed segments
    ck.load_group(g)
    assert np.array_equal(ck.forward_capture(T, probes=probes), tr)
    g_ck = ck.backward(c)
    for k in g_full:
        assert np.array_equal(g_full[k], g_ck[k]), k


def test_library_param_roundtrip_and_handles(Sim):
    g = _group()
    s = Sim(0)
    s.load_group(g)
    for key in LIB_KEYS:
        if key.split(".")[0] not in g.lib:
            continue
        v = s.get_param_array(key)
        mech, var = key.split(".")
        assert np.array_equal(v, g.lib[mech].fields[var]), key
    k = "NaTg.gNaTgbar"
    new = g.lib["NaTg"].fields["gNaTgbar"] * 1.5
    s.set_param_array(k, new)
    assert np.array_equal(s.get_param_array(k), new)
    h = s.get_variable_handle("NaTg", "gNaTgbar", 3)
    assert s.get_variables([h])[0] == new[3]
    # the changed densities take effect
    probes = _probes(g)
    tr = s.simulate(400, probes=probes)
    g2 = g.copy()
    g2.lib["NaTg"].fields["gNaTgbar"] = new
    ref, _ = O.forward(g2, 400, probe=probes)
    assert np.max(np.abs(tr - ref)) / np.max(np.abs(ref)) <= V_TOL


def _fd_view(g, key, u, T, probes, c, h):
    """d/de L(p (1 + e u)) at e = 0 for any parameter kind (model.param_view)."""
    mech, var = key.split(".")
    view = g.param_view(mech, var)
    p0 = view.copy()
    vals = []
    for e in (2 * h, h, -h, -2 * h):
        view[:] = p0 * (1.0 + e * u)
        vals.append(_loss(g, T, probes, c))
    view[:] = p0
    return (-vals[0] + 8 * vals[1] - 8 * vals[2] + vals[3]) / (12 * h)


@pytest.mark.parametrize("kind,tape_budget", [("event", 0), ("coupled", 0), ("event", 24 << 20)])
def test_library_cells_in_networks(Sim, kind, tape_budget):
    """Library cells wired into an event network (ExpSyn / Exp2Syn, NetStims)
    or a coupled one (HalfGap, gapjunction_lr / _noptr, graded synapses; the
    grid-synchronous launches): voltages and spikes against the oracle (itself
    bit-exact to the reference on these networks), and network and library
    gradients against finite differences of the oracle forward, full tape and
    checkpointed.  The event network's steps are relative 1e-5 (at 1e-3 a
    perturbed run already moves a spike across a step: the difference quotient
    is then not the local derivative; measured resolution at 1e-5: < 1e-6)."""
    h = 1e-5 if kind == "event" else 1e-3
    if kind == "event":
        g = synth.lib_network("event", ncell=6, seed=41, nstim=3, weight=(0.02, 0.08), stim_noise=1.0,
                              stim_interval=5.0)
        keys = ("Exp2Syn.weight", "ExpSyn.weight", "NaTg.gNaTgbar", "SKv3_1.gSKv3_1bar", "CaDynamics_E2.gamma")
    else:
        g = synth.lib_network("coupled", ncell=6, seed=42, ngap=4, ngapj=3, ngraded=8, ngapnp=3)
        keys = ("HalfGap.g", "gapjunction_noptr.weight", "neuron_to_neuron_syn_lr.w", "NaTg.gNaTgbar",
                "shl1_lr.w")
    T = 600
    probes = g.soma_nodes()
    s = Sim(0, tape_budget_bytes=tape_budget)
    s.load_group(g)
    tr = s.forward_capture(T, probes=probes)
    ref, st = O.forward(g, T, probe=probes)
    assert np.max(np.abs(tr - ref)) / np.max(np.abs(ref)) <= V_TOL
    gid, t = s.spikes()
    want = sorted((int(b), float(a)) for a, b in st["spikes"])
    got = sorted(zip(gid.tolist(), t.tolist()))
    assert len(got) == len(want) and len(want) > 0
    assert all(a[0] == b[0] and abs(a[1] - b[1]) <= g.dt for a, b in zip(got, want))
    rng = np.random.default_rng(23)
    c = rng.standard_normal((T + 1, probes.size)) * 1e-2
    c[0] = 0.0
    grads = s.backward(c, keys=keys)
    resolved = 0
    for key in keys:
        mech, var = key.split(".")
        p = g.param_view(mech, var)
        u = rng.standard_normal(p.size)
        fd = _fd_view(g, key, u, T, probes, c, h)
        noise = max(abs(fd - _fd_view(g, key, u, T, probes, c, 2 * h)), abs(fd - _fd_view(g, key, u, T, probes, c, h / 2)))
        ad = float(np.sum(grads[key] * p * u))
        assert abs(ad - fd) <= FD_TOL * abs(fd) + 4 * noise, (key, ad, fd, noise)
        resolved += noise <= 1e-3 * abs(fd)
    assert resolved >= len(keys) - 1
    s.close()
