"""GPU parity of the network path (synapses, spikes, NetStims, gaps, graded
synapses) against the CPU oracle, through the C ABI.

Tolerances as for single cells: voltages within 1e-9 of the trace scale,
gradients within 1e-7 of the largest oracle gradient of each kind, the spike
lists identical in gid with times within one dt.  The oracle itself is pinned
bit for bit to the reference's CPU integrator on these networks
(tests/test_oracle_pin.py).
"""
import numpy as np
import pytest

from heliox_b200 import synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu

V_TOL = 1e-9
G_TOL = 1e-7
GRAD_KINDS = ("hh.gnabar", "hh.gkbar", "hh.gl", "hh.el", "pas.g", "pas.e", "cm", "IClamp.amp")
NET_KINDS = ("ExpSyn.weight", "ExpSyn.e", "Exp2Syn.weight", "Exp2Syn.e", "HalfGap.g", "gapjunction_lr.g",
             "gapjunction_lr.w", "neuron_to_neuron_syn_lr.w")


@pytest.fixture(scope="module")
def Sim():
    from heliox_b200.runtime import Sim as S

    return S


def _check_v(tr, ref):
    err = np.max(np.abs(tr - ref)) / np.max(np.abs(ref))
    assert err <= V_TOL, err


def _check_spikes(sim, ref_spikes, dt):
    gid, t = sim.spikes()
    mine = sorted(zip(gid.tolist(), t.tolist()))
    ref = sorted((g, tt) for tt, g in ref_spikes)
    assert len(mine) == len(ref)
    for (gm, tm), (gr, tr) in zip(mine, ref):
        assert gm == gr and abs(tm - tr) <= dt


def _check_g(gg, gr, keys):
    for k in keys:
        ref = gr.get(k)
        if ref is None or ref.size == 0:
            continue
        scale = np.max(np.abs(ref))
        if scale == 0:
            assert np.max(np.abs(gg[k])) == 0, k
            continue
        err = np.max(np.abs(gg[k] - ref)) / scale
        assert err <= G_TOL, (k, err)


def _run(Sim, g, T, tape_budget=0, probes=None):
    s = Sim(0, tape_budget_bytes=tape_budget)
    s.load_group(g)
    p = g.soma_nodes() if probes is None else probes
    rng = np.random.default_rng(1)
    c = rng.standard_normal((T + 1, p.shape[0]))
    tr = s.forward_capture(T, probes=p)
    gg = s.backward(c)
    ref, gr = O.adjoint(g, T, c, probe=p)
    return s, tr, gg, ref, gr


def test_event_network_forward_spikes_and_gradients(Sim):
    g = synth.spiking_network(ncell=8, seed=11, nstim=6, weight=(0.02, 0.08), stim_noise=1.0, stim_interval=5.0)
    s, tr, gg, ref, gr = _run(Sim, g, 2400)
    _check_v(tr, ref)
    assert len(gr["spikes"]) >= 5
    _check_spikes(s, gr["spikes"], g.dt)
    _check_g(gg, gr, GRAD_KINDS + NET_KINDS)
    assert np.max(np.abs(gr["Exp2Syn.weight"])) > 0 and np.max(np.abs(gr["ExpSyn.weight"])) > 0


def test_event_network_checkpointed_equals_full(Sim):
    g = synth.spiking_network(ncell=6, seed=12, nstim=4, weight=(0.02, 0.08), stim_noise=1.0, stim_interval=4.0)
    T = 1600
    _, tr, gg, ref, gr = _run(Sim, g, T, tape_budget=8 << 20)
    _check_v(tr, ref)
    _check_g(gg, gr, GRAD_KINDS + NET_KINDS)
    _, tr2, gg2, _, _ = _run(Sim, g, T)
    assert np.array_equal(tr, tr2)
    for k in NET_KINDS + GRAD_KINDS:
        assert np.allclose(gg[k], gg2[k], rtol=1e-12, atol=0), k


def test_netstim_gpu_stream_mode(Sim):
    g = synth.spiking_network(ncell=6, seed=13, nstim=6, weight=(0.02, 0.08), stim_noise=1.0, stim_interval=5.0)
    g.netstim_rng = 1
    s, tr, gg, ref, gr = _run(Sim, g, 2000)
    _check_v(tr, ref)
    _check_spikes(s, gr["spikes"], g.dt)
    _check_g(gg, gr, NET_KINDS)


def test_coupled_network_forward_and_gradients(Sim):
    g = synth.coupled_network(ncell=6, seed=5, ngap=6, ngapj=3, ngraded=10)
    p = np.arange(g.nnode, dtype=np.int32)[::13]
    s, tr, gg, ref, gr = _run(Sim, g, 1500, probes=p)
    _check_v(tr, ref)
    _check_spikes(s, gr["spikes"], g.dt)
    _check_g(gg, gr, GRAD_KINDS + NET_KINDS)
    for k in ("HalfGap.g", "gapjunction_lr.w", "neuron_to_neuron_syn_lr.w"):
        assert np.max(np.abs(gr[k])) > 0


def test_coupled_network_checkpointed(Sim):
    g = synth.coupled_network(ncell=5, seed=9, ngap=4, ngapj=2, ngraded=8)
    _, tr, gg, ref, gr = _run(Sim, g, 1000, tape_budget=4 << 20)
    _check_v(tr, ref)
    _check_g(gg, gr, GRAD_KINDS + NET_KINDS)


def test_network_parameters_roundtrip(Sim):
    g = synth.spiking_network(ncell=4, seed=14, nstim=2)
    s = Sim(0)
    s.load_group(g)
    w = s.get_param_array("Exp2Syn.weight")
    assert np.array_equal(w, g.exp2syn.fields["weight"])
    w2 = w * 1.5
    s.set_param_array("Exp2Syn.weight", w2)
    assert np.array_equal(s.get_param_array("Exp2Syn.weight"), w2)
    # the changed weights drive the simulation exactly like an oracle run with them
    g2 = g.copy()
    g2.exp2syn.fields["weight"] = w2
    tr = s.simulate(1200)
    ref, _ = O.forward(g2, 1200)
    _check_v(tr, ref)


def test_gapjunction_noptr_forward_and_gradients(Sim):
    """gapjunction_noptr (i = weight (v - vpre), vpre from the gap transfer) on
    nodes that also carry HalfGap, gapjunction_lr and graded synapses (the
    golden case net_gapnoptr, whose oracle trace is the reference's bit for
    bit): voltages, spikes and every coupling gradient against the oracle, the
    weights settable through the handle API."""
    import importlib.util
    import os

    spec = importlib.util.spec_from_file_location(
        "make_golden", os.path.join(os.path.dirname(__file__), "golden", "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    g = mg.net_gapnoptr()
    p = np.arange(g.nnode, dtype=np.int32)[::11]
    s, tr, gg, ref, gr = _run(Sim, g, 1500, probes=p)
    _check_v(tr, ref)
    _check_spikes(s, gr["spikes"], g.dt)
    _check_g(gg, gr, GRAD_KINDS + NET_KINDS + ("gapjunction_noptr.weight",))
    assert np.max(np.abs(gr["gapjunction_noptr.weight"])) > 0
    w = s.get_param_array("gapjunction_noptr.weight")
    assert np.array_equal(w, g.gapnoptr.fields["weight"])
    g2 = g.copy()
    g2.gapnoptr.fields["weight"] = w * 1.7
    s.set_param_array("gapjunction_noptr.weight", g2.gapnoptr.fields["weight"])
    tr2 = s.simulate(600, probes=p)
    ref2, _ = O.forward(g2, 600, probe=p)
    _check_v(tr2, ref2)
    s.close()


def _coupled_run(Sim, g, T, grid_sync, tape_budget=0, probes=None):
    s = Sim(0, tape_budget_bytes=tape_budget)
    s.load_group(g)
    s.set_grid_sync(grid_sync)
    p = g.soma_nodes() if probes is None else probes
    c = np.random.default_rng(7).standard_normal((T + 1, p.shape[0]))
    tr = s.forward_capture(T, probes=p)
    gg = s.backward(c)
    window = s.window()
    s.close()
    return tr, gg, window


@pytest.mark.parametrize("tape_budget", [0, 16 << 20])
def test_coupled_grid_sync_equals_per_step_launches(Sim, tape_budget):
    """Coupled groups run whole windows in one cooperative launch with a grid
    barrier per step (forward, checkpoint recompute and reverse sweep); the
    traces and every gradient equal those of one launch per step bit for bit,
    and the oracle's within tolerance."""
    g = synth.coupled_network(ncell=40, seed=12, ngap=60, ngapj=10, ngraded=80, ngapnp=10)
    T = 800
    tr1, g1, w1 = _coupled_run(Sim, g, T, True, tape_budget)
    tr0, g0, w0 = _coupled_run(Sim, g, T, False, tape_budget)
    assert w0 == 1 and w1 > 1  # the grid-synchronous launch runs many steps
    assert np.array_equal(tr1, tr0)
    for k in g0:
        assert np.array_equal(g1[k], g0[k]), k
    ref, gr = O.adjoint(g, T, np.random.default_rng(7).standard_normal((T + 1, g.ncell)))
    _check_v(tr1, ref)
    _check_g(g1, gr, GRAD_KINDS + NET_KINDS + ("gapjunction_noptr.weight",))


def test_coupled_grid_barrier_wait_gives_up_and_context_recovers(Sim):
    """A grid-barrier wait of the coupled launches bounded to one ~100 ns sleep
    runs out (40 CTAs never all arrive within it at every step of 400): the
    forward reports the timeout instead of waiting; with the default bound the
    same context runs the forward to the oracle's trace."""
    from heliox_b200.runtime import HxError

    g = synth.coupled_network(ncell=40, seed=13, ngap=60, ngapj=0, ngraded=80)
    s = Sim(0)
    s.load_group(g)
    assert s.plan_stats()["npack"] >= 8
    s.set_split_barrier_limit(1)
    with pytest.raises(HxError, match="timed out"):
        s.simulate(400)
    s.set_split_barrier_limit(0)
    tr = s.simulate(400)
    ref, _ = O.forward(g, 400)
    _check_v(tr, ref)
    s.close()


def test_requested_gradient_kinds_only(Sim):
    """hx_set_grad_kinds: the reverse sweep accumulates only the requested
    kinds; those equal the all-kinds gradients bit for bit (each accumulator's
    arithmetic is its own), the others read as zero, and resetting restores
    all kinds."""
    g = synth.spiking_network(ncell=6, seed=21, nstim=4, weight=(0.02, 0.08), stim_noise=1.0, stim_interval=5.0)
    T = 1200
    s = Sim(0)
    s.load_group(g)
    p = g.soma_nodes()
    c = np.random.default_rng(3).standard_normal((T + 1, p.shape[0]))
    s.forward_capture(T, probes=p)
    full = s.backward(c)
    want = ("hh.gnabar", "Exp2Syn.weight")
    s.set_grad_kinds(want)
    part = s.backward(c)
    for k in part:
        if k in want or (k == "ExpSyn.weight"):  # ExpSyn and Exp2Syn weights share one accumulator
            assert np.array_equal(part[k], full[k]), k
        elif k in GRAD_KINDS + NET_KINDS:
            assert not np.any(part[k]), k
    assert np.max(np.abs(full["hh.gnabar"])) > 0 and np.max(np.abs(full["Exp2Syn.weight"])) > 0
    s.set_grad_kinds(None)
    again = s.backward(c)
    for k in full:
        assert np.array_equal(again[k], full[k]), k
    s.close()
