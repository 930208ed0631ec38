"""GPU parity of the CUDA path against the CPU oracle (through the C ABI).

Tolerances: voltages within 1e-9 relative to the trace's
scale (max |v_ref|), parameter gradients within 1e-7 relative to the largest
reference gradient of the same kind, spike counts identical with spike times
within one dt.
"""
import numpy as np
import pytest

from heliox_b200 import synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu

V_TOL = 1e-9
G_TOL = 1e-7


@pytest.fixture(scope="module")
def Sim():
    from heliox_b200.runtime import Sim as S

    return S


def _spikes(tr, dt):
    up = (tr[1:] > 0.0) & (tr[:-1] <= 0.0)
    return [np.nonzero(up[:, j])[0] * dt for j in range(tr.shape[1])]


def _check_v(tr_gpu, tr_ref, dt):
    scale = np.max(np.abs(tr_ref))
    err = np.max(np.abs(tr_gpu - tr_ref)) / scale
    assert err <= V_TOL, err
    for sg, sr in zip(_spikes(tr_gpu, dt), _spikes(tr_ref, dt)):
        assert len(sg) == len(sr)
        if len(sr):
            assert np.max(np.abs(sg - sr)) <= dt


def _check_g(gg, gr, keys):
    for k in keys:
        ref = gr[k]
        if ref.size == 0:
            continue
        scale = np.max(np.abs(ref))
        err = np.max(np.abs(gg[k] - ref)) / max(scale, 1e-300)
        assert err <= G_TOL, (k, err)


def test_forward_ball_and_stick(Sim):
    g = synth.ball_and_stick()
    s = Sim(0)
    s.load_group(g)
    probes = np.array([0, 1, 50, 100], dtype=np.int32)
    tr = s.simulate(4000, probes=probes)
    ref, _ = O.forward(g, 4000, probe=probes)
    _check_v(tr, ref, g.dt)
    assert len(_spikes(ref[:, :1], g.dt)[0]) >= 3


def test_forward_random_trees(Sim):
    g = synth.random_tree_batch(12, seed0=101)
    s = Sim(0, pack_target=200)
    s.load_group(g)
    rng = np.random.default_rng(0)
    probes = np.concatenate([g.soma_nodes(), rng.integers(g.ncell, g.nnode, 8)]).astype(np.int32)
    tr = s.simulate(4000, probes=probes)
    ref, _ = O.forward(g, 4000, probe=probes)
    _check_v(tr, ref, g.dt)


def _long_chain_and_star():
    """Two cells that exercise the solver's structural paths: a 1,500-node
    unbranched chain (cut into 63 segments of at most 24 nodes, solved by the
    reduced-tree form) and a star of 700 one-node arms (more segments than a
    CTA has threads: the level-by-level form)."""
    from heliox_b200.model import CellGroup, MechTable, _f64, _i32, concat_groups

    def cell(parent, seed):
        n = len(parent)
        rng = np.random.default_rng(seed)
        hh_nodes = np.arange(0, n, 7)
        pas_nodes = np.setdiff1d(np.arange(n), hh_nodes)
        hh = {k: _f64(np.full(hh_nodes.size, v)) for k, v in synth.HH_STD.items()}
        return CellGroup(
            ncell=1,
            parent=_i32(parent),
            a=_f64(-rng.uniform(5, 15, n)),
            b=_f64(-rng.uniform(5, 15, n)),
            area=_f64(np.full(n, 300.0)),
            cm=_f64(np.ones(n)),
            hh=MechTable(_i32(hh_nodes), hh),
            pas=MechTable(_i32(pas_nodes), {"g": _f64(np.full(pas_nodes.size, 1e-4)),
                                           "e": _f64(np.full(pas_nodes.size, -65.0))}),
            iclamp=MechTable(_i32([0]), {"del": _f64([1.0]), "dur": _f64([20.0]), "amp": _f64([0.8])}),
        )

    chain = cell(np.arange(-1, 1499), 1)
    star = cell(np.concatenate([[-1], np.zeros(700, dtype=np.int64)]), 2)
    return concat_groups([chain, star])


def test_segmented_chain_and_wide_star(Sim):
    g = _long_chain_and_star()
    s = Sim(0)
    s.load_group(g)
    probes = np.array([0, 700, 1499, 1500, 1600], dtype=np.int32)
    T = 1200
    tr = s.forward_capture(T, probes=probes)
    ref, _ = O.forward(g, T, probe=probes)
    _check_v(tr, ref, g.dt)
    rng = np.random.default_rng(4)
    dLdv = rng.standard_normal(tr.shape) * 1e-3
    gg = s.backward(dLdv)
    _, gr = O.adjoint(g, T, dLdv, probe=probes)
    _check_g(gg, gr, O.GRAD_KEYS)


def test_capture_trace_equals_simulate(Sim):
    g = synth.random_tree_batch(4, seed0=7)
    s = Sim(0)
    s.load_group(g)
    a = s.simulate(800)
    b = s.forward_capture(800)
    assert np.array_equal(a, b)


def test_backward_ball_and_stick_mse(Sim):
    g = synth.ball_and_stick()
    target, _ = O.forward(synth.ball_and_stick(gnabar_scale=1.1), 4000)
    s = Sim(0)
    s.load_group(g)
    tr = s.forward_capture(4000)
    T = 4000
    dLdv = np.zeros_like(tr)
    dLdv[1:] = 2.0 * (tr[1:] - target[1:]) / T
    gg = s.backward(dLdv)
    _, gr = O.adjoint(g, T, dLdv)
    _check_g(gg, gr, O.GRAD_KEYS)


def test_backward_random_trees(Sim):
    g = synth.random_tree_batch(6, seed0=55)
    T = 2000
    s = Sim(0)
    s.load_group(g)
    tr = s.forward_capture(T)
    rng = np.random.default_rng(5)
    dLdv = rng.standard_normal(tr.shape) * 1e-3
    gg = s.backward(dLdv)
    ref_tr, gr = O.adjoint(g, T, dLdv)
    _check_v(tr, ref_tr, g.dt)
    _check_g(gg, gr, O.GRAD_KEYS)


def test_checkpointed_backward_equals_full_tape(Sim):
    g = synth.random_tree_batch(5, seed0=21)
    T = 1000
    rng = np.random.default_rng(9)
    full = Sim(0)
    full.load_group(g)
    tr = full.forward_capture(T)
    dLdv = rng.standard_normal(tr.shape)
    g_full = full.backward(dLdv)
    per_step = (g.nnode + 3 * g.hh.n) * 8
    ck = Sim(0, tape_budget_bytes=per_step * 80)
    ck.load_group(g)
    tr2 = ck.forward_capture(T)
    g_ck = ck.backward(dLdv)
    assert np.array_equal(tr, tr2)
    for k in g_full:
        assert np.array_equal(g_full[k], g_ck[k]), k


def test_pinned_out_buffers(Sim):
    """forward_capture / backward / set_param_array with page-locked caller
    buffers (the bench's end-to-end path) give the same results as with
    freshly allocated arrays."""
    from heliox_b200.runtime import pinned_empty

    g = synth.random_tree_batch(4, seed0=77)
    T = 400
    s = Sim(0)
    s.load_group(g)
    x = pinned_empty(g.hh.n)
    x[:] = g.hh.fields["gnabar"] * 1.02
    s.set_param_array("hh.gnabar", x)
    assert np.array_equal(s.get_param_array("hh.gnabar"), x)
    tr = s.forward_capture(T)
    tr_p = pinned_empty(tr.shape)
    assert s.forward_capture(T, out=tr_p) is tr_p
    assert np.array_equal(tr, tr_p)
    rng = np.random.default_rng(3)
    dl = pinned_empty(tr.shape)
    dl[:] = rng.standard_normal(tr.shape) * 1e-3
    keys = ("hh.gnabar", "pas.g", "cm")
    gg = s.backward(np.array(dl), keys=keys)
    s.forward_capture(T, out=tr_p)
    out = {k: pinned_empty(gg[k].shape[0]) for k in keys}
    gp = s.backward(dl, keys=keys, out=out)
    for k in keys:
        assert gp[k] is out[k]
        assert np.array_equal(gg[k], out[k]), k
    with pytest.raises(ValueError):
        s.forward_capture(T, out=np.zeros((T, 2)))


def test_param_roundtrip_and_effect(Sim):
    g = synth.random_tree_batch(3, seed0=2)
    s = Sim(0)
    s.load_group(g)
    x = s.get_param_array("hh.gnabar")
    assert np.array_equal(x, g.hh.fields["gnabar"])
    y = x * 1.05
    s.set_param_array("hh.gnabar", y)
    assert np.array_equal(s.get_param_array("hh.gnabar"), y)
    g2 = g.copy()
    g2.hh.fields["gnabar"] = y
    tr = s.simulate(600)
    ref, _ = O.forward(g2, 600)
    _check_v(tr, ref, g.dt)


def test_reduce_grads_columns(Sim):
    g = synth.random_tree_batch(3, seed0=4)
    s = Sim(0)
    s.load_group(g)
    tr = s.forward_capture(500)
    dLdv = np.ones_like(tr) * 1e-2
    gg = s.backward(dLdv)
    rng = np.random.default_rng(2)
    n = 50
    idx = rng.integers(0, g.hh.n, n)
    handles = [s.get_variable_handle("hh", "gnabar", int(i)) for i in idx]
    dest = rng.integers(0, 7, n).astype(np.int32)
    scale = rng.uniform(0.5, 2, n).astype(np.float32)
    out = s.reduce_grads_f32(handles, dest, scale, 7)
    ref = np.zeros(7)
    for j in range(n):
        ref[dest[j]] += float(scale[j]) * gg["hh.gnabar"][idx[j]]
    np.testing.assert_allclose(out, ref.astype(np.float32), rtol=1e-6, atol=1e-30)


def test_simulate_and_adjoint_into(Sim):
    """The one-call entry (shape of LearnRuntime::simulate_and_replay_dw_dx_streaming_into)
    equals forward_capture + backward + the column reduction, scaled and clipped."""
    g = synth.random_tree_batch(3, seed0=9)
    T = 300
    probes = g.soma_nodes().astype(np.int32)
    rng = np.random.default_rng(6)
    dLtdv = (rng.standard_normal((T, probes.shape[0])) * 1e-2).astype(np.float32)
    n = 40
    idx = rng.integers(0, g.hh.n, n)
    dest = rng.integers(0, 5, n).astype(np.int32)
    scale = rng.uniform(0.5, 2, n).astype(np.float32)

    s = Sim(0)
    s.load_group(g)
    handles = [s.get_variable_handle("hh", "gkbar", int(i)) for i in idx]
    tr = s.forward_capture(T, probes=probes)
    dl = np.zeros_like(tr)
    dl[1:] = dLtdv
    gg = s.backward(dl, keys=("hh.gkbar",))
    ref = np.zeros(5)
    for j in range(n):
        ref[dest[j]] += float(scale[j]) * gg["hh.gkbar"][idx[j]]

    out = s.simulate_and_adjoint_into(dLtdv, probes, handles, dest, scale, 5, grad_scale=0.5)
    np.testing.assert_allclose(out, (0.5 * ref).astype(np.float32), rtol=1e-6, atol=1e-30)
    norm = float(np.linalg.norm(0.5 * ref))
    clipped = s.simulate_and_adjoint_into(dLtdv, probes, handles, dest, scale, 5, grad_scale=0.5,
                                          grad_l2norm_threshold=0.25 * norm, clip_strategy=1)
    np.testing.assert_allclose(np.linalg.norm(clipped.astype(np.float64)), 0.25 * norm, rtol=1e-5)
    np.testing.assert_allclose(clipped / np.linalg.norm(clipped), out / np.linalg.norm(out), rtol=1e-5, atol=1e-7)
    # input gradients are not produced: a dx buffer is an error
    from heliox_b200 import _lib

    dx = np.zeros(4, dtype=np.float32)
    rc = s._L.hx_simulate_and_adjoint_into(s._ctx, _lib.fptr(dLtdv), T, probes.shape[0], _lib.iptr(probes), 5,
                                           _lib.fptr(out), _lib.fptr(dx), 0, None, None, None, None,
                                           float(g.v_init), 1.0, 0.0, 0)
    assert rc != 0


def _golden_cases():
    import glob
    import importlib.util
    import os

    here = os.path.dirname(os.path.abspath(__file__))
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(here, "golden", "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    return mg, sorted(glob.glob(os.path.join(here, "golden", "*_perm3.npz")))


_MG, _PERM3 = _golden_cases()


@pytest.mark.parametrize("path", _PERM3, ids=[p.rsplit("/", 1)[-1][:-4] for p in _PERM3])
def test_forward_vs_reference_permute3(Sim, path):
    """The device forward against the reference run with its default node
    permutation (type 3), from the committed fixtures: voltages within 1e-9 of
    the trace scale, spike lists equal with times within dt.  The adjoint's
    gradients are those of the serial-order forward (the oracle), which the
    permute-3 forward matches to rounding (< 1e-10)."""
    name = path.rsplit("/", 1)[-1][: -len("_perm3.npz")]
    make, nstep, _ = _MG.CASES[name]
    d = np.load(path)
    g = make()
    s = Sim(0)
    s.load_group(g)
    tr = s.forward_capture(int(d["nstep"]), probes=d["probes"])
    _check_v(tr, d["trace"], g.dt)
    if g.has_network:
        gid, t = s.spikes()
        got = sorted(zip(t.tolist(), gid.tolist()))
        ref = [(float(a), int(b)) for a, b in d["spikes"]]
        assert [b for _, b in got] == [b for _, b in sorted(ref)]
        assert all(abs(a[0] - b[0]) <= g.dt for a, b in zip(got, sorted(ref)))
    s.close()
