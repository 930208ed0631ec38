"""GPU: device Adam against the reference-pinned Adam restatement, and the
heliox_learn-compatible gradient-method surface."""
import numpy as np
import pytest

from heliox_b200 import synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_device_adam_matches_reference_adam():
    from heliox_b200.runtime import Sim

    g = synth.random_tree_batch(2, seed0=9)
    s = Sim(0)
    s.load_group(g)
    idx = np.arange(0, g.hh.n, 3)
    handles = [s.get_variable_handle("hh", "gnabar", int(i)) for i in idx]
    opt = s.create_optimizer("adam", beta1=0.9, beta2=0.999, epsilon=1e-8)
    s.optimizer_add_external_grads(opt, handles, impedance=2.0)
    rng = np.random.default_rng(3)
    w0 = s.get_param_array("hh.gnabar")[idx]
    grads = (rng.standard_normal((6, idx.size)) * 10).astype(np.float32)
    for k in range(grads.shape[0]):
        s.optimizer_set_external_grads_f32(opt, grads[k])
        s.optimizer_step_with_inv_record_steps(opt, 1e-3, 0.25)
    w = s.get_param_array("hh.gnabar")[idx]
    ws, m, v = O.adam_port(w0, grads.astype(np.float64), 1e-3, 0.25, 0.9, 0.999, 1e-8, 2.0)
    assert np.array_equal(w, ws[-1])
    step, m2, v2, hyper = s.optimizer_get_adam_state(opt)
    assert step == 6 and np.array_equal(m2, m) and np.array_equal(v2, v)
    # untouched instances keep their values
    rest = np.setdiff1d(np.arange(g.hh.n), idx)
    assert np.array_equal(s.get_param_array("hh.gnabar")[rest], g.hh.fields["gnabar"][rest])


def test_adjoint_method_mapped_columns():
    from heliox_b200.learn import (AdjointCaptureSpec, AdjointMethod, AdjointRuntime, AdjointState, MappedSignal,
                                   mse_objective)

    g = synth.random_tree_batch(3, seed0=12)
    rt = AdjointRuntime(g)
    T = 600
    target, _ = O.forward(synth.perturb_conductances(g, 0.2, seed=4), T)
    handles = [rt.handle("hh", "gnabar", i) for i in range(g.hh.n)] + [rt.handle("pas", "g_pas", i) for i in range(g.pas.n)]
    cell = g.cell_of_node()
    dest = np.concatenate([cell[g.hh.nodes], g.ncell + cell[g.pas.nodes]]).astype(np.int32)
    scale = np.ones(len(handles), dtype=np.float32)
    st = AdjointState(AdjointCaptureSpec(g.soma_nodes(), T), MappedSignal("w", handles, dest, scale))
    m = AdjointMethod()
    assert m.spec.name == "adjoint"
    cap = m.capture(rt, state=st)
    loss, dl = mse_objective(cap.output_vs_tn, target)
    rg = m.backward(rt, captured=cap, dL_dprobe=dl, state=st)
    _, gr = O.adjoint(g, T, dl)
    ref = np.zeros(2 * g.ncell)
    np.add.at(ref, cell[g.hh.nodes], gr["hh.gnabar"])
    np.add.at(ref, g.ncell + cell[g.pas.nodes], gr["pas.g"])
    np.testing.assert_allclose(rg.dw_out_n, ref.astype(np.float32), rtol=1e-5)
    rt.close()


def test_train_adam_reduces_loss():
    from heliox_b200.learn import AdjointRuntime, train_adam

    g = synth.ball_and_stick()
    target, _ = O.forward(synth.ball_and_stick(gnabar_scale=1.1), 2000)
    rt = AdjointRuntime(g)
    h = [rt.handle("hh", "gnabar", 0), rt.handle("hh", "gkbar", 0)]
    hist = train_adam(rt, h, target, epochs=12, lr=2e-3)
    assert hist[-1] < 0.5 * hist[0], hist
    rt.close()
