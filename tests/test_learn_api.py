"""CPU: host-side pieces of the heliox_learn-compatible surface."""
import numpy as np
import pytest

from heliox_b200.learn import AdjointMethod, GradientMethod, MappedSignal, mse_objective


def test_mapped_signal_validation():
    MappedSignal("w", [1, 2], np.array([0, 1], np.int32), np.ones(2, np.float32))
    with pytest.raises(TypeError):
        MappedSignal("w", [1, 2], np.array([0, 1], np.int64), np.ones(2, np.float32))
    with pytest.raises(ValueError):
        MappedSignal("w", [1, 2, 3], np.array([0, 1], np.int32), np.ones(2, np.float32))


def test_adjoint_method_is_a_gradient_method():
    assert isinstance(AdjointMethod(), GradientMethod)
    assert AdjointMethod().spec.precise


def test_mse_objective_gradient_fd():
    rng = np.random.default_rng(0)
    tr = rng.standard_normal((11, 3))
    tg = rng.standard_normal((11, 3))
    loss, g = mse_objective(tr, tg)
    assert np.all(g[0] == 0)
    h = 1e-6
    e = np.zeros_like(tr)
    e[4, 1] = h
    fd = (mse_objective(tr + e, tg)[0] - mse_objective(tr - e, tg)[0]) / (2 * h)
    assert abs(fd - g[4, 1]) < 1e-8


def _reference_python_lib():
    import os

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    ref = os.environ.get("HX_REFERENCE") or os.path.join(os.path.dirname(root), "reference")
    lib = os.path.join(ref, "python_lib")
    return lib if os.path.isdir(os.path.join(lib, "heliox_learn")) else None


def test_adjoint_method_in_the_reference_plugin_slot():
    """With the reference's heliox_learn importable (its python_lib on the path),
    heliox_b200.learn uses the reference's own types: AdjointMethod is a
    heliox_learn.GradientMethod, MappedSignal and ReplayGrads are the
    reference's classes (checked in a fresh interpreter)."""
    import os
    import subprocess
    import sys

    lib = _reference_python_lib()
    if lib is None:
        pytest.skip("reference checkout not present")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = (
        "import sys; sys.path[:0] = [%r, %r]\n"
        "import numpy as np, heliox_learn\n"
        "from heliox_b200 import learn\n"
        "assert learn.REFERENCE_TYPES\n"
        "assert isinstance(learn.AdjointMethod(), heliox_learn.GradientMethod)\n"
        "assert learn.MappedSignal is heliox_learn.MappedSignal and learn.ReplayGrads is heliox_learn.ReplayGrads\n"
        "assert learn.MethodSpec is heliox_learn.MethodSpec and learn.AdjointMethod().spec.name == 'adjoint'\n"
        "p = heliox_learn.MappedSignal('w', [1, 2, 3], np.array([0, 2, 2], np.int32), np.ones(3, np.float32))\n"
        "assert learn.n_columns(p) == 3\n"
        "print('reference types ok')\n" % (root, lib))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True)
    assert r.returncode == 0 and "reference types ok" in r.stdout, r.stdout + r.stderr
