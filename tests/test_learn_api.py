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
