"""GPU: the device reciprocal the mechanism rate functions use instead of IEEE
division (rcp_nz: hardware estimate refined by two Newton-Raphson steps),
against IEEE 1/x over a wide sweep.  The bound is 1 ulp; the test reports the
largest error and the fraction of results that are not correctly rounded."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_rcp_nz_within_one_ulp_of_ieee():
    import torch

    from heliox_b200 import _lib

    L = _lib.load()
    rng = np.random.default_rng(17)
    n = 1 << 22
    # magnitudes log-uniform over the domain (normal x with a normal reciprocal),
    # both signs, plus dense samples near 1 and every power of two in range
    mag = 10.0 ** rng.uniform(-307.0, 307.0, n)
    near1 = 1.0 + rng.uniform(-0.5, 0.5, 1 << 20)
    pow2 = np.ldexp(1.0, np.arange(-1021, 1022))
    x = np.concatenate([mag, near1, pow2, np.nextafter(pow2, 0.0), np.nextafter(pow2, np.inf)])
    x = x * np.where(rng.random(x.shape[0]) < 0.5, -1.0, 1.0)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty_like(xd)
    assert L.hx_rcp_nz_dev(C.c_void_p(xd.data_ptr()), C.c_void_p(yd.data_ptr()), int(x.shape[0]), None) == 0
    torch.cuda.synchronize()
    y = yd.cpu().numpy()
    ref = 1.0 / x
    ulp = np.abs(y - ref) / np.spacing(np.abs(ref))
    worst = float(np.max(ulp))
    inexact = float(np.mean(ulp > 0))
    print(f"rcp_nz vs IEEE 1/x over {x.shape[0]} values: max {worst:.3f} ulp, not correctly rounded: {inexact:.2e}")
    assert np.all(np.isfinite(y))
    assert worst <= 1.0
