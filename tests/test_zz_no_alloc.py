"""GPU: the allocation-free MSE entry point against the allocating one.

hx_mse_loss_grad_noalloc serves callers that cannot let the library allocate
device memory (a host that owns all device memory through its own pool, or a
loop that must not meet cudaFree's implicit synchronisation); its scratch is a
static device array instead of a buffer the context allocates.  Two calls in a
row on different data must each match hx_mse_loss_grad_dev: the gradient
exactly (elementwise, same arithmetic) and the loss within 1e-12 relative (the
two reductions sum in different orders).  This file is collected last.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_noalloc_mse_matches_allocating_entry_twice():
    import torch

    from heliox_b200 import _lib, synth
    from heliox_b200.runtime import Sim

    L = _lib.load()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.Stream(dev)
    s = Sim(0)
    s.set_stream(stream.cuda_stream)
    s.load_group(synth.ball_and_stick())
    rng = np.random.default_rng(11)
    for call, (nrow, ncol) in enumerate(((4001, 1024), (1201, 37))):
        trace = torch.from_numpy(rng.standard_normal((nrow, ncol)) * 10 - 60).to(dev)
        target = torch.from_numpy(rng.standard_normal((nrow, ncol)) * 10 - 60).to(dev)
        g_ref = torch.full_like(trace, np.nan)
        g_new = torch.full_like(trace, np.nan)
        l_ref = torch.full((1,), np.nan, dtype=torch.float64, device=dev)
        l_new = torch.full((1,), np.nan, dtype=torch.float64, device=dev)
        with torch.cuda.stream(stream):
            s.mse_loss_grad_dev(trace.data_ptr(), target.data_ptr(), nrow, ncol, g_ref.data_ptr(), l_ref.data_ptr())
            rc = L.hx_mse_loss_grad_noalloc(C.c_void_p(trace.data_ptr()), C.c_void_p(target.data_ptr()), nrow, ncol,
                                            C.c_void_p(g_new.data_ptr()), C.c_void_p(l_new.data_ptr()),
                                            C.c_void_p(stream.cuda_stream))
        assert rc == 0, f"call {call}: rc={rc}"
        stream.synchronize()
        assert torch.equal(g_new, g_ref), f"call {call}: gradient differs"
        lr, ln = float(l_ref.item()), float(l_new.item())
        assert abs(ln - lr) <= 1e-12 * abs(lr), (call, lr, ln)
        err = (trace - target)[1:]
        assert abs(lr - float((err * err).mean())) <= 1e-10 * lr
    s.close()


def test_noalloc_rejects_oversize():
    import torch

    from heliox_b200 import _lib

    L = _lib.load()
    one = torch.zeros(1, dtype=torch.float64, device="cuda")
    p = C.c_void_p(one.data_ptr())
    # 2^28 + 1 rows x 1 column exceeds the static scratch; rejected before any access
    assert L.hx_mse_loss_grad_noalloc(p, p, (1 << 28) + 1, 1, p, p, None) == -2
