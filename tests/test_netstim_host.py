"""CPU: the library's host NetStim generator (csrc/hx_netstim.cpp through
hx_netstim_trains; no GPU) against the oracle's NetStim, which restates the
reference's (netstim.cpp:120-330, one shared Random123 stream) and is pinned
bit for bit to the reference through the network traces and spike lists:
the same firing instances in the same order at the same steps, in both
stream modes (0: the reference's CPU mode, 1: its GPU mode) and with and
without noise."""
import numpy as np
import pytest

from heliox_b200 import _lib, synth
from oracle import oracle as O


@pytest.mark.parametrize("rng_mode", [0, 1])
@pytest.mark.parametrize("noise,interval,seed", [(1.0, 5.0, 13), (0.5, 8.0, 14), (0.0, 3.0, 15)])
def test_host_netstim_trains_match_oracle(rng_mode, noise, interval, seed):
    g = synth.spiking_network(ncell=6, seed=seed, nstim=6, weight=(0.02, 0.08), stim_noise=noise,
                              stim_interval=interval)
    g.netstim_rng = rng_mode
    T = 2000
    ids, steps = _lib.netstim_trains(g, T)
    _, st = O.forward(g, T)
    ns = st["netstim_spikes"]
    assert len(ns) > 5
    assert ids.tolist() == [i for _, i in ns]
    k = np.array([t / g.dt for t, _ in ns])
    assert np.max(np.abs(k - np.round(k))) < 1e-6  # emissions fall on step times
    assert steps.tolist() == np.round(k).astype(int).tolist()
