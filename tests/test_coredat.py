"""CPU: CoreNEURON-format export and import (heliox_b200.coredat).

``write_coredat`` writes the files the reference's loader reads (checked by
running the reference on them, tests/test_oracle_pin.py); ``read_coredat``
reads them back.  A write -> read round trip must give back every node array,
every mechanism table (library mechanisms included) and the network wiring
exactly.
"""
import os

import numpy as np
import pytest

from heliox_b200 import coredat, synth

TABLES = ("hh", "pas", "iclamp", "expsyn", "exp2syn", "netstim", "halfgap", "gapjunction", "gapnoptr", "graded")


def _same(g, h):
    assert g.ncell == h.ncell
    for k in ("parent", "a", "b", "area", "cm", "ps_thresh"):
        assert np.array_equal(getattr(g, k), getattr(h, k)), k
    assert (g.dt, g.celsius, g.v_init) == (h.dt, h.celsius, h.v_init)
    for t in TABLES:
        x, y = getattr(g, t), getattr(h, t)
        assert np.array_equal(x.nodes, y.nodes), t
        for k, v in x.fields.items():
            assert np.array_equal(v, y.fields[k]), (t, k)
        for k, v in x.ifields.items():
            assert np.array_equal(v, y.ifields[k]), (t, k)
    assert sorted(g.lib) == sorted(h.lib)
    for t, x in g.lib.items():
        y = h.lib[t]
        assert np.array_equal(x.nodes, y.nodes), t
        for k, v in x.fields.items():
            assert np.array_equal(v, y.fields[k]), (t, k)
        for k, v in x.ifields.items():
            assert np.array_equal(v, y.ifields[k]), (t, k)


@pytest.mark.parametrize(
    "maker",
    [
        lambda: synth.ball_and_stick(),
        lambda: synth.random_tree_batch(6, seed0=17),
        lambda: synth.spiking_network(),
        lambda: synth.coupled_network(),
        lambda: synth.coupled_network(ncell=4, seed=9, ngapnp=4),
        lambda: synth.lib_network("coupled", ncell=4, seed=10, ngap=3, ngapj=2, ngraded=5, ngapnp=2),
        lambda: synth.lib_network("event", ncell=4, seed=11, nstim=2),
        lambda: synth.lib_tree_batch(2, seed0=8, nmax=150),
        lambda: synth.lib_tree_batch(2, seed0=9, nmax=150, cadyn="cainternm_lr"),
        lambda: _lib_mixed(),
    ],
)
def test_write_read_round_trip(maker, tmp_path):
    g = maker()
    path = coredat.write_coredat(g, str(tmp_path / "model"))
    _same(g, coredat.read_coredat(path))


def _lib_mixed():
    from heliox_b200.model import concat_groups

    g = concat_groups([synth.lib_tree_cell(4, ncomp=60), synth.random_tree_cell(5, ncomp=70)])
    g.lib["ca_ion"].ifields["nernst"][::2] = 0  # fixed eca on every other calcium node
    return g


def test_read_needs_a_group_id_for_several_groups(tmp_path):
    g = synth.ball_and_stick()
    path = coredat.write_coredat(g, str(tmp_path / "m"), file_id=3)
    with open(os.path.join(path, "files.dat"), "w") as f:
        f.write(f"{coredat.VERSION}\n2\n3\n4\n")
    with pytest.raises(ValueError):
        coredat.read_coredat(path)
    _same(g, coredat.read_coredat(path, file_id=3))


def test_read_rejects_unknown_version(tmp_path):
    path = coredat.write_coredat(synth.ball_and_stick(), str(tmp_path / "m"))
    with open(os.path.join(path, "files.dat"), "w") as f:
        f.write("1.2\n1\n0\n")
    with pytest.raises(ValueError):
        coredat.read_coredat(path)
