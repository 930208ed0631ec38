"""CoreNEURON-format export of a ``CellGroup`` (version 1.8 files).

Writes the files the reference loads with ``read_coredat``
(src/io/read_coredat.cpp:36-87): ``files.dat`` (read_filesdat :258-295),
``bbcore_mech.dat`` (read_mech :138-210), ``globals.dat``
(src/io/global_vars.cpp:12-80), ``<id>_1.dat`` (read_phase1 :312-400) and
``<id>_2.dat`` (read_phase2 :625-1120).  Every binary array is preceded by a
``chkpnt N`` line; N counts up across ``_1.dat`` and ``_2.dat`` of a group
(read_checkpoint_assert :223-240).

Mechanism data columns follow the offsets the reference reads
(``var_in_coredata_idx`` of hh_templated.cu:51-65, pas_templated.cu:13-14,
iclamp_templated.cu:25-27, capac.cpp:29, eion.cuh:81-86, expsyn.cpp:36-72,
exp2syn_temp.cuh:22-27, netstim.cpp:56-79, HalfGap.cu:43-47,
gapjunction_lr.cu:47-53, neuron_to_neuron_syn_lr.cu:70-86); the remaining
columns of NEURON's layouts are written as zeros.  Ion instances (na_ion, k_ion)
sit on every hh node and carry the reversal potentials; their ``iontype``
flags are 0 (fixed reversal potentials, eion.cuh:155-197).  Every cell gets a
spike-source PreSyn at its root (gid = cell index, threshold ``ps_thresh``),
which the loader requires for each real cell (read_coredat.cpp:911-915);
NetStim j gets PreSyn ``ncell + j`` (gid ``ncell + j``).  Point processes carry
dparams (area node, point-process slot[, POINTER target node]); POINTERs of
gapjunction_lr / neuron_to_neuron_syn_lr are voltages (empty pointer2type,
mech_template.cuh:431-455).  One NetCon per ExpSyn / Exp2Syn instance, ExpSyn
targets first, in instance order.  HalfGap's vgap is not in the files: the
reference wires it through Simulate::add_gap_source/add_gap_target
(simulate.cpp:995-1056); ``write_coredat`` writes the (instance, source node)
pairs to ``halfgap.i32`` for a driver to replay.
"""
from __future__ import annotations

import os
import struct
from typing import List, Tuple

import numpy as np

from .model import CellGroup

VERSION = "1.8"

# (type, name, pnttype, is_art, is_ion, dsize, pdsize, charge)
MECH_TABLE: List[Tuple[int, str, int, int, int, int, int, float]] = [
    (2, "morphology", 0, 0, 0, 1, 0, 0.0),
    (3, "capacitance", 0, 0, 0, 2, 0, 0.0),
    (4, "pas", 0, 0, 0, 3, 0, 0.0),
    (5, "na_ion", 0, 0, 1, 5, 1, 1.0),
    (6, "k_ion", 0, 0, 1, 5, 1, 1.0),
    (7, "hh", 0, 0, 0, 23, 0, 0.0),
    (8, "IClamp", 1, 0, 0, 4, 2, 0.0),
    (9, "ExpSyn", 2, 0, 0, 8, 2, 0.0),
    (10, "Exp2Syn", 3, 0, 0, 13, 2, 0.0),
    (11, "NetStim", 4, 1, 0, 9, 2, 0.0),
    (12, "HalfGap", 5, 0, 0, 5, 2, 0.0),
    (13, "gapjunction_lr", 6, 0, 0, 7, 3, 0.0),
    (14, "neuron_to_neuron_syn_lr", 7, 0, 0, 19, 3, 0.0),
]
# a NetStim's PreSyn is written as output_vindex -(type + USER_MOD_NUM * index)
# (read_coredat.cpp:930-940 with the loader's default user_mod_num 1000)
USER_MOD_NUM = 1000
TYPE = {m[1]: m[0] for m in MECH_TABLE}
DSIZE = {m[1]: m[5] for m in MECH_TABLE}
PDSIZE = {m[1]: m[6] for m in MECH_TABLE}



class _Writer:
    def __init__(self, path: str):
        self.f = open(path, "wb")

    def line(self, s) -> None:
        self.f.write((str(s) + "\n").encode())

    def array(self, chk: List[int], arr: np.ndarray) -> None:
        self.line(f"chkpnt {chk[0]}")
        chk[0] += 1
        self.f.write(np.ascontiguousarray(arr).tobytes())

    def close(self) -> None:
        self.f.close()


def write_coredat(g: CellGroup, path: str, file_id: int = 0) -> str:
    """Export ``g`` as a CoreNEURON data directory at ``path``; returns ``path``."""
    g.validate()
    os.makedirs(path, exist_ok=True)
    n = g.nnode
    # files.dat
    with open(os.path.join(path, "files.dat"), "w") as f:
        f.write(f"{VERSION}\n1\n{file_id}\n")
    # bbcore_mech.dat: types 2.. in order (types 0 and 1 are unused)
    with open(os.path.join(path, "bbcore_mech.dat"), "w") as f:
        f.write(f"{VERSION}\n{MECH_TABLE[-1][0] + 1}\n")
        for (t, name, pnt, art, ion, ds, pds, charge) in MECH_TABLE:
            f.write(f"{name} {t} {pnt} {art} {ion} {ds} {pds} 0\n")
            if ion:
                f.write(f"{charge}\n")
    # globals.dat
    with open(os.path.join(path, "globals.dat"), "w") as f:
        f.write(f"{VERSION}\n")
        f.write(f"celsius {g.celsius:.17g}\n")
        f.write(f"dt {g.dt:.17g}\n")
        f.write("0 0\n")
        f.write("secondorder 0\n")

    chk = [0]
    ncell = g.ncell
    nstim = g.netstim.n
    npre = ncell + nstim
    e1, e2 = g.expsyn, g.exp2syn
    nc_src = np.concatenate([e1.ifields["src"], e2.ifields["src"]]).astype(np.int32)
    nc_type = np.concatenate([np.full(e1.n, TYPE["ExpSyn"]), np.full(e2.n, TYPE["Exp2Syn"])]).astype(np.int32)
    nc_index = np.concatenate([np.arange(e1.n), np.arange(e2.n)]).astype(np.int32)
    nc_w = np.concatenate([e1.fields["weight"], e2.fields["weight"]])
    nc_d = np.concatenate([e1.fields["delay"], e2.fields["delay"]])
    # <id>_1.dat: PreSyns (cells, then NetStims; gid = index) and NetCon sources
    w = _Writer(os.path.join(path, f"{file_id}_1.dat"))
    w.line(VERSION)
    w.line(npre)  # n_presyn
    w.line(nc_src.shape[0])  # n_netcon
    w.array(chk, np.arange(npre, dtype=np.int32))  # output_gid
    w.array(chk, nc_src)  # netcon_srcgid
    w.close()

    # mechanism instance tables in type order
    hh, pas, ic = g.hh, g.pas, g.iclamp
    mechs = []  # (name, nodes, data[n, ds], pdata[n, pds] or None)
    mechs.append(("capacitance", np.arange(n, dtype=np.int32),
                  np.column_stack([g.cm, np.zeros(n)]), None))
    if pas.n:
        d = np.zeros((pas.n, DSIZE["pas"]))
        d[:, 0] = pas.fields["g"]
        d[:, 1] = pas.fields["e"]
        mechs.append(("pas", pas.nodes, d, None))
    if hh.n:
        for ion, key in (("na_ion", "ena"), ("k_ion", "ek")):
            d = np.zeros((hh.n, DSIZE[ion]))
            d[:, 0] = hh.fields[key]
            mechs.append((ion, hh.nodes, d, np.zeros((hh.n, 1), dtype=np.int32)))
        d = np.zeros((hh.n, DSIZE["hh"]))
        d[:, 0] = hh.fields["gnabar"]
        d[:, 1] = hh.fields["gkbar"]
        d[:, 2] = hh.fields["gl"]
        d[:, 3] = hh.fields["el"]
        d[:, 19] = hh.fields["ena"]
        d[:, 20] = hh.fields["ek"]
        mechs.append(("hh", hh.nodes, d, None))
    npnt = [0]

    def point(name, tab, cols, pointer=None, nodes=None):
        if not tab.n:
            return
        d = np.zeros((tab.n, DSIZE[name]))
        for c, key in cols:
            d[:, c] = tab.fields[key]
        pd = np.zeros((tab.n, PDSIZE[name]), dtype=np.int32)
        pd[:, 0] = tab.nodes if nodes is None else 0  # area of the node
        pd[:, 1] = np.arange(tab.n) + npnt[0]  # point-process slot in vdata
        if pointer is not None:
            pd[:, 2] = pointer
        npnt[0] += tab.n
        mechs.append((name, tab.nodes if nodes is None else nodes, d, pd))

    point("IClamp", ic, ((0, "del"), (1, "dur"), (2, "amp")))
    point("ExpSyn", e1, ((0, "tau"), (1, "e")))
    point("Exp2Syn", e2, ((0, "tau1"), (1, "tau2"), (2, "e")))
    point("NetStim", g.netstim, ((0, "interval"), (1, "number"), (2, "start"), (3, "noise")),
          nodes=np.zeros(0, dtype=np.int32))
    point("HalfGap", g.halfgap, ((0, "g"),))
    point("gapjunction_lr", g.gapjunction, ((0, "g"), (1, "w")), pointer=g.gapjunction.ifields["pre"])
    point("neuron_to_neuron_syn_lr", g.graded, ((0, "w"), (1, "g"), (2, "delta"), (3, "k"), (4, "Vth"), (5, "erev"),
                                                (6, "dvpre")), pointer=g.graded.ifields["pre"])
    npnt = npnt[0]
    counts = {name: (g.netstim.n if name == "NetStim" else int(nodes.shape[0])) for name, nodes, _, _ in mechs}

    # <id>_2.dat
    w = _Writer(os.path.join(path, f"{file_id}_2.dat"))
    w.line(VERSION)
    w.line(ncell)  # n_real_cell
    w.line(npre)  # n_outputgid (= n_presyn)
    w.line(ncell)  # n_real_output
    w.line(n)  # n_node
    w.line(0)  # n_diam
    w.line(len(mechs))
    for name, nodes, _, _ in mechs:
        w.line(TYPE[name])
        w.line(counts[name])
    w.line(0)  # nidata
    w.line(npnt)  # nvdata
    w.line(nc_src.shape[0])  # n_weight (pnt_receive_size 1 for ExpSyn and Exp2Syn)
    w.array(chk, g.parent.astype(np.int32))
    w.array(chk, g.a.astype(np.float64))
    w.array(chk, g.b.astype(np.float64))
    w.array(chk, g.area.astype(np.float64))
    w.array(chk, np.full(n, g.v_init, dtype=np.float64))
    for name, nodes, data, pdata in mechs:
        if name != "NetStim":  # artificial cells have no nodeindices (read_coredat.cpp:748-757)
            w.array(chk, np.ascontiguousarray(nodes, dtype=np.int32))
        w.array(chk, np.ascontiguousarray(data, dtype=np.float64).reshape(-1))
        if PDSIZE[name]:
            w.array(chk, np.ascontiguousarray(pdata, dtype=np.int32).reshape(-1))
            w.line(0)  # pointer2type size
            w.line(0)  # nmodlrandom size
    ovi = np.concatenate([np.arange(ncell), -(TYPE["NetStim"] + USER_MOD_NUM * np.arange(nstim))]).astype(np.int32)
    w.array(chk, ovi)  # output_vindex: root node of each cell, encoded NetStim instances
    w.array(chk, np.ascontiguousarray(g.ps_thresh, dtype=np.float64))  # output_threshold (real cells)
    w.array(chk, nc_type)  # pnttype
    w.array(chk, nc_index)  # pntindex
    w.array(chk, np.ascontiguousarray(nc_w, dtype=np.float64))  # weights
    w.array(chk, np.ascontiguousarray(nc_d, dtype=np.float64))  # delay
    w.line(0)  # BBCOREPOINTER count
    w.line(0)  # VecPlayContinuous count
    w.close()
    if g.halfgap.n:
        np.column_stack([np.arange(g.halfgap.n), g.halfgap.ifields["src"]]).astype(np.int32).tofile(
            os.path.join(path, "halfgap.i32"))
    return path
