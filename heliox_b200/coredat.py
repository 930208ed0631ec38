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
iclamp_templated.cu:25-27, capac.cpp:29, eion.cuh:81-86); the remaining
columns of NEURON's layouts are written as zeros.  Ion instances (na_ion, k_ion)
sit on every hh node and carry the reversal potentials; their ``iontype``
flags are 0 (fixed reversal potentials, eion.cuh:155-197).  Every cell gets a
spike-source PreSyn at its root (gid = cell index, threshold 10 mV), which the
loader requires for each real cell (read_coredat.cpp:911-915).
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
]
TYPE = {m[1]: m[0] for m in MECH_TABLE}
DSIZE = {m[1]: m[5] for m in MECH_TABLE}
PDSIZE = {m[1]: m[6] for m in MECH_TABLE}

SPIKE_THRESHOLD = 10.0


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
    # <id>_1.dat: one PreSyn per cell (gid = cell index), no NetCons
    w = _Writer(os.path.join(path, f"{file_id}_1.dat"))
    w.line(VERSION)
    w.line(ncell)  # n_presyn
    w.line(0)  # n_netcon
    w.array(chk, np.arange(ncell, dtype=np.int32))  # output_gid
    w.array(chk, np.zeros(0, dtype=np.int32))  # netcon_srcgid
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
    npnt = 0
    if ic.n:
        d = np.zeros((ic.n, DSIZE["IClamp"]))
        d[:, 0] = ic.fields["del"]
        d[:, 1] = ic.fields["dur"]
        d[:, 2] = ic.fields["amp"]
        pd = np.zeros((ic.n, 2), dtype=np.int32)
        pd[:, 0] = ic.nodes  # area of the node
        pd[:, 1] = np.arange(ic.n) + npnt  # point-process slot in vdata
        npnt += ic.n
        mechs.append(("IClamp", ic.nodes, d, pd))

    # <id>_2.dat
    w = _Writer(os.path.join(path, f"{file_id}_2.dat"))
    w.line(VERSION)
    w.line(ncell)  # n_real_cell
    w.line(ncell)  # n_outputgid (= n_presyn)
    w.line(ncell)  # n_real_output
    w.line(n)  # n_node
    w.line(0)  # n_diam
    w.line(len(mechs))
    for name, nodes, _, _ in mechs:
        w.line(TYPE[name])
        w.line(int(nodes.shape[0]))
    w.line(0)  # nidata
    w.line(npnt)  # nvdata
    w.line(0)  # n_weight
    w.array(chk, g.parent.astype(np.int32))
    w.array(chk, g.a.astype(np.float64))
    w.array(chk, g.b.astype(np.float64))
    w.array(chk, g.area.astype(np.float64))
    w.array(chk, np.full(n, g.v_init, dtype=np.float64))
    for name, nodes, data, pdata in mechs:
        w.array(chk, np.ascontiguousarray(nodes, dtype=np.int32))
        w.array(chk, np.ascontiguousarray(data, dtype=np.float64).reshape(-1))
        if PDSIZE[name]:
            w.array(chk, np.ascontiguousarray(pdata, dtype=np.int32).reshape(-1))
            w.line(0)  # pointer2type size
            w.line(0)  # nmodlrandom size
    w.array(chk, np.arange(ncell, dtype=np.int32))  # output_vindex: root node of each cell
    w.array(chk, np.full(ncell, SPIKE_THRESHOLD))  # output_threshold
    w.array(chk, np.zeros(0, dtype=np.int32))  # pnttype
    w.array(chk, np.zeros(0, dtype=np.int32))  # pntindex
    w.array(chk, np.zeros(0))  # weights
    w.array(chk, np.zeros(0))  # delay
    w.line(0)  # BBCOREPOINTER count
    w.line(0)  # VecPlayContinuous count
    w.close()
    return path
