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
gapjunction_lr.cu:47-53, gapjunction_noptr.cu:28-31,
neuron_to_neuron_syn_lr.cu:70-86); the remaining
columns of NEURON's layouts are written as zeros.  Ion instances (na_ion, k_ion)
sit on every hh node and carry the reversal potentials; their ``iontype``
flags are 0 (fixed reversal potentials, eion.cuh:155-197).  Every cell gets a
spike-source PreSyn at its root (gid = cell index, threshold ``ps_thresh``),
which the loader requires for each real cell (read_coredat.cpp:911-915);
NetStim j gets PreSyn ``ncell + j`` (gid ``ncell + j``).  Point processes carry
dparams (area node, point-process slot[, POINTER target node]); POINTERs of
gapjunction_lr / neuron_to_neuron_syn_lr are voltages (empty pointer2type,
mech_template.cuh:431-455).  One NetCon per ExpSyn / Exp2Syn instance, ExpSyn
targets first, in instance order.  HalfGap's vgap and gapjunction_noptr's
vpre are not in the files: the reference wires them through
Simulate::add_gap_source/add_gap_target (simulate.cpp:995-1056);
``write_coredat`` writes the (instance, source node) pairs to ``halfgap.i32``
and ``gapnoptr.i32`` for a driver to replay.
"""
from __future__ import annotations

import os
import struct
from typing import List, Tuple

import numpy as np

from .model import LIB_GLOBALS, CellGroup

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
    (14, "gapjunction_noptr", 7, 0, 0, 4, 2, 0.0),
    (15, "neuron_to_neuron_syn_lr", 8, 0, 0, 19, 3, 0.0),
]
# library mechanisms (written only for groups that carry them): ca_ion and the
# user-mech channel set; dsize covers the columns var_in_coredata_idx reads
# (CaDynamics_E2.cu:57-66, CA_HVA.cu, Ca_LVAst.cu, Im.cu, K_Pst.cu, K_Tst.cu,
# NaTg.cu:62-70, Nap_Et2.cu, SK_E2.cu:58-62, SKv3_1.cu)
LIB_MECH_TABLE: List[Tuple[int, str, int, int, int, int, int, float]] = [
    (16, "ca_ion", 0, 0, 1, 5, 1, 2.0),
    (17, "CaDynamics_E2", 0, 0, 0, 6, 0, 0.0),
    (18, "Ca_HVA", 0, 0, 0, 15, 0, 0.0),
    (19, "Ca_LVAst", 0, 0, 0, 10, 0, 0.0),
    (20, "Im", 0, 0, 0, 9, 0, 0.0),
    (21, "K_Pst", 0, 0, 0, 10, 0, 0.0),
    (22, "K_Tst", 0, 0, 0, 10, 0, 0.0),
    (23, "NaTg", 0, 0, 0, 9, 0, 0.0),
    (24, "Nap_Et2", 0, 0, 0, 5, 0, 0.0),
    (25, "SK_E2", 0, 0, 0, 4, 0, 0.0),
    (26, "SKv3_1", 0, 0, 0, 4, 0, 0.0),
    (27, "hd_la", 0, 0, 0, 11, 0, 0.0),
    (28, "km_la", 0, 0, 0, 13, 0, 0.0),
    (29, "kca_la", 0, 0, 0, 14, 0, 0.0),
    (30, "it2_la", 0, 0, 0, 16, 0, 0.0),
    (31, "kdr_la", 0, 0, 0, 8, 0, 0.0),
    (32, "sca_la", 0, 0, 0, 18, 0, 0.0),
    (33, "Ca", 0, 0, 0, 14, 0, 0.0),
    (34, "shl1_lr", 0, 0, 0, 24, 0, 0.0),
    (35, "kvs1_lr", 0, 0, 0, 20, 0, 0.0),
    (36, "irk_lr", 0, 0, 0, 16, 0, 0.0),
    (37, "egl36_lr", 0, 0, 0, 24, 0, 0.0),
    (38, "shk1_lr", 0, 0, 0, 20, 0, 0.0),
    (39, "egl2_lr", 0, 0, 0, 16, 0, 0.0),
    (40, "cca1_lr", 0, 0, 0, 20, 0, 0.0),
    (41, "egl19_lr", 0, 0, 0, 20, 0, 0.0),
    (42, "unc2_lr", 0, 0, 0, 20, 0, 0.0),
    (43, "kcnl_lr", 0, 0, 0, 16, 0, 0.0),
    (44, "nca_lr", 0, 0, 0, 9, 0, 0.0),
    (45, "kqt3_lr", 0, 0, 0, 27, 0, 0.0),
    (46, "cainternm_lr", 0, 0, 0, 6, 0, 0.0),
    (47, "shl1", 0, 0, 0, 12, 0, 0.0),
    (48, "kvs1", 0, 0, 0, 9, 0, 0.0),
    (49, "irk", 0, 0, 0, 6, 0, 0.0),
    (50, "egl36", 0, 0, 0, 12, 0, 0.0),
    (51, "shk1", 0, 0, 0, 9, 0, 0.0),
    (52, "egl2", 0, 0, 0, 6, 0, 0.0),
    (53, "cca1", 0, 0, 0, 9, 0, 0.0),
    (54, "egl19", 0, 0, 0, 9, 0, 0.0),
    (55, "unc2", 0, 0, 0, 9, 0, 0.0),
]
# data column of each library field (its var_in_coredata_idx); SK_E2.zTau is
# the GLOBAL zTau_SK_E2 of globals.dat (SK_E2.cu:65-66)
LIB_COLUMNS = {
    "CaDynamics_E2": {"gamma": 0, "decay": 1, "depth": 2, "minCai": 3},
    "Ca_HVA": {"gbar": 0}, "Ca_LVAst": {"gCa_LVAstbar": 0}, "Im": {"gImbar": 0}, "K_Pst": {"gK_Pstbar": 0},
    "K_Tst": {"gK_Tstbar": 0},
    "NaTg": {"gNaTgbar": 0, "vshifth": 1, "vshiftm": 2, "slopeh": 3, "slopem": 4},
    "Nap_Et2": {"gNap_Et2bar": 0}, "SK_E2": {"gSK_E2bar": 0}, "SKv3_1": {"gSKv3_1bar": 0},
    "hd_la": {"ghdbar": 0, "vhalfl": 1, "tau": 2}, "km_la": {"gbar": 0}, "kca_la": {"gbar": 0},
    "it2_la": {"gcabar": 0}, "kdr_la": {"gbar": 0}, "sca_la": {"inactF": 0, "actF": 1, "gbar": 2},
    "Ca": {"gCabar": 0},
    "shl1_lr": {"gbshl1": 0, "ek_tmp": 1, "w": 2, "dv": 3},
    "kvs1_lr": {"gbkvs1": 0, "ek_tmp": 1, "w": 2, "dv": 3},
    "irk_lr": {"gbirk": 0, "ek_tmp": 1, "w": 2, "dv": 3},
    "egl36_lr": {"gbegl36": 0, "ek_tmp": 1, "w": 2, "dv": 3},
    "shk1_lr": {"gbshk1": 0, "ek_tmp": 1, "w": 2, "dv": 3},
    "egl2_lr": {"gbegl2": 0, "ek_tmp": 1, "w": 2, "dv": 3},
    "cca1_lr": {"gbcca1": 0, "eca_tmp": 1, "w": 2, "dv": 3},
    "egl19_lr": {"gbegl19": 0, "eca_tmp": 1, "w": 2, "dv": 3},
    "unc2_lr": {"gbunc2": 0, "eca_tmp": 1, "w": 2, "dv": 3},
    "kcnl_lr": {"gbkcnl": 0, "w": 1, "dv": 2},
    "nca_lr": {"gbnca": 0, "ena_tmp": 1, "w": 2},
    "kqt3_lr": {"gbkqt3": 0, "ek_tmp": 1, "w": 2, "dv": 3},
    "cainternm_lr": {"vcell": 0},
    "shl1": {"gbshl1": 0}, "kvs1": {"gbkvs1": 0}, "irk": {"gbirk": 0}, "egl36": {"gbegl36": 0},
    "shk1": {"gbshk1": 0}, "egl2": {"gbegl2": 0}, "cca1": {"gbcca1": 0}, "egl19": {"gbegl19": 0},
    "unc2": {"gbunc2": 0},
}
# GLOBALs the loader requires of a mechanism that the dynamics do not read
# (km_la.cu:70-80: its table parameters), written with these values
LIB_EXTRA_GLOBALS = {"km_la": {"temp": 23.0, "q10": 2.3, "vmin": -120.0, "vmax": 100.0, "usetable": 0.0},
                     "kca_la": {"q10": 2.3, "temp": 23.0, "vmin": -120.0, "vmax": 100.0},
                     "it2_la": {"vmin": -120.0, "vmax": 100.0, "cao": 2.0, "cai": 2.4e-4},
                     "sca_la": {"temp": 23.0, "q10": 2.3, "vmin": -120.0, "vmax": 100.0, "cao": 2.5, "cai": 1e-4,
                                "usetable": 0.0}}
# ca_ion iontype with Nernst reversal potentials at finitialize and every step
# (eion.cuh:165, 181: bits 040 and 0100)
IONTYPE_NERNST = 0o140
# a NetStim's PreSyn is written as output_vindex -(type + USER_MOD_NUM * index)
# (read_coredat.cpp:930-940 with the loader's default user_mod_num 1000)
USER_MOD_NUM = 1000
TYPE = {m[1]: m[0] for m in MECH_TABLE + LIB_MECH_TABLE}
DSIZE = {m[1]: m[5] for m in MECH_TABLE + LIB_MECH_TABLE}
PDSIZE = {m[1]: m[6] for m in MECH_TABLE + LIB_MECH_TABLE}



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
    table = MECH_TABLE + (LIB_MECH_TABLE if g.lib else [])
    with open(os.path.join(path, "bbcore_mech.dat"), "w") as f:
        f.write(f"{VERSION}\n{table[-1][0] + 1}\n")
        for (t, name, pnt, art, ion, ds, pds, charge) in table:
            f.write(f"{name} {t} {pnt} {art} {ion} {ds} {pds} 0\n")
            if ion:
                f.write(f"{charge}\n")
    # globals.dat
    with open(os.path.join(path, "globals.dat"), "w") as f:
        f.write(f"{VERSION}\n")
        f.write(f"celsius {g.celsius:.17g}\n")
        f.write(f"dt {g.dt:.17g}\n")
        for nm, keys in LIB_GLOBALS.items():
            tab = g.lib.get(nm)
            if tab is None or not tab.n:
                continue
            for k in keys:
                f.write(f"{k}_{nm} {float(tab.fields[k][0]):.17g}\n")
            for k, val in LIB_EXTRA_GLOBALS.get(nm, {}).items():
                f.write(f"{k}_{nm} {val:.17g}\n")
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
    for ion, key in (("na_ion", "ena"), ("k_ion", "ek")):
        # instances on the hh nodes and the library's ion nodes (equal erev where both)
        lt = g.lib.get(ion)
        nodes = np.union1d(hh.nodes, lt.nodes if lt is not None else np.zeros(0, np.int32)).astype(np.int32)
        if not nodes.size:
            continue
        d = np.zeros((nodes.size, DSIZE[ion]))
        d[np.searchsorted(nodes, hh.nodes), 0] = hh.fields[key]
        if lt is not None and lt.n:
            d[np.searchsorted(nodes, lt.nodes), 0] = lt.fields[key]
        mechs.append((ion, nodes, d, np.zeros((nodes.size, 1), dtype=np.int32)))
    if hh.n:
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
    point("gapjunction_noptr", g.gapnoptr, ((0, "weight"),))
    point("neuron_to_neuron_syn_lr", g.graded, ((0, "w"), (1, "g"), (2, "delta"), (3, "k"), (4, "Vth"), (5, "erev"),
                                                (6, "dvpre")), pointer=g.graded.ifields["pre"])
    npnt = npnt[0]
    ca = g.lib.get("ca_ion")
    if ca is not None and ca.n:
        d = np.zeros((ca.n, DSIZE["ca_ion"]))
        d[:, 0], d[:, 1], d[:, 2] = ca.fields["eca"], ca.fields["cai"], ca.fields["cao"]
        it = np.where(ca.ifields["nernst"] != 0, IONTYPE_NERNST, 0).astype(np.int32).reshape(-1, 1)
        mechs.append(("ca_ion", ca.nodes, d, it))
    for name, cols in LIB_COLUMNS.items():
        tab = g.lib.get(name)
        if tab is None or not tab.n:
            continue
        d = np.zeros((tab.n, DSIZE[name]))
        for key, c in cols.items():
            d[:, c] = tab.fields[key]
        mechs.append((name, tab.nodes, d, None))
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
    for tab, fname in ((g.halfgap, "halfgap.i32"), (g.gapnoptr, "gapnoptr.i32")):
        if tab.n:
            np.column_stack([np.arange(tab.n), tab.ifields["src"]]).astype(np.int32).tofile(os.path.join(path, fname))
    return path


# ---------------------------------------------------------------- reader
class _Reader:
    def __init__(self, path: str):
        with open(path, "rb") as f:
            self.b = f.read()
        self.pos = 0
        self.path = path

    def line(self) -> str:
        end = self.b.index(b"\n", self.pos)
        s = self.b[self.pos:end].decode()
        self.pos = end + 1
        return s

    def int(self) -> int:
        return int(self.line().split()[0])

    def array(self, chk: List[int], dtype, count: int) -> np.ndarray:
        tag = self.line()
        if tag != f"chkpnt {chk[0]}":
            raise ValueError(f"{self.path}: expected 'chkpnt {chk[0]}', found {tag!r}")
        chk[0] += 1
        dt = np.dtype(dtype)
        a = np.frombuffer(self.b, dtype=dt, count=count, offset=self.pos).copy()
        self.pos += count * dt.itemsize
        return a


def read_coredat(path: str, file_id=None) -> CellGroup:
    """Load a CoreNEURON data directory (version 1.8 files) as a ``CellGroup``.

    Reads what ``write_coredat`` writes, in the order the reference's loader
    reads it (read_filesdat, read_mech, global_vars, read_phase1,
    read_phase2; src/io/read_coredat.cpp:258-1120): the node arrays, the
    capacitance, pas, na_ion / k_ion, hh, IClamp, ExpSyn, Exp2Syn, NetStim,
    HalfGap, gapjunction_lr, gapjunction_noptr and neuron_to_neuron_syn_lr instances, the
    library mechanisms (ca_ion, CaDynamics_E2 and the user-mech channel set),
    the PreSyns and one NetCon per ExpSyn / Exp2Syn instance.  HalfGap sources
    and gapjunction_noptr sources come from ``halfgap.i32`` / ``gapnoptr.i32``
    when present.  A file with other mechanisms, more
    than one NetCon on a synapse instance, per-node initial voltages or
    playback vectors is rejected with a ValueError naming what is not
    supported.  ``file_id``: the group to read (default: the only one listed in
    files.dat).
    """
    from .model import MechTable, _f64, _i32, empty_table, EXPSYN_FIELDS, EXP2SYN_FIELDS, NETSTIM_FIELDS, \
        HALFGAP_FIELDS, GAPJ_FIELDS, GAPNP_FIELDS, GRADED_FIELDS

    with open(os.path.join(path, "files.dat")) as f:
        toks = f.read().split()
    if toks[0] != VERSION:
        raise ValueError(f"files.dat version {toks[0]} (supported: {VERSION})")
    ngroup = int(toks[1])
    ids = [int(t) for t in toks[2:2 + ngroup]]
    if file_id is None:
        if len(ids) != 1:
            raise ValueError(f"files.dat lists {len(ids)} groups; pass file_id")
        file_id = ids[0]
    elif file_id not in ids:
        raise ValueError(f"group {file_id} not in files.dat")
    # bbcore_mech.dat: name type pnttype is_art is_ion dsize pdsize ...
    mech = {}
    with open(os.path.join(path, "bbcore_mech.dat")) as f:
        lines = [l for l in f.read().splitlines() if l.strip()]
    if lines[0].strip() != VERSION:
        raise ValueError(f"bbcore_mech.dat version {lines[0].strip()} (supported: {VERSION})")
    k = 2
    while k < len(lines):
        t = lines[k].split()
        name, typ, art, ion, ds, pds = t[0], int(t[1]), int(t[3]), int(t[4]), int(t[5]), int(t[6])
        mech[typ] = (name, art, ds, pds)
        k += 2 if ion else 1
    # globals.dat: "name value" lines up to "0 0", then "secondorder n"
    glob = {}
    with open(os.path.join(path, "globals.dat")) as f:
        glines = f.read().splitlines()
    for l in glines[1:]:
        t = l.split()
        if len(t) == 2 and t[0] == "0" and t[1] == "0":
            break
        if len(t) == 2:
            glob[t[0]] = float(t[1])

    chk = [0]
    r1 = _Reader(os.path.join(path, f"{file_id}_1.dat"))
    r1.line()
    n_presyn, n_netcon = r1.int(), r1.int()
    output_gid = r1.array(chk, np.int32, n_presyn)
    netcon_srcgid = r1.array(chk, np.int32, n_netcon)

    r = _Reader(os.path.join(path, f"{file_id}_2.dat"))
    r.line()
    ncell, n_outputgid, n_real_output, n = r.int(), r.int(), r.int(), r.int()
    n_diam, n_mech = r.int(), r.int()
    mtc = [(r.int(), r.int()) for _ in range(n_mech)]
    r.int()  # nidata
    r.int()  # nvdata
    n_weight = r.int()
    parent = r.array(chk, np.int32, n)
    a = r.array(chk, np.float64, n)
    b = r.array(chk, np.float64, n)
    area = r.array(chk, np.float64, n)
    v = r.array(chk, np.float64, n)
    if n_diam > 0:
        r.array(chk, np.float64, n)
    tabs = {}
    for typ, cnt in mtc:
        if typ not in mech:
            raise ValueError(f"mechanism type {typ} is not in bbcore_mech.dat")
        name, art, ds, pds = mech[typ]
        if name not in DSIZE:
            raise ValueError(f"mechanism {name} is not supported by heliox_b200")
        # artificial cells have no node (the model keeps node 0 as a placeholder)
        nodes = np.zeros(cnt, dtype=np.int32) if art else r.array(chk, np.int32, cnt)
        data = r.array(chk, np.float64, cnt * ds).reshape(cnt, ds) if ds else np.zeros((cnt, 0))
        pdata = None
        if pds:
            pdata = r.array(chk, np.int32, cnt * pds).reshape(cnt, pds)
            if r.int() != 0:
                raise ValueError(f"{name}: pointer2type entries are not supported")
            if r.int() != 0:
                raise ValueError(f"{name}: nmodlrandom entries are not supported")
        tabs[name] = (nodes, data, pdata)
    output_vindex = r.array(chk, np.int32, n_outputgid)
    output_threshold = r.array(chk, np.float64, n_real_output)
    pnttype = r.array(chk, np.int32, n_netcon)
    pntindex = r.array(chk, np.int32, n_netcon)
    weights = r.array(chk, np.float64, n_weight)
    delay = r.array(chk, np.float64, n_netcon)
    if r.int() != 0:
        raise ValueError("BBCOREPOINTER data is not supported")
    if r.int() != 0:
        raise ValueError("VecPlayContinuous playback is not supported")
    if n_weight != n_netcon:
        raise ValueError("only NetCons with one weight (ExpSyn, Exp2Syn targets) are supported")
    if n and not np.all(v == v[0]):
        raise ValueError("per-node initial voltages are not supported (one v_init per group)")

    def tab(name, cols, fields, inames=(), ifill=None):
        if name not in tabs:
            return empty_table(fields, inames)
        nodes, data, pdata = tabs[name]
        fl = {key: _f64(data[:, c]) for c, key in cols}
        for key in fields:
            fl.setdefault(key, _f64(np.zeros(data.shape[0])))
        ifl = {key: _i32(np.zeros(data.shape[0])) for key in inames}
        if ifill:
            ifl.update(ifill(pdata))
        return MechTable(_i32(nodes), fl, ifl)

    cm = tabs["capacitance"][1][:, 0].copy() if "capacitance" in tabs else np.ones(n)
    hh = tab("hh", ((0, "gnabar"), (1, "gkbar"), (2, "gl"), (3, "el"), (19, "ena"), (20, "ek")),
             ("gnabar", "gkbar", "gl", "el", "ena", "ek"))
    # the ions carry the reversal potentials the hh instances use
    for ion, key in (("na_ion", "ena"), ("k_ion", "ek")):
        if ion in tabs and hh.n:
            inodes, idata, _ = tabs[ion]
            pos = {int(x): i for i, x in enumerate(inodes)}
            hh.fields[key] = _f64([idata[pos[int(x)], 0] for x in hh.nodes])
    pas = tab("pas", ((0, "g"), (1, "e")), ("g", "e"))
    iclamp = tab("IClamp", ((0, "del"), (1, "dur"), (2, "amp")), ("del", "dur", "amp"))
    expsyn = tab("ExpSyn", ((0, "tau"), (1, "e")), EXPSYN_FIELDS, ("src",))
    exp2syn = tab("Exp2Syn", ((0, "tau1"), (1, "tau2"), (2, "e")), EXP2SYN_FIELDS, ("src",))
    netstim = tab("NetStim", ((0, "interval"), (1, "number"), (2, "start"), (3, "noise")), NETSTIM_FIELDS)
    halfgap = tab("HalfGap", ((0, "g"),), HALFGAP_FIELDS, ("src",))
    gapj = tab("gapjunction_lr", ((0, "g"), (1, "w")), GAPJ_FIELDS, ("pre",),
               lambda pd: {"pre": _i32(pd[:, 2])})
    gapnp = tab("gapjunction_noptr", ((0, "weight"),), GAPNP_FIELDS, ("src",))
    graded = tab("neuron_to_neuron_syn_lr", ((0, "w"), (1, "g"), (2, "delta"), (3, "k"), (4, "Vth"), (5, "erev"),
                                             (6, "dvpre")), GRADED_FIELDS, ("pre",),
                 lambda pd: {"pre": _i32(pd[:, 2])})
    # PreSyns: real cells (output_vindex >= 0, the root node) then artificial
    # cells (-(type + USER_MOD_NUM * index)); NetCon sources map to cell index /
    # ncell + NetStim index
    src_of_gid = {}
    for i in range(n_presyn):
        ov = int(output_vindex[i])
        if ov >= 0:
            if ov >= ncell or parent[ov] >= 0:
                raise ValueError("a PreSyn not at a cell root is not supported")
            src_of_gid[int(output_gid[i])] = ov
        else:
            typ, idx = (-ov) % USER_MOD_NUM, (-ov) // USER_MOD_NUM
            if mech.get(typ, ("",))[0] != "NetStim":
                raise ValueError("artificial-cell PreSyns other than NetStim are not supported")
            src_of_gid[int(output_gid[i])] = ncell + idx
    ps_thresh = np.full(ncell, 10.0)
    for i in range(min(n_real_output, n_presyn)):
        ov = int(output_vindex[i])
        if 0 <= ov < ncell:
            ps_thresh[ov] = output_threshold[i]
    seen = {TYPE["ExpSyn"]: np.zeros(expsyn.n, bool), TYPE["Exp2Syn"]: np.zeros(exp2syn.n, bool)}
    for j in range(n_netcon):
        t, idx = int(pnttype[j]), int(pntindex[j])
        name = mech.get(t, ("",))[0]
        if name not in ("ExpSyn", "Exp2Syn"):
            raise ValueError(f"NetCon target {name or t} is not supported")
        tb = expsyn if name == "ExpSyn" else exp2syn
        if seen[TYPE[name]][idx]:
            raise ValueError(f"more than one NetCon on {name} instance {idx} is not supported")
        seen[TYPE[name]][idx] = True
        g_src = int(netcon_srcgid[j])
        if g_src not in src_of_gid:
            raise ValueError(f"NetCon source gid {g_src} has no PreSyn in this group")
        tb.ifields["src"][idx] = src_of_gid[g_src]
        tb.fields["weight"][idx] = weights[j]
        tb.fields["delay"][idx] = delay[j]
    for name, s in seen.items():
        if not s.all():
            raise ValueError("a synapse instance without a NetCon is not supported")
    for tb, fname in ((halfgap, "halfgap.i32"), (gapnp, "gapnoptr.i32")):
        wpath = os.path.join(path, fname)
        if tb.n and os.path.exists(wpath):
            pairs = np.fromfile(wpath, dtype=np.int32).reshape(-1, 2)
            tb.ifields["src"][pairs[:, 0]] = pairs[:, 1]
    lib = _read_lib(tabs, glob)
    g = CellGroup(ncell=int(ncell), parent=_i32(parent), a=_f64(a), b=_f64(b), area=_f64(area), cm=_f64(cm),
                  hh=hh, pas=pas, iclamp=iclamp, celsius=glob.get("celsius", 6.3), dt=glob.get("dt", 0.025),
                  v_init=float(v[0]) if n else -65.0, name=os.path.basename(os.path.normpath(path)),
                  expsyn=expsyn, exp2syn=exp2syn, netstim=netstim, halfgap=halfgap, gapjunction=gapj,
                  gapnoptr=gapnp, graded=graded, ps_thresh=_f64(ps_thresh), lib=lib)
    g.validate()
    return g


def _read_lib(tabs, glob):
    """Library tables of a read group: the channels and CaDynamics_E2 from
    their data columns, ca_ion from the ion layout (eion.cuh:81-86) and its
    iontype (04: default concentrations at finitialize, 040 / 0100: Nernst
    eca at finitialize / every step, eion.cuh:155-186), na_ion / k_ion on the
    nodes of the library channels that use them."""
    import math

    from .model import LIB_IONS, MechTable, _f64, _i32

    lib = {}
    for name, cols in LIB_COLUMNS.items():
        if name not in tabs:
            continue
        nodes, data, _ = tabs[name]
        fl = {key: _f64(data[:, c]) for key, c in cols.items()}
        for k in LIB_GLOBALS.get(name, ()):
            if f"{k}_{name}" not in glob:
                raise ValueError(f"{name} needs the GLOBAL {k}_{name} in globals.dat")
            fl[k] = _f64(np.full(nodes.size, glob[f"{k}_{name}"]))
        lib[name] = MechTable(_i32(nodes), fl)
    if not lib:
        return lib
    if "ca_ion" in tabs:
        nodes, data, pdata = tabs["ca_ion"]
        it = pdata[:, 0] if pdata is not None else np.zeros(nodes.size, np.int32)
        eca, cai, cao = data[:, 0].copy(), data[:, 1].copy(), data[:, 2].copy()
        dflt = (it & 0o4) != 0
        cai[dflt], cao[dflt] = 5.e-5, 2.0
        every = (it & 0o100) != 0
        once = ((it & 0o40) != 0) & ~every
        if once.any():  # Nernst at finitialize only: a fixed eca from the initial concentrations
            ktf = 1000. * (1.380649e-23 * 6.02214076e+23) * (glob.get("celsius", 6.3) + 273.15) / (
                1.602176634e-19 * 6.02214076e+23)
            for j in np.nonzero(once)[0]:
                eca[j] = 1e6 if cai[j] <= 0. else -1e6 if cao[j] <= 0. else ktf / 2.0 * math.log(cao[j] / cai[j])
        lib["ca_ion"] = MechTable(_i32(nodes), {"cai": _f64(cai), "cao": _f64(cao), "eca": _f64(eca)},
                                  {"nernst": _i32(every.astype(np.int32))})
    for ion, key, tag in (("na_ion", "ena", "na"), ("k_ion", "ek", "k")):
        users = [lib[m].nodes for m, ions in LIB_IONS.items() if m in lib and tag in ions]
        if not users or ion not in tabs:
            continue
        want = np.unique(np.concatenate(users))
        nodes, data, _ = tabs[ion]
        keep = np.isin(nodes, want)
        lib[ion] = MechTable(_i32(nodes[keep]), {key: _f64(data[keep, 0])})
    return lib
