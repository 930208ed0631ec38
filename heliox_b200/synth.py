"""Seeded synthetic cell groups for the benchmark configurations.

NEURON (the only producer of the reference's CoreNEURON input files,
``python_lib/heliox_sim/manager.py:590-630``) is not available, so the
morphology -> (parent, a, b, area) discretisation is done here from cable
theory.  The rules (written once, used by every config):

* a section of length ``L`` um and ``nseg`` segments contributes ``nseg``
  compartments, each a cylinder of length ``L/nseg`` whose diameter is the
  section's diameter profile evaluated at the segment centre;
* ``area = pi * d * dx`` (um^2);
* the axial resistance between a node and its parent is the sum of the two
  half-segment resistances, ``ri = 1e-2 * Ra * (dx_i/2 / (pi r_i^2) + dx_p/2 / (pi r_p^2))``
  in MOhm (Ra in Ohm*cm, lengths in um);
* ``b[i] = -1e2 / (ri * area[i])`` and ``a[i] = -1e2 / (ri * area[parent])`` in
  S/cm^2, the NEURON sign convention the reference's matrix assembly consumes
  (``src/simulate.cpp:542-555``).

There are no zero-area section-end nodes; the reference consumes whatever arrays
it is given, so parity does not depend on this choice.
"""
from __future__ import annotations

import math
from typing import List, Tuple

import numpy as np

from .model import LIB_FIELDS, LIB_IONS, LIB_NAMES, CellGroup, MechTable, _f64, _i32, concat_groups

RA = 100.0  # Ohm*cm
HH_STD = dict(gnabar=0.12, gkbar=0.036, gl=3e-4, el=-54.3, ena=50.0, ek=-77.0)


class _Builder:
    """Accumulates compartments of one cell in a topological order."""

    def __init__(self):
        self.parent: List[int] = []
        self.dx: List[float] = []
        self.diam: List[float] = []
        self.kind: List[int] = []  # 0 soma, 1 axon/hillock, 2 dendrite
        self.path: List[float] = []  # path distance (um) of the node centre

    def add(self, parent: int, dx: float, diam: float, kind: int, path: float) -> int:
        self.parent.append(parent)
        self.dx.append(dx)
        self.diam.append(diam)
        self.kind.append(kind)
        self.path.append(path)
        return len(self.parent) - 1

    def add_section(self, parent_node: int, L: float, nseg: int, diam_fn, kind: int) -> List[int]:
        dx = L / nseg
        p0 = self.path[parent_node] if parent_node >= 0 else 0.0
        pdx = self.dx[parent_node] if parent_node >= 0 else 0.0
        nodes = []
        prev = parent_node
        for j in range(nseg):
            # centre of segment j measured from the section's 0-end
            xc = (j + 0.5) * dx
            path = p0 + 0.5 * pdx + xc
            prev = self.add(prev, dx, diam_fn(path), kind, path)
            nodes.append(prev)
        return nodes

    def finish(self) -> Tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray]:
        n = len(self.parent)
        parent = np.asarray(self.parent, dtype=np.int32)
        dx = np.asarray(self.dx)
        d = np.asarray(self.diam)
        area = math.pi * d * dx
        a = np.zeros(n)
        b = np.zeros(n)
        for i in range(1, n):
            p = parent[i]
            ri = 1e-2 * RA * (0.5 * dx[i] / (math.pi * (0.5 * d[i]) ** 2) + 0.5 * dx[p] / (math.pi * (0.5 * d[p]) ** 2))
            b[i] = -1e2 / (ri * area[i])
            a[i] = -1e2 / (ri * area[p])
        parent[0] = -1
        return parent, a, b, area


def _single_cell_group(bld: _Builder, hh_nodes, hh_par, pas_nodes, pas_par, ic, name, **kw) -> CellGroup:
    parent, a, b, area = bld.finish()
    n = len(parent)
    hh_nodes = np.asarray(hh_nodes, dtype=np.int64)
    o = np.argsort(hh_nodes, kind="stable")
    hh = MechTable(_i32(hh_nodes[o]), {k: _f64(np.asarray(v)[o]) for k, v in hh_par.items()})
    pas_nodes = np.asarray(pas_nodes, dtype=np.int64)
    o = np.argsort(pas_nodes, kind="stable")
    pas = MechTable(_i32(pas_nodes[o]), {k: _f64(np.asarray(v)[o]) for k, v in pas_par.items()})
    icl = MechTable(_i32(ic["nodes"]), {k: _f64(ic[k]) for k in ("del", "dur", "amp")})
    g = CellGroup(
        ncell=1,
        parent=parent,
        a=_f64(a),
        b=_f64(b),
        area=_f64(area),
        cm=_f64(np.ones(n)),
        hh=hh,
        pas=pas,
        iclamp=icl,
        name=name,
        **kw,
    )
    g.validate()
    return g


# ---------------------------------------------------------------- config 1
def ball_and_stick(gnabar_scale: float = 1.0, ndend: int = 100) -> CellGroup:
    """Config 1: soma (L=diam=20 um, hh) + 100-compartment dendrite (L=500, diam=1, pas).

    IClamp 0.5 nA at the soma, del 5 ms, dur 50 ms; cm 1, Ra 100, v_init -65,
    celsius 6.3 (NEURON default), ena 50, ek -77.
    """
    bld = _Builder()
    soma = bld.add(-1, 20.0, 20.0, 0, 0.0)
    dend = bld.add_section(soma, 500.0, ndend, lambda p: 1.0, 2)
    hh_par = {k: [v] for k, v in HH_STD.items()}
    hh_par["gnabar"] = [HH_STD["gnabar"] * gnabar_scale]
    pas_par = {"g": [1e-4] * len(dend), "e": [-65.0] * len(dend)}
    ic = {"nodes": [soma], "del": [5.0], "dur": [50.0], "amp": [0.5]}
    return _single_cell_group(bld, [soma], hh_par, dend, pas_par, ic, "ball_and_stick")


# ---------------------------------------------------------------- config 2/3
def random_tree_cell(
    seed: int,
    ncomp: int | None = None,
    nmin: int = 200,
    nmax: int = 1000,
    max_levels: int | None = None,
    seg_len: float = 10.0,
    amp: float | None = None,
) -> CellGroup:
    """One seeded random-tree cell.

    Soma (1 compartment, L=diam=20, standard hh) and an axon hillock section
    (L=20, diam 1.5, 4 segments, standard hh); dendritic sections of length
    U[20,200] um, each attached to the 1-end of a uniformly chosen existing
    dendrite section or the soma (subject to ``max_levels`` branch levels),
    ``nseg = max(1, round(L/seg_len))``.  Dendrite diameter tapers linearly from
    3 um at the soma to 0.3 um at the largest path distance.  Dendrites carry
    pas (g 1e-4, e -65) plus hh at 10 % of the standard conductance densities
    (gnabar, gkbar and gl scaled by 0.1).  The soma gets an IClamp with
    amplitude U[0.2, 1] nA, del 5 ms, dur 50 ms.
    """
    rng = np.random.default_rng(seed)
    if ncomp is None:
        ncomp = int(rng.integers(nmin, nmax + 1))
    if amp is None:
        amp = float(rng.uniform(0.2, 1.0))
    # --- topology of dendritic sections first (lengths, parents), then lay out
    ndend_target = ncomp - 1 - 4
    secs = []  # (parent_sec or -1 for soma, L, nseg, level)
    total = 0
    while total < ndend_target:
        if not secs or rng.random() < 0.08:
            par = -1
            lvl = 1
        else:
            cand = [i for i, s in enumerate(secs) if max_levels is None or s[3] < max_levels]
            if not cand:
                par, lvl = -1, 1
            else:
                par = int(cand[int(rng.integers(len(cand)))])
                lvl = secs[par][3] + 1
        L = float(rng.uniform(20.0, 200.0))
        nseg = max(1, int(round(L / seg_len)))
        if total + nseg > ndend_target:
            nseg = ndend_target - total
            L = nseg * seg_len
        secs.append((par, L, nseg, lvl))
        total += nseg
    # path distance of the far end of every section, to define the taper
    end_path = []
    for (par, L, nseg, lvl) in secs:
        base = 10.0 if par < 0 else end_path[par]
        end_path.append(base + L)
    pmax = max(end_path) if end_path else 1.0

    def taper(path):
        return 3.0 + (0.3 - 3.0) * min(1.0, path / pmax)

    bld = _Builder()
    soma = bld.add(-1, 20.0, 20.0, 0, 0.0)
    hill = bld.add_section(soma, 20.0, 4, lambda p: 1.5, 1)
    sec_last = []
    dend_nodes = []
    for (par, L, nseg, lvl) in secs:
        pnode = soma if par < 0 else sec_last[par]
        nodes = bld.add_section(pnode, L, nseg, taper, 2)
        sec_last.append(nodes[-1])
        dend_nodes.extend(nodes)
    hh_nodes = [soma] + hill + dend_nodes
    nh = len(hh_nodes)
    scale = np.array([1.0] * (1 + len(hill)) + [0.1] * len(dend_nodes))
    hh_par = {
        "gnabar": HH_STD["gnabar"] * scale,
        "gkbar": HH_STD["gkbar"] * scale,
        "gl": HH_STD["gl"] * scale,
        "el": np.full(nh, HH_STD["el"]),
        "ena": np.full(nh, HH_STD["ena"]),
        "ek": np.full(nh, HH_STD["ek"]),
    }
    pas_par = {"g": np.full(len(dend_nodes), 1e-4), "e": np.full(len(dend_nodes), -65.0)}
    ic = {"nodes": [soma], "del": [5.0], "dur": [50.0], "amp": [amp]}
    g = _single_cell_group(bld, hh_nodes, hh_par, dend_nodes, pas_par, ic, f"tree{seed}")
    g.meta["levels"] = max([s[3] for s in secs], default=0)
    return g


def random_tree_batch(ncell: int = 1024, seed0: int = 20240, **kw) -> CellGroup:
    """Config 2: ``ncell`` independent seeded random trees (seed ``seed0 + cell``)."""
    cells = [random_tree_cell(seed0 + c, **kw) for c in range(ncell)]
    g = concat_groups(cells, name=f"trees{ncell}")
    return g


def giant_cell(ncomp: int = 50000, max_levels: int = 40, seed: int = 7) -> CellGroup:
    """Config 3: one random tree of ``ncomp`` compartments with <= ``max_levels`` levels."""
    g = random_tree_cell(seed, ncomp=ncomp, max_levels=max_levels, seg_len=10.0, amp=0.5)
    g.name = f"giant{ncomp}"
    return g


# ---------------------------------------------------------------- library cells
# Channel densities (S/cm^2) of the user-mech channel set per region
# (soma, axon initial segment, dendrites), in the range of published layer-5
# pyramidal-cell fits; the ion parameters are the reference's ion defaults
# (eion.cuh:306-327) with ena 50, ek -85 and eca from the Nernst equation.
LIB_DENSITY = {
    "NaTg": (1.5, 3.0, 0.02),
    "Nap_Et2": (0.002, 0.006, 0.0),
    "K_Pst": (0.05, 0.9, 0.0),
    "K_Tst": (0.03, 0.08, 0.0),
    "SKv3_1": (0.3, 1.0, 0.004),
    "SK_E2": (0.05, 0.01, 0.001),
    "Im": (0.0, 0.0, 1e-4),
    "Ca_HVA": (1e-3, 1e-3, 5e-5),
    "Ca_LVAst": (3e-3, 5e-3, 1e-4),
    "hd_la": (5e-5, 0.0, 1e-4),
    "km_la": (10.0, 20.0, 0.0),  # pS/um^2 (km_la.cu:53)
    "kca_la": (5.0, 0.0, 1.0),  # pS/um^2
    "it2_la": (0.0, 0.0, 2e-4),
    "kdr_la": (0.0, 0.01, 0.0),
    "sca_la": (0.0, 0.0, 0.5),  # pS/um^2
    "Ca": (2e-4, 0.0, 0.0),
    # worm-lr channels: gb per region (w = 1 times the seeded lognormal factor)
    "shl1_lr": (1e-3, 0.0, 0.0),
    "kvs1_lr": (0.0, 0.0, 5e-5),
    "irk_lr": (1e-4, 0.0, 1e-4),
    "egl36_lr": (0.0, 0.0, 1e-4),
    "shk1_lr": (5e-4, 5e-4, 0.0),
    "egl2_lr": (0.0, 0.0, 5e-5),
    "cca1_lr": (0.0, 0.0, 1e-5),
    "egl19_lr": (0.0, 0.0, 1e-5),
    "unc2_lr": (0.0, 0.0, 1e-5),
    "kcnl_lr": (1e-4, 0.0, 1e-5),
    "nca_lr": (0.0, 0.0, 2e-6),
    "kqt3_lr": (2e-4, 0.0, 5e-5),
    # worm-mech channels: gb per region
    "shl1": (2e-4, 0.0, 0.0),
    "kvs1": (0.0, 0.0, 2e-5),
    "irk": (5e-5, 0.0, 5e-5),
    "egl36": (0.0, 0.0, 5e-5),
    "shk1": (1e-4, 1e-4, 0.0),
    "egl2": (0.0, 0.0, 2e-5),
    "cca1": (0.0, 0.0, 5e-6),
    "egl19": (0.0, 0.0, 5e-6),
    "unc2": (0.0, 0.0, 5e-6),
}
# GLOBALs of hd_la / km_la (one value per group; their published defaults,
# km_la's tadj = 2.3^((34 - 23) / 10)) and hd_la's per-instance vhalfl, tau
LIB_LA_GLOBALS = {
    "hd_la": dict(ehd=-30.0, kl=-8.0, vhalft=-75.0, a0t=0.011, zetat=2.2, gmt=0.4, q10=4.5, qtl=1.0),
    "km_la": dict(Ra=0.001, Rb=0.001, tha=-30.0, qa=9.0, tadj=2.3 ** 1.1),
    "kca_la": dict(Ra=0.01, Rb=0.02, caix=1.0, tadj=2.3 ** 1.1),
    "it2_la": dict(vshift=0.0, v12m=50.0, vwm=7.4, v12h=78.0, vwh=5.0, am=3.0, ah=85.0, vm1=25.0, vm2=100.0,
                   vh1=46.0, vh2=405.0, wm1=20.0, wm2=15.0, wh1=4.0, wh2=50.0),
    "sca_la": dict(vshift=0.0, tadj=2.3 ** 1.1),
    # kinetics of the worm-lr channels (C. elegans K currents; voltages mV, times ms)
    "shl1_lr": dict(vhm=-6.8, ka=14.1, vhh=-33.1, ki=8.3, atm=13.8, btm=-17.5, ctm=12.9, dtm=-3.7, etm=6.5, ftm=1.9,
                    athf=539.0, bthf=-28.2, cthf=4.9, dthf=27.3, aths=8422.0, bths=-37.7, cths=6.4, dths=118.9),
    "kvs1_lr": dict(vhm=57.1, ka=25.0, vhh=47.3, ki=11.1, atm=30.0, btm=18.1, ctm=20.0, dtm=1.0, ath=88.5, bth=50.0,
                    cth=-15.0, dth=53.4),
    "irk_lr": dict(vhm=-82.0, ka=13.0, atm=17.1, btm=-17.8, ctm=20.3, dtm=-43.4, etm=11.2, ftm=3.8),
    "egl36_lr": dict(vhm=63.0, ka=28.5, atms=1000.0, atmm=100.0, atmf=13.0),
    "shk1_lr": dict(vhm=20.4, ka=7.7, vhh=-7.0, ki=5.8, atm=26.6, btm=-33.7, ctm=15.8, dtm=-33.7, etm=15.4, ftm=2.0,
                    ath=1400.0),
    "egl2_lr": dict(vhm=-6.9, ka=14.9, atm=1845.8, btm=-122.6, ctm=13.8, dtm=1517.74),
    "cca1_lr": dict(vhm=-43.32, ka=7.6, vhh=-58.0, ki=7.0, atm=40.0, btm=-62.5, ctm=-12.6, dtm=0.7, ath=280.0, bth=-60.7, cth=8.5, dth=19.8),
    "egl19_lr": dict(vhm=5.6, ka=7.5, vhh=24.9, ki=12.0, vhhb=-20.5, kib=8.1, ahinf=1.43, bhinf=0.14, chinf=5.96, dhinf=0.6, atm=2.9, btm=5.2, ctm=6.0, dtm=1.9, etm=1.4, ftm=30.0, gtm=2.3, ath=0.4, bth=44.6, cth=-23.0, dth=5.0, eth=36.4, fth=28.7, gth=3.7, hth=43.1),
    "kcnl_lr": dict(kca=2e-4, a=50.0, ek_tmp=-80.0),
    "kvs1": dict(vhm=57.1, ka=25.0, vhh=47.3, ki=11.1, atm=30.0, btm=18.1, ctm=20.0, dtm=1.0, ath=88.5, bth=50.0,
                 cth=-15.0, dth=53.4),
    "kqt3_lr": dict(vhm=-12.8, ka=15.8, vhw=-1.1, kiw=28.8, aw=0.5, bw=0.5, vhs=-45.3, kis=12.3, bs=0.7,
                    atmf=395.3, btmf=38.1, ctmf=33.59, atms=5503.0, btms=-5345.4, ctms=0.02827, dtms=-23.9,
                    etms=-4590.6, ftms=0.0357, gtms=14.2, atw=0.5, btw=2.9, ctw=-48.09, dtw=48.83, ats=500.0,
                    **{"as": 0.3}),
    "unc2_lr": dict(vhm=-12.2, ka=4.0, vhh=-52.5, ki=5.6, atm=1.5, btm=-8.2, ctm=9.1, dtm=15.4, etm=0.1, ath=83.8, bth=52.9, cth=-3.5, dth=72.1, eth=23.9, fth=-3.6),
}
LIB_CADYN = (dict(gamma=5e-4, decay=460.0), dict(gamma=5e-4, decay=100.0), dict(gamma=5e-4, decay=80.0))
# cainternm_lr (the worm-lr calcium dynamics): vcell per instance, GLOBALs f, tca (ms), caeq (mM)
LIB_CAINTERNM = dict(vcell=31.16, f=0.05, tca=50.0, caeq=5e-5)
LIB_GBAR_FIELD = {nm: LIB_FIELDS[nm][0] for nm in LIB_DENSITY}


# the user-mech set the library started from (a layer-5 pyramidal-cell
# composition): bench config 6 uses it
LIB_BBP_CHANNELS = ("NaTg", "Nap_Et2", "K_Pst", "K_Tst", "SKv3_1", "SK_E2", "Im", "Ca_HVA", "Ca_LVAst")


def lib_tree_cell(seed: int, ncomp: int | None = None, nmin: int = 100, nmax: int = 400,
                  amp: float | None = None, channels=None, cadyn: str = "CaDynamics_E2") -> CellGroup:
    """One seeded random-tree cell carrying the user-mech channel set.

    The morphology is ``random_tree_cell``'s (soma, a 4-compartment axon
    initial segment, tapering dendrites).  Every compartment gets pas
    (g 3e-5, e -75); the channels of ``LIB_DENSITY`` (the user-mech set and
    hd_la, km_la, kca_la, it2_la, kdr_la, sca_la, Ca and eleven worm-lr
    channels, with the GLOBALs of
    ``LIB_LA_GLOBALS``) go where their region's density is nonzero, scaled
    by a seeded lognormal factor (sigma 0.1);
    CaDynamics_E2 sits with the Ca channels (depth 0.1 um, minCai 1e-4 mM);
    na_ion / k_ion / ca_ion sit on every compartment that a mechanism needs
    them on (ca_ion: cai 5e-5, cao 2 mM, eca by the Nernst equation each
    step).  IClamp at the soma, del 5 ms, dur 50 ms, amplitude U[0.2, 1] nA.
    celsius 34 (the channels' temperature: their rate factors hard-code it).
    ``channels``: the subset of ``LIB_DENSITY`` to place (default: all).
    ``cadyn``: the calcium dynamics on the calcium nodes, CaDynamics_E2 or
    cainternm_lr (``LIB_CAINTERNM``, vcell times a seeded lognormal factor).
    """
    rng = np.random.default_rng(seed + 7_000_000)
    base = random_tree_cell(seed, ncomp=ncomp, nmin=nmin, nmax=nmax, amp=amp)
    n = base.nnode
    region = np.full(n, 2)
    region[0] = 0
    region[1:5] = 1
    lib = {}
    need = {"na": np.zeros(n, bool), "k": np.zeros(n, bool), "ca": np.zeros(n, bool)}
    for nm, dens in LIB_DENSITY.items():
        if channels is not None and nm not in channels:
            continue
        d = np.asarray(dens)[region]
        nodes = np.nonzero(d > 0)[0]
        gbar = d[nodes] * np.exp(0.1 * rng.standard_normal(nodes.size))
        f = {LIB_GBAR_FIELD[nm]: _f64(gbar)}
        if nm.endswith("_lr"):  # w (learned) carries the seeded factor, gb the region's density
            erev = {"eca_tmp": 60.0, "ena_tmp": 30.0}
            f = {"w": _f64(gbar / d[nodes]), LIB_FIELDS[nm][1]: _f64(d[nodes])}
            for k in LIB_FIELDS[nm][2:]:
                if k.endswith("_tmp") and k not in LIB_LA_GLOBALS.get(nm, {}):
                    f[k] = _f64(np.full(nodes.size, erev.get(k, -80.0)))
                elif k == "dv":
                    f[k] = _f64(np.full(nodes.size, 1e-3))
        if nm == "NaTg":
            f.update(vshifth=_f64(np.zeros(nodes.size)), vshiftm=_f64(np.zeros(nodes.size)),
                     slopeh=_f64(np.full(nodes.size, 6.0)), slopem=_f64(np.full(nodes.size, 6.0)))
        if nm == "SK_E2":
            f["zTau"] = _f64(np.ones(nodes.size))
        if nm == "hd_la":
            f.update(vhalfl=_f64(np.full(nodes.size, -81.0)), tau=_f64(np.ones(nodes.size)))
        if nm == "sca_la":
            f.update(inactF=_f64(np.full(nodes.size, 3.0)), actF=_f64(np.ones(nodes.size)))
        for k, val in LIB_LA_GLOBALS.get(nm, {}).items():
            f[k] = _f64(np.full(nodes.size, val))
        lib[nm] = MechTable(_i32(nodes), f)
        for ion in LIB_IONS[nm]:
            need[ion][nodes] = True
    ca_nodes = np.nonzero(need["ca"])[0]
    if cadyn == "cainternm_lr":
        ci = LIB_CAINTERNM
        lib["cainternm_lr"] = MechTable(_i32(ca_nodes), {
            "vcell": _f64(ci["vcell"] * np.exp(0.1 * rng.standard_normal(ca_nodes.size))),
            **{k: _f64(np.full(ca_nodes.size, ci[k])) for k in ("f", "tca", "caeq")}})
    elif cadyn == "CaDynamics_E2":
        cad = [LIB_CADYN[r] for r in region[ca_nodes]]
        lib["CaDynamics_E2"] = MechTable(_i32(ca_nodes), {
            "gamma": _f64([c["gamma"] for c in cad]), "decay": _f64([c["decay"] for c in cad]),
            "depth": _f64(np.full(ca_nodes.size, 0.1)), "minCai": _f64(np.full(ca_nodes.size, 1e-4))})
    else:
        raise ValueError(f"unknown calcium dynamics {cadyn!r}")
    na = np.nonzero(need["na"])[0]
    k = np.nonzero(need["k"])[0]
    lib["na_ion"] = MechTable(_i32(na), {"ena": _f64(np.full(na.size, 50.0))})
    lib["k_ion"] = MechTable(_i32(k), {"ek": _f64(np.full(k.size, -85.0))})
    lib["ca_ion"] = MechTable(_i32(ca_nodes), {"cai": _f64(np.full(ca_nodes.size, 5e-5)),
                                               "cao": _f64(np.full(ca_nodes.size, 2.0)),
                                               "eca": _f64(np.full(ca_nodes.size, 132.5))},
                              {"nernst": _i32(np.ones(ca_nodes.size))})
    g = CellGroup(ncell=1, parent=base.parent, a=base.a, b=base.b, area=base.area, cm=base.cm,
                  hh=MechTable(_i32([]), {k2: _f64([]) for k2 in HH_STD}),
                  pas=MechTable(_i32(np.arange(n)), {"g": _f64(np.full(n, 3e-5)), "e": _f64(np.full(n, -75.0))}),
                  iclamp=base.iclamp, celsius=34.0, v_init=-75.0, name=f"libtree{seed}",
                  lib={nm: lib[nm] for nm in LIB_NAMES if nm in lib and lib[nm].n})
    g.validate()
    return g


def lib_tree_batch(ncell: int = 64, seed0: int = 51000, **kw) -> CellGroup:
    """``ncell`` seeded library cells (seed ``seed0 + cell``) in one group."""
    g = concat_groups([lib_tree_cell(seed0 + c, **kw) for c in range(ncell)], name=f"libtrees{ncell}")
    g.v_init = -75.0
    return g


def perturb_lib(g: CellGroup, sigma: float = 0.2, seed: int = 98) -> CellGroup:
    """Teacher copy: every library channel density multiplied by exp(sigma*N(0,1))."""
    rng = np.random.default_rng(seed)
    t = g.copy()
    for nm, key in LIB_GBAR_FIELD.items():
        if nm in t.lib:
            v = t.lib[nm].fields[key]
            t.lib[nm].fields[key] = _f64(v * np.exp(sigma * rng.standard_normal(v.size)))
    return t


# ---------------------------------------------------------------- teachers
def perturb_conductances(g: CellGroup, sigma: float = 0.2, seed: int = 99) -> CellGroup:
    """Teacher copy: every hh gnabar/gkbar/gl and pas g multiplied by exp(sigma*N(0,1))."""
    rng = np.random.default_rng(seed)
    t = g.copy()
    for k in ("gnabar", "gkbar", "gl"):
        t.hh.fields[k] = _f64(t.hh.fields[k] * np.exp(sigma * rng.standard_normal(t.hh.n)))
    t.pas.fields["g"] = _f64(t.pas.fields["g"] * np.exp(sigma * rng.standard_normal(t.pas.n)))
    return t


# ---------------------------------------------------------------- networks
def _table(nodes, fields, ifields=None) -> MechTable:
    """Instance table sorted by node (stable), the layout the exporter writes."""
    nodes = np.asarray(nodes, dtype=np.int64)
    o = np.argsort(nodes, kind="stable")
    return MechTable(_i32(nodes[o]), {k: _f64(np.asarray(v, dtype=np.float64)[o]) for k, v in fields.items()},
                     {k: _i32(np.asarray(v)[o]) for k, v in (ifields or {}).items()})


def _cell_nodes(g: CellGroup) -> List[np.ndarray]:
    cell = g.cell_of_node()
    order = np.argsort(cell, kind="stable")
    bounds = np.searchsorted(cell[order], np.arange(g.ncell + 1))
    return [order[bounds[c]:bounds[c + 1]] for c in range(g.ncell)]


def spiking_network(ncell: int = 8, seed: int = 11, nmin: int = 40, nmax: int = 120, syn_per_cell: int = 6,
                    nstim: int = 4, exp_frac: float = 0.3, weight: Tuple[float, float] = (0.005, 0.03),
                    delay: Tuple[float, float] = (1.0, 5.0), drive_frac: float = 0.5,
                    stim_interval: float = 8.0, stim_number: float = 20.0, stim_noise: float = 0.5,
                    cell=None) -> CellGroup:
    """A small event-driven network of random-tree cells (test scale).

    Every cell receives ``syn_per_cell`` synapses at uniformly drawn nodes of
    its own tree (a fraction ``exp_frac`` ExpSyn with tau 2 ms, the rest
    Exp2Syn with tau1 0.5, tau2 5 ms), each driven by one NetCon from a random
    other cell (80 % excitatory, e = 0 mV; 20 % inhibitory, e = -80 mV) with
    delay U[delay] and weight U[weight] uS.  ``nstim`` NetStims (interval,
    number, start 1 ms, noise) each drive one extra Exp2Syn at the soma of
    cell ``i % ncell``.  Only a fraction ``drive_frac`` of the cells keep
    their somatic IClamp.  ``cell(seed, nmin, nmax)`` builds each cell
    (default ``random_tree_cell``; ``lib_network`` passes library cells).
    """
    rng = np.random.default_rng(seed)
    make = cell or (lambda sd, lo, hi: random_tree_cell(sd, nmin=lo, nmax=hi))
    cells = [make(seed * 1000 + c, nmin, nmax) for c in range(ncell)]
    g = concat_groups(cells, name=f"net{ncell}")
    amp = g.iclamp.fields["amp"].copy()
    amp[rng.random(amp.shape[0]) >= drive_frac] = 0.0
    g.iclamp.fields["amp"] = _f64(amp)
    per_cell = _cell_nodes(g)
    e1 = {"nodes": [], "tau": [], "e": [], "delay": [], "weight": [], "src": []}
    e2 = {"nodes": [], "tau1": [], "tau2": [], "e": [], "delay": [], "weight": [], "src": []}
    for c in range(ncell):
        for _ in range(syn_per_cell):
            node = int(rng.choice(per_cell[c]))
            src = int(rng.integers(ncell - 1))
            src = src + 1 if src >= c else src
            e = 0.0 if rng.random() < 0.8 else -80.0
            d = float(rng.uniform(*delay))
            w = float(rng.uniform(*weight))
            if rng.random() < exp_frac:
                for k, v in zip(("nodes", "tau", "e", "delay", "weight", "src"), (node, 2.0, e, d, w, src)):
                    e1[k].append(v)
            else:
                for k, v in zip(("nodes", "tau1", "tau2", "e", "delay", "weight", "src"),
                                (node, 0.5, 5.0, e, d, w, src)):
                    e2[k].append(v)
    for i in range(nstim):
        for k, v in zip(("nodes", "tau1", "tau2", "e", "delay", "weight", "src"),
                        (i % ncell, 0.5, 5.0, 0.0, float(rng.uniform(*delay)), 2 * weight[1], ncell + i)):
            e2[k].append(v)
    g.expsyn = _table(e1["nodes"], {k: e1[k] for k in ("tau", "e", "delay", "weight")}, {"src": e1["src"]})
    g.exp2syn = _table(e2["nodes"], {k: e2[k] for k in ("tau1", "tau2", "e", "delay", "weight")}, {"src": e2["src"]})
    g.netstim = MechTable(_i32(np.zeros(nstim)), {
        "interval": _f64(np.full(nstim, stim_interval)), "number": _f64(np.full(nstim, stim_number)),
        "start": _f64(np.full(nstim, 1.0)), "noise": _f64(np.full(nstim, stim_noise))})
    g.validate()
    return g


def network_config4(ncell: int = 10000, seed: int = 4, syn_per_cell: int = 100, nmin: int = 400, nmax: int = 600,
                    rate_hz: float = 5.0) -> CellGroup:
    """Config 4: ``ncell`` random-tree cells, ``syn_per_cell`` Exp2Syn each.

    80/20 excitatory/inhibitory sources (e = 0 / -80 mV), tau1 0.5, tau2 5 ms,
    weight exp(N(-7, 1)) uS, random presynaptic cell, delay U[1, 5] ms; one
    NetStim per cell (``rate_hz``, noise 1, start 0, unlimited number) drives
    one more Exp2Syn at the soma.  Seeded; the reference quotes no data set.
    """
    return network_config4_shard(ncell, 0, 1, seed=seed, syn_per_cell=syn_per_cell, nmin=nmin, nmax=nmax,
                                 rate_hz=rate_hz)


def config4_cell_range(total: int, rank: int, nranks: int) -> Tuple[int, int]:
    """Cells [c0, c1) of rank ``rank``: contiguous, counts differing by at most one."""
    return total * rank // nranks, total * (rank + 1) // nranks


def network_config4_shard(total: int, rank: int, nranks: int, seed: int = 4, syn_per_cell: int = 100,
                          nmin: int = 400, nmax: int = 600, rate_hz: float = 5.0,
                          teacher_sigma: float = 0.2) -> CellGroup:
    """Rank ``rank``'s part of the config-4 network of ``total`` cells.

    The network does not depend on how it is split: cell c (global id) has
    its morphology seeded by c, and its synapses -- location, presynaptic
    source over all ``total`` cells, sign, delay, weight, plus the synapse of
    its NetStim -- drawn from a generator seeded by (seed, c).  Rank r builds
    only its cells ``config4_cell_range(total, r, nranks)`` with their
    synapses (global NetCon sources) and the whole NetStim table (one per
    global cell, ids total + c).  ``meta`` records ``gid_base``,
    ``nsrc_cells`` and ``teacher_weight``: the weights lognormally perturbed
    (sigma ``teacher_sigma``, generator seeded by (seed, 7, c)) in the
    group's synapse order, the teacher network of the loss.
    """
    c0, c1 = config4_cell_range(total, rank, nranks)
    ncell = c1 - c0
    cells = [random_tree_cell(seed * 100000 + c, nmin=nmin, nmax=nmax) for c in range(c0, c1)]
    g = concat_groups(cells, name=f"net{total}.r{rank}of{nranks}")
    cell = g.cell_of_node()
    order = np.argsort(cell, kind="stable")
    bounds = np.searchsorted(cell[order], np.arange(ncell + 1))
    k = syn_per_cell
    nodes = np.empty(ncell * (k + 1), np.int64)
    src = np.empty_like(nodes)
    e = np.empty(nodes.shape[0])
    d = np.empty_like(e)
    w = np.empty_like(e)
    wt = np.empty_like(e)
    for i in range(ncell):
        gc = c0 + i
        rng = np.random.default_rng([seed, gc])
        sl = slice(i * (k + 1), (i + 1) * (k + 1))
        nloc = bounds[i + 1] - bounds[i]
        pick = bounds[i] + (rng.random(k) * nloc).astype(np.int64)
        s = rng.integers(0, total - 1, k)
        s = np.where(s >= gc, s + 1, s)  # no self-connection
        exc = rng.random(k) < 0.8
        # synapses of cell gc, then the one its NetStim drives at the soma
        nodes[sl] = np.concatenate([order[pick], [i]])
        src[sl] = np.concatenate([s, [total + gc]])
        e[sl] = np.concatenate([np.where(exc, 0.0, -80.0), [0.0]])
        d[sl] = rng.uniform(1.0, 5.0, k + 1)
        w[sl] = np.concatenate([np.exp(rng.normal(-7.0, 1.0, k)), [0.01]])
        wt[sl] = w[sl] * np.exp(teacher_sigma * np.random.default_rng([seed, 7, gc]).standard_normal(k + 1))
    n = nodes.shape[0]
    o = np.argsort(nodes, kind="stable")  # the table order _table gives
    g.exp2syn = _table(nodes, {"tau1": np.full(n, 0.5), "tau2": np.full(n, 5.0), "e": e, "delay": d, "weight": w},
                       {"src": src})
    g.netstim = MechTable(_i32(np.zeros(total)), {
        "interval": _f64(np.full(total, 1000.0 / rate_hz)), "number": _f64(np.full(total, 1e9)),
        "start": _f64(np.zeros(total)), "noise": _f64(np.ones(total))})
    g.meta["gid_base"] = c0
    g.meta["nsrc_cells"] = total
    g.meta["teacher_weight"] = _f64(wt[o])
    g.validate()
    return g


def coupled_network(ncell: int = 6, seed: int = 5, nmin: int = 50, nmax: int = 150, ngap: int = 6,
                    ngapj: int = 3, ngraded: int = 10, drive_frac: float = 0.4,
                    gap_g: Tuple[float, float] = (1e-4, 1e-3), graded_w: Tuple[float, float] = (2e-4, 2e-3),
                    ngapnp: int = 0, cell=None) -> CellGroup:
    """Config 5 style network: cells coupled by gap junctions and graded synapses.

    ``ngap`` HalfGap pairs (two instances per pair at random nodes of two
    different cells, each copying the other's voltage, g U[gap_g] uS),
    ``ngapj`` gapjunction_lr pairs (w 1, g U[gap_g]), ``ngraded``
    neuron_to_neuron_syn_lr synapses from a random cell's soma onto a random
    node of another cell (w = +-U[graded_w], 80 % positive; delta 5 mV,
    Vth -20 mV, the MOD defaults otherwise), ``ngapnp`` gapjunction_noptr
    pairs (weight U[gap_g], vpre from the partner node; drawn after the others,
    so the rest of the network does not depend on it).  A fraction
    ``drive_frac`` of the cells keep their somatic IClamp.  ``cell`` as in
    ``spiking_network``.
    """
    rng = np.random.default_rng(seed)
    make = cell or (lambda sd, lo, hi: random_tree_cell(sd, nmin=lo, nmax=hi))
    cells = [make(seed * 1000 + c, nmin, nmax) for c in range(ncell)]
    g = concat_groups(cells, name=f"coupled{ncell}")
    amp = g.iclamp.fields["amp"].copy()
    amp[rng.random(amp.shape[0]) >= drive_frac] = 0.0
    g.iclamp.fields["amp"] = _f64(amp)
    per_cell = _cell_nodes(g)

    def two_cells():
        a = int(rng.integers(ncell))
        b = int(rng.integers(ncell - 1))
        return a, (b + 1 if b >= a else b)

    hn, hs, hg = [], [], []
    for _ in range(ngap):
        a, b = two_cells()
        na, nb = int(rng.choice(per_cell[a])), int(rng.choice(per_cell[b]))
        gg = float(rng.uniform(*gap_g))
        hn += [na, nb]
        hs += [nb, na]
        hg += [gg, gg]
    jn, jp, jg = [], [], []
    for _ in range(ngapj):
        a, b = two_cells()
        na, nb = int(rng.choice(per_cell[a])), int(rng.choice(per_cell[b]))
        gg = float(rng.uniform(*gap_g))
        jn += [na, nb]
        jp += [nb, na]
        jg += [gg, gg]
    rn, rp, rw = [], [], []
    for _ in range(ngraded):
        a, b = two_cells()
        rn.append(int(rng.choice(per_cell[b])))
        rp.append(a)
        w = float(rng.uniform(*graded_w))
        rw.append(w if rng.random() < 0.8 else -w)
    nn_, ns_, nw_ = [], [], []
    for _ in range(ngapnp):
        a, b = two_cells()
        na, nb = int(rng.choice(per_cell[a])), int(rng.choice(per_cell[b]))
        gg = float(rng.uniform(*gap_g))
        nn_ += [na, nb]
        ns_ += [nb, na]
        nw_ += [gg, gg]
    g.gapnoptr = _table(nn_, {"weight": nw_}, {"src": ns_})
    g.halfgap = _table(hn, {"g": hg}, {"src": hs})
    g.gapjunction = _table(jn, {"g": jg, "w": np.ones(len(jn))}, {"pre": jp})
    ng = len(rn)
    g.graded = _table(rn, {"w": rw, "g": np.full(ng, 4.9), "delta": np.full(ng, 5.0), "k": np.full(ng, 0.5),
                           "Vth": np.full(ng, -20.0), "erev": np.full(ng, 30.0), "dvpre": np.full(ng, 1e-3)},
                      {"pre": rp})
    g.validate()
    return g


def lib_network(kind: str = "event", ncell: int = 6, seed: int = 41, channels=None, cadyn: str = "CaDynamics_E2",
                **kw) -> CellGroup:
    """A network of library cells (``lib_tree_cell``: the channel set, ions,
    calcium dynamics): ``kind`` "event" wires them like ``spiking_network``
    (ExpSyn / Exp2Syn, NetCons, NetStims), "coupled" like ``coupled_network``
    (HalfGap, gapjunction_lr / _noptr, graded synapses) -- the worm networks
    with learned channels of the reference's worm-lr set."""
    def make(sd, lo, hi):
        return lib_tree_cell(sd, nmin=lo, nmax=hi, channels=channels, cadyn=cadyn)

    kw.setdefault("nmin", 60)
    kw.setdefault("nmax", 140)
    g = (spiking_network if kind == "event" else coupled_network)(ncell=ncell, seed=seed, cell=make, **kw)
    g.v_init = -75.0
    g.name = f"lib{kind}{ncell}"
    return g


def worm_config5(ncell: int = 302, seed: int = 5) -> CellGroup:
    """Config 5: 302 cells of U[50,150] compartments, 900 gap pairs, 2000 graded synapses."""
    return coupled_network(ncell=ncell, seed=seed, nmin=50, nmax=150, ngap=900, ngapj=0, ngraded=2000,
                           drive_frac=0.3)
