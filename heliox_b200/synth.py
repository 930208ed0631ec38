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

from .model import CellGroup, MechTable, _f64, _i32, concat_groups

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


# ---------------------------------------------------------------- teachers
def perturb_conductances(g: CellGroup, sigma: float = 0.2, seed: int = 99) -> CellGroup:
    """Teacher copy: every hh gnabar/gkbar/gl and pas g multiplied by exp(sigma*N(0,1))."""
    rng = np.random.default_rng(seed)
    t = g.copy()
    for k in ("gnabar", "gkbar", "gl"):
        t.hh.fields[k] = _f64(t.hh.fields[k] * np.exp(sigma * rng.standard_normal(t.hh.n)))
    t.pas.fields["g"] = _f64(t.pas.fields["g"] * np.exp(sigma * rng.standard_normal(t.pas.n)))
    return t
