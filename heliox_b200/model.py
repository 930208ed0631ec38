"""Cell-group container: the arrays the forward integrator and the adjoint consume.

A ``CellGroup`` holds exactly what the reference's ``HelioXroupData`` holds for the
hot path (``src/neuron.h:19-130``): the node arrays ``a``, ``b``, ``area``,
``parent`` (``v_parent_index``) and capacitance ``cm`` in NEURON/CoreNEURON node
order, with the first ``ncell`` nodes being the cell roots and every other node
having ``parent[i] < i`` (``src/simulate.cpp:542-555`` relies on this), plus one
instance table per mechanism, each sorted by node index like the reference's
``nodeindices`` (``src/permute.cpp:593-622``).

Units follow NEURON: ``area`` in um^2, ``a``/``b`` in S/cm^2 (negative, the
NEURON sign convention consumed at ``src/simulate.cpp:544-555``), ``cm`` in
uF/cm^2, conductances in S/cm^2, currents of point processes in nA, times in ms,
voltages in mV.

Mechanism order inside one step is the CoreNEURON type order that the reference
keeps in ``mech_current_list`` (``src/io/coredat_to_innerdat.cpp:179-181``):
capacitance, pas, hh, IClamp, ExpSyn, Exp2Syn, HalfGap, graded synapse.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, Optional

import numpy as np

F64 = np.float64
I32 = np.int32

# Mechanism names used in handles (``Sim.get_variable_handle``) and in the
# C-ABI parameter kinds.
HH_PARAMS = ("gnabar", "gkbar", "gl", "el")
PAS_PARAMS = ("g", "e")
ICLAMP_PARAMS = ("del", "dur", "amp")


def _f64(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=F64))


def _i32(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=I32))


@dataclass
class MechTable:
    """Instances of one mechanism: ``nodes`` (sorted, int32) + per-instance fields."""

    nodes: np.ndarray
    fields: Dict[str, np.ndarray] = field(default_factory=dict)

    @property
    def n(self) -> int:
        return int(self.nodes.shape[0])

    def copy(self) -> "MechTable":
        return MechTable(self.nodes.copy(), {k: v.copy() for k, v in self.fields.items()})


@dataclass
class CellGroup:
    """One group of cells in reference node order (roots first, parent[i] < i)."""

    ncell: int
    parent: np.ndarray  # int32[nnode], -1 for roots
    a: np.ndarray  # f64[nnode]
    b: np.ndarray  # f64[nnode]
    area: np.ndarray  # f64[nnode] um^2
    cm: np.ndarray  # f64[nnode] uF/cm^2
    hh: MechTable  # fields: gnabar gkbar gl el ena ek
    pas: MechTable  # fields: g e
    iclamp: MechTable  # fields: del dur amp
    celsius: float = 6.3
    dt: float = 0.025
    v_init: float = -65.0
    name: str = "group"
    meta: Dict[str, object] = field(default_factory=dict)

    # ------------------------------------------------------------------ basics
    @property
    def nnode(self) -> int:
        return int(self.parent.shape[0])

    def cell_of_node(self) -> np.ndarray:
        """Cell id of every node (roots are cells 0..ncell-1)."""
        c = np.empty(self.nnode, dtype=I32)
        c[: self.ncell] = np.arange(self.ncell, dtype=I32)
        p = self.parent
        for i in range(self.ncell, self.nnode):
            c[i] = c[p[i]]
        return c

    def soma_nodes(self) -> np.ndarray:
        return np.arange(self.ncell, dtype=I32)

    def validate(self) -> None:
        n = self.nnode
        if self.ncell <= 0 or self.ncell > n:
            raise ValueError("ncell out of range")
        for arr, nm in ((self.a, "a"), (self.b, "b"), (self.area, "area"), (self.cm, "cm")):
            if arr.shape != (n,) or arr.dtype != F64:
                raise ValueError(f"{nm} must be float64[{n}]")
        if self.parent.dtype != I32:
            raise ValueError("parent must be int32")
        if np.any(self.parent[: self.ncell] != -1):
            raise ValueError("roots (first ncell nodes) must have parent -1")
        idx = np.arange(self.ncell, n)
        if np.any(self.parent[self.ncell:] < 0) or np.any(self.parent[self.ncell:] >= idx):
            raise ValueError("parent[i] must satisfy 0 <= parent[i] < i for non-roots")
        if np.any(self.area <= 0):
            raise ValueError("area must be positive")
        for tab, nm, uniq in ((self.hh, "hh", True), (self.pas, "pas", True), (self.iclamp, "IClamp", False)):
            if tab.n and (np.any(tab.nodes < 0) or np.any(tab.nodes >= n)):
                raise ValueError(f"{nm} node index out of range")
            if tab.n > 1 and np.any(np.diff(tab.nodes) < 0):
                raise ValueError(f"{nm} nodes must be sorted")
            if uniq and tab.n > 1 and np.any(np.diff(tab.nodes) == 0):
                raise ValueError(f"density mechanism {nm} has two instances on one node")
            for k, v in tab.fields.items():
                if v.shape != (tab.n,) or v.dtype != F64:
                    raise ValueError(f"{nm}.{k} must be float64[{tab.n}]")

    def copy(self) -> "CellGroup":
        return CellGroup(
            ncell=self.ncell,
            parent=self.parent.copy(),
            a=self.a.copy(),
            b=self.b.copy(),
            area=self.area.copy(),
            cm=self.cm.copy(),
            hh=self.hh.copy(),
            pas=self.pas.copy(),
            iclamp=self.iclamp.copy(),
            celsius=self.celsius,
            dt=self.dt,
            v_init=self.v_init,
            name=self.name,
            meta=dict(self.meta),
        )

    # ------------------------------------------------------------ parameters
    def param_view(self, mech: str, var: str) -> np.ndarray:
        """The live array of one learnable/settable parameter."""
        tab = {"hh": self.hh, "pas": self.pas, "IClamp": self.iclamp}.get(mech)
        if tab is None:
            if mech == "capacitance" and var == "cm":
                return self.cm
            raise KeyError(f"unknown mechanism {mech!r}")
        key = {"g_pas": "g", "e_pas": "e", "delay": "del"}.get(var, var)
        if key not in tab.fields:
            raise KeyError(f"unknown variable {mech}.{var}")
        return tab.fields[key]


def empty_table(names) -> MechTable:
    return MechTable(_i32([]), {k: _f64([]) for k in names})


def concat_groups(groups, name: str = "group") -> CellGroup:
    """Concatenate cell groups into one group in reference order (roots first).

    Roots of all groups come first (in group order), followed by the non-root
    nodes of each group in turn, so a multi-cell group built this way has the
    same layout NEURON's CoreNEURON writer produces for a thread with several
    cells.
    """
    groups = list(groups)
    ncell = sum(g.ncell for g in groups)
    nn = sum(g.nnode for g in groups)
    # new index of every old node
    maps = []
    root_off = 0
    rest_off = ncell
    for g in groups:
        m = np.empty(g.nnode, dtype=np.int64)
        m[: g.ncell] = root_off + np.arange(g.ncell)
        nr = g.nnode - g.ncell
        m[g.ncell:] = rest_off + np.arange(nr)
        root_off += g.ncell
        rest_off += nr
        maps.append(m)
    parent = np.full(nn, -1, dtype=I32)
    a = np.zeros(nn)
    b = np.zeros(nn)
    area = np.zeros(nn)
    cm = np.zeros(nn)
    for g, m in zip(groups, maps):
        pp = g.parent.astype(np.int64)
        newp = np.where(pp >= 0, m[np.maximum(pp, 0)], -1)
        parent[m] = newp
        a[m] = g.a
        b[m] = g.b
        area[m] = g.area
        cm[m] = g.cm

    def cat_tab(attr, names):
        nodes = []
        fields = {k: [] for k in names}
        for g, m in zip(groups, maps):
            t = getattr(g, attr)
            nodes.append(m[t.nodes])
            for k in names:
                fields[k].append(t.fields[k])
        nodes = np.concatenate(nodes) if nodes else np.zeros(0, np.int64)
        order = np.argsort(nodes, kind="stable")
        return MechTable(
            _i32(nodes[order]),
            {k: _f64(np.concatenate(v)[order]) if v else _f64([]) for k, v in fields.items()},
        )

    hh = cat_tab("hh", ("gnabar", "gkbar", "gl", "el", "ena", "ek"))
    pas = cat_tab("pas", ("g", "e"))
    ic = cat_tab("iclamp", ("del", "dur", "amp"))
    g0 = groups[0]
    out = CellGroup(
        ncell=ncell,
        parent=parent,
        a=_f64(a),
        b=_f64(b),
        area=_f64(area),
        cm=_f64(cm),
        hh=hh,
        pas=pas,
        iclamp=ic,
        celsius=g0.celsius,
        dt=g0.dt,
        v_init=g0.v_init,
        name=name,
    )
    out.validate()
    return out
