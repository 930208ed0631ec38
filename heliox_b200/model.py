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

Mechanism order inside one step is the order of the CoreNEURON mechanism list
that the reference keeps in ``mech_current_list``
(``src/io/coredat_to_innerdat.cpp:179-181``); the exporter here writes it as
capacitance, pas, hh, IClamp, ExpSyn, Exp2Syn, NetStim, HalfGap,
gapjunction_lr, gapjunction_noptr, neuron_to_neuron_syn_lr.

Network parts (all optional, empty by default):

* ``expsyn`` / ``exp2syn``: event-driven synapses (fields tau / tau1, tau2, e),
  each instance the target of exactly one NetCon: ``ifields['src']`` is the
  spike source (0..ncell-1: the PreSyn of that cell; ncell+j: NetStim j),
  ``fields['delay']`` (ms) and ``fields['weight']`` (uS) -- the per-instance
  ``spk_vec_idx``/``delay``/``weights`` the reference fills in
  ``initSynapse`` (coredat_to_innerdat.cpp:348-376);
* ``ps_thresh``: spike threshold (mV) of each cell's PreSyn, detected at the
  cell's root node (``PreSyn::threshold_detect_cpu``, presyn.cpp:133-177);
* ``netstim``: artificial spike sources (fields interval, number, start,
  noise; netstim.cpp), ``netstim_rng`` selects the initial random stream
  (0: the reference's CPU mode, 1: its GPU mode);
* ``halfgap``: HalfGap point processes (field g, ``ifields['src']`` the node
  whose voltage is copied into vgap; HalfGap.cu, simulate.cpp:953-966);
* ``gapjunction``: gapjunction_lr (fields g, w, ``ifields['pre']``,
  gapjunction_lr.cu:58-65);
* ``gapnoptr``: gapjunction_noptr (field weight, ``ifields['src']`` the node
  whose voltage the reference's gap transfer copies into vpre after every
  update; i = weight (v - vpre), worm-mech/gapjunction_noptr.cu:33-36);
* ``graded``: neuron_to_neuron_syn_lr (fields w, g, delta, k, Vth, erev,
  dvpre, ``ifields['pre']``, neuron_to_neuron_syn_lr.cu:97-145).
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
EXPSYN_FIELDS = ("tau", "e", "delay", "weight")
EXP2SYN_FIELDS = ("tau1", "tau2", "e", "delay", "weight")
NETSTIM_FIELDS = ("interval", "number", "start", "noise")
HALFGAP_FIELDS = ("g",)
GAPJ_FIELDS = ("g", "w")
GAPNP_FIELDS = ("weight",)
GRADED_FIELDS = ("w", "g", "delta", "k", "Vth", "erev", "dvpre")
SPIKE_THRESHOLD = 10.0

# Library mechanisms: the ions and the user-mech channel set (name, fields,
# number of leading trainable fields), in CoreNEURON type order.  Field names
# are the reference's RANGE names (src/mech/user-mech/<name>.cu
# var_in_coredata_idx); ion fields follow eion.cuh:81-86 (cai is the initial
# concentration, ifields['nernst'] = 1 recomputes eca from cai/cao every step,
# eion.cuh:155-166).  na_ion / k_ion on an hh node must carry hh's ena / ek.
KQT3_GLOBALS = ("vhm", "ka", "vhw", "kiw", "aw", "bw", "vhs", "kis", "as", "bs", "atmf", "btmf", "ctmf", "atms", "btms", "ctms", "dtms", "etms", "ftms", "gtms", "atw", "btw", "ctw", "dtw", "ats")
LIB_MECHS = (
    ("na_ion", ("ena",), 0),
    ("k_ion", ("ek",), 0),
    ("ca_ion", ("cai", "cao", "eca"), 0),
    ("CaDynamics_E2", ("gamma", "decay", "depth", "minCai"), 4),
    ("Ca_HVA", ("gbar",), 1),
    ("Ca_LVAst", ("gCa_LVAstbar",), 1),
    ("Im", ("gImbar",), 1),
    ("K_Pst", ("gK_Pstbar",), 1),
    ("K_Tst", ("gK_Tstbar",), 1),
    ("NaTg", ("gNaTgbar", "vshifth", "vshiftm", "slopeh", "slopem"), 1),
    ("Nap_Et2", ("gNap_Et2bar",), 1),
    ("SK_E2", ("gSK_E2bar", "zTau"), 1),
    ("SKv3_1", ("gSKv3_1bar",), 1),
    ("hd_la", ("ghdbar", "vhalfl", "tau", "ehd", "kl", "vhalft", "a0t", "zetat", "gmt", "q10", "qtl"), 1),
    ("km_la", ("gbar", "Ra", "Rb", "tha", "qa", "tadj"), 1),
    ("kca_la", ("gbar", "Ra", "Rb", "caix", "tadj"), 1),
    ("it2_la", ("gcabar", "vshift", "v12m", "vwm", "v12h", "vwh", "am", "ah", "vm1", "vm2", "vh1", "vh2", "wm1",
                "wm2", "wh1", "wh2"), 1),
    ("kdr_la", ("gbar",), 1),
    ("sca_la", ("gbar", "inactF", "actF", "vshift", "tadj"), 1),
    ("Ca", ("gCabar",), 1),
    # worm-lr channels (src/mech/worm-lr-mech): current w * (gb * gates * (v - ek_tmp)); w is the weight the
    # reference's LRDS learns, gb, ek_tmp, dv per instance, the kinetics GLOBALs
    ("shl1_lr", ("w", "gbshl1", "ek_tmp", "dv", "vhm", "ka", "vhh", "ki", "atm", "btm", "ctm", "dtm", "etm", "ftm", "athf", "bthf", "cthf", "dthf", "aths", "bths", "cths", "dths"), 1),
    ("kvs1_lr", ("w", "gbkvs1", "ek_tmp", "dv", "vhm", "ka", "vhh", "ki", "atm", "btm", "ctm", "dtm", "ath", "bth", "cth", "dth"), 1),
    ("irk_lr", ("w", "gbirk", "ek_tmp", "dv", "vhm", "ka", "atm", "btm", "ctm", "dtm", "etm", "ftm"), 1),
    ("egl36_lr", ("w", "gbegl36", "ek_tmp", "dv", "vhm", "ka", "atms", "atmm", "atmf"), 1),
    ("shk1_lr", ("w", "gbshk1", "ek_tmp", "dv", "vhm", "ka", "vhh", "ki", "atm", "btm", "ctm", "dtm", "etm", "ftm", "ath"), 1),
    ("egl2_lr", ("w", "gbegl2", "ek_tmp", "dv", "vhm", "ka", "atm", "btm", "ctm", "dtm"), 1),
    ("cca1_lr", ("w", "gbcca1", "eca_tmp", "dv", "vhm", "ka", "vhh", "ki", "atm", "btm", "ctm", "dtm", "ath", "bth", "cth", "dth"), 1),
    ("egl19_lr", ("w", "gbegl19", "eca_tmp", "dv", "vhm", "ka", "vhh", "ki", "vhhb", "kib", "ahinf", "bhinf", "chinf", "dhinf", "atm", "btm", "ctm", "dtm", "etm", "ftm", "gtm", "ath", "bth", "cth", "dth", "eth", "fth", "gth", "hth"), 1),
    ("unc2_lr", ("w", "gbunc2", "eca_tmp", "dv", "vhm", "ka", "vhh", "ki", "atm", "btm", "ctm", "dtm", "etm", "ath", "bth", "cth", "dth", "eth", "fth"), 1),
    ("kcnl_lr", ("w", "gbkcnl", "dv", "kca", "a", "ek_tmp"), 1),
    ("nca_lr", ("w", "gbnca", "ena_tmp"), 1),
    # kqt3_lr: w (gb (0.3 mf + 0.7 ms) ww s (v - ek)) with k_ion's ek; ek_tmp is carried, not read
    ("kqt3_lr", ("w", "gbkqt3", "ek_tmp", "dv") + KQT3_GLOBALS, 1),
    # cainternm_lr (calcium dynamics of the worm-lr set): vcell per instance, GLOBALs f, tca, caeq
    ("cainternm_lr", ("vcell", "f", "tca", "caeq"), 1),
    # worm-mech channels (src/mech/worm-mech): gb ... (v + 80) with the kinetics hard-coded in setparames
    # (kvs1: GLOBALs), gb trainable
    ("shl1", ("gbshl1",), 1),
    ("kvs1", ("gbkvs1",) + ("vhm", "ka", "vhh", "ki", "atm", "btm", "ctm", "dtm", "ath", "bth", "cth", "dth"), 1),
    ("irk", ("gbirk",), 1),
    ("egl36", ("gbegl36",), 1),
    ("shk1", ("gbshk1",), 1),
    ("egl2", ("gbegl2",), 1),
    ("cca1", ("gbcca1",), 1),  # calcium: gb ... (v - 60), current into ica
    ("egl19", ("gbegl19",), 1),
    ("unc2", ("gbunc2",), 1),
)
# fields that are GLOBALs of their mechanism in the reference (one value per
# group, written to globals.dat as <field>_<mechanism>)
LIB_GLOBALS = {
    "SK_E2": ("zTau",),
    "hd_la": ("ehd", "kl", "vhalft", "a0t", "zetat", "gmt", "q10", "qtl"),
    "km_la": ("Ra", "Rb", "tha", "qa", "tadj"),
    "kca_la": ("Ra", "Rb", "caix", "tadj"),
    "it2_la": ("vshift", "v12m", "vwm", "v12h", "vwh", "am", "ah", "vm1", "vm2", "vh1", "vh2", "wm1", "wm2", "wh1",
               "wh2"),
    "sca_la": ("vshift", "tadj"),
    "shl1_lr": ("vhm", "ka", "vhh", "ki", "atm", "btm", "ctm", "dtm", "etm", "ftm", "athf", "bthf", "cthf", "dthf", "aths", "bths", "cths", "dths",),
    "kvs1_lr": ("vhm", "ka", "vhh", "ki", "atm", "btm", "ctm", "dtm", "ath", "bth", "cth", "dth",),
    "irk_lr": ("vhm", "ka", "atm", "btm", "ctm", "dtm", "etm", "ftm",),
    "egl36_lr": ("vhm", "ka", "atms", "atmm", "atmf",),
    "shk1_lr": ("vhm", "ka", "vhh", "ki", "atm", "btm", "ctm", "dtm", "etm", "ftm", "ath",),
    "egl2_lr": ("vhm", "ka", "atm", "btm", "ctm", "dtm",),
    "cca1_lr": ("vhm", "ka", "vhh", "ki", "atm", "btm", "ctm", "dtm", "ath", "bth", "cth", "dth",),
    "egl19_lr": ("vhm", "ka", "vhh", "ki", "vhhb", "kib", "ahinf", "bhinf", "chinf", "dhinf", "atm", "btm", "ctm", "dtm", "etm", "ftm", "gtm", "ath", "bth", "cth", "dth", "eth", "fth", "gth", "hth",),
    "unc2_lr": ("vhm", "ka", "vhh", "ki", "atm", "btm", "ctm", "dtm", "etm", "ath", "bth", "cth", "dth", "eth", "fth",),
    "kcnl_lr": ("kca", "a", "ek_tmp"),
    "kqt3_lr": KQT3_GLOBALS,
    "cainternm_lr": ("f", "tca", "caeq"),
    "kvs1": ("vhm", "ka", "vhh", "ki", "atm", "btm", "ctm", "dtm", "ath", "bth", "cth", "dth"),
}
LIB_NAMES = tuple(m[0] for m in LIB_MECHS)
LIB_FIELDS = {m[0]: m[1] for m in LIB_MECHS}
LIB_NTRAIN = {m[0]: m[2] for m in LIB_MECHS}
# which ion each library mechanism reads (erev / concentration) or writes
LIB_IONS = {
    "CaDynamics_E2": ("ca",), "Ca_HVA": ("ca",), "Ca_LVAst": ("ca",), "Im": ("k",), "K_Pst": ("k",),
    "K_Tst": ("k",), "NaTg": ("na",), "Nap_Et2": ("na",), "SK_E2": ("k", "ca"), "SKv3_1": ("k",),
    "hd_la": (), "km_la": ("k",), "kca_la": ("k", "ca"), "it2_la": ("ca",), "kdr_la": ("k",), "sca_la": ("ca",),
    "Ca": ("ca",),
    "shl1_lr": ("k",),
    "kvs1_lr": ("k",),
    "irk_lr": ("k",),
    "egl36_lr": ("k",),
    "shk1_lr": ("k",),
    "egl2_lr": ("k",),
    "cca1_lr": ("ca",),
    "egl19_lr": ("ca",),
    "unc2_lr": ("ca",),
    "kcnl_lr": ("k", "ca"),
    "nca_lr": ("na",),
    "kqt3_lr": ("k",),
    "cainternm_lr": ("ca",),
    "shl1": ("k",), "kvs1": ("k",), "irk": ("k",), "egl36": ("k",), "shk1": ("k",), "egl2": ("k",),
    "cca1": ("ca",), "egl19": ("ca",), "unc2": ("ca",),
}


def _f64(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=F64))


def _i32(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=I32))


@dataclass
class MechTable:
    """Instances of one mechanism: ``nodes`` (sorted, int32) + per-instance fields.

    ``fields`` are float64 per-instance values; ``ifields`` are int32
    per-instance values (a partner node, a spike source).
    """

    nodes: np.ndarray
    fields: Dict[str, np.ndarray] = field(default_factory=dict)
    ifields: Dict[str, np.ndarray] = field(default_factory=dict)

    @property
    def n(self) -> int:
        return int(self.nodes.shape[0])

    def copy(self) -> "MechTable":
        return MechTable(self.nodes.copy(), {k: v.copy() for k, v in self.fields.items()},
                         {k: v.copy() for k, v in self.ifields.items()})


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
    expsyn: Optional[MechTable] = None
    exp2syn: Optional[MechTable] = None
    netstim: Optional[MechTable] = None
    halfgap: Optional[MechTable] = None
    gapjunction: Optional[MechTable] = None
    gapnoptr: Optional[MechTable] = None
    graded: Optional[MechTable] = None
    ps_thresh: Optional[np.ndarray] = None
    netstim_rng: int = 0
    lib: Dict[str, MechTable] = field(default_factory=dict)

    def __post_init__(self):
        if self.expsyn is None:
            self.expsyn = empty_table(EXPSYN_FIELDS, ("src",))
        if self.exp2syn is None:
            self.exp2syn = empty_table(EXP2SYN_FIELDS, ("src",))
        if self.netstim is None:
            self.netstim = empty_table(NETSTIM_FIELDS)
        if self.halfgap is None:
            self.halfgap = empty_table(HALFGAP_FIELDS, ("src",))
        if self.gapjunction is None:
            self.gapjunction = empty_table(GAPJ_FIELDS, ("pre",))
        if self.gapnoptr is None:
            self.gapnoptr = empty_table(GAPNP_FIELDS, ("src",))
        if self.graded is None:
            self.graded = empty_table(GRADED_FIELDS, ("pre",))
        if self.ps_thresh is None:
            self.ps_thresh = np.full(self.ncell, SPIKE_THRESHOLD)

    @property
    def has_network(self) -> bool:
        """True if any event, gap or graded coupling is present."""
        return bool(self.expsyn.n or self.exp2syn.n or self.netstim.n or self.halfgap.n or self.gapjunction.n
                    or self.gapnoptr.n or self.graded.n)

    @property
    def coupled(self) -> bool:
        """True if voltages of other nodes enter a step's currents or states (gaps, graded synapses)."""
        return bool(self.halfgap.n or self.gapjunction.n or self.gapnoptr.n or self.graded.n)

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
        # a shard of a multi-GPU network keeps global NetCon sources
        nsrc = int(self.meta.get("nsrc_cells", self.ncell)) + self.netstim.n
        for tab, nm, fl in ((self.expsyn, "ExpSyn", EXPSYN_FIELDS), (self.exp2syn, "Exp2Syn", EXP2SYN_FIELDS),
                            (self.halfgap, "HalfGap", HALFGAP_FIELDS), (self.gapjunction, "gapjunction_lr",
                                                                        GAPJ_FIELDS),
                            (self.gapnoptr, "gapjunction_noptr", GAPNP_FIELDS),
                            (self.graded, "neuron_to_neuron_syn_lr", GRADED_FIELDS)):
            if tab.n and (np.any(tab.nodes < 0) or np.any(tab.nodes >= n)):
                raise ValueError(f"{nm} node index out of range")
            if tab.n > 1 and np.any(np.diff(tab.nodes) < 0):
                raise ValueError(f"{nm} nodes must be sorted")
            for k in fl:
                v = tab.fields.get(k)
                if v is None or v.shape != (tab.n,) or v.dtype != F64:
                    raise ValueError(f"{nm}.{k} must be float64[{tab.n}]")
            for k, v in tab.ifields.items():
                if v.shape != (tab.n,) or v.dtype != I32:
                    raise ValueError(f"{nm}.{k} must be int32[{tab.n}]")
        for tab, nm in ((self.expsyn, "ExpSyn"), (self.exp2syn, "Exp2Syn")):
            src = tab.ifields.get("src")
            if src is None or (tab.n and (np.any(src < 0) or np.any(src >= nsrc))):
                raise ValueError(f"{nm}.src must index a cell PreSyn (0..ncell-1) or a NetStim (ncell..)")
            if tab.n and np.any(tab.fields["delay"] < self.dt):
                raise ValueError(f"{nm}: NetCon delays must be at least dt (one step)")
        for tab, nm, key in ((self.halfgap, "HalfGap", "src"), (self.gapjunction, "gapjunction_lr", "pre"),
                             (self.gapnoptr, "gapjunction_noptr", "src"),
                             (self.graded, "neuron_to_neuron_syn_lr", "pre")):
            pv = tab.ifields.get(key)
            if pv is None or (tab.n and (np.any(pv < 0) or np.any(pv >= n))):
                raise ValueError(f"{nm}.{key} must be a node index")
        if self.exp2syn.n and np.any(self.exp2syn.fields["tau2"] <= 0):
            raise ValueError("Exp2Syn.tau2 must be positive")
        if self.expsyn.n and np.any(self.expsyn.fields["tau"] <= 0):
            raise ValueError("ExpSyn.tau must be positive")
        if self.ps_thresh.shape != (self.ncell,) or self.ps_thresh.dtype != F64:
            raise ValueError(f"ps_thresh must be float64[{self.ncell}]")
        self._validate_lib()

    def _validate_lib(self) -> None:
        n = self.nnode
        for nm, tab in self.lib.items():
            if nm not in LIB_FIELDS:
                raise ValueError(f"unknown library mechanism {nm!r}")
            if tab.n and (np.any(tab.nodes < 0) or np.any(tab.nodes >= n)):
                raise ValueError(f"{nm} node index out of range")
            if tab.n > 1 and np.any(np.diff(tab.nodes) <= 0):
                raise ValueError(f"{nm} nodes must be sorted, one instance per node")
            for k in LIB_FIELDS[nm]:
                v = tab.fields.get(k)
                if v is None or v.shape != (tab.n,) or v.dtype != F64:
                    raise ValueError(f"{nm}.{k} must be float64[{tab.n}]")
        if "ca_ion" in self.lib:
            nz = self.lib["ca_ion"].ifields.get("nernst")
            if nz is None or nz.shape != (self.lib["ca_ion"].n,) or nz.dtype != I32:
                raise ValueError("ca_ion.nernst must be int32[n]")
            if np.any(self.lib["ca_ion"].fields["cai"] <= 0):
                raise ValueError("ca_ion.cai must be positive")
        for nm, ions in LIB_IONS.items():
            tab = self.lib.get(nm)
            if tab is None or not tab.n:
                continue
            for ion in ions:
                it = self.lib.get(ion + "_ion")
                if it is None or not np.all(np.isin(tab.nodes, it.nodes)):
                    raise ValueError(f"{nm} needs {ion}_ion on each of its nodes")
        cad, cin = self.lib.get("CaDynamics_E2"), self.lib.get("cainternm_lr")
        if cad is not None and cin is not None and np.intersect1d(cad.nodes, cin.nodes).size:
            raise ValueError("CaDynamics_E2 and cainternm_lr on one node: one calcium dynamics per node")
        for ion, key in (("na_ion", "ena"), ("k_ion", "ek")):
            it = self.lib.get(ion)
            if it is None or not it.n or not self.hh.n:
                continue
            common, ia, ib = np.intersect1d(it.nodes, self.hh.nodes, return_indices=True)
            if common.size and not np.array_equal(it.fields[key][ia], self.hh.fields[key][ib]):
                raise ValueError(f"{ion}.{key} differs from hh.{key} on a shared node")
        for nm, keys in LIB_GLOBALS.items():
            tab = self.lib.get(nm)
            if tab is None or not tab.n:
                continue
            for k in keys:
                if np.any(tab.fields[k] != tab.fields[k][0]):
                    raise ValueError(f"{nm}.{k} is a GLOBAL of the mechanism: one value for all instances")

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
            expsyn=self.expsyn.copy(),
            exp2syn=self.exp2syn.copy(),
            netstim=self.netstim.copy(),
            halfgap=self.halfgap.copy(),
            gapjunction=self.gapjunction.copy(),
            gapnoptr=self.gapnoptr.copy(),
            graded=self.graded.copy(),
            ps_thresh=self.ps_thresh.copy(),
            netstim_rng=self.netstim_rng,
            lib={k: v.copy() for k, v in self.lib.items()},
        )

    # ------------------------------------------------------------ parameters
    def param_view(self, mech: str, var: str) -> np.ndarray:
        """The live array of one learnable/settable parameter."""
        tab = {"hh": self.hh, "pas": self.pas, "IClamp": self.iclamp, "ExpSyn": self.expsyn,
               "Exp2Syn": self.exp2syn, "NetStim": self.netstim, "HalfGap": self.halfgap,
               "gapjunction_lr": self.gapjunction, "gapjunction_noptr": self.gapnoptr,
               "neuron_to_neuron_syn_lr": self.graded}.get(mech)
        if tab is None:
            if mech == "capacitance" and var == "cm":
                return self.cm
            if mech in self.lib and var in self.lib[mech].fields:
                return self.lib[mech].fields[var]
            raise KeyError(f"unknown mechanism {mech!r}")
        key = {"g_pas": "g", "e_pas": "e", "delay": "del"}.get(var, var)
        if key not in tab.fields:
            raise KeyError(f"unknown variable {mech}.{var}")
        return tab.fields[key]


def lib_par_matrix(g: "CellGroup", name: str) -> np.ndarray:
    """float64[n, npar] parameter columns of library table ``name`` in the
    order of the C tables (LIB_FIELDS, then ca_ion's nernst flag as 0/1);
    an absent table gives shape (0, npar)."""
    cols = list(LIB_FIELDS[name])
    tab = g.lib.get(name)
    n = tab.n if tab is not None else 0
    npar = len(cols) + (1 if name == "ca_ion" else 0)
    out = np.zeros((n, npar))
    if n:
        for c, k in enumerate(cols):
            out[:, c] = tab.fields[k]
        if name == "ca_ion":
            out[:, -1] = tab.ifields["nernst"] != 0
    return out


# states per library table, in the order the forward keeps them
LIB_STATES = {"ca_ion": ("cai",), "Ca_HVA": ("m", "h"), "Ca_LVAst": ("m", "h"), "Im": ("m",), "K_Pst": ("m", "h"),
              "K_Tst": ("m", "h"), "NaTg": ("m", "h"), "Nap_Et2": ("m", "h"), "SK_E2": ("z",), "SKv3_1": ("m",),
              "hd_la": ("l",), "km_la": ("n",), "kca_la": ("n",), "it2_la": ("m", "h"), "kdr_la": ("m",),
              "sca_la": ("m", "h"), "Ca": ("m", "h"),
              "shl1_lr": ("m", "hf", "hs",),
              "kvs1_lr": ("m", "h",),
              "irk_lr": ("m",),
              "egl36_lr": ("mf", "mm", "ms",),
              "shk1_lr": ("m", "h",),
              "egl2_lr": ("m",),
              "cca1_lr": ("m", "h"),
              "egl19_lr": ("m", "h"),
              "unc2_lr": ("m", "h"),
              "kcnl_lr": ("m",),
              "kqt3_lr": ("mf", "ms", "ww", "s"),
              "shl1": ("m", "hf", "hs"), "kvs1": ("m", "h"), "irk": ("m",), "egl36": ("mf", "mm", "ms"),
              "shk1": ("m", "h"), "egl2": ("m",), "cca1": ("m", "h"), "egl19": ("m", "h"), "unc2": ("m", "h"),
}


def empty_table(names, inames=()) -> MechTable:
    return MechTable(_i32([]), {k: _f64([]) for k in names}, {k: _i32([]) for k in inames})


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
    lib = {}
    for nm in LIB_NAMES:
        parts = [(g.lib[nm], m) for g, m in zip(groups, maps) if nm in g.lib]
        if not parts:
            continue
        nodes = np.concatenate([m[t.nodes] for t, m in parts])
        order = np.argsort(nodes, kind="stable")
        t0 = parts[0][0]
        lib[nm] = MechTable(
            _i32(nodes[order]),
            {k: _f64(np.concatenate([t.fields[k] for t, _ in parts])[order]) for k in t0.fields},
            {k: _i32(np.concatenate([t.ifields[k] for t, _ in parts])[order]) for k in t0.ifields},
        )
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
        lib=lib,
    )
    out.validate()
    return out
