"""ctypes binding of ``libhx_b200.so`` (declarations in include/heliox_b200.h).

There is no fallback: if the native library or a CUDA device is missing, the
calls raise.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libhx_b200.so")

_dp = C.POINTER(C.c_double)
_ip = C.POINTER(C.c_int)
_fp = C.POINTER(C.c_float)

HX_P = {
    "hh.gnabar": 0,
    "hh.gkbar": 1,
    "hh.gl": 2,
    "hh.el": 3,
    "pas.g": 4,
    "pas.e": 5,
    "cm": 6,
    "IClamp.amp": 7,
    "ExpSyn.weight": 8,
    "ExpSyn.e": 9,
    "Exp2Syn.weight": 10,
    "Exp2Syn.e": 11,
    "HalfGap.g": 12,
    "gapjunction_lr.g": 13,
    "gapjunction_lr.w": 14,
    "neuron_to_neuron_syn_lr.w": 15,
    "CaDynamics_E2.gamma": 16,
    "CaDynamics_E2.decay": 17,
    "CaDynamics_E2.depth": 18,
    "CaDynamics_E2.minCai": 19,
    "Ca_HVA.gbar": 20,
    "Ca_LVAst.gCa_LVAstbar": 21,
    "Im.gImbar": 22,
    "K_Pst.gK_Pstbar": 23,
    "K_Tst.gK_Tstbar": 24,
    "NaTg.gNaTgbar": 25,
    "Nap_Et2.gNap_Et2bar": 26,
    "SK_E2.gSK_E2bar": 27,
    "SKv3_1.gSKv3_1bar": 28,
    "hd_la.ghdbar": 29,
    "km_la.gbar": 30,
    "kca_la.gbar": 31,
    "it2_la.gcabar": 32,
    "kdr_la.gbar": 33,
    "sca_la.gbar": 34,
    "Ca.gCabar": 35,
    "shl1_lr.w": 36,
    "kvs1_lr.w": 37,
    "irk_lr.w": 38,
    "egl36_lr.w": 39,
    "shk1_lr.w": 40,
    "egl2_lr.w": 41,
    "cca1_lr.w": 42,
    "egl19_lr.w": 43,
    "unc2_lr.w": 44,
    "kcnl_lr.w": 45,
    "nca_lr.w": 46,
    "kqt3_lr.w": 47,
    "cainternm_lr.vcell": 48,
    "shl1.gbshl1": 49,
    "kvs1.gbkvs1": 50,
    "irk.gbirk": 51,
    "egl36.gbegl36": 52,
    "shk1.gbshk1": 53,
    "egl2.gbegl2": 54,
    "cca1.gbcca1": 55,
    "egl19.gbegl19": 56,
    "unc2.gbunc2": 57,
    "gapjunction_noptr.weight": 58,
}
HX_P_COUNT = 59
HX_LIB_NTYPE = 42


class LibTable(C.Structure):
    _fields_ = [("n", C.c_int), ("node", _ip), ("par", _dp)]


class LibDesc(C.Structure):
    _fields_ = [("t", LibTable * HX_LIB_NTYPE)]


class GroupDesc(C.Structure):
    _fields_ = [
        ("ncell", C.c_int),
        ("nnode", C.c_int),
        ("parent", _ip),
        ("a", _dp),
        ("b", _dp),
        ("area", _dp),
        ("cm", _dp),
        ("celsius", C.c_double),
        ("dt", C.c_double),
        ("nhh", C.c_int),
        ("hh_node", _ip),
        ("hh_gnabar", _dp),
        ("hh_gkbar", _dp),
        ("hh_gl", _dp),
        ("hh_el", _dp),
        ("hh_ena", _dp),
        ("hh_ek", _dp),
        ("npas", C.c_int),
        ("pas_node", _ip),
        ("pas_g", _dp),
        ("pas_e", _dp),
        ("nic", C.c_int),
        ("ic_node", _ip),
        ("ic_del", _dp),
        ("ic_dur", _dp),
        ("ic_amp", _dp),
        ("gid_base", C.c_int), ("nsrc_cells", C.c_int),
        ("ps_thresh", _dp),
        ("nexpsyn", C.c_int), ("expsyn_node", _ip), ("expsyn_src", _ip),
        ("expsyn_tau", _dp), ("expsyn_e", _dp), ("expsyn_delay", _dp), ("expsyn_weight", _dp),
        ("nexp2syn", C.c_int), ("exp2syn_node", _ip), ("exp2syn_src", _ip),
        ("exp2syn_tau1", _dp), ("exp2syn_tau2", _dp), ("exp2syn_e", _dp), ("exp2syn_delay", _dp),
        ("exp2syn_weight", _dp),
        ("nnetstim", C.c_int), ("ns_interval", _dp), ("ns_number", _dp), ("ns_start", _dp), ("ns_noise", _dp),
        ("netstim_rng", C.c_int),
        ("nhalfgap", C.c_int), ("hg_node", _ip), ("hg_src", _ip), ("hg_g", _dp),
        ("ngapj", C.c_int), ("gj_node", _ip), ("gj_pre", _ip), ("gj_g", _dp), ("gj_w", _dp),
        ("ngapnp", C.c_int), ("gn_node", _ip), ("gn_src", _ip), ("gn_weight", _dp),
        ("ngraded", C.c_int), ("gr_node", _ip), ("gr_pre", _ip), ("gr_w", _dp), ("gr_delta", _dp), ("gr_vth", _dp),
        ("lib", C.POINTER(LibDesc)),
    ]


# int (*)(void* user, const void* send_dev, void* recv_dev, int cap_entries, void* stream)
EXCHANGE_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p)
# int (*)(void* user, double* grad_dev, int n, void* stream)
ALLREDUCE_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p)


class PlanStats(C.Structure):
    _fields_ = [
        ("npack", C.c_int),
        ("max_pack_nodes", C.c_int),
        ("max_pack_hh", C.c_int),
        ("max_levels", C.c_int),
        ("max_crit_nodes", C.c_int),
        ("nbranch", C.c_int),
        ("imbalance", C.c_double),
        ("smem_fwd", C.c_size_t),
        ("smem_bwd", C.c_size_t),
        ("nsub", C.c_int),
        ("est_max", C.c_double),
        ("est_mean", C.c_double),
    ]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


# name -> (restype, argtypes)
SIGNATURES = {
    "hx_abi_version": (C.c_int, []),
    "hx_create": (C.c_int, [C.POINTER(C.c_void_p), C.c_int]),
    "hx_destroy": (C.c_int, [C.c_void_p]),
    "hx_last_error": (C.c_char_p, [C.c_void_p]),
    "hx_set_stream": (C.c_int, [C.c_void_p, C.c_void_p]),
    "hx_set_pack_target": (C.c_int, [C.c_void_p, C.c_int]),
    "hx_set_tape_budget": (C.c_int, [C.c_void_p, C.c_size_t]),
    "hx_set_split_barrier_limit": (C.c_int, [C.c_void_p, C.c_longlong]),
    "hx_set_grid_sync": (C.c_int, [C.c_void_p, C.c_int]),
    "hx_set_grad_kinds": (C.c_int, [C.c_void_p, _ip, C.c_int]),
    "hx_load_group": (C.c_int, [C.c_void_p, C.POINTER(GroupDesc)]),
    "hx_get_plan_stats": (C.c_int, [C.c_void_p, C.POINTER(PlanStats)]),
    "hx_plan_check": (C.c_int, [C.POINTER(GroupDesc), C.c_int, C.POINTER(PlanStats), _dp, _dp]),
    "hx_plan_check_cap": (C.c_int, [C.POINTER(GroupDesc), C.c_int, C.c_int, C.POINTER(PlanStats), _dp, _dp]),
    "hx_simulate_and_adjoint_into": (C.c_int, [C.c_void_p, _fp, C.c_int, C.c_int, _ip, C.c_int, _fp, _fp, C.c_int,
                                               _ip, _ip, _ip, _fp, C.c_double, C.c_double, C.c_double, C.c_int]),
    "hx_plan_check_sm": (C.c_int, [C.POINTER(GroupDesc), C.c_int, C.c_int, C.c_int, C.POINTER(PlanStats), _dp, _dp]),
    "hx_set_param": (C.c_int, [C.c_void_p, C.c_int, _dp, C.c_int]),
    "hx_get_param": (C.c_int, [C.c_void_p, C.c_int, _dp, C.c_int]),
    "hx_simulate": (C.c_int, [C.c_void_p, C.c_int, C.c_double, C.c_int, _ip, _dp]),
    "hx_forward_capture": (C.c_int, [C.c_void_p, C.c_int, C.c_double, C.c_int, _ip, _dp]),
    "hx_forward_capture_dev": (C.c_int, [C.c_void_p, C.c_int, C.c_double, C.c_int, _ip, C.c_void_p]),
    "hx_backward": (C.c_int, [C.c_void_p, _dp, C.POINTER(_dp)]),
    "hx_backward_dev": (C.c_int, [C.c_void_p, C.c_void_p, C.POINTER(C.c_void_p)]),
    "hx_reduce_grads_f32": (C.c_int, [C.c_void_p, C.c_int, _ip, _ip, _ip, _fp, _fp, C.c_int]),
    "hx_mse_loss_grad_dev": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
    "hx_mse_loss_grad_noalloc": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                            C.c_void_p]),
    "hx_last_kernel_ms": (C.c_int, [C.c_void_p, C.c_int, _dp, _ip]),
    "hx_rcp_nz_dev": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]),
    "hx_opt_create_adam": (C.c_int, [C.c_void_p, C.c_double, C.c_double, C.c_double]),
    "hx_opt_add_params": (C.c_int, [C.c_void_p, C.c_int, C.c_int, _ip, _ip, C.c_double]),
    "hx_opt_set_grads_f32": (C.c_int, [C.c_void_p, C.c_int, _fp, C.c_int]),
    "hx_opt_grads_from_backward": (C.c_int, [C.c_void_p, C.c_int, C.c_double]),
    "hx_opt_grad_buffer": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_void_p), _ip]),
    "hx_opt_step": (C.c_int, [C.c_void_p, C.c_int, C.c_double, C.c_double]),
    "hx_opt_set_allreduce": (C.c_int, [C.c_void_p, C.c_int, ALLREDUCE_FN, C.c_void_p]),
    "hx_opt_get_adam_state": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_longlong), _dp, _dp, C.c_int, _dp]),
    "hx_opt_set_adam_state": (C.c_int, [C.c_void_p, C.c_int, C.c_longlong, _dp, _dp, C.c_int, _dp]),
    "hx_opt_reset": (C.c_int, [C.c_void_p, C.c_int]),
    "hx_get_spikes": (C.c_int, [C.c_void_p, C.c_int, _ip, _dp, _ip]),
    "hx_netstim_trains": (C.c_int, [C.POINTER(GroupDesc), C.c_int, C.c_int, _ip, _ip, _ip]),
    "hx_set_exchange": (C.c_int, [C.c_void_p, EXCHANGE_FN, C.c_void_p, C.c_int, C.c_int]),
    "hx_set_window": (C.c_int, [C.c_void_p, C.c_int]),
    "hx_get_window": (C.c_int, [C.c_void_p, _ip]),
    "hx_exchange_merge_status": (C.c_int, [_ip, C.c_int, _ip, _ip, _ip, _ip]),
}

_LIB = None


def load(path: str = LIB_PATH):
    """Load the native library (raises if it has not been built)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(path):
        raise RuntimeError(f"heliox_b200 native library missing: {path} (run heliox_b200/build.py)")
    L = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _LIB = L
    return L


def dptr(x: np.ndarray):
    return x.ctypes.data_as(_dp)


def iptr(x: np.ndarray):
    return x.ctypes.data_as(_ip)


def fptr(x: np.ndarray):
    return x.ctypes.data_as(_fp)


class BoundGroup:
    """A GroupDesc pointing at contiguous numpy copies of a CellGroup's arrays.

    ``gid_base`` / ``nsrc_cells``: this group's first global cell id and the
    number of cells over all groups of a multi-GPU job (0 = the group alone).
    """

    def __init__(self, g, gid_base: int = 0, nsrc_cells: int = 0):
        self.keep = []

        def D(x):
            x = np.ascontiguousarray(x, dtype=np.float64)
            self.keep.append(x)
            return dptr(x)

        def I(x):
            x = np.ascontiguousarray(x, dtype=np.int32)
            self.keep.append(x)
            return iptr(x)

        s = GroupDesc()
        s.ncell, s.nnode = g.ncell, g.nnode
        s.parent = I(g.parent)
        s.a, s.b, s.area, s.cm = D(g.a), D(g.b), D(g.area), D(g.cm)
        s.celsius, s.dt = float(g.celsius), float(g.dt)
        h = g.hh
        s.nhh = h.n
        s.hh_node = I(h.nodes)
        s.hh_gnabar, s.hh_gkbar, s.hh_gl, s.hh_el = (D(h.fields[k]) for k in ("gnabar", "gkbar", "gl", "el"))
        s.hh_ena, s.hh_ek = D(h.fields["ena"]), D(h.fields["ek"])
        p = g.pas
        s.npas = p.n
        s.pas_node = I(p.nodes)
        s.pas_g, s.pas_e = D(p.fields["g"]), D(p.fields["e"])
        c = g.iclamp
        s.nic = c.n
        s.ic_node = I(c.nodes)
        s.ic_del, s.ic_dur, s.ic_amp = D(c.fields["del"]), D(c.fields["dur"]), D(c.fields["amp"])
        # network parts (all empty for a group without them)
        s.gid_base = int(gid_base)
        s.nsrc_cells = int(nsrc_cells) if nsrc_cells else g.ncell
        s.ps_thresh = D(g.ps_thresh) if g.has_network else _dp()
        e1, e2 = g.expsyn, g.exp2syn
        s.nexpsyn, s.expsyn_node, s.expsyn_src = e1.n, I(e1.nodes), I(e1.ifields["src"])
        s.expsyn_tau, s.expsyn_e, s.expsyn_delay, s.expsyn_weight = (
            D(e1.fields[k]) for k in ("tau", "e", "delay", "weight"))
        s.nexp2syn, s.exp2syn_node, s.exp2syn_src = e2.n, I(e2.nodes), I(e2.ifields["src"])
        s.exp2syn_tau1, s.exp2syn_tau2, s.exp2syn_e, s.exp2syn_delay, s.exp2syn_weight = (
            D(e2.fields[k]) for k in ("tau1", "tau2", "e", "delay", "weight"))
        ns = g.netstim
        s.nnetstim = ns.n
        s.ns_interval, s.ns_number, s.ns_start, s.ns_noise = (
            D(ns.fields[k]) for k in ("interval", "number", "start", "noise"))
        s.netstim_rng = int(g.netstim_rng)
        hg = g.halfgap
        s.nhalfgap, s.hg_node, s.hg_src, s.hg_g = hg.n, I(hg.nodes), I(hg.ifields["src"]), D(hg.fields["g"])
        gj = g.gapjunction
        s.ngapj, s.gj_node, s.gj_pre = gj.n, I(gj.nodes), I(gj.ifields["pre"])
        s.gj_g, s.gj_w = D(gj.fields["g"]), D(gj.fields["w"])
        gn = g.gapnoptr
        s.ngapnp, s.gn_node, s.gn_src, s.gn_weight = gn.n, I(gn.nodes), I(gn.ifields["src"]), D(gn.fields["weight"])
        gr = g.graded
        s.ngraded, s.gr_node, s.gr_pre = gr.n, I(gr.nodes), I(gr.ifields["pre"])
        s.gr_w, s.gr_delta, s.gr_vth = D(gr.fields["w"]), D(gr.fields["delta"]), D(gr.fields["Vth"])
        self.lib = None
        if any(t.n for t in g.lib.values()):
            from .model import LIB_NAMES, lib_par_matrix

            lb = LibDesc()
            for t, nm in enumerate(LIB_NAMES):
                tab = g.lib.get(nm)
                lb.t[t].n = tab.n if tab is not None else 0
                lb.t[t].node = I(tab.nodes if tab is not None else np.zeros(0, np.int32))
                lb.t[t].par = D(lib_par_matrix(g, nm).reshape(-1))
            self.lib = lb
            s.lib = C.pointer(lb)
        self.desc = s


def netstim_trains(g, nstep: int):
    """NetStim spike trains of ``g`` from the native host generator (no GPU):
    arrays (instance, step) in emission order."""
    L = load()
    b = BoundGroup(g)
    n = C.c_int(0)
    rc = L.hx_netstim_trains(C.byref(b.desc), int(nstep), 0, _ip(), _ip(), C.byref(n))
    if rc != 0:
        raise ValueError("hx_netstim_trains failed")
    cap = int(n.value)
    ids = np.zeros(max(cap, 1), dtype=np.int32)
    steps = np.zeros(max(cap, 1), dtype=np.int32)
    rc = L.hx_netstim_trains(C.byref(b.desc), int(nstep), cap, iptr(ids), iptr(steps), C.byref(n))
    if rc != 0:
        raise ValueError("hx_netstim_trains failed")
    return ids[:cap], steps[:cap]


def plan_check(g, nodes_per_pack: int = 0, max_pack_nodes: int = 0, nsm: int = 0):
    """Host-only plan build + CPU check of the planned Hines order (no GPU needed).

    nsm > 0 plans for a device of that many SMs (CTAs balanced over waves)."""
    L = load()
    b = BoundGroup(g)
    st = PlanStats()
    diff = C.c_double(-1.0)
    pq = C.c_double(-1.0)
    rc = L.hx_plan_check_sm(C.byref(b.desc), int(nodes_per_pack), int(max_pack_nodes), int(nsm), C.byref(st),
                            C.byref(diff), C.byref(pq))
    if rc != 0:
        raise ValueError(f"hx_plan_check failed (rc={rc})")
    d = st.as_dict()
    d["pq_rel_diff"] = float(pq.value)
    return d, float(diff.value)
