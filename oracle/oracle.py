"""ctypes wrapper of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may
import this module; the product package never does.  See ``hx_oracle.h`` for
what the oracle restates and how it is pinned to the reference.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from typing import Dict, Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

_dp = C.POINTER(C.c_double)
_ip = C.POINTER(C.c_int)


class _Net(C.Structure):
    _fields_ = [
        ("nexp", C.c_int), ("exp_node", _ip), ("exp_src", _ip),
        ("exp_tau", _dp), ("exp_e", _dp), ("exp_delay", _dp), ("exp_w", _dp),
        ("nexp2", C.c_int), ("exp2_node", _ip), ("exp2_src", _ip),
        ("exp2_tau1", _dp), ("exp2_tau2", _dp), ("exp2_e", _dp), ("exp2_delay", _dp), ("exp2_w", _dp),
        ("ps_thresh", _dp),
        ("nstim", C.c_int), ("ns_interval", _dp), ("ns_number", _dp), ("ns_start", _dp), ("ns_noise", _dp),
        ("rng_mode", C.c_int),
        ("nhg", C.c_int), ("hg_node", _ip), ("hg_src", _ip), ("hg_g", _dp),
        ("ngj", C.c_int), ("gj_node", _ip), ("gj_pre", _ip), ("gj_g", _dp), ("gj_w", _dp),
        ("ngn", C.c_int), ("gn_node", _ip), ("gn_src", _ip), ("gn_w", _dp),
        ("ngr", C.c_int), ("gr_node", _ip), ("gr_pre", _ip), ("gr_w", _dp), ("gr_g", _dp), ("gr_delta", _dp),
        ("gr_k", _dp), ("gr_vth", _dp), ("gr_erev", _dp),
        ("spike_cap", C.c_int), ("spike_gid", _ip), ("spike_t", _dp), ("nspike", C.c_int),
        ("ns_spike_cap", C.c_int), ("ns_spike_id", _ip), ("ns_spike_t", _dp), ("ns_nspike", C.c_int),
    ]


class _LibTable(C.Structure):
    _fields_ = [("n", C.c_int), ("node", _ip), ("par", _dp)]


class _Lib(C.Structure):
    _fields_ = [("t", _LibTable * 42)]


class _Group(C.Structure):
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
        ("net", C.POINTER(_Net)),
        ("lib", C.POINTER(_Lib)),
    ]


class _Grads(C.Structure):
    _fields_ = [
        ("hh_gnabar", _dp),
        ("hh_gkbar", _dp),
        ("hh_gl", _dp),
        ("hh_el", _dp),
        ("pas_g", _dp),
        ("pas_e", _dp),
        ("cm", _dp),
        ("ic_amp", _dp),
        ("exp_w", _dp), ("exp_e", _dp), ("exp2_w", _dp), ("exp2_e", _dp),
        ("hg_g", _dp), ("gj_g", _dp), ("gj_w", _dp), ("gr_w", _dp),
        ("gn_w", _dp),
    ]


REF_LIB = os.path.join(_HERE, "_ref", "hxref_run")


def ref_available() -> bool:
    """True when the reference's own CPU integrator was compiled into oracle/_ref."""
    return os.path.exists(REF_LIB)


def ref_forward(g, nstep: int, probe: Optional[Sequence[int]] = None, v_init: Optional[float] = None,
                workdir: Optional[str] = None, permute_type: int = 0, timing: bool = False):
    """Run the reference's own CPU integrator (oracle/_ref/hxref_run) on ``g``.

    The group is exported in CoreNEURON format (heliox_b200.coredat) and loaded
    by the reference's read_coredat/data_format_trans with node permutation
    ``permute_type`` (0, 1 or 3); returns (trace[(nstep+1), nprobe], spikes
    list of (t, gid)), plus, with ``timing``, the seconds the reference spent
    in finitialize and its fadvance loop (measured inside the harness:
    loading, export and output are not counted).
    """
    import shutil
    import tempfile

    from heliox_b200.coredat import write_coredat

    if not ref_available():
        raise RuntimeError("reference harness not built (oracle/ref_build.sh)")
    probe = np.ascontiguousarray(g.soma_nodes() if probe is None else probe, dtype=np.int32)
    tmp = tempfile.mkdtemp(prefix="hxref_", dir=workdir)
    try:
        data = os.path.join(tmp, "data")
        write_coredat(g, data)
        pf = os.path.join(tmp, "probes.i32")
        probe.tofile(pf)
        tf = os.path.join(tmp, "trace.f64")
        spk = os.path.join(tmp, "spk")
        vi = float(g.v_init if v_init is None else v_init)
        r = subprocess.run([REF_LIB, data, str(int(permute_type)), repr(float(g.dt)), str(int(nstep)), repr(vi), pf,
                            tf, spk], capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"reference run failed ({r.returncode}):\n{r.stdout[-2000:]}\n{r.stderr[-2000:]}")
        trace = np.fromfile(tf, dtype=np.float64).reshape(nstep + 1, probe.shape[0])
        spikes = []
        sf = os.path.join(spk, "spk.dat")
        if os.path.exists(sf):
            for line in open(sf):
                t, gid = line.split()
                spikes.append((float(t), int(gid)))
        if timing:
            secs = [float(line.split()[1]) for line in r.stdout.splitlines() if line.startswith("HXREF_FADVANCE_S")]
            return trace, spikes, secs[-1]
        return trace, spikes
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


REF_GPU = os.path.join(_HERE, "_ref", "hxref_run_gpu")


def ref_forward_gpu(g, nstep: int, probe: Optional[Sequence[int]] = None, v_init: Optional[float] = None,
                    timing_only: bool = False, permute_type: int = 0):
    """Run the reference's GPU integrator (Simulate(GPU): fadvance_gpu and its
    kernels, oracle/_ref/hxref_run_gpu) on ``g`` with node permutation
    ``permute_type`` (0: cuda_solve_matrix, 3: its cop_solve_kernel); needs a
    CUDA device.

    Returns (trace, spikes, seconds): with ``timing_only`` the trace holds only
    the initial and final rows and the seconds are the fadvance loop between
    two device synchronisations; otherwise every step is recorded (a copy of
    v back to the host per step) and the seconds include those copies.
    """
    import shutil
    import tempfile

    from heliox_b200.coredat import write_coredat

    if not os.path.exists(REF_GPU):
        raise RuntimeError("reference GPU harness not built (oracle/ref_build.sh)")
    probe = np.ascontiguousarray(g.soma_nodes() if probe is None else probe, dtype=np.int32)
    tmp = tempfile.mkdtemp(prefix="hxrefg_")
    try:
        data = os.path.join(tmp, "data")
        write_coredat(g, data)
        pf = os.path.join(tmp, "probes.i32")
        probe.tofile(pf)
        tf = os.path.join(tmp, "trace.f64")
        spk = os.path.join(tmp, "spk")
        vi = float(g.v_init if v_init is None else v_init)
        r = subprocess.run([REF_GPU, data, str(int(permute_type)), repr(float(g.dt)), str(int(nstep)), repr(vi), pf,
                            tf, spk, "gpu-time" if timing_only else "gpu"], capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"reference GPU run failed ({r.returncode}):\n{r.stdout[-2000:]}\n{r.stderr[-2000:]}")
        trace = np.fromfile(tf, dtype=np.float64).reshape(nstep + 1, probe.shape[0])
        spikes = []
        sf = os.path.join(spk, "spk.dat")
        if os.path.exists(sf):
            for line in open(sf):
                t, gid = line.split()
                spikes.append((float(t), int(gid)))
        secs = [float(x.split()[1]) for x in r.stdout.splitlines() if x.startswith("HXREF_FADVANCE_S")]
        return trace, spikes, secs[-1]
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


def adam_port(w0, grads, lr, inv_record_steps, beta1=0.9, beta2=0.999, eps=1e-8, impedance=1.0):
    """Restatement of AdamOptimizer::step_cpu (src/optimizer/optimizer.cpp:351-397)
    for one weight per entry, same operation order.  Returns (weights after each
    step [steps, n], m, v)."""
    import math

    w = np.array(w0, dtype=np.float64)
    m = np.zeros_like(w)
    v = np.zeros_like(w)
    out = []
    for s, g in enumerate(np.asarray(grads, dtype=np.float64), start=1):
        sg = (g / 1.0) * impedance * inv_record_steps
        m = beta1 * m + (1.0 - beta1) * sg
        v = beta2 * v + (1.0 - beta2) * sg * sg
        b1 = math.pow(beta1, float(s))
        b2 = math.pow(beta2, float(s))
        mh = m / (1.0 - b1)
        vh = v / (1.0 - b2)
        w = w - lr * mh / (np.sqrt(vh) + eps)
        out.append(w.copy())
    return np.array(out), m, v


def adam_ref(w0, grads, lr, inv_record_steps, beta1=0.9, beta2=0.999, eps=1e-8, impedance=1.0):
    """The reference's own AdamOptimizer (CPU mode) through the harness."""
    import tempfile

    w0 = np.asarray(w0, dtype=np.float64)
    grads = np.asarray(grads, dtype=np.float64)
    n, steps = w0.shape[0], grads.shape[0]
    with tempfile.TemporaryDirectory() as d:
        fi, fo = os.path.join(d, "in.f64"), os.path.join(d, "out.f64")
        np.concatenate([w0, grads.ravel()]).tofile(fi)
        r = subprocess.run([REF_LIB, "--adam", str(n), str(steps), repr(lr), repr(inv_record_steps), repr(beta1),
                            repr(beta2), repr(eps), repr(impedance), fi, fo], capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"reference Adam failed ({r.returncode}): {r.stderr[-500:]}")
        out = np.fromfile(fo, dtype=np.float64)
    ws = out[: steps * n].reshape(steps, n)
    return ws, out[steps * n: steps * n + n], out[steps * n + n:]


def build() -> str:
    """Compile the oracle (make) and return the .so path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return os.path.join(_HERE, "libhxoracle.so")


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "libhxoracle.so")
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        L.hxo_forward.argtypes = [C.POINTER(_Group), C.c_double, C.c_int, C.c_int, _ip, _dp, _dp, _dp, _dp, _dp]
        L.hxo_forward.restype = C.c_int
        L.hxo_adjoint.argtypes = [C.POINTER(_Group), C.c_double, C.c_int, C.c_int, _ip, _dp, _dp, C.POINTER(_Grads)]
        L.hxo_adjoint.restype = C.c_int
        L.hxo_forward_lib.argtypes = [C.POINTER(_Group), C.c_double, C.c_int, C.c_int, _ip, _dp, _dp, C.c_int]
        L.hxo_forward_lib.restype = C.c_int
        L.hxo_last_reverse_seconds.argtypes = []
        L.hxo_last_reverse_seconds.restype = C.c_double
        _LIB = L
    return _LIB


def _d(x):
    return x.ctypes.data_as(_dp)


def _i(x):
    return x.ctypes.data_as(_ip)


class _Bound:
    """Keeps numpy arrays alive while the ctypes struct points at them."""

    def __init__(self, g):
        self.keep = []

        def D(x):
            x = np.ascontiguousarray(x, dtype=np.float64)
            self.keep.append(x)
            return _d(x)

        def I(x):
            x = np.ascontiguousarray(x, dtype=np.int32)
            self.keep.append(x)
            return _i(x)

        s = _Group()
        s.ncell = g.ncell
        s.nnode = g.nnode
        s.parent = I(g.parent)
        s.a, s.b, s.area, s.cm = D(g.a), D(g.b), D(g.area), D(g.cm)
        s.celsius = g.celsius
        s.dt = g.dt
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
        self.net = None
        if g.has_network:
            n = _Net()
            e1, e2 = g.expsyn, g.exp2syn
            n.nexp, n.exp_node, n.exp_src = e1.n, I(e1.nodes), I(e1.ifields["src"])
            n.exp_tau, n.exp_e, n.exp_delay, n.exp_w = (D(e1.fields[k]) for k in ("tau", "e", "delay", "weight"))
            n.nexp2, n.exp2_node, n.exp2_src = e2.n, I(e2.nodes), I(e2.ifields["src"])
            n.exp2_tau1, n.exp2_tau2, n.exp2_e, n.exp2_delay, n.exp2_w = (
                D(e2.fields[k]) for k in ("tau1", "tau2", "e", "delay", "weight"))
            n.ps_thresh = D(g.ps_thresh)
            ns = g.netstim
            n.nstim = ns.n
            n.ns_interval, n.ns_number, n.ns_start, n.ns_noise = (
                D(ns.fields[k]) for k in ("interval", "number", "start", "noise"))
            n.rng_mode = int(g.netstim_rng)
            hg = g.halfgap
            n.nhg, n.hg_node, n.hg_src, n.hg_g = hg.n, I(hg.nodes), I(hg.ifields["src"]), D(hg.fields["g"])
            gj = g.gapjunction
            n.ngj, n.gj_node, n.gj_pre = gj.n, I(gj.nodes), I(gj.ifields["pre"])
            n.gj_g, n.gj_w = D(gj.fields["g"]), D(gj.fields["w"])
            gn = g.gapnoptr
            n.ngn, n.gn_node, n.gn_src, n.gn_w = gn.n, I(gn.nodes), I(gn.ifields["src"]), D(gn.fields["weight"])
            gr = g.graded
            n.ngr, n.gr_node, n.gr_pre = gr.n, I(gr.nodes), I(gr.ifields["pre"])
            n.gr_w, n.gr_g, n.gr_delta, n.gr_k, n.gr_vth, n.gr_erev = (
                D(gr.fields[k]) for k in ("w", "g", "delta", "k", "Vth", "erev"))
            cap = 1 << 16
            self.spk_gid = np.zeros(cap, dtype=np.int32)
            self.spk_t = np.zeros(cap)
            n.spike_cap, n.spike_gid, n.spike_t, n.nspike = cap, _i(self.spk_gid), _d(self.spk_t), 0
            self.ns_id = np.zeros(cap, dtype=np.int32)
            self.ns_t = np.zeros(cap)
            n.ns_spike_cap, n.ns_spike_id, n.ns_spike_t, n.ns_nspike = cap, _i(self.ns_id), _d(self.ns_t), 0
            self.net = n
            s.net = C.pointer(n)
        self.lib = None
        if g.lib:
            from heliox_b200.model import LIB_NAMES, lib_par_matrix

            lb = _Lib()
            for t, nm in enumerate(LIB_NAMES):
                tab = g.lib.get(nm)
                lb.t[t].n = tab.n if tab is not None else 0
                lb.t[t].node = I(tab.nodes if tab is not None else np.zeros(0, np.int32))
                lb.t[t].par = D(lib_par_matrix(g, nm).reshape(-1))
            self.lib = lb
            s.lib = C.pointer(lb)
        self.s = s

    def netstim_spikes(self):
        """NetStim spikes as a list of (t, instance) in emission order."""
        if self.net is None:
            return []
        k = min(self.net.ns_nspike, self.net.ns_spike_cap)
        return [(float(self.ns_t[i]), int(self.ns_id[i])) for i in range(k)]

    def spikes(self):
        """Detected PreSyn spikes as a list of (t, gid) in detection order."""
        if self.net is None:
            return []
        k = min(self.net.nspike, self.net.spike_cap)
        return [(float(self.spk_t[i]), int(self.spk_gid[i])) for i in range(k)]


def forward(g, nstep: int, probe: Optional[Sequence[int]] = None, v_init: Optional[float] = None):
    """Run finitialize + nstep steps; returns (trace[(nstep+1), nprobe], final_state dict)."""
    L = lib()
    probe = np.ascontiguousarray(g.soma_nodes() if probe is None else probe, dtype=np.int32)
    b = _Bound(g)
    trace = np.zeros((nstep + 1, probe.shape[0]))
    vf = np.zeros(g.nnode)
    nh = max(g.hh.n, 1)
    mf, hf, nf = np.zeros(nh), np.zeros(nh), np.zeros(nh)
    rc = L.hxo_forward(C.byref(b.s), float(g.v_init if v_init is None else v_init), int(nstep), int(probe.shape[0]),
                       _i(probe), _d(trace), _d(vf), _d(mf), _d(hf), _d(nf))
    if rc != 0:
        raise RuntimeError("oracle forward failed")
    return trace, {"v": vf, "m": mf[: g.hh.n], "h": hf[: g.hh.n], "n": nf[: g.hh.n], "spikes": b.spikes(),
                   "netstim_spikes": b.netstim_spikes()}


def forward_lib(g, nstep: int, probe: Optional[Sequence[int]] = None, v_init: Optional[float] = None):
    """Forward of a group with library mechanisms; returns (trace, final
    library states {"<mech>.<state>": array per instance})."""
    from heliox_b200.model import LIB_NAMES, LIB_STATES

    L = lib()
    probe = np.ascontiguousarray(g.soma_nodes() if probe is None else probe, dtype=np.int32)
    b = _Bound(g)
    trace = np.zeros((nstep + 1, probe.shape[0]))
    sizes = [(nm, g.lib[nm].n, LIB_STATES[nm]) for nm in LIB_NAMES if nm in g.lib and nm in LIB_STATES]
    buf = np.zeros(sum(n * len(st) for _, n, st in sizes) + 1)
    rc = L.hxo_forward_lib(C.byref(b.s), float(g.v_init if v_init is None else v_init), int(nstep),
                           int(probe.shape[0]), _i(probe), _d(trace), _d(buf), int(buf.shape[0]))
    if rc != 0:
        raise RuntimeError("oracle forward failed")
    out, k = {}, 0
    for nm, n, st in sizes:
        blk = buf[k: k + n * len(st)].reshape(n, len(st))
        k += n * len(st)
        for c, sn in enumerate(st):
            out[f"{nm}.{sn}"] = blk[:, c].copy()
    return trace, out


GRAD_KEYS = ("hh.gnabar", "hh.gkbar", "hh.gl", "hh.el", "pas.g", "pas.e", "cm", "IClamp.amp")
NET_GRAD_KEYS = ("ExpSyn.weight", "ExpSyn.e", "Exp2Syn.weight", "Exp2Syn.e", "HalfGap.g", "gapjunction_lr.g",
                 "gapjunction_lr.w", "neuron_to_neuron_syn_lr.w", "gapjunction_noptr.weight")


def adjoint(g, nstep: int, dLdv: np.ndarray, probe: Optional[Sequence[int]] = None, v_init: Optional[float] = None):
    """Forward + reverse sweep; returns (trace, grads dict keyed by GRAD_KEYS).
    ``grads["reverse_s"]`` is the wall time of the reverse sweep alone."""
    L = lib()
    probe = np.ascontiguousarray(g.soma_nodes() if probe is None else probe, dtype=np.int32)
    dLdv = np.ascontiguousarray(dLdv, dtype=np.float64)
    if dLdv.shape != (nstep + 1, probe.shape[0]):
        raise ValueError("dLdv must have shape (nstep+1, nprobe)")
    b = _Bound(g)
    trace = np.zeros((nstep + 1, probe.shape[0]))
    out: Dict[str, np.ndarray] = {
        "hh.gnabar": np.zeros(g.hh.n),
        "hh.gkbar": np.zeros(g.hh.n),
        "hh.gl": np.zeros(g.hh.n),
        "hh.el": np.zeros(g.hh.n),
        "pas.g": np.zeros(g.pas.n),
        "pas.e": np.zeros(g.pas.n),
        "cm": np.zeros(g.nnode),
        "IClamp.amp": np.zeros(g.iclamp.n),
    }
    gs = _Grads()
    gs.hh_gnabar, gs.hh_gkbar, gs.hh_gl, gs.hh_el = (_d(out[k]) for k in GRAD_KEYS[:4])
    gs.pas_g, gs.pas_e, gs.cm, gs.ic_amp = (_d(out[k]) for k in GRAD_KEYS[4:])
    if g.has_network:
        sizes = (g.expsyn.n, g.expsyn.n, g.exp2syn.n, g.exp2syn.n, g.halfgap.n, g.gapjunction.n, g.gapjunction.n,
                 g.graded.n, g.gapnoptr.n)
        for k, nsz in zip(NET_GRAD_KEYS, sizes):
            out[k] = np.zeros(nsz)
        gs.exp_w, gs.exp_e, gs.exp2_w, gs.exp2_e, gs.hg_g, gs.gj_g, gs.gj_w, gs.gr_w, gs.gn_w = (
            _d(out[k]) for k in NET_GRAD_KEYS)
    rc = L.hxo_adjoint(C.byref(b.s), float(g.v_init if v_init is None else v_init), int(nstep), int(probe.shape[0]),
                       _i(probe), _d(dLdv), _d(trace), C.byref(gs))
    if rc != 0:
        raise RuntimeError("oracle adjoint failed")
    if g.has_network:
        out["spikes"] = b.spikes()
    out["reverse_s"] = float(L.hxo_last_reverse_seconds())
    return trace, out
