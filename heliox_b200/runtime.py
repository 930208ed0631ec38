"""Host-side mirror of the reference's ``Sim`` operator surface for the hot path.

The reference exposes a nanobind class ``Sim`` (src/python_api/PyBindings.cpp:12-266)
whose learning entry points run a forward capture and a gradient replay through
``LearnRuntime`` (src/runtime_api/learn/LearnRuntime.h:21-293).  ``Sim`` here keeps
the same verbs -- variable handles, simulate, capture, backward, the
MappedSignal column reduction and the external-gradient Adam optimizer -- and
calls the native library (include/heliox_b200.h) for every computation.
"""
from __future__ import annotations

import ctypes as C
from typing import Dict, Iterable, Optional, Sequence

import numpy as np

from . import _lib
from .model import CellGroup

_MECH_VAR = {
    ("hh", "gnabar"): "hh.gnabar",
    ("hh", "gkbar"): "hh.gkbar",
    ("hh", "gl"): "hh.gl",
    ("hh", "el"): "hh.el",
    ("pas", "g_pas"): "pas.g",
    ("pas", "g"): "pas.g",
    ("pas", "e_pas"): "pas.e",
    ("pas", "e"): "pas.e",
    ("capacitance", "cm"): "cm",
    ("IClamp", "amp"): "IClamp.amp",
    ("ExpSyn", "weight"): "ExpSyn.weight",
    ("ExpSyn", "e"): "ExpSyn.e",
    ("Exp2Syn", "weight"): "Exp2Syn.weight",
    ("Exp2Syn", "e"): "Exp2Syn.e",
    ("HalfGap", "g"): "HalfGap.g",
    ("gapjunction_lr", "g"): "gapjunction_lr.g",
    ("gapjunction_lr", "w"): "gapjunction_lr.w",
    ("gapjunction_noptr", "weight"): "gapjunction_noptr.weight",
    ("neuron_to_neuron_syn_lr", "w"): "neuron_to_neuron_syn_lr.w",
}
# library mechanisms: every HX_P key "<mech>.<var>" is also its handle name
for _k in _lib.HX_P:
    _m, _, _v = _k.partition(".")
    if _m in ("CaDynamics_E2", "Ca_HVA", "Ca_LVAst", "Im", "K_Pst", "K_Tst", "NaTg", "Nap_Et2", "SK_E2", "SKv3_1",
              "hd_la", "km_la", "kca_la", "it2_la", "kdr_la", "sca_la", "Ca", "shl1_lr", "kvs1_lr", "irk_lr",
              "egl36_lr", "shk1_lr", "egl2_lr", "cca1_lr", "egl19_lr", "unc2_lr", "kcnl_lr", "nca_lr", "kqt3_lr",
              "cainternm_lr", "shl1", "kvs1", "irk", "egl36", "shk1", "egl2", "cca1", "egl19", "unc2"):
        _MECH_VAR[(_m, _v)] = _k
_HANDLE_SHIFT = 24


def make_handle(key: str, index: int) -> int:
    return (_lib.HX_P[key] << _HANDLE_SHIFT) | int(index)


def split_handle(h: int):
    return int(h) >> _HANDLE_SHIFT, int(h) & ((1 << _HANDLE_SHIFT) - 1)


class HxError(RuntimeError):
    pass


def pinned_empty(shape, dtype=np.float64) -> np.ndarray:
    """Uninitialised page-locked host array (host<->device copies at full link
    rate and without first-touch page faults); torch provides the allocation."""
    import torch

    shape = (int(shape),) if np.isscalar(shape) else tuple(int(x) for x in shape)
    t = torch.empty(shape, dtype=torch.from_numpy(np.zeros(0, dtype=dtype)).dtype, pin_memory=True)
    return t.numpy()  # the array keeps the tensor (its base) alive


def _out_array(out: Optional[np.ndarray], shape) -> np.ndarray:
    if out is None:
        return np.zeros(shape)
    if out.dtype != np.float64 or out.shape != tuple(shape) or not out.flags["C_CONTIGUOUS"] or not out.flags["WRITEABLE"]:
        raise ValueError(f"out must be a writeable C-contiguous float64 array of shape {tuple(shape)}")
    return out


class Sim:
    """One simulation/learning runtime bound to one CUDA device."""

    def __init__(self, device: int = 0, pack_target: int = 0, tape_budget_bytes: int = 0):
        self._L = _lib.load()
        ctx = C.c_void_p()
        rc = self._L.hx_create(C.byref(ctx), int(device))
        if rc != 0:
            raise HxError(f"hx_create failed (rc={rc}): no usable CUDA device {device}")
        self._ctx = ctx
        self.device = int(device)
        self._check(self._L.hx_set_pack_target(ctx, int(pack_target)), "hx_set_pack_target")
        self._check(self._L.hx_set_tape_budget(ctx, int(tape_budget_bytes)), "hx_set_tape_budget")
        self.group: Optional[CellGroup] = None
        self._bound = None
        self._nstep = None
        self._probes = None
        self._opt_hyper: Dict[int, tuple] = {}
        self._arfn: Dict[int, object] = {}  # ctypes callbacks of the optimizers' all-reduce hooks

    # ------------------------------------------------------------------ basics
    def _check(self, rc: int, what: str):
        if rc != 0:
            msg = self._L.hx_last_error(self._ctx)
            raise HxError(f"{what} failed (rc={rc}): {msg.decode() if msg else ''}")

    def close(self):
        if getattr(self, "_ctx", None):
            self._L.hx_destroy(self._ctx)
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_stream(self, stream_handle: int):
        """Launch on an existing CUDA stream (e.g. ``torch.cuda.current_stream().cuda_stream``)."""
        self._check(self._L.hx_set_stream(self._ctx, C.c_void_p(int(stream_handle))), "hx_set_stream")

    def load_group(self, group: CellGroup, gid_base: int = 0, nsrc_cells: int = 0):
        """Load a cell group.  For one shard of a multi-GPU network, ``gid_base``
        is the global id of its first cell and ``nsrc_cells`` the number of cells
        over all shards (NetCon sources and NetStims then use global ids)."""
        group.validate()
        self.group = group
        self._bound = _lib.BoundGroup(group, gid_base=gid_base, nsrc_cells=nsrc_cells)
        self._check(self._L.hx_load_group(self._ctx, C.byref(self._bound.desc)), "hx_load_group")

    def plan_stats(self) -> dict:
        st = _lib.PlanStats()
        self._check(self._L.hx_get_plan_stats(self._ctx, C.byref(st)), "hx_get_plan_stats")
        return st.as_dict()

    # ------------------------------------------------------------------ handles / parameters
    def get_variable_handle(self, mech: str, var: str, idx: int) -> int:
        """Handle of one parameter instance (mirrors Sim.get_variable_handle)."""
        key = _MECH_VAR.get((mech, var))
        if key is None:
            raise KeyError(f"{mech}.{var} is not a parameter of the adjoint path")
        n = self._count(key)
        if not 0 <= idx < n:
            raise IndexError(f"{mech}.{var}[{idx}] out of range (n={n})")
        return make_handle(key, idx)

    def _count(self, key: str) -> int:
        g = self.group
        mech = key.split(".")[0]
        tab = {"hh": g.hh, "pas": g.pas, "IClamp": g.iclamp, "ExpSyn": g.expsyn, "Exp2Syn": g.exp2syn,
               "HalfGap": g.halfgap, "gapjunction_lr": g.gapjunction, "gapjunction_noptr": g.gapnoptr,
               "neuron_to_neuron_syn_lr": g.graded}.get(mech)
        if key == "cm":
            return g.nnode
        if tab is None:
            lt = g.lib.get(mech)
            return lt.n if lt is not None else 0
        return tab.n

    # ------------------------------------------------------------------ network
    def spikes(self):
        """Spikes of the group's PreSyns in the last forward: (gid int32[n], t float64[n]),
        in detection order (the reference's spk.dat holds the same pairs)."""
        n = C.c_int(0)
        self._check(self._L.hx_get_spikes(self._ctx, 0, _lib._ip(), _lib._dp(), C.byref(n)), "hx_get_spikes")
        k = int(n.value)
        gid = np.zeros(max(k, 1), dtype=np.int32)
        t = np.zeros(max(k, 1))
        self._check(self._L.hx_get_spikes(self._ctx, k, _lib.iptr(gid), _lib.dptr(t), C.byref(n)), "hx_get_spikes")
        return gid[:k], t[:k]

    def set_exchange(self, fn, nranks: int, cap_entries: int = 0):
        """Install the multi-GPU spike exchange: ``fn(send_ptr, recv_ptr, cap_entries, stream_ptr)``
        must all-gather ``cap_entries`` (gid, step) int pairs per rank from
        ``send_ptr`` into ``recv_ptr`` on the given stream (``None`` removes it).
        ``cap_entries`` is the initial window buffer size, the same on every
        rank (0: the library's default; it grows on overflow)."""
        if fn is None:
            self._xfn = None
            self._check(self._L.hx_set_exchange(self._ctx, _lib.EXCHANGE_FN(), None, 1, 0), "hx_set_exchange")
            return

        def cb(user, send, recv, cap, stream):
            try:
                fn(int(send or 0), int(recv or 0), int(cap), int(stream or 0))
                return 0
            except Exception:  # an exception must not cross the C boundary
                import traceback

                traceback.print_exc()
                return -1

        self._xfn = _lib.EXCHANGE_FN(cb)
        self._check(self._L.hx_set_exchange(self._ctx, self._xfn, None, int(nranks), int(cap_entries)),
                    "hx_set_exchange")

    def set_split_barrier_limit(self, sleeps: int = 0):
        """Bound of a split-cell grid-barrier wait, in ~100 ns sleeps (0 = default, ~2 s)."""
        self._check(self._L.hx_set_split_barrier_limit(self._ctx, int(sleeps)), "hx_set_split_barrier_limit")

    def set_grad_kinds(self, keys=None):
        """Accumulate only these gradient kinds in the next backward passes (None: all); the others read as zero."""
        if not keys:
            self._check(self._L.hx_set_grad_kinds(self._ctx, None, 0), "hx_set_grad_kinds")
            return
        k = np.array([_lib.HX_P[key] for key in keys], dtype=np.int32)
        self._check(self._L.hx_set_grad_kinds(self._ctx, _lib.iptr(k), int(k.shape[0])), "hx_set_grad_kinds")

    def set_grid_sync(self, enable: bool = True):
        """Coupled groups: many steps a launch with a grid barrier per step (True, when the packs fit) or one launch per step."""
        self._check(self._L.hx_set_grid_sync(self._ctx, 1 if enable else 0), "hx_set_grid_sync")

    def set_window(self, steps: int):
        self._check(self._L.hx_set_window(self._ctx, int(steps)), "hx_set_window")

    def window(self) -> int:
        w = C.c_int(0)
        self._check(self._L.hx_get_window(self._ctx, C.byref(w)), "hx_get_window")
        return int(w.value)

    def set_param_array(self, key: str, values: np.ndarray):
        v = np.ascontiguousarray(values, dtype=np.float64)
        self._check(self._L.hx_set_param(self._ctx, _lib.HX_P[key], _lib.dptr(v), int(v.shape[0])), "hx_set_param")

    def get_param_array(self, key: str) -> np.ndarray:
        out = np.zeros(self._count(key))
        self._check(self._L.hx_get_param(self._ctx, _lib.HX_P[key], _lib.dptr(out), int(out.shape[0])), "hx_get_param")
        return out

    def set_variables(self, handles: Sequence[int], values: Sequence[float]):
        by_kind: Dict[int, list] = {}
        for h, v in zip(handles, values):
            k, i = split_handle(h)
            by_kind.setdefault(k, []).append((i, float(v)))
        inv = {v: k for k, v in _lib.HX_P.items()}
        for k, items in by_kind.items():
            key = inv[k]
            arr = self.get_param_array(key)
            for i, v in items:
                arr[i] = v
            self.set_param_array(key, arr)

    def get_variables(self, handles: Sequence[int]) -> np.ndarray:
        inv = {v: k for k, v in _lib.HX_P.items()}
        cache: Dict[int, np.ndarray] = {}
        out = np.zeros(len(handles))
        for j, h in enumerate(handles):
            k, i = split_handle(h)
            if k not in cache:
                cache[k] = self.get_param_array(inv[k])
            out[j] = cache[k][i]
        return out

    # ------------------------------------------------------------------ forward
    def _probe_arr(self, probes) -> np.ndarray:
        if probes is None:
            probes = self.group.soma_nodes()
        return np.ascontiguousarray(probes, dtype=np.int32)

    def simulate(self, nstep: int, v_init: Optional[float] = None, probes=None) -> np.ndarray:
        """finitialize + nstep steps; returns v at the probes, shape (nstep+1, nprobe)."""
        p = self._probe_arr(probes)
        tr = np.zeros((nstep + 1, p.shape[0]))
        vi = self.group.v_init if v_init is None else v_init
        self._check(self._L.hx_simulate(self._ctx, int(nstep), float(vi), int(p.shape[0]), _lib.iptr(p), _lib.dptr(tr)),
                    "hx_simulate")
        return tr

    def forward_capture(self, nstep: int, v_init: Optional[float] = None, probes=None,
                        out: Optional[np.ndarray] = None) -> np.ndarray:
        """Forward that records the tape for ``backward``; returns the probe trace.

        ``out``: optional C-contiguous float64 array of shape (nstep+1, nprobe)
        to write the trace into (e.g. from ``pinned_empty``, for full-rate
        copies); otherwise a new array is returned."""
        p = self._probe_arr(probes)
        tr = _out_array(out, (nstep + 1, p.shape[0]))
        vi = self.group.v_init if v_init is None else v_init
        self._check(
            self._L.hx_forward_capture(self._ctx, int(nstep), float(vi), int(p.shape[0]), _lib.iptr(p), _lib.dptr(tr)),
            "hx_forward_capture")
        self._nstep, self._probes = int(nstep), p
        return tr

    # ------------------------------------------------------------------ backward
    def backward(self, dLdv: np.ndarray, keys: Iterable[str] = tuple(_lib.HX_P),
                 out: Optional[Dict[str, np.ndarray]] = None) -> Dict[str, np.ndarray]:
        """Exact adjoint of the last capture; dLdv shape (nstep+1, nprobe).

        ``out``: optional dict of C-contiguous float64 arrays (one per key, of
        the parameter's instance count) to write the gradients into."""
        if self._nstep is None:
            raise HxError("backward needs a preceding forward_capture")
        d = np.ascontiguousarray(dLdv, dtype=np.float64)
        if d.shape != (self._nstep + 1, self._probes.shape[0]):
            raise ValueError(f"dLdv must have shape {(self._nstep + 1, self._probes.shape[0])}")
        out = out or {}
        outs = {k: _out_array(out.get(k), (self._count(k),)) for k in keys}
        arr = (_lib._dp * _lib.HX_P_COUNT)()
        for k, v in outs.items():
            arr[_lib.HX_P[k]] = _lib.dptr(v)
        self._check(self._L.hx_backward(self._ctx, _lib.dptr(d), arr), "hx_backward")
        return outs

    def reduce_grads_f32(self, handles: Sequence[int], dest: np.ndarray, scale: np.ndarray, n_out: int) -> np.ndarray:
        """MappedSignal column reduction of the last backward: out[dest[j]] += scale[j]*grad[handle j]."""
        hk = np.array([split_handle(h)[0] for h in handles], dtype=np.int32)
        hi = np.array([split_handle(h)[1] for h in handles], dtype=np.int32)
        dest = np.ascontiguousarray(dest, dtype=np.int32)
        scale = np.ascontiguousarray(scale, dtype=np.float32)
        out = np.zeros(int(n_out), dtype=np.float32)
        self._check(
            self._L.hx_reduce_grads_f32(self._ctx, int(hk.shape[0]), _lib.iptr(hk), _lib.iptr(hi), _lib.iptr(dest),
                                        _lib.fptr(scale), _lib.fptr(out), int(n_out)), "hx_reduce_grads_f32")
        return out

    def simulate_and_adjoint_into(self, dLtdv: np.ndarray, probes, handles: Sequence[int], dest: np.ndarray,
                                  scale: np.ndarray, n_out: int, v_init: Optional[float] = None,
                                  grad_scale: float = 1.0, grad_l2norm_threshold: float = 0.0,
                                  clip_strategy: int = 0) -> np.ndarray:
        """One call in the shape of the reference's simulate_and_replay_dw_dx_streaming_into:
        forward (probes recorded), exact adjoint of dL/d(probe trace) = dLtdv
        (float32, nstep x nprobe; row t is step t+1), column reduction
        out[dest[j]] += scale[j] * grad[handle j] times grad_scale, optional
        L2-norm clipping of the result.  Returns out (float32[n_out])."""
        p = self._probe_arr(probes)
        d = np.ascontiguousarray(dLtdv, dtype=np.float32)
        if d.ndim != 2 or d.shape[1] != p.shape[0]:
            raise ValueError("dLtdv must have shape (nstep, nprobe)")
        hk = np.array([split_handle(h)[0] for h in handles], dtype=np.int32)
        hi = np.array([split_handle(h)[1] for h in handles], dtype=np.int32)
        dest = np.ascontiguousarray(dest, dtype=np.int32)
        scale = np.ascontiguousarray(scale, dtype=np.float32)
        out = np.zeros(int(n_out), dtype=np.float32)
        vi = self.group.v_init if v_init is None else v_init
        self._check(
            self._L.hx_simulate_and_adjoint_into(self._ctx, _lib.fptr(d), int(d.shape[0]), int(p.shape[0]),
                                                 _lib.iptr(p), int(n_out), _lib.fptr(out), None,
                                                 int(hk.shape[0]), _lib.iptr(hk), _lib.iptr(hi), _lib.iptr(dest),
                                                 _lib.fptr(scale), float(vi), float(grad_scale),
                                                 float(grad_l2norm_threshold), int(clip_strategy)),
            "hx_simulate_and_adjoint_into")
        self._nstep, self._probes = int(d.shape[0]), p
        return out

    # ------------------------------------------------------------------ device-pointer variants
    def forward_capture_dev(self, nstep: int, trace_ptr: int, v_init: Optional[float] = None, probes=None):
        """Forward + tape with the probe trace written to a device buffer ((nstep+1) x nprobe doubles)."""
        p = self._probe_arr(probes)
        vi = self.group.v_init if v_init is None else v_init
        self._check(self._L.hx_forward_capture_dev(self._ctx, int(nstep), float(vi), int(p.shape[0]), _lib.iptr(p),
                                                   C.c_void_p(int(trace_ptr))), "hx_forward_capture_dev")
        self._nstep, self._probes = int(nstep), p

    def backward_dev(self, dLdv_ptr: int, grad_ptrs: Dict[str, int]):
        """Adjoint of the last capture; dL/dv and the per-kind gradients are device buffers."""
        arr = (C.c_void_p * _lib.HX_P_COUNT)()
        for k, ptr in grad_ptrs.items():
            arr[_lib.HX_P[k]] = C.c_void_p(int(ptr))
        self._check(self._L.hx_backward_dev(self._ctx, C.c_void_p(int(dLdv_ptr)), arr), "hx_backward_dev")

    def mse_loss_grad_dev(self, trace_ptr: int, target_ptr: int, nrow: int, ncol: int, dLdv_ptr: int, loss_ptr: int):
        self._check(self._L.hx_mse_loss_grad_dev(self._ctx, C.c_void_p(int(trace_ptr)), C.c_void_p(int(target_ptr)),
                                                 int(nrow), int(ncol), C.c_void_p(int(dLdv_ptr)),
                                                 C.c_void_p(int(loss_ptr))), "hx_mse_loss_grad_dev")

    # ------------------------------------------------------------------ optimizer
    # Mirrors Sim.create_optimizer / configure_optimizer / optimizer_add_external_grads /
    # optimizer_set_external_grads_f32 / optimizer_step_with_inv_record_steps /
    # optimizer_get/set_adam_state / optimizer_reset_state
    # (src/python_api/PyBindings.cpp:43-65, SimWrapper.cpp:284-451).
    def create_optimizer(self, kind: str = "adam", beta1: float = 0.9, beta2: float = 0.999,
                         epsilon: float = 1e-8) -> int:
        if kind.lower() != "adam":
            raise HxError(f"optimizer {kind!r} is not provided (Adam is the training step of this path)")
        oid = self._L.hx_opt_create_adam(self._ctx, float(beta1), float(beta2), float(epsilon))
        if oid < 0:
            self._check(oid, "hx_opt_create_adam")
        self._opt_hyper[oid] = (float(beta1), float(beta2), float(epsilon))
        return oid

    def configure_optimizer(self, opt: int, momentum: float = 0.9, beta1: float = 0.9, beta2: float = 0.999,
                            epsilon: float = 1e-8):
        self._opt_hyper[opt] = (float(beta1), float(beta2), float(epsilon))
        n = self._opt_n(opt)
        if n:
            step, m, v, _ = self.optimizer_get_adam_state(opt)
            self.optimizer_set_adam_state(opt, step, m, v, beta1, beta2, epsilon)

    def _opt_n(self, opt: int) -> int:
        ptr = C.c_void_p()
        n = C.c_int(0)
        if self._L.hx_opt_grad_buffer(self._ctx, int(opt), C.byref(ptr), C.byref(n)) != 0:
            return 0
        return int(n.value)

    def optimizer_add_external_grads(self, opt: int, weight_handles: Sequence[int], impedance: float = 1.0):
        kinds = np.array([split_handle(h)[0] for h in weight_handles], dtype=np.int32)
        idx = np.array([split_handle(h)[1] for h in weight_handles], dtype=np.int32)
        self._check(self._L.hx_opt_add_params(self._ctx, int(opt), int(kinds.shape[0]), _lib.iptr(kinds),
                                              _lib.iptr(idx), float(impedance)), "hx_opt_add_params")
        b1, b2, eps = self._opt_hyper.get(opt, (0.9, 0.999, 1e-8))
        n = int(kinds.shape[0])
        self.optimizer_set_adam_state(opt, 0, np.zeros(n), np.zeros(n), b1, b2, eps)

    def optimizer_set_external_grads_f32(self, opt: int, grads: np.ndarray):
        g = np.ascontiguousarray(grads, dtype=np.float32)
        self._check(self._L.hx_opt_set_grads_f32(self._ctx, int(opt), _lib.fptr(g), int(g.shape[0])),
                    "hx_opt_set_grads_f32")

    def optimizer_grads_from_backward(self, opt: int, scale: float = 1.0):
        """Slot gradients := the last backward's gradients of the bound parameters (device, fp64)."""
        self._check(self._L.hx_opt_grads_from_backward(self._ctx, int(opt), float(scale)), "hx_opt_grads_from_backward")

    def optimizer_grad_buffer(self, opt: int):
        """(device pointer, n) of the slot gradients, e.g. for an all-reduce across ranks."""
        ptr = C.c_void_p()
        n = C.c_int(0)
        self._check(self._L.hx_opt_grad_buffer(self._ctx, int(opt), C.byref(ptr), C.byref(n)), "hx_opt_grad_buffer")
        return int(ptr.value or 0), int(n.value)

    def optimizer_set_allreduce(self, opt: int, fn):
        """Install the data-parallel gradient all-reduce of optimizer ``opt``:
        ``fn(grad_ptr, n, stream_ptr)`` must replace the n fp64 slot gradients
        at ``grad_ptr`` by their sum over ranks on the given stream
        (``shard.allreduce_sum``); each step calls it before Adam.  ``None``
        removes it."""
        if fn is None:
            self._arfn.pop(opt, None)
            self._check(self._L.hx_opt_set_allreduce(self._ctx, int(opt), _lib.ALLREDUCE_FN(), None),
                        "hx_opt_set_allreduce")
            return

        def cb(user, grad, n, stream):
            try:
                fn(int(grad or 0), int(n), int(stream or 0))
                return 0
            except Exception:  # an exception must not cross the C boundary
                import traceback

                traceback.print_exc()
                return -1

        self._arfn[opt] = _lib.ALLREDUCE_FN(cb)
        self._check(self._L.hx_opt_set_allreduce(self._ctx, int(opt), self._arfn[opt], None), "hx_opt_set_allreduce")

    def optimizer_step_with_inv_record_steps(self, opt: int, learning_rate: float, inv_record_steps: float = 1.0):
        self._check(self._L.hx_opt_step(self._ctx, int(opt), float(learning_rate), float(inv_record_steps)),
                    "hx_opt_step")

    def optimizer_get_adam_state(self, opt: int):
        n = self._opt_n(opt)
        m = np.zeros(max(n, 1))
        v = np.zeros(max(n, 1))
        step = C.c_longlong(0)
        hyper = np.zeros(3)
        self._check(self._L.hx_opt_get_adam_state(self._ctx, int(opt), C.byref(step), _lib.dptr(m), _lib.dptr(v), n,
                                                  _lib.dptr(hyper)), "hx_opt_get_adam_state")
        return int(step.value), m[:n], v[:n], tuple(float(x) for x in hyper)

    def optimizer_set_adam_state(self, opt: int, step: int, m, v, beta1: float = 0.9, beta2: float = 0.999,
                                 epsilon: float = 1e-8):
        m = np.ascontiguousarray(m, dtype=np.float64)
        v = np.ascontiguousarray(v, dtype=np.float64)
        hyper = np.array([beta1, beta2, epsilon], dtype=np.float64)
        self._check(self._L.hx_opt_set_adam_state(self._ctx, int(opt), int(step), _lib.dptr(m), _lib.dptr(v),
                                                  int(m.shape[0]), _lib.dptr(hyper)), "hx_opt_set_adam_state")
        self._opt_hyper[opt] = (float(beta1), float(beta2), float(epsilon))

    def optimizer_reset_state(self, opt: int):
        self._check(self._L.hx_opt_reset(self._ctx, int(opt)), "hx_opt_reset")

    def synchronize(self):
        """Wait for the context's work (the optimizer step is asynchronous)."""
        self.get_param_array("cm")

    def last_kernel_ms(self, which: int):
        ms = C.c_double()
        n = C.c_int()
        self._check(self._L.hx_last_kernel_ms(self._ctx, int(which), C.byref(ms), C.byref(n)), "hx_last_kernel_ms")
        return float(ms.value), int(n.value)
