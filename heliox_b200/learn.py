"""``heliox_learn``-compatible surface for the exact adjoint.

The reference's learning package defines a gradient-method plugin slot
(``GradientMethod``: ``spec``, ``capture(runtime, state)``,
``backward(runtime, captured, dL_dprobe)``, python_lib/heliox_learn/method.py:
15-32), column mappings of runtime handles (``MappedSignal``, signals.py:9-37)
and the result type ``ReplayGrads(dw_out_n, dx_lr_it)`` (signals.py:94-99).
``AdjointMethod`` plugs the exact discrete adjoint into that slot: ``capture``
runs the forward with tape, ``backward`` runs the reverse sweep and reduces the
per-instance gradients into the N columns of a ``MappedSignal`` on the device
(the reference's batch_scatter_add, src/runtime_api/core/kernels/
batch_scatter_add.cu:4-27).  ``train_adam`` is the loop the reference drives
through ``Sim.optimizer_*`` (SimWrapper.cpp:284-451), run on the device.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional, Protocol, Sequence, Tuple, runtime_checkable

import numpy as np

from .model import CellGroup
from .runtime import Sim


try:
    # The reference's own plugin types, when its package is installed beside
    # this one: AdjointMethod then satisfies heliox_learn.GradientMethod,
    # accepts heliox_learn.MappedSignal and returns heliox_learn.ReplayGrads.
    from heliox_learn.method import GradientMethod, MethodSpec  # type: ignore
    from heliox_learn.signals import MappedSignal, ReplayGrads  # type: ignore

    REFERENCE_TYPES = True
except ImportError:
    # The same types restated (field names, validation and messages of
    # python_lib/heliox_learn/method.py:7-32 and signals.py:9-37, 94-99) for
    # hosts without the reference package.
    REFERENCE_TYPES = False

    @dataclass(frozen=True)
    class MethodSpec:  # type: ignore[no-redef]
        name: str
        precise: bool = True

    @runtime_checkable
    class GradientMethod(Protocol):  # type: ignore[no-redef]
        @property
        def spec(self) -> MethodSpec: ...

        def capture(self, runtime: Any, *, state: Any) -> Any: ...

        def backward(self, runtime: Any, *, captured: Any, dL_dprobe: Any) -> Any: ...

    @dataclass(frozen=True)
    class MappedSignal:  # type: ignore[no-redef]
        """Handles gathered and scatter-added into N columns: out[dest[j]] += scale[j] * x[handles[j]]."""

        name: str
        handles: Sequence[int]
        dest: np.ndarray  # int32 (len(handles),)
        scale: np.ndarray  # float32 (len(handles),)

        def __post_init__(self) -> None:
            if self.dest.ndim != 1 or self.scale.ndim != 1:
                raise ValueError(f"MappedSignal({self.name}): dest/scale must be 1D arrays")
            if int(self.dest.shape[0]) != len(self.handles) or int(self.scale.shape[0]) != len(self.handles):
                raise ValueError(f"MappedSignal({self.name}): size mismatch")
            if self.dest.dtype != np.int32:
                raise TypeError(f"MappedSignal({self.name}): dest must be int32 (got {self.dest.dtype})")
            if self.scale.dtype != np.float32:
                raise TypeError(f"MappedSignal({self.name}): scale must be float32 (got {self.scale.dtype})")

    @dataclass(frozen=True)
    class ReplayGrads:  # type: ignore[no-redef]
        dw_out_n: np.ndarray  # float32 (N,)
        dx_lr_it: Optional[np.ndarray] = None


def n_columns(p: MappedSignal) -> int:
    """Columns N of a mapping: 1 + the largest destination column."""
    return int(p.dest.max()) + 1 if p.dest.size else 0


@dataclass(frozen=True)
class AdjointCaptureSpec:
    """Forward capture: voltages at probe nodes over ``total_steps`` steps."""

    probe_nodes: Sequence[int]
    total_steps: int
    v_init: Optional[float] = None


@dataclass
class CapturedTrace:
    output_vs_tn: np.ndarray  # float64 (total_steps+1, n_output)

    @property
    def total_steps(self) -> int:
        return int(self.output_vs_tn.shape[0]) - 1

    @property
    def n_output(self) -> int:
        return int(self.output_vs_tn.shape[1])


class AdjointRuntime:
    """A loaded cell group on one GPU (the counterpart of heliox_learn.Runtime)."""

    def __init__(self, group: CellGroup, device: int = 0, **sim_kwargs):
        self.group = group
        self.sim = Sim(device, **sim_kwargs)
        self.sim.load_group(group)

    @property
    def loaded(self) -> bool:
        return True

    @property
    def dt_ms(self) -> float:
        return float(self.group.dt)

    @property
    def v_init(self) -> float:
        return float(self.group.v_init)

    def handle(self, mech: str, var: str, idx: int) -> int:
        return self.sim.get_variable_handle(mech, var, idx)

    def close(self) -> None:
        self.sim.close()


@dataclass
class AdjointState:
    spec: AdjointCaptureSpec
    params: MappedSignal


class AdjointMethod:
    """Exact discrete adjoint in the GradientMethod slot."""

    @property
    def spec(self) -> MethodSpec:
        return MethodSpec("adjoint", precise=True)

    def capture(self, runtime: AdjointRuntime, *, state: AdjointState) -> CapturedTrace:
        sp = state.spec
        tr = runtime.sim.forward_capture(int(sp.total_steps), v_init=sp.v_init,
                                         probes=np.asarray(sp.probe_nodes, dtype=np.int32))
        return CapturedTrace(tr)

    def backward(self, runtime: AdjointRuntime, *, captured: CapturedTrace, dL_dprobe: np.ndarray,
                 state: Optional[AdjointState] = None) -> ReplayGrads:
        if state is None:
            raise ValueError("AdjointMethod.backward needs the state with the parameter mapping")
        runtime.sim.backward(np.asarray(dL_dprobe, dtype=np.float64), keys=())
        p = state.params
        dw = runtime.sim.reduce_grads_f32(list(p.handles), p.dest, p.scale, n_columns(p))
        return ReplayGrads(dw_out_n=dw, dx_lr_it=None)


def mse_objective(trace: np.ndarray, target: np.ndarray) -> Tuple[float, np.ndarray]:
    """Soma-voltage MSE over steps 1..T and its gradient dL/dtrace (row 0 is the initial state)."""
    err = trace[1:] - target[1:]
    n = err.size
    loss = float(np.sum(err * err) / n)
    g = np.zeros_like(trace)
    g[1:] = (2.0 / n) * err
    return loss, g


def train_adam(runtime: AdjointRuntime, handles: Sequence[int], target: np.ndarray, epochs: int,
               lr: float = 1e-3, probes: Optional[Sequence[int]] = None, total_steps: Optional[int] = None,
               allreduce: Optional[Callable[[int, int, int], None]] = None,
               on_epoch: Optional[Callable[[int, float], None]] = None) -> List[float]:
    """Fit the parameters behind ``handles`` to ``target`` with the device Adam.

    Each epoch: forward capture, MSE against ``target`` on the host, reverse
    sweep, gradients of the bound parameters copied into the optimizer's slots
    on the device, one Adam step.  With data-parallel replicas (one trial or
    teacher per rank) ``allreduce`` is the optimizer's all-reduce hook
    (``shard.allreduce_sum()``): each step first sums the slot gradients over
    the ranks on the library's stream.  Returns the loss history.
    """
    sim = runtime.sim
    probes = runtime.group.soma_nodes() if probes is None else np.asarray(probes, dtype=np.int32)
    T = int(total_steps if total_steps is not None else target.shape[0] - 1)
    opt = sim.create_optimizer("adam")
    sim.optimizer_add_external_grads(opt, list(handles), impedance=1.0)
    if allreduce is not None:
        sim.optimizer_set_allreduce(opt, allreduce)
    hist = []
    for ep in range(int(epochs)):
        tr = sim.forward_capture(T, probes=probes)
        loss, g = mse_objective(tr, target)
        sim.backward(g, keys=())
        sim.optimizer_grads_from_backward(opt)
        sim.optimizer_step_with_inv_record_steps(opt, lr, 1.0)
        hist.append(loss)
        if on_epoch:
            on_epoch(ep, loss)
    sim.synchronize()
    return hist
