"""Multi-GPU partition of an event network and the spike exchange between ranks.

A network is split by cell: rank r owns a contiguous range of cells, the
synapses on those cells (each synapse lives with its postsynaptic cell) and a
copy of the whole NetStim table (NetStim trains are generated identically on
every rank and routed only to local synapses).  NetCon sources keep their
global ids (cells 0..ncell-1, NetStims ncell..), so a rank needs nothing of
another rank but its spikes: after every forward window the ranks all-gather
their window spike buffers ((gid, step) int pairs padded with -1).  The
backward needs no exchange -- weight gradients are local to the postsynaptic
rank and the spike schedule is fixed.  Gap junctions and graded synapses that
cross ranks are not partitioned (such networks run as replicas).

This follows the reference's division of a network into groups with one
PreSyn table and a spike exchange per step (Simulate::network_spike_send_cpu /
network_spike_receive_cpu, src/simulate.cpp:858-951), with one collective per
minimum-delay window instead of a host queue per step.
"""
from __future__ import annotations

from typing import List, Tuple

import numpy as np

from .model import CellGroup, MechTable, _f64, _i32


def cell_ranges(g: CellGroup, nranks: int) -> List[Tuple[int, int]]:
    """Contiguous cell ranges balanced by compartment count."""
    cell = g.cell_of_node()
    sizes = np.bincount(cell, minlength=g.ncell).astype(np.float64)
    cum = np.concatenate([[0.0], np.cumsum(sizes)])
    total = cum[-1]
    cuts = [0]
    for r in range(1, nranks):
        cuts.append(int(np.searchsorted(cum, total * r / nranks)))
    cuts.append(g.ncell)
    for r in range(1, len(cuts)):
        cuts[r] = max(cuts[r], cuts[r - 1])
    return [(cuts[r], cuts[r + 1]) for r in range(nranks)]


def shard(g: CellGroup, nranks: int, rank: int) -> Tuple[CellGroup, int, int]:
    """The part of ``g`` that rank ``rank`` of ``nranks`` owns.

    Returns (group, gid_base, nsrc_cells): the shard's cells in the original
    order (roots first), its synapses with global NetCon sources, the whole
    NetStim table; ``gid_base`` is the global id of its first cell and
    ``nsrc_cells`` the number of cells over all shards.  The group's
    ``meta["global_index"]`` maps its synapse and library-mechanism instances
    to the network's.
    """
    if g.coupled:
        raise ValueError("gap junctions and graded synapses are not partitioned across ranks")
    c0, c1 = cell_ranges(g, nranks)[rank]
    cell = g.cell_of_node()
    keep = np.nonzero((cell >= c0) & (cell < c1))[0]
    roots = keep[keep < g.ncell]
    rest = keep[keep >= g.ncell]
    order = np.concatenate([roots, rest])
    new = np.full(g.nnode, -1, dtype=np.int64)
    new[order] = np.arange(order.shape[0])
    par = g.parent[order].astype(np.int64)
    parent = np.where(par >= 0, new[np.maximum(par, 0)], -1)

    global_index = {}

    def sub(tab: MechTable, name: str = "") -> MechTable:
        m = np.isin(tab.nodes, keep)
        nodes = new[tab.nodes[m]]
        o = np.argsort(nodes, kind="stable")
        if name:
            global_index[name] = np.nonzero(m)[0][o]
        return MechTable(_i32(nodes[o]), {k: _f64(v[m][o]) for k, v in tab.fields.items()},
                         {k: _i32(v[m][o]) for k, v in tab.ifields.items()})

    out = CellGroup(
        ncell=int(roots.shape[0]),
        parent=_i32(parent),
        a=_f64(g.a[order]),
        b=_f64(g.b[order]),
        area=_f64(g.area[order]),
        cm=_f64(g.cm[order]),
        hh=sub(g.hh),
        pas=sub(g.pas),
        iclamp=sub(g.iclamp),
        celsius=g.celsius,
        dt=g.dt,
        v_init=g.v_init,
        name=f"{g.name}.rank{rank}of{nranks}",
        expsyn=sub(g.expsyn, "ExpSyn"),
        exp2syn=sub(g.exp2syn, "Exp2Syn"),
        netstim=g.netstim.copy(),
        ps_thresh=_f64(g.ps_thresh[c0:c1]),
        netstim_rng=g.netstim_rng,
        lib={nm: sub(tab, nm) for nm, tab in g.lib.items()},
    )
    # instance i of the shard's ExpSyn / Exp2Syn table is global instance
    # meta["global_index"][mech][i]
    out.meta["global_index"] = global_index
    out.meta["nsrc_cells"] = g.ncell
    out.meta["gid_base"] = c0
    # NetCon sources stay global: validate against the global source count
    nsrc = g.ncell + g.netstim.n
    for tab in (out.expsyn, out.exp2syn):
        s = tab.ifields["src"]
        if s.size and (s.min() < 0 or s.max() >= nsrc):
            raise ValueError("NetCon source out of range")
    return out, c0, g.ncell


def window_of(g: CellGroup) -> int:
    """Steps per forward window of an event network: no longer than the
    smallest NetCon delay (the rule the library applies to one group);
    without synapses the window is free and the library keeps it at 256."""
    d = np.concatenate([g.expsyn.fields["delay"], g.exp2syn.fields["delay"]])
    if d.size == 0:
        return 256
    lag = np.floor((d.min() - 0.5 * g.dt) / g.dt) - 1.0
    return int(max(1.0, lag))


def exchange_capacity(g: CellGroup, nranks: int, window: int) -> int:
    """The bound on one window's spikes of the largest shard: its cells times
    ceil(window/2) (a PreSyn fires at most every other step) plus one.  A
    window buffer this large never overflows; ``Sim.set_exchange`` may start
    far smaller (0: the library's default), growing on overflow."""
    most = max(c1 - c0 for c0, c1 in cell_ranges(g, nranks))
    return most * ((window + 1) // 2) + 1


class _DevView:
    """A device buffer (pointer, count, numpy type string) seen by torch without a copy."""

    def __init__(self, ptr: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 3}


def _wrap(ptr: int, n: int, ctype, device: str):
    """torch view of n elements at ``ptr``: device memory ("cuda") or host memory
    ("cpu", for hooks tested with the gloo backend)."""
    import ctypes as C

    import torch

    if device == "cpu":
        arr = np.ctypeslib.as_array(C.cast(ptr, C.POINTER(ctype)), shape=(n,))
        return torch.from_numpy(arr)
    typestr = {C.c_int: "<i4", C.c_double: "<f8"}[ctype]
    return torch.as_tensor(_DevView(ptr, n, typestr), device="cuda")


def _on_stream(stream_ptr: int, device: str):
    """Context that makes the library's launch stream torch's current stream, so
    the collective is ordered after the kernels that wrote its input and before
    the ones that read its output, whatever stream the caller had current."""
    import contextlib

    import torch

    if device != "cuda" or not stream_ptr:
        return contextlib.nullcontext()
    return torch.cuda.stream(torch.cuda.ExternalStream(stream_ptr))


def allgather_exchange(group=None, device: str = "cuda"):
    """Exchange hook for ``Sim.set_exchange`` over ``torch.distributed``.

    The library hands over its window send buffer and a receive buffer of
    nranks times its size (``cap`` (gid, step) int32 pairs per rank; ``cap`` is
    2 for the status after the last window) and its launch stream; the hook
    wraps the buffers without copying and all-gathers on that stream.
    ``device="cpu"`` takes host buffers (gloo tests of the protocol).
    """
    import ctypes as C

    import torch.distributed as dist

    def fn(send_ptr: int, recv_ptr: int, cap: int, stream_ptr: int) -> None:
        ws = dist.get_world_size(group)
        send = _wrap(send_ptr, 2 * cap, C.c_int, device)
        recv = _wrap(recv_ptr, 2 * cap * ws, C.c_int, device)
        with _on_stream(stream_ptr, device):
            dist.all_gather_into_tensor(recv, send, group=group)

    return fn


def allreduce_sum(group=None, device: str = "cuda"):
    """Gradient hook for ``Sim.optimizer_set_allreduce``: the optimizer's n fp64
    slot gradients are summed over the ranks of ``group`` in place, on the
    library's launch stream, before every Adam step (data-parallel replicas,
    e.g. one trial or teacher per GPU)."""
    import ctypes as C

    import torch.distributed as dist

    def fn(grad_ptr: int, n: int, stream_ptr: int) -> None:
        g = _wrap(grad_ptr, n, C.c_double, device)
        with _on_stream(stream_ptr, device):
            dist.all_reduce(g, op=dist.ReduceOp.SUM, group=group)

    return fn


def merge_status(status: np.ndarray) -> Tuple[int, int, int, int]:
    """(flags, bucket need, window need, first_rank) of the gathered per-rank
    status (4 ints per rank), by the library's own rule
    (``hx_exchange_merge_status``; host only)."""
    import ctypes as C

    from . import _lib

    L = _lib.load()
    st = np.ascontiguousarray(status, dtype=np.int32).reshape(-1)
    f, nd, wn, r = C.c_int(0), C.c_int(0), C.c_int(0), C.c_int(0)
    if L.hx_exchange_merge_status(_lib.iptr(st), st.shape[0] // 4, C.byref(f), C.byref(nd), C.byref(wn),
                                  C.byref(r)) != 0:
        raise ValueError("bad status array")
    return int(f.value), int(nd.value), int(wn.value), int(r.value)


def pad_spikes(gid: np.ndarray, step: np.ndarray, cap: int) -> np.ndarray:
    """The window buffer layout: cap (gid, step) int32 pairs, unused ones (-1, -1)."""
    out = np.full((cap, 2), -1, dtype=np.int32)
    n = min(cap, gid.shape[0])
    out[:n, 0] = gid[:n]
    out[:n, 1] = step[:n]
    return out
