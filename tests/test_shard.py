"""CPU: partition of an event network across ranks and the window spike
exchange format (gloo, world size 2)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from heliox_b200 import shard, synth


def _net():
    return synth.spiking_network(ncell=7, seed=21, nstim=3, weight=(0.02, 0.06))


@pytest.mark.parametrize("nranks", [1, 2, 3])
def test_shards_cover_the_network(nranks):
    g = _net()
    parts = [shard.shard(g, nranks, r) for r in range(nranks)]
    assert sum(p.ncell for p, _, _ in parts) == g.ncell
    assert sum(p.nnode for p, _, _ in parts) == g.nnode
    assert sum(p.exp2syn.n for p, _, _ in parts) == g.exp2syn.n
    assert sum(p.expsyn.n for p, _, _ in parts) == g.expsyn.n
    bases = [b for _, b, _ in parts]
    assert bases == sorted(bases) and bases[0] == 0
    for p, base, nsrc in parts:
        p.validate()
        assert nsrc == g.ncell
        assert p.netstim.n == g.netstim.n  # every rank generates every NetStim train
        # synapse weights and sources are carried unchanged (global source ids)
        assert set(p.exp2syn.ifields["src"].tolist()) <= set(g.exp2syn.ifields["src"].tolist())
        assert np.all(p.parent[: p.ncell] == -1)
    # the multiset of (src, delay, weight) over shards equals the network's
    allsyn = sorted(zip(np.concatenate([p.exp2syn.ifields["src"] for p, _, _ in parts]).tolist(),
                        np.concatenate([p.exp2syn.fields["weight"] for p, _, _ in parts]).tolist()))
    assert allsyn == sorted(zip(g.exp2syn.ifields["src"].tolist(), g.exp2syn.fields["weight"].tolist()))


@pytest.mark.parametrize("nranks", [2, 3])
def test_shards_carry_library_mechanisms(nranks):
    """Library cells in an event network: every library table is partitioned
    with its cells (instance counts add up, each instance's fields travel with
    it, global_index maps back), and every shard is a valid group."""
    g = synth.lib_network("event", ncell=5, seed=12, nstim=2)
    parts = [shard.shard(g, nranks, r) for r in range(nranks)]
    for nm, tab in g.lib.items():
        assert sum(p.lib[nm].n for p, _, _ in parts) == tab.n, nm
        for p, _, _ in parts:
            gi = p.meta["global_index"][nm]
            for k, v in p.lib[nm].fields.items():
                assert np.array_equal(v, tab.fields[k][gi]), (nm, k)
    for p, _, _ in parts:
        p.validate()


def test_shard_rejects_coupled_networks():
    with pytest.raises(ValueError):
        shard.shard(synth.coupled_network(ncell=4), 2, 0)


def test_window_matches_min_delay():
    g = _net()
    d = min(g.expsyn.fields["delay"].min(), g.exp2syn.fields["delay"].min())
    w = shard.window_of(g)
    assert 1 <= w and w * g.dt <= d - 0.5 * g.dt


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _spawn(target, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=timeout) for _ in procs], key=lambda x: x[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return res


def _init(rank, world, port):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    return dist


def _exchange_worker(rank, world, port, q):
    import ctypes as C

    dist = _init(rank, world, port)
    try:
        fn = shard.allgather_exchange(device="cpu")
        cap = 5
        rng = np.random.default_rng(rank)
        n = 2 + rank
        gid = rng.integers(0, 100, n).astype(np.int32)
        step = rng.integers(0, 50, n).astype(np.int32)
        send = shard.pad_spikes(gid, step, cap)
        recv = np.zeros((world * cap, 2), np.int32)
        # the library's call: window buffer pointers, entries per rank, stream
        fn(send.ctypes.data_as(C.c_void_p).value, recv.ctypes.data_as(C.c_void_p).value, cap, 0)
        q.put((rank, recv.tolist(), gid.tolist(), step.tolist()))
    finally:
        dist.destroy_process_group()


def test_window_exchange_roundtrip_gloo():
    """The exchange hook all-gathers every rank's window buffer (host buffers over gloo)."""
    res = _spawn(_exchange_worker)
    sent = {r: list(zip(g, s)) for r, _, g, s in res}
    for r, recv, _, _ in res:
        recv = np.asarray(recv)
        valid = [tuple(x) for x in recv if x[0] >= 0]
        assert valid == sent[0] + sent[1]
        assert recv.shape == (2 * 5, 2)


# status bits of include/heliox_b200.h
XS_LATE, XS_BUCKET, XS_WINDOW, XS_ABORT = 1, 2, 4, 8


def _status_worker(rank, world, port, q):
    """After the last window every rank all-gathers its status -- (bits,
    bucket need), (window need, 0) -- and applies the library's merge rule.
    Scenario 1 injects a host failure on rank 1 (it reports HX_XS_ABORT, as
    the library does for a rank that stopped launching work) while rank 0's
    buckets overflowed; scenario 2 has only overflows of different sizes."""
    import ctypes as C

    dist = _init(rank, world, port)
    try:
        fn = shard.allgather_exchange(device="cpu")
        out = []
        for mine in ({0: (XS_BUCKET, 40, 300, 0), 1: (XS_ABORT, 0, 0, 0)},
                     {0: (XS_BUCKET, 40, 300, 0), 1: (XS_BUCKET | XS_WINDOW, 90, 2500, 0)}):
            send = np.array(mine[rank], np.int32)
            recv = np.zeros(4 * world, np.int32)
            fn(send.ctypes.data_as(C.c_void_p).value, recv.ctypes.data_as(C.c_void_p).value, 2, 0)
            out.append(shard.merge_status(recv))
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_status_exchange_agrees_on_failure_gloo():
    res = _spawn(_status_worker)
    (_, a), (_, b) = res
    assert a == b  # every rank reaches the same decision
    assert a[0] == (XS_BUCKET | XS_ABORT, 40, 300, 1)  # fail together, naming rank 1
    assert a[1] == (XS_BUCKET | XS_WINDOW, 90, 2500, 0)  # rerun together with the largest needs


def test_merge_status_rule():
    assert shard.merge_status(np.array([[0, 3, 5, 0], [0, 7, 2, 0]])) == (0, 7, 5, -1)
    assert shard.merge_status(np.array([[XS_BUCKET, 3, 0, 0], [XS_WINDOW, 0, 9, 0], [XS_LATE, 1, 0, 0]])) == (7, 3, 9, 2)


def _allreduce_worker(rank, world, port, q):
    """Data-parallel Adam: each rank's gradient (its own trial) summed by the
    optimizer hook over gloo, then the reference's Adam update on every rank."""
    import ctypes as C

    from oracle import oracle as O

    dist = _init(rank, world, port)
    try:
        fn = shard.allreduce_sum(device="cpu")
        w0 = np.array([0.12, 0.036, 3e-4])
        rng = np.random.default_rng(100 + rank)
        grads = rng.standard_normal((3, 3))
        summed = []
        for g in grads:
            buf = np.array(g, dtype=np.float64)  # a copy: the hook sums in place
            fn(buf.ctypes.data_as(C.c_void_p).value, buf.shape[0], 0)
            summed.append(buf.copy())
        ws, _, _ = O.adam_port(w0, np.array(summed), 1e-3, 1.0)
        q.put((rank, grads.tolist(), np.array(summed).tolist(), ws.tolist()))
    finally:
        dist.destroy_process_group()


def test_gradient_allreduce_before_adam_gloo():
    res = _spawn(_allreduce_worker)
    g0, g1 = np.array(res[0][1]), np.array(res[1][1])
    for r in res:
        assert np.array_equal(np.array(r[2]), g0 + g1)  # each rank holds the sum
    assert np.array_equal(np.array(res[0][3]), np.array(res[1][3]))  # identical updates


def test_config4_network_independent_of_rank_count():
    """The strong-scaling network: its union over any number of ranks is the same network."""

    def key(g):
        cell = g.cell_of_node()
        base = g.meta["gid_base"]
        e = g.exp2syn
        return sorted(zip((base + cell[e.nodes]).tolist(), e.ifields["src"].tolist(), e.fields["weight"].tolist(),
                          e.fields["delay"].tolist(), g.meta["teacher_weight"].tolist()))

    one = synth.network_config4_shard(9, 0, 1)
    for n in (2, 3):
        parts = [synth.network_config4_shard(9, r, n) for r in range(n)]
        assert sum(p.nnode for p in parts) == one.nnode
        assert sorted(sum((key(p) for p in parts), [])) == key(one)
        assert [p.meta["gid_base"] for p in parts] == [synth.config4_cell_range(9, r, n)[0] for r in range(n)]
