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


def _worker(rank, world, port, q):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        cap = 5
        rng = np.random.default_rng(rank)
        n = 2 + rank
        gid = rng.integers(0, 100, n).astype(np.int32)
        step = rng.integers(0, 50, n).astype(np.int32)
        buf = torch.from_numpy(shard.pad_spikes(gid, step, cap).reshape(-1))
        out = [torch.zeros_like(buf) for _ in range(world)]
        dist.all_gather(out, buf)
        recv = torch.cat(out).numpy().reshape(-1, 2)
        q.put((rank, recv.tolist(), gid.tolist(), step.tolist()))
    finally:
        dist.destroy_process_group()


def test_window_exchange_roundtrip_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    sent = {r: list(zip(g, s)) for r, _, g, s in res}
    for r, recv, _, _ in res:
        recv = np.asarray(recv)
        valid = [tuple(x) for x in recv if x[0] >= 0]
        assert valid == sent[0] + sent[1]
        assert recv.shape == (2 * 5, 2)
