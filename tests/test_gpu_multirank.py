"""Two GPUs: a sharded event network whose ranks exchange window spikes over
NCCL (through the library's exchange hook) reproduces the oracle run of the
whole network -- traces, spikes and weight gradients.  Skipped with fewer than
two GPUs."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

T = 1600


def _net():
    from heliox_b200 import synth

    return synth.spiking_network(ncell=8, seed=31, nstim=4, weight=(0.02, 0.08), stim_noise=1.0, stim_interval=5.0)


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

    from heliox_b200 import shard
    from heliox_b200.runtime import Sim

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        g = _net()
        part, base, nsrc = shard.shard(g, world, rank)
        stream = torch.cuda.Stream()
        torch.cuda.set_stream(stream)
        s = Sim(rank)
        s.set_stream(stream.cuda_stream)
        s.load_group(part, gid_base=base, nsrc_cells=nsrc)
        W = shard.window_of(g)
        s.set_window(W)
        s.set_exchange(shard.allgather_exchange(), world, shard.exchange_capacity(g, world, W))
        c = np.random.default_rng(1).standard_normal((T + 1, g.ncell))[:, base:base + part.ncell]
        tr = s.forward_capture(T)
        gr = s.backward(np.ascontiguousarray(c), keys=("Exp2Syn.weight", "ExpSyn.weight", "hh.gnabar"))
        gid, t = s.spikes()
        torch.cuda.synchronize()
        q.put((rank, base, tr, {k: v for k, v in gr.items()}, part.meta["global_index"], gid.tolist(), t.tolist(),
               part.hh.nodes.tolist()))
        s.set_exchange(None, 1)
        s.close()
    finally:
        dist.destroy_process_group()


def test_two_rank_network_matches_oracle():
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from oracle import oracle as O

    g = _net()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=180) for _ in procs], key=lambda x: x[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    c = np.random.default_rng(1).standard_normal((T + 1, g.ncell))
    ref, gr = O.adjoint(g, T, c)
    tr = np.concatenate([r[2] for r in res], axis=1)
    assert np.max(np.abs(tr - ref)) / np.max(np.abs(ref)) <= 1e-9
    spikes = sorted((gid, t) for r in res for gid, t in zip(r[5], r[6]))
    want = sorted((gid, t) for t, gid in gr["spikes"])
    assert len(spikes) == len(want) and len(want) > 0
    assert all(a[0] == b[0] and abs(a[1] - b[1]) <= g.dt for a, b in zip(spikes, want))
    for key, mech in (("Exp2Syn.weight", "Exp2Syn"), ("ExpSyn.weight", "ExpSyn")):
        full = np.zeros_like(gr[key])
        for r in res:
            full[r[4][mech]] = r[3][key]
        scale = np.max(np.abs(gr[key]))
        assert scale > 0
        assert np.max(np.abs(full - gr[key])) / scale <= 1e-7, key
