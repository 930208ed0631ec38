"""Two GPUs, one process each, NCCL through the library's hooks (skipped with
fewer than two GPUs; NVLS is off, the multi-rank tests use plain NCCL).

* a sharded event network whose ranks exchange window spikes reproduces the
  oracle run of the whole network -- traces, spikes and weight gradients --
  both for a partition of a given network (shard.shard) and for the config-4
  network built per rank (synth.network_config4_shard, the bench's strong
  scaling layout, window agreed over the ranks, a window buffer started far
  too small so that every rank grows it and reruns together);
* a host-side failure on one rank (injected into its status pair) makes every
  rank's forward return the error, with no rank left waiting, and the next
  forward runs normally;
* data-parallel replicas (a different teacher per rank): the optimizer's
  all-reduce hook sums the slot gradients over the ranks before Adam, so both
  ranks apply the same update, the one the reference's Adam gives for the
  summed oracle gradients.
"""
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


def _init(rank, world, port):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    return dist


def _sim_on_stream(rank):
    import torch

    from heliox_b200.runtime import Sim

    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    s = Sim(rank)
    s.set_stream(stream.cuda_stream)
    return s


def _agreed_window(dist, w):
    import torch

    t = torch.tensor([w], dtype=torch.int64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return int(t.item())


def _worker(rank, world, port, q, mode):
    import torch

    from heliox_b200 import shard, synth
    from heliox_b200.runtime import HxError

    dist = _init(rank, world, port)
    try:
        s = _sim_on_stream(rank)
        if mode == "config4":
            part = synth.network_config4_shard(12, rank, world)
            base, nsrc = part.meta["gid_base"], part.meta["nsrc_cells"]
            W = _agreed_window(dist, shard.window_of(part))
            cap = 2  # far below the window's spikes: the ranks grow it together and rerun
            ncell_all = 12
        else:
            g = _net()
            part, base, nsrc = shard.shard(g, world, rank)
            W = shard.window_of(g)
            cap = shard.exchange_capacity(g, world, W)
            ncell_all = g.ncell
        s.load_group(part, gid_base=base, nsrc_cells=nsrc)
        s.set_window(W)
        hook = shard.allgather_exchange()
        if mode == "abort":
            import ctypes as C

            def failing(send, recv, cap_, stream):
                if cap_ == 2 and rank == 1:  # rank 1 reports a failed host step in its status
                    t = shard._wrap(send, 2, C.c_int, "cuda")
                    with shard._on_stream(stream, "cuda"):
                        t[0:1].bitwise_or_(8)
                hook(send, recv, cap_, stream)

            s.set_exchange(failing, world, cap)
            try:
                s.forward_capture(T)
                err = ""
            except HxError as e:
                err = str(e)
            s.set_exchange(hook, world, cap)  # the next forward runs normally on both ranks
            tr = s.forward_capture(T)
            torch.cuda.synchronize()
            q.put((rank, err, bool(np.all(np.isfinite(tr)))))
            return
        s.set_exchange(hook, world, cap)
        c = np.random.default_rng(1).standard_normal((T + 1, ncell_all))[:, base:base + part.ncell]
        tr = s.forward_capture(T)
        gr = s.backward(np.ascontiguousarray(c), keys=("Exp2Syn.weight", "ExpSyn.weight", "hh.gnabar"))
        gid, t = s.spikes()
        torch.cuda.synchronize()
        q.put((rank, base, tr, {k: v for k, v in gr.items()}, part.meta.get("global_index"), gid.tolist(), t.tolist(),
               (part.exp2syn.ifields["src"].tolist(), part.exp2syn.fields["weight"].tolist())))
        s.set_exchange(None, 1)
        s.close()
    finally:
        dist.destroy_process_group()


def _run(mode, world=2, timeout=240):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker if mode != "adam" else _adam_worker, args=(r, world, port, q, mode))
             for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=timeout) for _ in procs], key=lambda x: x[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return res


def _check_network(g, res, remap):
    from oracle import oracle as O

    c = np.random.default_rng(1).standard_normal((T + 1, g.ncell))
    ref, gr = O.adjoint(g, T, c)
    tr = np.concatenate([r[2] for r in res], axis=1)
    assert np.max(np.abs(tr - ref)) / np.max(np.abs(ref)) <= 1e-9
    spikes = sorted((gid, t) for r in res for gid, t in zip(r[5], r[6]))
    want = sorted((gid, t) for t, gid in gr["spikes"])
    assert len(spikes) == len(want) and len(want) > 0
    assert all(a[0] == b[0] and abs(a[1] - b[1]) <= g.dt for a, b in zip(spikes, want))
    for key, mech in (("Exp2Syn.weight", "Exp2Syn"), ("ExpSyn.weight", "ExpSyn")):
        if not gr[key].size:
            continue
        full = np.full_like(gr[key], np.nan)
        for r in res:
            full[remap(r, mech)] = r[3][key]
        scale = np.max(np.abs(gr[key]))
        assert scale > 0
        assert np.max(np.abs(full - gr[key])) / scale <= 1e-7, key


def test_two_rank_network_matches_oracle():
    res = _run("shard")
    _check_network(_net(), res, lambda r, mech: r[4][mech])


def test_two_rank_config4_network_matches_oracle():
    from heliox_b200 import synth

    whole = synth.network_config4_shard(12, 0, 1)
    # synapses are identified by (source, weight): the weights are distinct draws
    pos = {(s, w): i for i, (s, w) in enumerate(zip(whole.exp2syn.ifields["src"].tolist(),
                                                    whole.exp2syn.fields["weight"].tolist()))}
    res = _run("config4")
    _check_network(whole, res, lambda r, mech: [pos[k] for k in zip(*r[7])])


def test_rank_failure_reported_on_every_rank():
    res = _run("abort", timeout=180)
    (_, e0, ok0), (_, e1, ok1) = res
    assert e0 and e1  # both ranks returned the error; neither waited for the other
    assert "rank 1" in e0
    assert ok0 and ok1  # and the next forward ran on both


def _adam_worker(rank, world, port, q, mode):
    import torch

    from heliox_b200 import shard, synth
    from heliox_b200.learn import mse_objective

    dist = _init(rank, world, port)
    try:
        g = synth.random_tree_batch(3, seed0=70, nmin=60, nmax=120)
        teacher = synth.perturb_conductances(g, 0.2, seed=500 + rank)  # each rank fits its own trial
        Tn = 1200
        s = _sim_on_stream(rank)
        s.load_group(teacher)
        target = s.simulate(Tn)
        s.close()
        s = _sim_on_stream(rank)
        s.load_group(g)
        h = [s.get_variable_handle("hh", "gnabar", i) for i in range(g.hh.n)]
        opt = s.create_optimizer("adam")
        s.optimizer_add_external_grads(opt, h, impedance=1.0)
        s.optimizer_set_allreduce(opt, shard.allreduce_sum())
        tr = s.forward_capture(Tn)
        _, dl = mse_objective(tr, target)
        s.backward(dl, keys=())
        s.optimizer_grads_from_backward(opt)
        s.optimizer_step_with_inv_record_steps(opt, 1e-3, 1.0)
        w = s.get_param_array("hh.gnabar")
        step, m, v, _ = s.optimizer_get_adam_state(opt)
        torch.cuda.synchronize()
        q.put((rank, dl, w, m, target))
        s.close()
    finally:
        dist.destroy_process_group()


def test_gradient_allreduce_before_adam_two_ranks():
    from heliox_b200 import synth
    from oracle import oracle as O

    res = _run("adam")
    g = synth.random_tree_batch(3, seed0=70, nmin=60, nmax=120)
    # the oracle gradient of each rank's loss, summed: what the all-reduce must produce
    gsum = np.zeros(g.hh.n)
    for r in res:
        _, gr = O.adjoint(g, 1200, r[1])
        gsum += gr["hh.gnabar"]
    w0 = g.hh.fields["gnabar"]
    ws, m_ref, _ = O.adam_port(w0, gsum[None, :], 1e-3, 1.0)
    (_, _, w0_gpu, m0, _), (_, _, w1_gpu, m1, _) = res
    assert np.array_equal(w0_gpu, w1_gpu) and np.array_equal(m0, m1)  # one update on both ranks
    assert np.max(np.abs(m0 - m_ref)) <= 1e-7 * np.max(np.abs(m_ref))  # m = (1 - beta1) * summed gradient
    assert np.max(np.abs(w0_gpu - ws[0])) <= 1e-10
