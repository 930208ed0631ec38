"""Regenerates the golden fixtures from the reference's own CPU integrator.

Needs the reference sources (to build oracle/_ref/hxref_run with
oracle/ref_build.sh); run from the repository root:

    python tests/golden/make_golden.py [case ...]   (case or case_perm3)

Each case exports a seeded synthetic group in CoreNEURON format
(heliox_b200.coredat), runs the reference (read_coredat -> data_format_trans ->
Simulate(CPU) finitialize + fadvance) and stores the voltage trace at the
probes together with the spike list the reference writes (spk.dat: time with
8 significant digits, gid).
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from heliox_b200 import synth  # noqa: E402
from oracle import oracle as O  # noqa: E402

CASES = {
    "ball_and_stick": (lambda: synth.ball_and_stick(), 4000, [0, 1, 25, 50, 100]),
    "ball_and_stick_teacher": (lambda: synth.ball_and_stick(gnabar_scale=1.1), 4000, [0]),
    "trees3": (lambda: synth.random_tree_batch(3, seed0=20240), 4000, None),
    "tree_deep": (lambda: synth.random_tree_cell(77, ncomp=400, max_levels=40), 2000, None),
    # event-driven network: ExpSyn/Exp2Syn, PreSyn detection, NetCon delays, NetStims (noise 1)
    "net_spiking": (lambda: synth.spiking_network(nstim=6, weight=(0.02, 0.08), stim_noise=1.0, stim_interval=5.0),
                    2400, None),
    # HalfGap + gapjunction_lr + neuron_to_neuron_syn_lr coupling
    "net_coupled": (lambda: synth.coupled_network(), 2000, None),
    # gapjunction_noptr (vpre through the gap transfer) on nodes that also carry
    # HalfGap, gapjunction_lr and graded synapses: the per-node current order
    "net_gapnoptr": (lambda: net_gapnoptr(), 2000, None),
    # library cells (channels, ions, calcium dynamics) coupled by gaps and graded synapses
    "lib_net_coupled": (lambda: synth.lib_network("coupled", ncell=5, seed=44, ngap=4, ngapj=3, ngraded=8,
                                                  ngapnp=3), 1600, None),
    # user-mech channel set with calcium dynamics (spiking library cells)
    "lib_cells": (lambda: synth.lib_tree_batch(2, seed0=700, nmax=200), 2000, None),
    # hh cells and library cells in one group
    "lib_mixed": (lambda: _lib_mixed(), 1200, None),
    # library cells with the worm-lr calcium dynamics cainternm_lr
    "lib_cainternm": (lambda: synth.lib_tree_batch(2, seed0=710, nmax=200, cadyn="cainternm_lr"), 2000, None),
}


def net_gapnoptr():
    """A coupled network plus gapjunction_noptr instances on every node that
    carries a graded synapse, a gapjunction_lr or a HalfGap (weight
    U[1e-4, 1e-3] uS, vpre from the root of the next cell), and five pairs at
    random nodes."""
    from heliox_b200.synth import _table

    g = synth.coupled_network(ncell=5, seed=31, ngap=5, ngapj=4, ngraded=12, ngapnp=5)
    cell = g.cell_of_node()
    nodes = list(g.gapnoptr.nodes) + list(g.graded.nodes) + list(g.gapjunction.nodes) + list(g.halfgap.nodes)
    src = list(g.gapnoptr.ifields["src"]) + [int(np.nonzero(cell == (cell[n] + 1) % g.ncell)[0][0])
                                             for n in nodes[g.gapnoptr.n:]]
    w = list(g.gapnoptr.fields["weight"]) + list(np.random.default_rng(1).uniform(1e-4, 1e-3, len(nodes) - g.gapnoptr.n))
    g.gapnoptr = _table(nodes, {"weight": w}, {"src": src})
    g.validate()
    return g


def _lib_mixed():
    from heliox_b200.model import concat_groups

    g = concat_groups([synth.lib_tree_cell(11, ncomp=80), synth.random_tree_cell(12, ncomp=90)])
    g.celsius = 20.0
    return g


# cases also run with the reference's node permutation type 3 (its default in
# python_lib/heliox_learn/runtime.py:13: the branch split of
# permute_order.cpp:641-1170 solved by cpu_solve_permute3, simulate.cpp:631-713),
# stored as <case>_perm3.npz
PERM3 = ("ball_and_stick", "trees3", "tree_deep", "net_spiking", "lib_cells")

ADAM = dict(n=64, steps=25, lr=1e-3, inv_record_steps=0.25, beta1=0.9, beta2=0.999, eps=1e-8, impedance=2.0, seed=5)


def adam_inputs():
    rng = np.random.default_rng(ADAM["seed"])
    w0 = rng.uniform(0.01, 0.2, ADAM["n"])
    grads = rng.standard_normal((ADAM["steps"], ADAM["n"])) * 10.0
    return w0, grads


def main(names=None):
    """Regenerate every fixture, or only the named cases."""
    if names:
        for name in names:
            make_case(name)
        return
    w0, grads = adam_inputs()
    ws, m, v = O.adam_ref(w0, grads, ADAM["lr"], ADAM["inv_record_steps"], ADAM["beta1"], ADAM["beta2"], ADAM["eps"],
                          ADAM["impedance"])
    np.savez_compressed(os.path.join(HERE, "adam.npz"), w0=w0, grads=grads, weights=ws, m=m, v=v)
    print("adam", ws.shape)
    for name in CASES:
        make_case(name)
    for name in PERM3:
        make_case(name, permute_type=3)


def make_case(name, permute_type=0):
    if name.endswith("_perm3"):
        name, permute_type = name[: -len("_perm3")], 3
    make, nstep, probes = CASES[name]
    g = make()
    p = np.asarray(probes if probes is not None else list(g.soma_nodes()) + [g.nnode - 1], dtype=np.int32)
    tr, spk = O.ref_forward(g, nstep, probe=p, permute_type=permute_type)
    out = f"{name}_perm{permute_type}.npz" if permute_type else f"{name}.npz"
    np.savez_compressed(os.path.join(HERE, out), trace=tr, probes=p, nstep=nstep, permute_type=permute_type,
                        spikes=np.asarray(spk, dtype=np.float64).reshape(-1, 2))
    print(out, tr.shape, len(spk))


if __name__ == "__main__":
    main(sys.argv[1:])
