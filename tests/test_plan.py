"""CPU: the host planner (cell packing + branch-level Hines schedule).

``hx_plan_check`` builds the execution plan the kernels use and replays the
planned triangularisation/back-substitution order on the CPU; it must equal the
reference's solve_serial (src/simulate.cpp:558-581) bit for bit, for the
forward and the transposed system.
"""
import numpy as np
import pytest

from heliox_b200 import _lib, synth
from heliox_b200.model import CellGroup, MechTable, _f64, _i32, concat_groups


def _chain_group(n, ncell=1):
    cells = []
    for c in range(ncell):
        parent = np.arange(-1, n - 1, dtype=np.int32)
        g = CellGroup(
            ncell=1,
            parent=parent,
            a=_f64(-np.linspace(1, 2, n)),
            b=_f64(-np.linspace(2, 3, n)),
            area=_f64(np.full(n, 100.0)),
            cm=_f64(np.ones(n)),
            hh=MechTable(_i32([0]), {k: _f64([v]) for k, v in synth.HH_STD.items()}),
            pas=MechTable(_i32(np.arange(1, n)), {"g": _f64(np.full(n - 1, 1e-4)), "e": _f64(np.full(n - 1, -65.0))}),
            iclamp=MechTable(_i32([]), {k: _f64([]) for k in ("del", "dur", "amp")}),
        )
        cells.append(g)
    return concat_groups(cells) if ncell > 1 else cells[0]


def _star_group(arms=40, arm_len=3):
    parent = [-1]
    for a in range(arms):
        prev = 0
        for j in range(arm_len):
            parent.append(prev)
            prev = len(parent) - 1
    n = len(parent)
    rng = np.random.default_rng(0)
    return CellGroup(
        ncell=1,
        parent=_i32(parent),
        a=_f64(-rng.uniform(1, 3, n)),
        b=_f64(-rng.uniform(1, 3, n)),
        area=_f64(np.full(n, 50.0)),
        cm=_f64(np.ones(n)),
        hh=MechTable(_i32([0]), {k: _f64([v]) for k, v in synth.HH_STD.items()}),
        pas=MechTable(_i32([]), {"g": _f64([]), "e": _f64([])}),
        iclamp=MechTable(_i32([]), {k: _f64([]) for k in ("del", "dur", "amp")}),
    )


@pytest.mark.parametrize(
    "maker,target",
    [
        (lambda: synth.ball_and_stick(), 0),
        (lambda: _chain_group(1), 0),
        (lambda: _chain_group(2), 0),
        (lambda: _chain_group(7, ncell=5), 0),
        (lambda: _star_group(), 0),
        (lambda: synth.random_tree_batch(24, seed0=11), 0),
        (lambda: synth.random_tree_batch(24, seed0=11), 4096),
        (lambda: synth.random_tree_cell(3, ncomp=3000, max_levels=40), 0),
        (lambda: _chain_group(1500), 0),  # 63 segments of <= 24 nodes
        (lambda: _star_group(arms=700, arm_len=1), 0),  # more segments than a CTA's threads
    ],
)
def test_planned_solve_bit_exact(maker, target):
    g = maker()
    stats, diff = _lib.plan_check(g, target)
    assert diff == 0.0
    assert stats["pq_rel_diff"] <= 1e-13
    assert stats["npack"] >= 1
    assert stats["max_pack_nodes"] >= 1


def test_packing_balance_and_coverage():
    g = synth.random_tree_batch(96, seed0=3)
    stats, diff = _lib.plan_check(g, 0)
    assert diff == 0.0
    # packs hold whole cells in 16-warp CTAs; node counts stay within 1.6x of the mean
    assert stats["imbalance"] < 1.6
    assert stats["nbranch"] >= g.ncell
    assert stats["max_pack_nodes"] >= 1000 or stats["npack"] == 1


def test_invalid_group_rejected():
    g = synth.ball_and_stick()
    bad = g.copy()
    bad.parent = bad.parent.copy()
    bad.parent[5] = 7  # parent after child
    with pytest.raises(ValueError):
        _lib.plan_check(bad)


@pytest.mark.parametrize("ncell,cap,nsm", [(296, 4500, 148), (1024, 4500, 148), (700, 2000, 64), (40, 4500, 148)])
def test_balanced_packing_over_sms(ncell, cap, nsm):
    """Device-aware plan (hx_load_group's default): whole cells dealt over
    whole waves of nsm CTAs within the node capacity, warps by the step-time
    model; the planned solve stays bit-exact."""
    g = synth.random_tree_batch(ncell, seed0=101)
    stats, diff = _lib.plan_check(g, 0, cap, nsm)
    assert diff == 0.0
    assert stats["pq_rel_diff"] <= 1e-13
    assert stats["max_pack_nodes"] <= cap
    total = g.nnode
    waves = -(-total // (nsm * int(cap * 0.96)))
    assert stats["npack"] <= max(waves * nsm, -(-ncell // 16))
    assert stats["npack"] >= min(ncell, nsm) or stats["npack"] * cap >= total
    assert stats["est_mean"] > 0
    if ncell >= 2 * nsm:  # several cells a CTA: the slowest CTA's modelled step time stays near the mean
        assert stats["est_max"] <= 1.35 * stats["est_mean"]
    if ncell <= nsm:  # fewer cells than SMs: one cell a CTA
        assert stats["npack"] == ncell


def test_balanced_plan_is_deterministic():
    g = synth.random_tree_batch(300, seed0=5)
    a, _ = _lib.plan_check(g, 0, 4000, 148)
    b, _ = _lib.plan_check(g, 0, 4000, 148)
    assert a == b
