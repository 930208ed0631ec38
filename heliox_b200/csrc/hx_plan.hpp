// hx_plan.hpp -- host-side execution plan: cell packing, warp groups and the
// branch-level Hines schedule consumed by the CUDA kernels.
//
// The reference orders nodes for its GPU solvers with permute types 1 and 3
// (src/permute_order.cpp:145-210, 465-1170) and applies the order with
// src/permute.cpp:256-622.  Here the order is designed for one CTA per "cell
// pack": a pack holds whole cells, each cell owns a group of warps of the CTA
// (1..8, by size) and synchronises only with itself (named barrier), so cells
// of one CTA never wait for each other.  Inside a cell the nodes are laid out
// branch by branch (an unbranched chain is contiguous, head first), branches
// sorted by branch level; the triangularisation walks the cell's levels
// deepest-first, one thread per branch, and the back-substitution walks them
// root-first.  Child branches fold into their parent node in descending
// reference index, the order solve_serial (src/simulate.cpp:558-581) applies
// them, so the planned solve replayed in division form is bit-identical to the
// serial one.
#pragma once

#include <cstddef>
#include <string>
#include <vector>

#include "heliox_b200.h"

namespace hx {

constexpr int kWarpsPerCta = 16;
constexpr int kSegMax = 24;  // longest branch segment (longer unbranched chains are cut)

struct Plan {
    int ncell = 0, nnode = 0, nhh = 0, npas = 0, nic = 0;
    int npack = 0;
    // per pack (size npack+1) prefix offsets
    std::vector<int> pack_node_off;   // GPU node ids
    std::vector<int> pack_slot_off;   // cell slots
    std::vector<int> pack_br_off;     // global branch ids
    std::vector<int> pack_bch_off;    // into br_child
    std::vector<int> pack_nch_off;    // into node_child
    // cell slots, in pack order
    std::vector<int> cs_node0, cs_nnode;    // pack-local first node, node count
    std::vector<int> cs_warp0, cs_nwarp;    // warp range inside the CTA
    std::vector<int> cs_bar;                // named-barrier id (1..15), 0 for one-warp cells
    std::vector<int> cs_lvl_off, cs_nlev;   // cell's level table in level_br_off (nlev+1 entries)
    std::vector<int> cs_cell;               // cell id
    std::vector<int> level_br_off;          // pack-local branch ids
    // branches (global id = pack_br_off[p] + pack-local id); node ids pack-local
    std::vector<int> br_head, br_end, br_parent;
    std::vector<int> br_child_off;     // size nbranch+1, global offsets into br_child
    std::vector<int> br_child;         // child-head node ids, descending reference index
    std::vector<int> br_child_br;      // the same children as pack-local branch ids (-1: another unit)
    // nodes in GPU order (global id = pack_node_off[p] + pack-local id)
    std::vector<int> node_parent;      // pack-local, -1 for roots
    std::vector<int> node_child_off;   // size nnode+1, global offsets into node_child
    std::vector<int> node_child;       // pack-local, ascending reference index
    std::vector<int> gpu2ref, ref2gpu; // node permutation
    std::vector<int> node_hh;          // hh instance (reference id) or -1
    std::vector<int> node_pas;         // pas instance (reference id) or -1
    std::vector<int> node_ic_off;      // size nnode+1
    std::vector<int> node_ic;          // GPU IClamp instance ids
    std::vector<int> ic_gpu2ref;
    std::vector<int> node_cell;        // GPU node -> cell id
    // split cell (one cell larger than a CTA): pack 0 holds the top unit, the
    // other packs hold subtree units; links between them are coded in
    // node_parent / node_child / br_parent / br_child as -(2 + subtree id)
    int warps = kWarpsPerCta;  // warps a CTA of this plan
    int nsub = 0;
    std::vector<int> sub_root;    // GPU node of each subtree root
    std::vector<int> sub_parent;  // GPU node (in pack 0) of its parent
    // statistics
    int max_pack_nodes = 0, max_pack_hh = 0, max_levels = 0, max_crit = 0;
    int max_pack_branches = 0, max_pack_bch = 0, max_pack_nch = 0;
    double imbalance = 1.0;
    double est_max = 0.0, est_mean = 0.0;  // modelled cycles of one forward + backward step: slowest / mean CTA
};

// Validates the group and builds the plan.  nodes_per_warp: target cell nodes
// per warp (0 = default); max_pack_nodes: node capacity of one CTA (shared
// memory), 0 = unlimited; nsm: SMs of the device (0 = unknown).  With nsm and
// a capacity but no explicit nodes_per_warp the CTAs are balanced over whole
// waves of nsm CTAs.  warps_per_cta: CTA width the plan is built for (at most
// that many cells a CTA).  Returns "" on success, else a reason.
std::string build_plan(const hx_group_desc& g, int nodes_per_warp, int max_pack_nodes, Plan& out, int nsm = 0,
                       int warps_per_cta = kWarpsPerCta);

// CPU emulation of the kernels' planned Hines solve on GPU-ordered arrays
// (a, b, d, rhs are GPU-ordered and pack-contiguous).  transposed swaps a/b.
void planned_solve_cpu(const Plan& P, const double* a, const double* b, double* d, double* rhs, bool transposed);

// CPU emulation of the kernels' division-free form of the same schedule (the
// p/q recurrence of hines_cell in hx_step.cuh, with exact reciprocals in
// place of the device's batch-inverted Newton reciprocals).  Output: rhs holds
// the solution.
void planned_solve_pq_cpu(const Plan& P, const double* a, const double* b, double* d, double* rhs, bool transposed);

// CPU emulation of hines_rt (hx_step.cuh): the three-phase reduced-tree solve
// per cell, exact reciprocals; for plans without a split cell.  Output: rhs
// holds the solution.
void planned_solve_rt_cpu(const Plan& P, const double* a, const double* b, double* d, double* rhs, bool transposed);

}  // namespace hx
