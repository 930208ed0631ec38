// hx_plan.hpp -- host-side execution plan: cell packing and the branch-level
// Hines schedule consumed by the CUDA kernels.
//
// The reference orders nodes for its GPU solvers with permute types 1 and 3
// (src/permute_order.cpp:145-210, 465-1170) and applies the order with
// src/permute.cpp:256-622.  Here the order is designed for one CTA per "cell
// pack": each pack holds whole cells; inside a pack the nodes are laid out
// branch by branch (an unbranched chain is contiguous, head first), branches
// sorted by branch level.  The triangularisation walks levels deepest-first, one
// thread per branch, and the back-substitution walks them root-first; child
// branches are folded into their parent node in descending reference index,
// which is the order solve_serial (src/simulate.cpp:558-581) applies them, so
// the planned solve is bit-identical to the serial one.
#pragma once

#include <cstddef>
#include <string>
#include <vector>

#include "heliox_b200.h"

namespace hx {

struct Plan {
    int ncell = 0, nnode = 0, nhh = 0, npas = 0, nic = 0;
    int npack = 0;
    // per pack (size npack+1): prefix offsets
    std::vector<int> pack_node_off, pack_hh_off, pack_br_off, pack_lvl_off;
    std::vector<int> pack_nlev;        // size npack
    // level -> [first branch, last branch) of the pack, pack-local branch ids;
    // entries pack_lvl_off[p] .. pack_lvl_off[p] + nlev_p (inclusive)
    std::vector<int> level_br_off;
    // branches (global id = pack_br_off[p] + local id); node ids pack-local
    std::vector<int> br_head, br_end, br_parent;
    std::vector<int> br_child_off;     // size nbranch+1
    std::vector<int> br_child;         // pack-local child-head node ids, descending reference index
    // nodes in GPU order (global id = pack_node_off[p] + local id)
    std::vector<int> node_parent;      // pack-local, -1 for roots
    std::vector<int> node_child_off;   // size nnode+1
    std::vector<int> node_child;       // pack-local, ascending reference index
    std::vector<int> gpu2ref, ref2gpu; // node permutation
    std::vector<int> node_hh;          // pack-local hh instance or -1
    std::vector<int> node_pas;         // global GPU pas instance or -1
    std::vector<int> node_ic_off;      // size nnode+1
    std::vector<int> node_ic;          // global GPU IClamp instance ids
    std::vector<int> hh_gpu2ref, pas_gpu2ref, ic_gpu2ref;
    std::vector<int> node_cell;        // GPU node -> cell id
    // statistics
    int max_pack_nodes = 0, max_pack_hh = 0, max_levels = 0, max_crit = 0;
    double imbalance = 1.0;
};

// Validates the group and builds the plan.  Returns "" on success, else a reason.
std::string build_plan(const hx_group_desc& g, int nodes_per_pack, Plan& out);

// CPU emulation of the kernels' planned Hines solve on GPU-ordered arrays
// (a, b, d, rhs are GPU-ordered and pack-contiguous).  transposed swaps a/b.
void planned_solve_cpu(const Plan& P, const double* a, const double* b, double* d, double* rhs, bool transposed);

}  // namespace hx
