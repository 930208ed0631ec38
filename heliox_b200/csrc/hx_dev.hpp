// hx_dev.hpp -- POD views of device buffers passed by value to the kernels.
#pragma once

#include <cstddef>

namespace hx {

constexpr int kThreads = 256;  // threads per CTA (one CTA per cell pack, 8 warps)

enum NodeFlag : int { kHasPas = 1, kHasHH = 2 };

// The execution plan and the model parameters.  Node arrays are in GPU
// (pack-contiguous, cell-contiguous) order; density-mechanism parameters are
// node-indexed (zero where the mechanism is absent, selected by node_flags).
struct DevGroup {
    int npack, nnode, nic;
    // shared-memory table sizes (maxima over packs)
    int smem_n, smem_br, smem_bch, smem_nch, smem_lvl;
    const int *pack_node_off, *pack_slot_off, *pack_br_off, *pack_bch_off, *pack_nch_off;
    const int *cs_node0, *cs_nnode, *cs_warp0, *cs_nwarp, *cs_bar, *cs_lvl_off, *cs_nlev;
    const int* level_br_off;
    const int *br_head, *br_end, *br_parent, *br_child_off, *br_child;
    const int *node_parent, *node_child_off, *node_child, *node_flags, *node_ic_off, *node_ic;
    const double *a, *b, *cm, *area;
    const double *hh_gnabar, *hh_gkbar, *hh_gl, *hh_el, *hh_ena, *hh_ek;
    const double *pas_g, *pas_e;
    const double *ic_del, *ic_dur, *ic_amp;
    double dt, cfac, q10;
};

// Simulation state in global memory (between windows); gates node-indexed.
struct DevState {
    double *v, *m, *h, *n;
};

// Forward tape: state at the start of step k lives in row (k - k_base); every
// row holds nnode values of v and of each gate.
struct DevTape {
    double* v;
    double *m, *h, *n;
    int k_base;
};

// Probe (recorded voltage) layout: per pack list of (pack-local node, column).
struct DevProbe {
    const int* pack_off;  // npack+1
    const int* local;
    const int* slot;
    int nprobe;
};

// Adjoint state (between windows), node-indexed.
struct DevAdj {
    double *lv, *lm, *lh, *ln;
};

// Gradient accumulators: node-indexed except ic_amp (per IClamp instance).
struct DevGrad {
    double *hh_gnabar, *hh_gkbar, *hh_gl, *hh_el;
    double *pas_g, *pas_e, *cm, *ic_amp;
};

}  // namespace hx
