// hx_dev.hpp -- POD views of device buffers passed by value to the kernels.
#pragma once

#include <cstddef>

namespace hx {

constexpr int kThreads = 256;  // threads per CTA (one CTA per cell pack)

// The execution plan and the model parameters, GPU (pack-contiguous) order.
struct DevGroup {
    int npack, nnode, nhh, npas, nic;
    int smem_n, smem_nh;  // shared-memory array strides (max pack nodes / hh instances)
    const int *pack_node_off, *pack_hh_off, *pack_br_off, *pack_lvl_off, *pack_nlev, *level_br_off;
    const int *br_head, *br_end, *br_parent, *br_child_off, *br_child;
    const int *node_parent, *node_child_off, *node_child;
    const int *node_hh, *node_pas, *node_ic_off, *node_ic;
    const double *a, *b, *cm, *area;
    const double *hh_gnabar, *hh_gkbar, *hh_gl, *hh_el, *hh_ena, *hh_ek;
    const double *pas_g, *pas_e;
    const double *ic_del, *ic_dur, *ic_amp;
    double dt, cfac, q10;
};

// Simulation state in global memory (between windows).
struct DevState {
    double *v, *m, *h, *n;
};

// Forward tape: state at the start of step k lives in row (k - k_base).
struct DevTape {
    double* v;           // rows x nnode
    double *m, *h, *n;   // rows x nhh
    int k_base;
};

// Probe (recorded voltage) layout: per pack list of (pack-local node, column).
struct DevProbe {
    const int* pack_off;  // npack+1
    const int* local;
    const int* slot;
    int nprobe;
};

// Adjoint state (between windows) and gradient accumulators (GPU order).
struct DevAdj {
    double *lv, *lm, *lh, *ln;
};

struct DevGrad {
    double *hh_gnabar, *hh_gkbar, *hh_gl, *hh_el;
    double *pas_g, *pas_e, *cm, *ic_amp;
};

}  // namespace hx
