// hx_dev.hpp -- POD views of device buffers passed by value to the kernels.
#pragma once

#include <cstddef>

namespace hx {

constexpr int kThreads = 512;  // threads per CTA (one CTA per cell pack, 16 warps, one CTA per SM)
// split-cell kernels: 8 warps a CTA, so that their larger state fits the
// registers (232 a thread) without spilling
constexpr int kSplitThreads = 256;

// kHasSyn: the node carries ExpSyn / Exp2Syn instances; kHasCpl: HalfGap,
// gapjunction_lr or graded-synapse instances; kHasIn: it is the partner
// (source / presynaptic node) of such an instance.  The per-node network
// loops run only on flagged nodes.
enum NodeFlag : int { kHasPas = 1, kHasHH = 2, kHasSyn = 4, kHasCpl = 8, kHasIn = 16 };

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
    const int *br_head, *br_end, *br_parent, *br_child_off, *br_child, *br_child_br;
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
    const int* slot_off;  // per cell slot (nslot+1): the slot's probes, sorted by (local node, probe index)
    const int* local;     // pack-local node
    const int* slot;      // output column
    int nprobe;
};

// Adjoint state (between windows), node-indexed; lA/lB per synapse.
struct DevAdj {
    double *lv, *lm, *lh, *ln;
    double *lA, *lB;
};

// Gradient accumulators: node-indexed except ic_amp (per IClamp instance)
// and the network kinds (per instance in GPU order).
struct DevGrad {
    double *hh_gnabar, *hh_gkbar, *hh_gl, *hh_el;
    double *pas_g, *pas_e, *cm, *ic_amp;
    double *syn_w, *syn_e;             // exponential synapses (ExpSyn then Exp2Syn per node)
    double *hg_g, *gj_g, *gj_w, *gr_w;  // HalfGap, gapjunction_lr, neuron_to_neuron_syn_lr
    // accumulators the caller did not ask for (bit 1 << HX_P_* kind, kinds
    // 0..15): neither read nor written, so the reverse sweep moves only the
    // requested gradients
    unsigned skip;
};

// A cell split across CTAs (hx_plan.hpp): pack 0 holds the top part, the
// other packs its subtrees.  Per subtree id, the interface values that cross
// CTAs each step go through these arrays; the grid barrier counter lives in
// bar[0..1] and err records a barrier that gave up waiting.
struct DevSplit {
    int nsub, nblocks;
    const int *sub_root, *sub_parent;  // GPU node ids
    double *xd, *xrhs;                 // eliminated diagonal / rhs of each subtree root
    double *xx;                        // solution at each root's parent (dv forward, w backward)
    double *xv;                        // root value read by the top part (v forward, w backward)
    double *xvp;                       // v of each root's parent (forward)
    unsigned* bar;
    int* err;
    // sleeps of ~100 ns a barrier wait takes before it gives up and sets *err
    long long spin_limit;
};
constexpr long long kSplitSpinLimitDefault = 20000000LL;  // ~2 s

// Network parts of a group (step kernels instantiated with kNet = true).
// Instance arrays are in GPU order: sorted by GPU node, ExpSyn before Exp2Syn
// on a node, then by reference instance -- the order in which the reference's
// mechanism loop accumulates them into one node's rhs/d.
struct DevNet {
    // exponential synapses: B' = B + fB w, A' = A + fA w at an event;
    // x <- x + c (0 - x) per step (c = 1 - exp(-dt/tau)); i = (B - A)(v - e)
    // Synapse states, their adjoints and gradients live in global memory and
    // are read and written only by the thread that owns the synapse's node
    // (delivery, current, decay and the event weight gradients alike).
    int nsyn, npack;
    const int *node_syn_off, *pack_syn_off;
    const int* syn_node;  // GPU node of synapse j
    const double *syn_e, *syn_w, *syn_cA, *syn_cB, *syn_fA, *syn_fB;
    double *sA, *sB;  // state
    double *tA, *tB;  // tape rows (k - k_base) x nsyn after the step's deliveries; null = no tape
    // events: bucket (k, p) holds the synapses of pack p that receive an event
    // at step k: ev_cnt[k * npack + p] entries from ev_syn[(k * npack + p) * ev_cap]
    const int *ev_cnt, *ev_syn;
    int ev_cap;
    // PreSyn threshold detection (one per cell slot; -1: none)
    const int *cs_ps_node, *cs_gid;
    const double* cs_ps_thr;
    int* cs_ps_flag;
    int2* win_spk;  // (source gid, step) of the window's spikes
    int* win_n;
    int win_cap, detect;
    // HalfGap (electrode): i = (v[src] - v) g
    const int *node_hg_off, *hg_src;
    const double* hg_g;
    // gapjunction_lr: i = w (g (v - v[pre]))
    const int *node_gj_off, *gj_pre;
    const double *gj_g, *gj_w;
    // neuron_to_neuron_syn_lr: i = |w| (g s (v - erev)), s' = inf + (s - inf) exp(-dt/tau)
    const int *node_gr_off, *gr_pre;
    const double *gr_w, *gr_g, *gr_k, *gr_erev, *gr_delta, *gr_vth;
    int ngr;
    double *gr_s, *lS;  // state s (s_{k-1} entering step k), adjoint of s
    double* tS;         // tape: row 0 = s_{k_base-1}, row k-k_base+1 = s_k
    int coupled;             // gaps or graded synapses present: partner voltages every step
    const double* vpeer;     // v_k of every node (read-only during a coupled launch)
    double* vout;            // v_{k+1} written by a coupled forward launch
    // reverse-sweep coupling: per-instance contributions to the partner's
    // dL/dv, written by the launch of step k, read by the launch of step k-1
    double *x_hg_out, *x_gj_out, *x_gr_out;
    const double *x_hg_in, *x_gj_in, *x_gr_in;
    const int *node_in_off, *node_in;  // incoming (kind << 28 | instance) per node
    // grid-synchronous coupled launches (cooperative, every pack co-resident):
    // one launch runs many steps with one bounded grid barrier per step;
    // v_k of every node in vbuf[k & 1] (forward), the reverse contributions
    // of step k in xbuf[k & 1] (HalfGap, gapjunction, graded instances,
    // xstride apart)
    int gsync, nhg, ngj;
    double* vbuf;
    double* xbuf;
    size_t xstride;
    unsigned* gbar;    // arrival count, generation (zeroed before each launch)
    int* gerr;         // set when a barrier wait gave up
    long long gspin;   // sleeps of ~100 ns a wait takes before it gives up
};

// Library mechanisms of a group (step kernels instantiated with kLib = true).
// Entries are the mechanism instances in GPU node order, on one node in
// CoreNEURON type order (ions, CaDynamics_E2, channels): entry e has code
// type << 24 | instance (GPU instance order of its type), its states at
// ent_st[e] of the flat state array (ca_ion: cai; channels: their gates) and
// its fixed parameters at ent_fix[e] of fix (entries of a type with equal
// values share one copy) (ions: erev / concentrations;
// NaTg: vshifth, vshiftm, slopeh, slopem; SK_E2: zTau; hd_la: vhalfl, tau,
// ehd, kl, vhalft, a0t, zetat, gmt and qtl q10^((celsius - 33)/10) a0t;
// km_la: Ra, Rb, tha, qa, tadj; kca_la: Ra, Rb, caix, tadj; it2_la: vshift,
// v12m, vwm, v12h, vwh, am, ah, vm1, vm2, vh1, vh2, wm1, wm2, wh1, wh2;
// sca_la: inactF, actF, vshift, tadj; worm-lr: gb, ek_tmp, dv, kinetics).  Trainable
// parameters (HX_P_CADYN_GAMMA .. HX_P_NCA_LR_W) live per instance in
// prm[kind - HX_P_CADYN_GAMMA], their gradients in grad[...].
constexpr int kLibKinds = 42;
struct DevLib {
    int nst;
    const int *node_off, *ent, *ent_st, *ent_fix;  // node_off: nnode + 1; ent_st: nent + 1
    const unsigned long long* mask;  // per node: bit t set when the node has an entry of type t
    const double* fix;
    const double* prm[kLibKinds];
    double* grad[kLibKinds];
    double* st;     // states at the current step
    double* lam;    // adjoints of the states (backward)
    double* nica;   // per node: calcium current of the forward's current step
    double* nlica;  // per node: adjoint of the step's calcium current (backward)
    double* tape;   // rows x nst: states at the start of each step, row 0 = step k_base
    int k_base;
    double ktf;  // 1000 R (celsius + 273.15) / F (eion.cuh:38-41)
    double dt;
};

}  // namespace hx
