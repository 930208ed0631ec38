/*
 * hx_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the reference's fixed-step forward integrator and a
 * discrete adjoint of exactly that step sequence.  It is the checker for the
 * CUDA path: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * leg may load it.  The product library never links or calls it.
 *
 * Parity pin: the forward is checked bit-for-bit/within 1e-12 against the
 * reference's own CPU integrator compiled from its sources (oracle/ref_build.sh
 * -> oracle/_ref/libhxref.so); the adjoint is checked against central finite
 * differences of that forward (the reference has no exact gradient,
 * src/runtime_api/learn/LearnRuntime.cpp:208-210).
 */
#ifndef HX_ORACLE_H
#define HX_ORACLE_H

#ifdef __cplusplus
extern "C" {
#endif

/* Network parts (optional; hxo_group.net may be NULL).  Synapse instance
 * tables are node-sorted like the reference's nodeindices; every ExpSyn /
 * Exp2Syn instance is the target of one NetCon (src, delay, weight).  Sources
 * 0..ncell-1 are the cells' PreSyns (threshold detection at the cell's root
 * node), sources ncell.. are the NetStims in instance order. */
typedef struct hxo_net {
    int nexp;
    const int *exp_node, *exp_src;
    const double *exp_tau, *exp_e, *exp_delay, *exp_w;
    int nexp2;
    const int *exp2_node, *exp2_src;
    const double *exp2_tau1, *exp2_tau2, *exp2_e, *exp2_delay, *exp2_w;
    const double* ps_thresh; /* ncell */
    int nstim;
    const double *ns_interval, *ns_number, *ns_start, *ns_noise;
    int rng_mode; /* 0: reference CPU mode (zero-initialised Random123 state), 1: GPU mode (sequence 0) */
    int nhg;
    const int *hg_node, *hg_src;
    const double* hg_g;
    int ngj;
    const int *gj_node, *gj_pre;
    const double *gj_g, *gj_w;
    int ngn; /* gapjunction_noptr: vpre copied from v of node gn_src by the gap transfer */
    const int *gn_node, *gn_src;
    const double* gn_w;
    int ngr;
    const int *gr_node, *gr_pre;
    const double *gr_w, *gr_g, *gr_delta, *gr_k, *gr_vth, *gr_erev;
    /* outputs of the forward: spikes of the cells' PreSyns (gid = cell, time) */
    int spike_cap;
    int* spike_gid;
    double* spike_t;
    int nspike; /* total detected (may exceed spike_cap) */
    /* NetStim spikes (instance, time) in emission order */
    int ns_spike_cap;
    int* ns_spike_id;
    double* ns_spike_t;
    int ns_nspike;
} hxo_net;

/* Library mechanisms (optional; hxo_group.lib may be NULL): the ions and the
 * user-mech channel set, CoreNEURON types after the network mechanisms in
 * this order.  Table t holds n instances on sorted, distinct nodes; par holds
 * HXO_LIB_NPAR columns per instance (row-major):
 *   na_ion: ena | k_ion: ek | ca_ion: cai (initial), cao, eca, nernst (0/1)
 *   CaDynamics_E2: gamma, decay, depth, minCai
 *   Ca_HVA, Ca_LVAst, Im, K_Pst, K_Tst, Nap_Et2, SKv3_1: gbar
 *   NaTg: gbar, vshifth, vshiftm, slopeh, slopem | SK_E2: gbar, zTau
 *   hd_la: ghdbar, vhalfl, tau, ehd, kl, vhalft, a0t, zetat, gmt, q10, qtl
 *   km_la: gbar, Ra, Rb, tha, qa, tadj
 *   kca_la: gbar, Ra, Rb, caix, tadj
 *   it2_la: gcabar, vshift, v12m, vwm, v12h, vwh, am, ah, vm1, vm2, vh1, vh2,
 *           wm1, wm2, wh1, wh2
 *   kdr_la: gbar
 *   sca_la: gbar, inactF, actF, vshift, tadj | Ca: gCabar
 *   worm-lr (shl1_lr, kvs1_lr, irk_lr, egl36_lr, shk1_lr, egl2_lr, cca1_lr,
 *   egl19_lr, unc2_lr): w, gb, ek_tmp / eca_tmp, dv, then the kinetics GLOBALs
 *   in the mechanism's order
 *   kcnl_lr: w, gbkcnl, dv, kca, a, ek_tmp | nca_lr: w, gbnca, ena_tmp */
enum {
    HXO_NA_ION = 0, HXO_K_ION, HXO_CA_ION, HXO_CADYN, HXO_CA_HVA, HXO_CA_LVAST, HXO_IM, HXO_K_PST, HXO_K_TST,
    HXO_NATG, HXO_NAP_ET2, HXO_SK_E2, HXO_SKV3_1, HXO_HD_LA, HXO_KM_LA, HXO_KCA_LA, HXO_IT2_LA, HXO_KDR_LA,
    HXO_SCA_LA, HXO_CA, HXO_SHL1_LR, HXO_KVS1_LR, HXO_IRK_LR, HXO_EGL36_LR, HXO_SHK1_LR, HXO_EGL2_LR,
    HXO_CCA1_LR, HXO_EGL19_LR, HXO_UNC2_LR, HXO_KCNL_LR, HXO_NCA_LR,
    HXO_KQT3_LR, HXO_CAINTERNM_LR, HXO_SHL1, HXO_KVS1, HXO_IRK, HXO_EGL36, HXO_SHK1, HXO_EGL2,
    HXO_CCA1, HXO_EGL19, HXO_UNC2, HXO_LIB_NTYPE
};
typedef struct hxo_lib_table {
    int n;
    const int* node;
    const double* par;
} hxo_lib_table;
typedef struct hxo_lib {
    hxo_lib_table t[HXO_LIB_NTYPE];
} hxo_lib;

typedef struct hxo_group {
    int ncell, nnode;
    const int* parent;            /* -1 for the ncell roots, parent[i] < i otherwise */
    const double *a, *b, *area, *cm;
    double celsius, dt;
    int nhh;
    const int* hh_node;
    const double *hh_gnabar, *hh_gkbar, *hh_gl, *hh_el, *hh_ena, *hh_ek;
    int npas;
    const int* pas_node;
    const double *pas_g, *pas_e;
    int nic;
    const int* ic_node;
    const double *ic_del, *ic_dur, *ic_amp;
    hxo_net* net;
    const hxo_lib* lib;
} hxo_group;

/* Gradient outputs; any pointer may be NULL.  Each array is per instance of its
 * mechanism (cm: per node).  Accumulated with '=' (zeroed first). */
typedef struct hxo_grads {
    double *hh_gnabar, *hh_gkbar, *hh_gl, *hh_el;
    double *pas_g, *pas_e;
    double *cm;
    double *ic_amp;
    double *exp_w, *exp_e, *exp2_w, *exp2_e; /* per ExpSyn / Exp2Syn instance */
    double *hg_g, *gj_g, *gj_w, *gr_w;       /* per HalfGap / gapjunction_lr / graded instance */
    double* gn_w;                            /* per gapjunction_noptr instance */
} hxo_grads;

/* Forward: finitialize(v_init) then nstep fadvance steps.
 * trace: (nstep+1) x nprobe, row 0 = state after finitialize.
 * v_final (nnode), m/h/n_final (nhh): optional final state. */
int hxo_forward(const hxo_group* g, double v_init, int nstep, int nprobe, const int* probe,
                double* trace, double* v_final, double* m_final, double* h_final, double* n_final);

/* Forward that also returns the library states after the last step: for
 * every table t in type order, its instances' states (Ca_HVA, Ca_LVAst,
 * K_Pst, K_Tst, NaTg, Nap_Et2, it2_la, sca_la, Ca: m, h; Im, SKv3_1, kdr_la: m; SK_E2: z;
 * hd_la: l; km_la, kca_la: n; shl1_lr: m, hf, hs; kvs1_lr, shk1_lr: m, h;
 * irk_lr, egl2_lr, kcnl_lr: m; egl36_lr: mf, mm, ms; cca1_lr, egl19_lr, unc2_lr: m, h;
 * ca_ion: cai)
 * appended to lib_final (nlib_final doubles available; -2 if too small). */
int hxo_forward_lib(const hxo_group* g, double v_init, int nstep, int nprobe, const int* probe, double* trace,
                    double* lib_final, int nlib_final);

/* Forward + reverse sweep (groups without library mechanisms; -2 otherwise).  dLdv: (nstep+1) x nprobe, dL/d(trace).  The trace of
 * the forward is written to trace (may be NULL). */
int hxo_adjoint(const hxo_group* g, double v_init, int nstep, int nprobe, const int* probe,
                const double* dLdv, double* trace, hxo_grads* grads);
/* Wall time (s) of the reverse sweep of this thread's last hxo_adjoint call
 * (after its taped forward), for the CPU baseline's timing. */
double hxo_last_reverse_seconds(void);

#ifdef __cplusplus
}
#endif
#endif
