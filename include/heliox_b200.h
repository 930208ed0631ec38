/*
 * heliox_b200.h -- C ABI of the B200-native forward + exact-adjoint library
 * (heliox_b200/libhx_b200.so).
 *
 * Plain C: opaque context, POD arguments, int status codes (0 ok, <0 error,
 * reason in hx_last_error), caller-owned output buffers ("_into" convention of
 * the reference's LearnRuntime, src/runtime_api/learn/LearnRuntime.h:21-293).
 * Pointers are HOST pointers unless the function name ends in "_dev", in which
 * case they are device pointers on the context's device.
 *
 * Which reference interface each entry replaces is given beside it.
 */
#ifndef HELIOX_B200_H
#define HELIOX_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HX_ABI_VERSION 8

typedef struct hx_ctx hx_ctx;

/* One cell group in reference node order: first ncell nodes are roots
 * (parent -1), parent[i] < i otherwise.  Mirrors the arrays HelioXroupData
 * holds after data_format_trans (src/neuron.h:19-130,
 * src/io/coredat_to_innerdat.cpp:569-603).  Mechanism instance tables are
 * sorted by node like the reference's nodeindices. */
/* Library mechanisms: the ions and the user-mech channel set, CoreNEURON
 * types after the network mechanisms in this order (src/mech/eion.cuh,
 * src/mech/user-mech/{CaDynamics_E2,CA_HVA,Ca_LVAst,Im,K_Pst,K_Tst,NaTg,
 * Nap_Et2,SK_E2,SKv3_1,hd_la,km_la,kca_la,it2_la,kdr_la,sca_la,Ca}.cu through MechTemp, src/mech/mech_template.cuh:
 * 589-767).  Each table holds n instances on sorted, distinct reference nodes;
 * par holds the type's columns instance by instance (row-major):
 *   HX_LIB_NA_ION: ena | HX_LIB_K_ION: ek
 *   HX_LIB_CA_ION: cai (initial), cao, eca, nernst (1: eca from cai/cao at
 *                  finitialize and every step, eion.cuh:155-186; 0: fixed eca)
 *   HX_LIB_CADYN (CaDynamics_E2): gamma, decay, depth, minCai
 *   HX_LIB_CA_HVA .. HX_LIB_SKV3_1: gbar (the mechanism's gXbar RANGE)
 *   HX_LIB_NATG: gbar, vshifth, vshiftm, slopeh, slopem
 *   HX_LIB_SK_E2: gbar, zTau (one value: the mechanism's GLOBAL)
 *   HX_LIB_HD_LA (hd_la.cu): ghdbar, vhalfl, tau, then its GLOBALs ehd, kl,
 *                  vhalft, a0t, zetat, gmt, q10, qtl (one value each)
 *   HX_LIB_KM_LA (km_la.cu): gbar (pS/um2), then its GLOBALs Ra, Rb, tha, qa,
 *                  tadj (one value each)
 *   HX_LIB_KCA_LA (kca_la.cu): gbar (pS/um2), then its GLOBALs Ra, Rb, caix,
 *                  tadj
 *   HX_LIB_IT2_LA (it2_la.cu): gcabar, then its GLOBALs vshift, v12m, vwm,
 *                  v12h, vwh, am, ah, vm1, vm2, vh1, vh2, wm1, wm2, wh1, wh2
 *   HX_LIB_KDR_LA (kdr_la.cu): gbar
 *   HX_LIB_SCA_LA (sca_la.cu): gbar (pS/um2), inactF, actF, then its GLOBALs
 *                  vshift, tadj
 *   HX_LIB_CA (Ca.cu): gCabar
 *   HX_LIB_SHL1_LR .. HX_LIB_UNC2_LR (src/mech/worm-lr-mech/<name>.cu): w,
 *                  gb, ek_tmp (eca_tmp for cca1_lr, egl19_lr, unc2_lr, whose
 *                  current enters ica), dv, then the kinetics GLOBALs in the
 *                  mechanism's order (shl1_lr: vhm ka vhh ki atm btm ctm dtm
 *                  etm ftm athf bthf cthf dthf aths bths cths dths; kvs1_lr:
 *                  vhm ka vhh ki atm btm ctm dtm ath bth cth dth; irk_lr: vhm
 *                  ka atm btm ctm dtm etm ftm; egl36_lr: vhm ka atms atmm atmf;
 *                  shk1_lr: vhm ka vhh ki atm btm ctm dtm etm ftm ath; egl2_lr:
 *                  vhm ka atm btm ctm dtm; cca1_lr: vhm ka vhh ki atm btm ctm
 *                  dtm ath bth cth dth; egl19_lr: vhm ka vhh ki vhhb kib ahinf
 *                  bhinf chinf dhinf atm btm ctm dtm etm ftm gtm ath bth cth dth
 *                  eth fth gth hth; unc2_lr: vhm ka vhh ki atm btm ctm dtm etm
 *                  ath bth cth dth eth fth); current w (gb gates (v - ek_tmp)),
 *   HX_LIB_KCNL_LR: w, gbkcnl, dv, then its GLOBALs kca, a, ek_tmp (gate from
 *                  cai); HX_LIB_NCA_LR: w, gbnca, ena_tmp (no gate)
 *                  w the trainable weight
 *   HX_LIB_KQT3_LR (kqt3_lr.cu): w, gbkqt3, ek_tmp (carried, not read: the
 *                  current uses k_ion's ek), dv, then its GLOBALs vhm ka vhw
 *                  kiw aw bw vhs kis as bs atmf btmf ctmf atms btms ctms dtms
 *                  etms ftms gtms atw btw ctw dtw ats
 *   HX_LIB_CAINTERNM_LR (cainternm_lr.cu): vcell, then its GLOBALs f, tca,
 *                  caeq; calcium dynamics (writes cai in the state phase), at
 *                  most one of it and HX_LIB_CADYN per node
 *   HX_LIB_SHL1, HX_LIB_IRK, HX_LIB_EGL36, HX_LIB_SHK1, HX_LIB_EGL2
 *                  (src/mech/worm-mech/<name>.cu): gb (the kinetics are
 *                  hard-coded in the mechanism, erev -80 mV); HX_LIB_KVS1: gb,
 *                  then its GLOBALs vhm ka vhh ki atm btm ctm dtm ath bth cth
 *                  dth; these need k_ion on their node
 *   HX_LIB_CCA1, HX_LIB_EGL19, HX_LIB_UNC2 (src/mech/worm-mech/<name>.cu):
 *                  gb (hard-coded kinetics, erev 60 mV, current into ica);
 *                  they need ca_ion on their node
 * A channel needs its ion on its node (Na: NaTg, Nap_Et2; K: Im, K_Pst,
 * K_Tst, SK_E2, SKv3_1, km_la, kca_la, kdr_la; Ca: CaDynamics_E2, Ca_HVA,
 * Ca_LVAst, it2_la, sca_la, Ca, SK_E2 and kca_la (cai)); the worm-lr
 * channels need k_ion (ca_ion for cca1_lr, egl19_lr, unc2_lr) on their node
 * (the reference maps their ion current) but use their own ek_tmp / eca_tmp; hd_la's current is nonspecific
 * (its own ehd);
 * na_ion / k_ion on an hh node carry hh's ena / ek. */
enum hx_lib_type {
    HX_LIB_NA_ION = 0,
    HX_LIB_K_ION = 1,
    HX_LIB_CA_ION = 2,
    HX_LIB_CADYN = 3,
    HX_LIB_CA_HVA = 4,
    HX_LIB_CA_LVAST = 5,
    HX_LIB_IM = 6,
    HX_LIB_K_PST = 7,
    HX_LIB_K_TST = 8,
    HX_LIB_NATG = 9,
    HX_LIB_NAP_ET2 = 10,
    HX_LIB_SK_E2 = 11,
    HX_LIB_SKV3_1 = 12,
    HX_LIB_HD_LA = 13,
    HX_LIB_KM_LA = 14,
    HX_LIB_KCA_LA = 15,
    HX_LIB_IT2_LA = 16,
    HX_LIB_KDR_LA = 17,
    HX_LIB_SCA_LA = 18,
    HX_LIB_CA = 19,
    HX_LIB_SHL1_LR = 20,
    HX_LIB_KVS1_LR = 21,
    HX_LIB_IRK_LR = 22,
    HX_LIB_EGL36_LR = 23,
    HX_LIB_SHK1_LR = 24,
    HX_LIB_EGL2_LR = 25,
    HX_LIB_CCA1_LR = 26,
    HX_LIB_EGL19_LR = 27,
    HX_LIB_UNC2_LR = 28,
    HX_LIB_KCNL_LR = 29,
    HX_LIB_NCA_LR = 30,
    HX_LIB_KQT3_LR = 31,
    HX_LIB_CAINTERNM_LR = 32,
    HX_LIB_SHL1 = 33,
    HX_LIB_KVS1 = 34,
    HX_LIB_IRK = 35,
    HX_LIB_EGL36 = 36,
    HX_LIB_SHK1 = 37,
    HX_LIB_EGL2 = 38,
    HX_LIB_CCA1 = 39,
    HX_LIB_EGL19 = 40,
    HX_LIB_UNC2 = 41,
    HX_LIB_NTYPE = 42
};
typedef struct hx_lib_table {
    int n;
    const int* node;
    const double* par;
} hx_lib_table;
typedef struct hx_lib_desc {
    hx_lib_table t[HX_LIB_NTYPE];
} hx_lib_desc;

typedef struct hx_group_desc {
    int ncell, nnode;
    const int* parent;
    const double *a, *b, *area, *cm;
    double celsius, dt;
    /* hh (src/mech/user-mech/hh_templated.cu) */
    int nhh;
    const int* hh_node;
    const double *hh_gnabar, *hh_gkbar, *hh_gl, *hh_el, *hh_ena, *hh_ek;
    /* pas (src/mech/user-mech/pas_templated.cu) */
    int npas;
    const int* pas_node;
    const double *pas_g, *pas_e;
    /* IClamp (src/mech/user-mech/iclamp_templated.cu) */
    int nic;
    const int* ic_node;
    const double *ic_del, *ic_dur, *ic_amp;

    /* ---- network (all counts may be 0; the pointers are then ignored) ----
     * Spike sources are global ids: gid_base + local cell (this group's
     * cells' PreSyns, threshold detection at the cell's root node,
     * src/spike/presyn.cpp:133-177), 0..nsrc_cells-1 over all groups of a
     * multi-GPU job, then nsrc_cells + j for NetStim j.  Every ExpSyn /
     * Exp2Syn instance is the target of exactly one NetCon (src, delay ms,
     * weight uS): the per-instance spk_vec_idx / delay / weights the
     * reference fills in initSynapse (src/io/coredat_to_innerdat.cpp:348-376). */
    int gid_base, nsrc_cells;       /* 0, 0 = this group alone (nsrc_cells = ncell) */
    const double* ps_thresh;        /* ncell thresholds (mV); NULL = 10 mV */
    /* ExpSyn (src/spike/postsyn_mech/expsyn.cpp) */
    int nexpsyn;
    const int *expsyn_node, *expsyn_src;
    const double *expsyn_tau, *expsyn_e, *expsyn_delay, *expsyn_weight;
    /* Exp2Syn (src/spike/user_postsyn_mech/exp2syn_temp.cuh) */
    int nexp2syn;
    const int *exp2syn_node, *exp2syn_src;
    const double *exp2syn_tau1, *exp2syn_tau2, *exp2syn_e, *exp2syn_delay, *exp2syn_weight;
    /* NetStim (src/spike/netstim.cpp): the same table on every rank */
    int nnetstim;
    const double *ns_interval, *ns_number, *ns_start, *ns_noise;
    int netstim_rng; /* 0: the reference's CPU-mode stream (zeroed state), 1: GPU mode (sequence 0) */
    /* HalfGap (src/mech/user-mech/HalfGap.cu): vgap follows v of node hg_src */
    int nhalfgap;
    const int *hg_node, *hg_src;
    const double* hg_g;
    /* gapjunction_lr (src/mech/worm-lr-mech/gapjunction_lr.cu): vpre = v of node gj_pre */
    int ngapj;
    const int *gj_node, *gj_pre;
    const double *gj_g, *gj_w;
    /* gapjunction_noptr (src/mech/worm-mech/gapjunction_noptr.cu:33-36):
     * i = weight (v - vpre), vpre copied from v of node gn_src by the
     * reference's gap transfer (simulate.cpp:953-966) */
    int ngapnp;
    const int *gn_node, *gn_src;
    const double* gn_weight;
    /* neuron_to_neuron_syn_lr (src/mech/worm-lr-mech/neuron_to_neuron_syn_lr.cu) */
    int ngraded;
    const int *gr_node, *gr_pre;
    const double *gr_w, *gr_delta, *gr_vth;

    /* ---- library mechanisms (NULL = none; not on a cell split across CTAs;
     * with network parts their currents follow the network mechanisms') */
    const hx_lib_desc* lib;
} hx_group_desc;

/* Parameter / gradient kinds (per mechanism instance; HX_P_CM per node). */
enum hx_param_kind {
    HX_P_HH_GNABAR = 0,
    HX_P_HH_GKBAR = 1,
    HX_P_HH_GL = 2,
    HX_P_HH_EL = 3,
    HX_P_PAS_G = 4,
    HX_P_PAS_E = 5,
    HX_P_CM = 6,
    HX_P_IC_AMP = 7,
    HX_P_EXPSYN_W = 8,    /* NetCon weight into ExpSyn instance i */
    HX_P_EXPSYN_E = 9,
    HX_P_EXP2SYN_W = 10,  /* NetCon weight into Exp2Syn instance i */
    HX_P_EXP2SYN_E = 11,
    HX_P_HALFGAP_G = 12,
    HX_P_GAPJ_G = 13,
    HX_P_GAPJ_W = 14,
    HX_P_GRADED_W = 15,
    /* library mechanisms: per instance of the table, reference order */
    HX_P_CADYN_GAMMA = 16,
    HX_P_CADYN_DECAY = 17,
    HX_P_CADYN_DEPTH = 18,
    HX_P_CADYN_MINCAI = 19,
    HX_P_CA_HVA_G = 20,
    HX_P_CA_LVAST_G = 21,
    HX_P_IM_G = 22,
    HX_P_K_PST_G = 23,
    HX_P_K_TST_G = 24,
    HX_P_NATG_G = 25,
    HX_P_NAP_ET2_G = 26,
    HX_P_SK_E2_G = 27,
    HX_P_SKV3_1_G = 28,
    HX_P_HD_LA_G = 29,
    HX_P_KM_LA_G = 30,
    HX_P_KCA_LA_G = 31,
    HX_P_IT2_LA_G = 32,
    HX_P_KDR_LA_G = 33,
    HX_P_SCA_LA_G = 34,
    HX_P_CA_G = 35,
    HX_P_SHL1_LR_W = 36, /* worm-lr: the weight w per instance */
    HX_P_KVS1_LR_W = 37,
    HX_P_IRK_LR_W = 38,
    HX_P_EGL36_LR_W = 39,
    HX_P_SHK1_LR_W = 40,
    HX_P_EGL2_LR_W = 41,
    HX_P_CCA1_LR_W = 42,
    HX_P_EGL19_LR_W = 43,
    HX_P_UNC2_LR_W = 44,
    HX_P_KCNL_LR_W = 45,
    HX_P_NCA_LR_W = 46,
    HX_P_KQT3_LR_W = 47,
    HX_P_CAINTERNM_LR_VCELL = 48, /* cainternm_lr: vcell per instance */
    HX_P_SHL1_G = 49,             /* worm-mech: gb per instance */
    HX_P_KVS1_G = 50,
    HX_P_IRK_G = 51,
    HX_P_EGL36_G = 52,
    HX_P_SHK1_G = 53,
    HX_P_EGL2_G = 54,
    HX_P_CCA1_G = 55,
    HX_P_EGL19_G = 56,
    HX_P_UNC2_G = 57,
    HX_P_GAPNP_W = 58, /* gapjunction_noptr weight per instance */
    HX_P_COUNT = 59
};

/* Statistics of the execution plan built at load time. */
typedef struct hx_plan_stats {
    int npack;            /* CTAs (cell packs of 8 warps) */
    int max_pack_nodes;   /* largest pack */
    int max_pack_hh;
    int max_levels;       /* branch levels of the deepest pack */
    int max_crit_nodes;   /* longest root->leaf chain (nodes) of any pack */
    int nbranch;          /* branches over all packs */
    double imbalance;     /* max pack nodes / mean pack nodes */
    size_t smem_fwd, smem_bwd; /* dynamic shared memory per CTA (bytes) */
    int nsub;             /* subtrees of a cell split across CTAs (0: no split) */
    double est_max;       /* modelled cycles of a forward + backward step: slowest CTA */
    double est_mean;      /* the same, mean over CTAs */
} hx_plan_stats;

/* ---- context ------------------------------------------------------------ */
/* Replaces SimRuntimeCore construction + Simulate(mode=GPU)
 * (src/runtime_api/core/SimRuntimeCore.h:24-219, src/simulate.h:17-80). */
int hx_create(hx_ctx** out, int device);
int hx_destroy(hx_ctx* ctx);
const char* hx_last_error(hx_ctx* ctx);
int hx_abi_version(void);
/* Launch on this CUDA stream (cudaStream_t passed as void*); NULL = the context's own stream. */
int hx_set_stream(hx_ctx* ctx, void* stream);
/* CTA layout.  0 (default): one 16-warp CTA per SM and as few waves as the
 * shared memory allows, cells dealt to CTAs by a step-time model and warps
 * given to the slowest cell of each CTA.  > 0: target cell nodes per warp;
 * cells are packed first-fit into CTAs of 16 x that many nodes.  Must be
 * called before hx_load_group. */
int hx_set_pack_target(hx_ctx* ctx, int nodes_per_warp);
/* Upper bound on device bytes the forward tape may use; when the full tape
 * does not fit, the backward recomputes checkpointed segments.  0 = default
 * (60% of free device memory at load time). */
int hx_set_tape_budget(hx_ctx* ctx, size_t bytes);
/* How long a grid-barrier wait lasts before it gives up -- the split-cell
 * kernels (a cell larger than one CTA) and the grid-synchronous launches of
 * coupled networks: `sleeps` waits of ~100 ns (0 = default, 20,000,000:
 * ~2 s).  A wait that gives up sets an error flag, later barriers return at
 * once, the launch finishes, and the forward or backward returns -1 with "a
 * grid barrier of the ... kernels timed out"; the context stays usable.
 * Takes effect at the next launch.  (The reference's intra-cell parallel
 * solvers synchronise inside one kernel, simulate.cu:119-189; this bounds the
 * cross-CTA form.) */
int hx_set_split_barrier_limit(hx_ctx* ctx, long long sleeps);
/* The parameter kinds whose gradients the next backward passes accumulate
 * (n <= 0: all kinds, the default).  The reverse sweep then neither reads nor
 * writes the accumulators of the other cell and network kinds (library kinds
 * are always accumulated), and their gradients read as zero -- through
 * hx_backward, hx_reduce_grads_f32 or an optimizer alike.  Persists until
 * changed.  (The reference's replay computes only the requested handles'
 * columns, LearnRuntime.h:72-100.) */
int hx_set_grad_kinds(hx_ctx* ctx, const int* kinds, int n);
/* Groups coupled by gap junctions or graded synapses exchange voltages every
 * step.  enable = 1 (default): when every cell pack can be co-resident, a
 * launch runs a whole window of steps with one grid barrier per step
 * (cooperative launch); 0: one launch per step.  Results are identical.
 * (Replaces the per-step gap transfer of simulate.cpp:953-966 between
 * mechanism launches.) */
int hx_set_grid_sync(hx_ctx* ctx, int enable);

/* ---- model ---------------------------------------------------------------- */
/* Replaces SimRuntimeCore::load_model -> read_coredat -> data_format_trans
 * (src/runtime_api/core/SimRuntimeCore.cpp:109-147). */
int hx_load_group(hx_ctx* ctx, const hx_group_desc* desc);
int hx_get_plan_stats(hx_ctx* ctx, hx_plan_stats* out);
/* Build the execution plan on the host only (no device needed): validates the
 * group, reports statistics and checks, on the CPU, the planned branch
 * schedule against solve_serial (src/simulate.cpp:558-581) on seeded
 * diagonally dominant systems, forward and transposed.  *max_abs_diff: largest
 * difference of the schedule replayed in the reference's division form (0 when
 * bit-exact).  *pq_rel_diff: largest difference, relative to max |x|, of the
 * forms the kernels use (projective chains; reduced tree of segments). */
int hx_plan_check(const hx_group_desc* desc, int nodes_per_warp, hx_plan_stats* out, double* max_abs_diff,
                  double* pq_rel_diff);
/* The same with a per-CTA node capacity (0 = unlimited): a group of one cell
 * larger than the capacity is split into a top part and subtrees, one CTA
 * each, as hx_load_group does when a cell exceeds a CTA's shared memory. */
int hx_plan_check_cap(const hx_group_desc* desc, int nodes_per_warp, int max_pack_nodes, hx_plan_stats* out,
                      double* max_abs_diff, double* pq_rel_diff);
/* The same for a device of nsm SMs: with nodes_per_warp = 0 the CTAs are
 * balanced over whole waves of nsm CTAs, as hx_load_group plans them. */
int hx_plan_check_sm(const hx_group_desc* desc, int nodes_per_warp, int max_pack_nodes, int nsm, hx_plan_stats* out,
                     double* max_abs_diff, double* pq_rel_diff);

/* Parameter access in reference instance order (replaces the handle-based
 * Sim.set/get_variable path, src/python_api/PyBindings.cpp:80-81). */
int hx_set_param(hx_ctx* ctx, int kind, const double* values, int n);
int hx_get_param(hx_ctx* ctx, int kind, double* values, int n);

/* ---- forward ------------------------------------------------------------------ */
/* finitialize(v_init) + nstep fixed steps, recording v at nprobe reference
 * nodes into trace ((nstep+1) x nprobe, row 0 = initial state).  No tape.
 * Replaces Simulate::finitialize + Simulate::run (src/simulate.cpp:106-141,
 * 343-371) and LearnRuntime::simulate_output_vs_into. */
int hx_simulate(hx_ctx* ctx, int nstep, double v_init, int nprobe, const int* probe_nodes, double* trace);
/* Same, but also records the forward tape (or its checkpoints) for hx_backward.
 * Replaces LearnRuntime::simulate_and_capture_mapped_signals_cached
 * (src/runtime_api/learn/LearnRuntime.cpp:1619-1985). */
int hx_forward_capture(hx_ctx* ctx, int nstep, double v_init, int nprobe, const int* probe_nodes, double* trace);
int hx_forward_capture_dev(hx_ctx* ctx, int nstep, double v_init, int nprobe, const int* probe_nodes,
                           double* trace_dev);

/* ---- network ------------------------------------------------------------------ */
/* Spikes of this group's PreSyns detected by the last forward, in detection
 * order: global source gid and time (ms).  *n receives the total count (which
 * may exceed cap).  Replaces Simulate::output_spikes / rec_spikes
 * (src/simulate.cpp:881-899). */
int hx_get_spikes(hx_ctx* ctx, int cap, int* gid, double* t, int* n);
/* Multi-GPU spike exchange.  A group whose NetCons name sources of other
 * groups (nsrc_cells > ncell) advances in windows no longer than the smallest
 * NetCon delay; after every window the library calls
 *   exchange(user, send_dev, recv_dev, cap_entries, stream)
 * where send_dev holds this group's window spikes as cap_entries int pairs
 * (global source gid, step) padded with (-1, -1), and recv_dev (nranks x
 * cap_entries pairs) must receive every rank's send buffer (an all-gather on
 * `stream`, e.g. ncclAllGather) before the callback returns.  All ranks must
 * use the same window (hx_set_window) and call the forward together.  The
 * reference exchanges through its host spike queue
 * (Simulate::network_spike_send_cpu / network_spike_receive_cpu,
 * src/simulate.cpp:858-951). */
/* NetStim spike trains of a group over finitialize + nstep steps, computed on
 * the host (no device needed): NetStim instance and the step at whose start
 * it fires (0 for the delivery at finitialize), in emission order.  *n gets
 * the total count (may exceed cap).  These are the artificial-cell events of
 * the reference's NetStim (src/spike/netstim.cpp:207-330). */
int hx_netstim_trains(const hx_group_desc* desc, int nstep, int cap, int* id, int* step, int* n);
typedef int (*hx_exchange_fn)(void* user, const void* send_dev, void* recv_dev, int cap_entries, void* stream);
/* cap_entries: the window buffer size every rank starts with (identical on
 * every rank; 0 = 1024 entries).  Most windows carry far fewer spikes than
 * the bound (cells) * ceil(window / 2) (a PreSyn fires at most every other
 * step), so the buffer stays small; a window that overflows it on any rank
 * makes every rank rerun the forward with the agreed larger size, which is
 * kept for later forwards.  The hook is called once per window with the
 * current cap_entries and, after the last window, once more with
 * cap_entries = 2: every rank's status -- (HX_XS_* bits, largest event-bucket
 * count), (largest window spike count, 0) -- is all-gathered, so that all
 * ranks return the same outcome (a rank whose host work failed keeps
 * exchanging empty windows until then and reports HX_XS_ABORT; a bucket or
 * window overflow on any rank reruns the forward on every rank).  A hook that
 * returns nonzero ends the forward on that rank at once; its peers' next
 * collective then ends by the process group's timeout. */
int hx_set_exchange(hx_ctx* ctx, hx_exchange_fn exchange, void* user, int nranks, int cap_entries);
/* Status bits of a rank after the last window of a multi-rank forward. */
#define HX_XS_LATE_EVENT 1 /* an event fell inside an already simulated window */
#define HX_XS_BUCKET 2     /* a per-step event bucket overflowed (the forward is rerun) */
#define HX_XS_WINDOW 4     /* the window spike buffer overflowed (the forward is rerun) */
#define HX_XS_ABORT 8      /* the rank's host work failed; it only kept exchanging */
/* Merge of the gathered status (4 ints per rank r: status[4 r] bits,
 * status[4 r + 1] bucket need, status[4 r + 2] window need, status[4 r + 3]
 * unused): *flags = OR of the bits, *need and *win_need = the largest needs,
 * *first_rank = the lowest rank with a bit other than the overflow bits set
 * (else the lowest with an overflow bit, else -1).  Host only; the rule every
 * rank applies, exposed for hosts that drive their own exchange. */
int hx_exchange_merge_status(const int* status, int nranks, int* flags, int* need, int* win_need, int* first_rank);
/* Steps per forward window of an event network (0 = derived from the smallest
 * NetCon delay of this group); returns the effective value with hx_get_window. */
int hx_set_window(hx_ctx* ctx, int steps);
int hx_get_window(hx_ctx* ctx, int* steps);

/* ---- backward ------------------------------------------------------------------ */
/* Exact discrete adjoint of the captured forward.  dLdv: (nstep+1) x nprobe,
 * dL/d(trace).  grads[kind] (may be NULL per kind) receives dL/d(param) in
 * reference instance order.  Replaces LearnRuntime::
 * replay_compute_dw_dx_from_cached_signals_into (LearnRuntime.cpp:1986-2297),
 * whose LRDS approximation it supersedes. */
int hx_backward(hx_ctx* ctx, const double* dLdv, double* const* grads);
int hx_backward_dev(hx_ctx* ctx, const double* dLdv_dev, double* const* grads_dev);

/* Column reduction of per-instance gradients ("MappedSignal" gather +
 * scatter-add, src/runtime_api/core/kernels/batch_scatter_add.cu:4-27):
 * out[dest[j]] += scale[j] * grad(kind[j], index[j]); out has n_out floats,
 * zeroed first.  Must follow hx_backward*. */
int hx_reduce_grads_f32(hx_ctx* ctx, int n, const int* kind, const int* index, const int32_t* dest,
                        const float* scale, float* out, int n_out);

/* One-call exact-adjoint counterpart of LearnRuntime::
 * simulate_and_replay_dw_dx_streaming_into (src/runtime_api/learn/
 * LearnRuntime.h:72-100): a forward of nstep steps from v_init recording the
 * n_output probe nodes poutput, the exact adjoint of dL/d(probe trace) given
 * by dLtdv (float32, nstep x n_output; row t is step t+1, the initial state
 * carries no loss), then dw_out_n[dest[j]] += scale[j] * dL/d(param j) for the
 * n_param handles (kind, index) -- the reference's pure_i / didv / didvpre
 * handle lists passed as one list -- times grad_scale (dw_out_n, N floats,
 * zeroed first).  With clip_strategy != 0, dw_out_n is scaled down to L2 norm
 * grad_l2norm_threshold when above it (the exact adjoint needs no clipping
 * inside the sweep; the reference clips its LRDS sensitivities there).  The
 * LRDS-only knobs (k_mul, percise, eps, clip_check_every) have no counterpart;
 * input gradients are not produced: dx must be NULL. */
int hx_simulate_and_adjoint_into(hx_ctx* ctx, const float* dLtdv, int nstep, int n_output, const int32_t* poutput,
                                 int N, float* dw_out_n, float* dx, int n_param, const int* kind, const int* index,
                                 const int32_t* dest, const float* scale, double v_init, double grad_scale,
                                 double grad_l2norm_threshold, int clip_strategy);

/* ---- optimizer ---------------------------------------------------------------------- */
/* Adam over parameter instances, updating the device parameters in place.
 * Mirrors Simulate::create_optimizer / configure_optimizer /
 * optimizer_step_with_inv_record_steps (src/simulate.cpp:1102-1280) and the
 * external-gradient binding of SimWrapper (src/python_api/SimWrapper.cpp:
 * 284-451): one slot per parameter, g = grad * impedance * inv_record_steps,
 * bias-corrected moments (AdamOptimizer::step_cpu, src/optimizer/optimizer.cpp:
 * 351-397), gradients zeroed after each step.  Returns an optimizer id >= 0. */
int hx_opt_create_adam(hx_ctx* ctx, double beta1, double beta2, double eps);
/* Binds n parameter instances (kind, reference index), replacing any previous binding. */
int hx_opt_add_params(hx_ctx* ctx, int opt, int n, const int* kind, const int* index, double impedance);
/* Host float32 gradients for the bound slots (optimizer_set_external_grads_f32). */
int hx_opt_set_grads_f32(hx_ctx* ctx, int opt, const float* grads, int n);
/* Device: slot gradients := the last backward's gradients of the bound instances times scale. */
int hx_opt_grads_from_backward(hx_ctx* ctx, int opt, double scale);
/* Device pointer and length of the slot gradients (e.g. for an all-reduce before hx_opt_step). */
int hx_opt_grad_buffer(hx_ctx* ctx, int opt, double** dev_ptr, int* n);
/* Data-parallel replicas (e.g. one trial or teacher per GPU): hx_opt_step
 * first calls allreduce(user, grad_dev, n, stream), which must replace the n
 * fp64 slot gradients at grad_dev by their sum over all ranks (an in-place
 * ncclAllReduce on `stream`) before it returns; then every rank applies the
 * same Adam update.  NULL removes the hook.  The reference has one process
 * and no collective; its Adam (src/optimizer/optimizer.cpp:351-397) receives
 * the summed gradient here. */
typedef int (*hx_allreduce_fn)(void* user, double* grad_dev, int n, void* stream);
int hx_opt_set_allreduce(hx_ctx* ctx, int opt, hx_allreduce_fn fn, void* user);
int hx_opt_step(hx_ctx* ctx, int opt, double lr, double inv_record_steps);
/* hyper3 = {beta1, beta2, eps}; optimizer_get/set_adam_state (SimWrapper.cpp:419-451). */
int hx_opt_get_adam_state(hx_ctx* ctx, int opt, long long* step, double* m, double* v, int n, double* hyper3);
int hx_opt_set_adam_state(hx_ctx* ctx, int opt, long long step, const double* m, const double* v, int n,
                          const double* hyper3);
int hx_opt_reset(hx_ctx* ctx, int opt);

/* ---- objective -------------------------------------------------------------------- */
/* Mean squared error of a probe trace against a target trace ((nrow x ncol),
 * rows 1..nrow-1 count; row 0 is the initial state) and its gradient
 * dLdv = 2 (trace - target) / ((nrow-1) ncol), row 0 = 0.  All device pointers;
 * *loss_dev receives the loss.  Deterministic reduction.  The device-side
 * counterpart of the Python objectives the reference's trainer evaluates
 * (python_lib/heliox_learn/objective.py:15-30). */
int hx_mse_loss_grad_dev(hx_ctx* ctx, const double* trace_dev, const double* target_dev, int nrow, int ncol,
                         double* dLdv_dev, double* loss_dev);

/* The same loss and gradient as hx_mse_loss_grad_dev for callers that cannot
 * let the library allocate device memory (a host that owns every device byte
 * through its own pool, or a loop that must not meet cudaFree's implicit
 * synchronisation).  No context and no allocation: the per-chunk partial sums
 * live in a static device array of 4,096 doubles (32 KiB per device, held until
 * the process exits), so nrow*ncol may be at most 4,096 * 65,536 = 2^28
 * elements; larger inputs return -2 (with a message on stderr) and do no work.
 * Work is enqueued on `stream` (NULL = the legacy default stream) of the
 * current device.  Every call made outside stream capture resolves the
 * scratch array's device address (so a cudaDeviceReset in between is
 * harmless); a call during capture reuses the last one, so make the first
 * call on a device before any stream capture.  All calls on a device share
 * the array: calls that overlap on the GPU race.  Returns 0, -1 bad argument,
 * -2 size beyond the maximum, -3 CUDA error of this call's launches, -4 an
 * earlier CUDA error is pending (left for the caller, no work done).  It has
 * no counterpart in the reference. */
int hx_mse_loss_grad_noalloc(const double* trace_dev, const double* target_dev, int nrow, int ncol, double* dLdv_dev,
                             double* loss_dev, void* stream);

/* ---- verification -------------------------------------------------------------- */
/* y[i] = the reciprocal the step kernels use in place of IEEE division in the
 * mechanism rate functions (hardware estimate + two Newton-Raphson steps), for
 * device arrays of n doubles on the current device; work on `stream`.  Its
 * domain is normal |x| whose reciprocal is normal (about 2^-1022 .. 2^1022);
 * subnormal inputs flush to zero.  Returns 0, -1 bad argument, -3 CUDA error.
 * No reference counterpart (the reference divides). */
int hx_rcp_nz_dev(const double* x_dev, double* y_dev, int n, void* stream);

/* ---- timing (CUDA events on the launch stream) ---------------------------------- */
/* Milliseconds of the last forward-capture / backward kernel work, measured with
 * events recorded around the launches.  which: 0 forward, 1 backward (with the
 * recompute of checkpointed segments), 2 the reverse kernel's launches alone
 * (summed; *launches = their count). */
int hx_last_kernel_ms(hx_ctx* ctx, int which, double* ms, int* launches);

#ifdef __cplusplus
}
#endif
#endif
