/*
 * hx_oracle.c -- TEST INFRASTRUCTURE ONLY (see hx_oracle.h).
 *
 * Restates, in plain C compiled with -ffp-contract=off like the reference's CPU
 * build (CMakeLists.txt:26-31), the reference's fixed-step integrator:
 *   Simulate::fadvance_cpu            src/simulate.cpp:410-442
 *   setup_tree_matrix_cpu             src/simulate.cpp:455-556
 *   solve_serial (permute type 0)     src/simulate.cpp:558-581
 *   update_cpu                        src/simulate.cpp:759-770
 *   last_part_cpu / nonvint_cpu       src/simulate.cpp:772-852
 *   MechTemp::current_cpu (FD g)      src/mech/mech_template.cuh:589-648
 *   hh                                src/mech/user-mech/hh_templated.cu:76-164
 *   pas                               src/mech/user-mech/pas_templated.cu:27-31
 *   IClamp                            src/mech/user-mech/iclamp_templated.cu:29-40
 *   capacitance                       src/mech/build-in-mech/capac.cpp:54-78
 *   ExpSyn                            src/spike/postsyn_mech/expsyn.cpp:80-150
 *   Exp2Syn                           src/spike/user_postsyn_mech/exp2syn_temp.cuh:29-67
 *   spike detection / delivery        presyn.cpp:133-177, postsyn.cpp:43-114,
 *                                     simulate.cpp:445-449, 858-951, spike.h:113-136
 *   NetStim                           src/spike/netstim.cpp:120-330 (Random123
 *                                     Philox4x32-10 stream, utils/nrnran123.cpp)
 *   HalfGap + gap transfer            src/mech/user-mech/HalfGap.cu:56-68,
 *                                     simulate.cpp:953-966
 *   gapjunction_lr                    src/mech/worm-lr-mech/gapjunction_lr.cu:58-65
 *   gapjunction_noptr (gap transfer)  src/mech/worm-mech/gapjunction_noptr.cu:33-36
 *   neuron_to_neuron_syn_lr           src/mech/worm-lr-mech/neuron_to_neuron_syn_lr.cu:97-145
 * and the discrete adjoint of that step sequence (no reference counterpart).
 * The adjoint holds the spike/event schedule of the forward fixed (events are
 * discrete; their times do not move under an infinitesimal parameter change
 * that crosses no threshold).
 */
#define _POSIX_C_SOURCE 199309L /* clock_gettime under -std=c11 */
#include "hx_oracle.h"
#include "hx_oracle_lib.h"

#include <math.h>
#include <stdint.h>
#include <time.h>
#include <stdlib.h>
#include <string.h>

#define FD_EPS 0.001 /* mech_template.cuh:616,626 */

/* ---------------------------------------------------------------- hh */
/* hh_templated.cu:76-85 */
static double vtrap(double x, double y) {
    if (fabs(x / y) < 1e-6) return y * (1 - x / y / 2);
    return x / (exp(x / y) - 1);
}
/* d vtrap / dx, derivative of the branch vtrap() takes.  Near the removable
 * singularity (1e-6 <= |u| < 0.05, u = x/y) the numerator exp(u) - 1 - u exp(u)
 * is taken from its series -sum_{n>=2} (n-1) u^n / n! and the denominator from
 * expm1: the direct difference loses ~1e-16/u^2 of it to cancellation. */
static double dvtrap(double x, double y) {
    double u = x / y;
    if (fabs(u) < 1e-6) return -0.5;
    if (fabs(u) < 0.05) {
        static const double c[10] = {1.0 / 2, 2.0 / 6, 3.0 / 24, 4.0 / 120, 5.0 / 720, 6.0 / 5040,
                                     7.0 / 40320, 8.0 / 362880, 9.0 / 3628800, 10.0 / 39916800};
        double t = c[9];
        for (int n = 8; n >= 0; n--) t = t * u + c[n];
        double em1 = expm1(u);
        return -(u * u) * t / (em1 * em1);
    }
    double e = exp(u);
    double em1 = e - 1;
    return (em1 - u * e) / (em1 * em1);
}

typedef struct {
    double minf, mtau, hinf, htau, ninf, ntau;
} hh_rates_t;

/* hh_templated.cu:87-109 (same expression order) */
static void hh_rates(double v, double celsius, hh_rates_t* r) {
    double q10, alpha, beta, sum;
    q10 = pow(3.0, (celsius - 6.3) / 10);
    alpha = 0.1 * vtrap(-(v + 40), 10);
    beta = 4 * exp(-(v + 65) / 18);
    sum = alpha + beta;
    r->mtau = 1.0 / (q10 * sum);
    r->minf = alpha / sum;
    alpha = 0.07 * exp(-(v + 65) / 20);
    beta = 1.0 / (exp(-(v + 35) / 10) + 1);
    sum = alpha + beta;
    r->htau = 1.0 / (q10 * sum);
    r->hinf = alpha / sum;
    alpha = 0.01 * vtrap(-(v + 55), 10);
    beta = 0.125 * exp(-(v + 65) / 80);
    sum = alpha + beta;
    r->ntau = 1.0 / (q10 * sum);
    r->ninf = alpha / sum;
}

/* hh_templated.cu:125-135 */
static double hh_current(double v, double gnabar, double gkbar, double gl, double m, double h, double n,
                         double ena, double ek, double el, double* gna_o, double* gk_o) {
    double gna = gnabar * m * m * m * h;
    double ina = gna * (v - ena);
    double gk = gkbar * n * n * n * n;
    double ik = gk * (v - ek);
    double il = gl * (v - el);
    if (gna_o) *gna_o = gna;
    if (gk_o) *gk_o = gk;
    return ina + ik + il;
}

/* one cnexp gate update, hh_templated.cu:161-163 */
static double gate_step(double x, double inf, double tau, double dt) {
    return x + (1.0 - exp(dt * (-1.0 / tau))) * ((inf / tau) / (1.0 / tau) - x);
}

/* Derivatives needed by the state VJP: for each gate, with s = alpha+beta,
 * inf = alpha/s, tau = 1/(q10 s):  d inf/dv and d s/dv. */
typedef struct {
    double dinf[3], ds[3], q10;
} hh_drates_t;

static void hh_drates(double v, double celsius, hh_drates_t* d) {
    double q10 = pow(3.0, (celsius - 6.3) / 10);
    double al, be, dal, dbe, s;
    /* m */
    al = 0.1 * vtrap(-(v + 40), 10);
    dal = -0.1 * dvtrap(-(v + 40), 10);
    be = 4 * exp(-(v + 65) / 18);
    dbe = -be / 18;
    s = al + be;
    d->dinf[0] = (dal * be - al * dbe) / (s * s);
    d->ds[0] = dal + dbe;
    /* h */
    al = 0.07 * exp(-(v + 65) / 20);
    dal = -al / 20;
    {
        double u = exp(-(v + 35) / 10);
        be = 1.0 / (u + 1);
        dbe = u / (10 * (u + 1) * (u + 1));
    }
    s = al + be;
    d->dinf[1] = (dal * be - al * dbe) / (s * s);
    d->ds[1] = dal + dbe;
    /* n */
    al = 0.01 * vtrap(-(v + 55), 10);
    dal = -0.01 * dvtrap(-(v + 55), 10);
    be = 0.125 * exp(-(v + 65) / 80);
    dbe = -be / 80;
    s = al + be;
    d->dinf[2] = (dal * be - al * dbe) / (s * s);
    d->ds[2] = dal + dbe;
    d->q10 = q10;
}

/* ---------------------------------------------------------------- Random123 */
/* Philox4x32-10 (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as easy
 * as 1, 2, 3", SC11): ten rounds of two 32x32->64 multiplications, the key
 * bumped by the Weyl constants between rounds.  The reference draws NetStim
 * intervals from it through nrnran123 (utils/nrnran123.cpp:108-140): a
 * counter c, the current block r = philox(c, key 0) and a word selector. */
static void philox4x32_10(const uint32_t in[4], uint32_t out[4]) {
    uint32_t c0 = in[0], c1 = in[1], c2 = in[2], c3 = in[3];
    uint32_t k0 = 0, k1 = 0;
    for (int r = 0; r < 10; r++) {
        if (r) {
            k0 += 0x9E3779B9u;
            k1 += 0xBB67AE85u;
        }
        uint64_t p0 = (uint64_t)0xD2511F53u * c0;
        uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
        uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
        uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
        c0 = n0;
        c1 = (uint32_t)p1;
        c2 = n2;
        c3 = (uint32_t)p0;
    }
    out[0] = c0;
    out[1] = c1;
    out[2] = c2;
    out[3] = c3;
}

typedef struct {
    uint32_t c[4], r[4];
    int which;
} ran123;

static void ran123_init(ran123* s, int mode) {
    memset(s, 0, sizeof(*s));
    /* mode 0: the state NetStim allocates (value-initialised: all zero, so
     * the first block is never computed, netstim.cpp:88); mode 1: the GPU
     * path's set_seed(0) -> nrnran123_setseq(s, 0) (netstim.cpp:243). */
    if (mode == 1) philox4x32_10(s->c, s->r);
}

static uint32_t ran123_ipick(ran123* s) {
    uint32_t v = s->r[s->which++];
    if (s->which > 3) {
        s->which = 0;
        for (int i = 0; i < 4; i++)
            if (++s->c[i]) break;
        philox4x32_10(s->c, s->r);
    }
    return v;
}

static double ran123_negexp(ran123* s) {
    static const double SHIFT32 = 1.0 / 4294967297.0; /* nrnran123.cpp:122 */
    double u = ((double)ran123_ipick(s) + 1.0) * SHIFT32;
    return -log(u);
}

/* ---------------------------------------------------------------- state */
enum { SPK_INVALID = -1, SPK_NORMAL = 0, SPK_SELF = 1, SPK_INIT = 2 };

typedef struct {
    double t;
    int id, flag;
} ns_event;

typedef struct {
    double t;
    int syn;
} syn_event;

typedef struct {
    double* v;
    double* rhs;
    double* d;
    double* m;
    double* h;
    double* n;
    double t;
    /* network */
    int nsyn; /* ExpSyn instances then Exp2Syn instances */
    double *sA, *sB;           /* Exp2Syn A, B; ExpSyn: A = 0, B = g */
    double *s_tau1, *s_factor; /* Exp2Syn: tau1 after the INITIAL clamp, factor */
    int *spk_flag;
    double* spk_t;     /* spike vector: one slot per source (spike.h:66-118) */
    int* pre_flag;     /* PreSyn hysteresis flags (presyn.cpp:150-170) */
    syn_event* pend;   /* the synapses' spike buffers */
    int npend, cappend;
    ns_event* nsq;     /* NetStim self-event buffer */
    int nnsq, capnsq;
    double *ns_event, *ns_on, *ns_ispike, *ns_noise;
    ran123 rng;
    double* vgap;      /* HalfGap vgap */
    double* vpre_np;   /* gapjunction_noptr vpre */
    double *gr_s, *gr_g, *gr_k, *gr_erev;
    /* event recording for the adjoint: (step, synapse) of every delivery */
    int rec_step; /* step whose deliveries are being recorded, -1 = off */
    int* ev;      /* pairs (step, synapse) */
    int nev, capev;
    struct hxo_libstate* lib; /* library mechanisms (hx_oracle_lib.c) */
} hxo_state;

static int grow(void** p, int* cap, int need, size_t el) {
    if (need <= *cap) return 0;
    int nc = *cap ? *cap : 64;
    while (nc < need) nc *= 2;
    void* q = realloc(*p, el * (size_t)nc);
    if (!q) return -1;
    *p = q;
    *cap = nc;
    return 0;
}

static int state_alloc(const hxo_group* g, hxo_state* s) {
    memset(s, 0, sizeof(*s));
    s->v = (double*)calloc((size_t)g->nnode, sizeof(double));
    s->rhs = (double*)calloc((size_t)g->nnode, sizeof(double));
    s->d = (double*)calloc((size_t)g->nnode, sizeof(double));
    size_t nh = g->nhh > 0 ? (size_t)g->nhh : 1;
    s->m = (double*)calloc(nh, sizeof(double));
    s->h = (double*)calloc(nh, sizeof(double));
    s->n = (double*)calloc(nh, sizeof(double));
    s->rec_step = -1;
    if (!(s->v && s->rhs && s->d && s->m && s->h && s->n)) return -1;
    if (hxo_lib_alloc(g, &s->lib)) return -1;
    const hxo_net* N = g->net;
    if (N) {
        s->nsyn = N->nexp + N->nexp2;
        size_t ns = (size_t)s->nsyn + 1, nsrc = (size_t)g->ncell + (size_t)N->nstim + 1;
        size_t nst = (size_t)N->nstim + 1;
        s->sA = (double*)calloc(ns, sizeof(double));
        s->sB = (double*)calloc(ns, sizeof(double));
        s->s_tau1 = (double*)calloc(ns, sizeof(double));
        s->s_factor = (double*)calloc(ns, sizeof(double));
        s->spk_flag = (int*)calloc(nsrc, sizeof(int));
        s->spk_t = (double*)calloc(nsrc, sizeof(double));
        s->pre_flag = (int*)calloc((size_t)g->ncell, sizeof(int));
        s->ns_event = (double*)calloc(nst, sizeof(double));
        s->ns_on = (double*)calloc(nst, sizeof(double));
        s->ns_ispike = (double*)calloc(nst, sizeof(double));
        s->ns_noise = (double*)calloc(nst, sizeof(double));
        s->vgap = (double*)calloc((size_t)N->nhg + 1, sizeof(double));
        s->vpre_np = (double*)calloc((size_t)N->ngn + 1, sizeof(double));
        size_t ng = (size_t)N->ngr + 1;
        s->gr_s = (double*)calloc(ng, sizeof(double));
        s->gr_g = (double*)calloc(ng, sizeof(double));
        s->gr_k = (double*)calloc(ng, sizeof(double));
        s->gr_erev = (double*)calloc(ng, sizeof(double));
        if (!(s->sA && s->sB && s->s_tau1 && s->s_factor && s->spk_flag && s->spk_t && s->pre_flag && s->ns_event &&
              s->ns_on && s->ns_ispike && s->ns_noise && s->vgap && s->vpre_np && s->gr_s && s->gr_g && s->gr_k &&
              s->gr_erev))
            return -1;
    }
    return 0;
}

static void state_free(hxo_state* s) {
    free(s->v);
    free(s->rhs);
    free(s->d);
    free(s->m);
    free(s->h);
    free(s->n);
    free(s->sA);
    free(s->sB);
    free(s->s_tau1);
    free(s->s_factor);
    free(s->spk_flag);
    free(s->spk_t);
    free(s->pre_flag);
    free(s->pend);
    free(s->nsq);
    free(s->ns_event);
    free(s->ns_on);
    free(s->ns_ispike);
    free(s->ns_noise);
    free(s->vgap);
    free(s->vpre_np);
    free(s->gr_s);
    free(s->gr_g);
    free(s->gr_k);
    free(s->gr_erev);
    free(s->ev);
    hxo_lib_free(s->lib);
}

/* ---------------------------------------------------------------- network */
static int syn_src(const hxo_net* N, int j) { return j < N->nexp ? N->exp_src[j] : N->exp2_src[j - N->nexp]; }
static double syn_delay(const hxo_net* N, int j) {
    return j < N->nexp ? N->exp_delay[j] : N->exp2_delay[j - N->nexp];
}

/* net_receive of ExpSyn (expsyn.cpp:137-149: g += w) and Exp2Syn
 * (exp2syn_temp.cuh:60-66: A += w*factor, B += w*factor) */
static void syn_receive(const hxo_net* N, hxo_state* s, int j) {
    if (j < N->nexp) {
        s->sB[j] += N->exp_w[j];
    } else {
        double w = N->exp2_w[j - N->nexp], f = s->s_factor[j];
        s->sA[j] = s->sA[j] + w * f;
        s->sB[j] = s->sB[j] + w * f;
    }
    if (s->rec_step >= 0) {
        if (grow((void**)&s->ev, &s->capev, 2 * (s->nev + 1), sizeof(int))) return;
        s->ev[2 * s->nev] = s->rec_step;
        s->ev[2 * s->nev + 1] = j;
        s->nev++;
    }
}

/* the spike buffer order of spike.h:113-136 for NetStim self events
 * (same syn_type): earlier deliver_time first (1e-9 tolerance), then syn_id */
static int ns_before(const ns_event* a, const ns_event* b) {
    if (fabs(a->t - b->t) > 1e-9) return a->t < b->t;
    return a->id < b->id;
}

static void ns_push(hxo_state* s, double t, int id, int flag) {
    if (grow((void**)&s->nsq, &s->capnsq, s->nnsq + 1, sizeof(ns_event))) return;
    s->nsq[s->nnsq].t = t;
    s->nsq[s->nnsq].id = id;
    s->nsq[s->nnsq].flag = flag;
    s->nnsq++;
}

/* NetStim::invl (netstim.cpp:134-147) */
static double ns_invl(hxo_state* s, double interval, double noise) {
    if (interval <= 0.0) interval = 0.01;
    if (noise == 0) return interval;
    return (1.0 - noise) * interval + noise * interval * ran123_negexp(&s->rng);
}

/* NetStim::init_sequence (netstim.cpp:120-132): every instance */
static void ns_init_sequence(const hxo_net* N, hxo_state* s) {
    for (int i = 0; i < N->nstim; i++)
        if (N->ns_number[i] > 0.0) {
            s->ns_event[i] = 0.0;
            s->ns_on[i] = 1.0;
            s->ns_ispike[i] = 0.0;
        }
}

/* NetStim::next_invl (netstim.cpp:149-164): redraws every instance's interval */
static void ns_next_invl(const hxo_net* N, hxo_state* s) {
    for (int i = 0; i < N->nstim; i++) {
        if (N->ns_number[i] > 0) s->ns_event[i] = ns_invl(s, N->ns_interval[i], s->ns_noise[i]);
        if (s->ns_ispike[i] >= N->ns_number[i]) s->ns_on[i] = 0.0;
    }
}

/* NetStim::initialize_cpu (netstim.cpp:207-239) */
static void ns_initialize(const hxo_group* g, hxo_state* s) {
    const hxo_net* N = g->net;
    ran123_init(&s->rng, N->rng_mode);
    s->nnsq = 0;
    for (int i = 0; i < N->nstim; i++) {
        s->ns_on[i] = 0.0;
        s->ns_ispike[i] = 0.0;
        double noise = N->ns_noise[i];
        if (noise < 0.0) noise = 0.0;
        if (noise > 1.0) noise = 1.0;
        s->ns_noise[i] = noise;
        if (N->ns_start[i] >= 0.0 && N->ns_number[i] > 0) {
            s->ns_on[i] = 1.0;
            double ev = N->ns_start[i] + ns_invl(s, N->ns_interval[i], noise) - N->ns_interval[i] * (1.0 - noise);
            if (ev < 0.0) ev = 0.0;
            s->ns_event[i] = ev;
            ns_push(s, ev, i, SPK_INIT);
        }
    }
}

/* post_spike_receive_cpu + NetStim::net_receive_cpu (postsyn.cpp:43-61,
 * netstim.cpp:275-320); returns send_count > 0 */
static int ns_receive(const hxo_group* g, hxo_state* s, double t, double tt) {
    const hxo_net* N = g->net;
    int nb = 0, capb = 0;
    ns_event* batch = NULL;
    for (;;) {
        int best = -1;
        for (int e = 0; e < s->nnsq; e++)
            if (best < 0 || ns_before(&s->nsq[e], &s->nsq[best])) best = e;
        if (best < 0 || s->nsq[best].t > tt) break;
        if (grow((void**)&batch, &capb, nb + 1, sizeof(ns_event))) break;
        batch[nb++] = s->nsq[best];
        s->nsq[best] = s->nsq[--s->nnsq];
    }
    int send = 0;
    for (int b = 0; b < nb; b++) {
        int i = batch[b].id, flag = batch[b].flag;
        /* NORMAL events into a NetStim need an incoming NetCon; there are none */
        if (flag == SPK_INIT) {
            if (s->ns_on[i] == 1.0) {
                ns_init_sequence(N, s);
                ns_push(s, t + 0.0, i, SPK_SELF);
                send++;
            }
        }
        if (flag == SPK_SELF && s->ns_on[i] == 1.0) {
            s->ns_ispike[i] += 1.0;
            /* net_send NORMAL_EVENT: the NetStim's slot in the spike vector */
            s->spk_flag[g->ncell + i] = SPK_NORMAL;
            s->spk_t[g->ncell + i] = t;
            {
                hxo_net* Nm = g->net;
                if (Nm->ns_nspike < Nm->ns_spike_cap) {
                    Nm->ns_spike_id[Nm->ns_nspike] = i;
                    Nm->ns_spike_t[Nm->ns_nspike] = t;
                }
                Nm->ns_nspike++;
            }
            ns_next_invl(N, s);
            if (s->ns_on[i] == 1.0) {
                ns_push(s, t + s->ns_event[i], i, SPK_SELF);
                send++;
            }
        }
    }
    free(batch);
    return send > 0;
}

/* Simulate::spike_deliver_cpu (simulate.cpp:445-449): threshold detection of
 * every PreSyn, then the receive loop of network_spike_receive_cpu
 * (simulate.cpp:916-941) until no NetStim sends again. */
static void spike_deliver(const hxo_group* g, hxo_state* s) {
    hxo_net* N = g->net;
    if (!N) return;
    const double t = s->t;
    for (int c = 0; c < g->ncell; c++) {
        double pv = s->v[c];
        if (pv > N->ps_thresh[c] && !s->pre_flag[c]) {
            s->spk_flag[c] = SPK_NORMAL;
            s->spk_t[c] = t;
            s->pre_flag[c] = 1;
            if (N->nspike < N->spike_cap) {
                N->spike_gid[N->nspike] = c;
                N->spike_t[N->nspike] = t;
            }
            N->nspike++;
        } else if (pv <= N->ps_thresh[c]) {
            s->pre_flag[c] = 0;
        }
    }
    const double tt = t + g->dt / 2;
    const int nsrc = g->ncell + N->nstim;
    int sent;
    do {
        sent = 0;
        /* get_spike_from_vec_common (postsyn.cpp:94-114) */
        for (int j = 0; j < s->nsyn; j++) {
            int src = syn_src(N, j);
            if (s->spk_flag[src] == SPK_NORMAL) {
                if (grow((void**)&s->pend, &s->cappend, s->npend + 1, sizeof(syn_event))) return;
                s->pend[s->npend].t = s->spk_t[src] + syn_delay(N, j);
                s->pend[s->npend].syn = j;
                s->npend++;
            }
        }
        for (int k = 0; k < nsrc; k++)
            if (s->spk_flag[k] == SPK_NORMAL) s->spk_flag[k] = SPK_INVALID;
        /* ExpSyn and Exp2Syn: deliver what is due (independent per synapse) */
        for (int e = 0; e < s->npend;) {
            if (s->pend[e].t <= tt) {
                syn_receive(N, s, s->pend[e].syn);
                s->pend[e] = s->pend[--s->npend];
            } else {
                e++;
            }
        }
        if (N->nstim) sent |= ns_receive(g, s, t, tt);
    } while (sent);
}

/* neuron_to_neuron_syn_lr rates (neuron_to_neuron_syn_lr.cu:97-100) */
static double gr_inf(const hxo_net* N, int j, double v) {
    return 1.0 / (1.0 + exp((N->gr_vth[j] - v) / N->gr_delta[j]));
}

/* gap_transfer_cpu, simulate.cpp:953-966: every wired target (HalfGap vgap,
 * gapjunction_noptr vpre) takes the voltage of its source node */
static void gap_transfer(const hxo_net* N, hxo_state* s, const double* v) {
    for (int j = 0; j < N->nhg; j++) s->vgap[j] = v[N->hg_src[j]];
    for (int j = 0; j < N->ngn; j++) s->vpre_np[j] = v[N->gn_src[j]];
}

/* finitialize_cpu, simulate.cpp:271-339: v = v_init, gap transfer, mech INITIAL
 * in mech_current_list order, then one spike delivery at t = 0. */
static void finitialize(const hxo_group* g, hxo_state* s, double v_init) {
    s->t = 0;
    for (int i = 0; i < g->nnode; i++) s->v[i] = v_init;
    const hxo_net* N = g->net;
    if (N) gap_transfer(N, s, s->v);
    for (int j = 0; j < g->nhh; j++) {
        hh_rates_t r;
        hh_rates(s->v[g->hh_node[j]], g->celsius, &r);
        s->m[j] = r.minf;
        s->h[j] = r.hinf;
        s->n[j] = r.ninf;
    }
    hxo_lib_init(g, s->lib, s->v);
    if (!N) return;
    for (int j = 0; j < N->nexp; j++) s->sA[j] = s->sB[j] = 0.0;
    for (int q = 0; q < N->nexp2; q++) {
        int j = N->nexp + q;
        double tau1 = N->exp2_tau1[q], tau2 = N->exp2_tau2[q];
        if (tau1 / tau2 > 0.9999) tau1 = 0.9999 * tau2;
        if (tau1 / tau2 < 1e-9) tau1 = tau2 * 1e-9;
        s->s_tau1[j] = tau1;
        s->sA[j] = 0.0;
        s->sB[j] = 0.0;
        double tp = (tau1 * tau2) / (tau2 - tau1) * log(tau2 / tau1);
        s->s_factor[j] = 1.0 / (-exp(-tp / tau1) + exp(-tp / tau2));
    }
    if (N->nstim) ns_initialize(g, s);
    for (int j = 0; j < N->ngr; j++) {
        s->gr_s[j] = gr_inf(N, j, s->v[N->gr_pre[j]]);
        if (N->gr_w[j] > 0.0) {
            s->gr_g[j] = 4.9;
            s->gr_k[j] = 0.5;
            s->gr_erev[j] = 30.0;
        } else {
            s->gr_g[j] = 2.0;
            s->gr_k[j] = 0.015000001;
            s->gr_erev[j] = -70.0;
        }
    }
    /* clearAllSpikes_cpu, then spike_deliver_cpu at t = 0 */
    int nsrc = g->ncell + N->nstim;
    for (int k = 0; k < nsrc; k++) s->spk_flag[k] = SPK_INVALID;
    for (int c = 0; c < g->ncell; c++) s->pre_flag[c] = 0;
    s->npend = 0;
    spike_deliver(g, s);
}

static int iclamp_on(const hxo_group* g, int j, double t) {
    return (t < g->ic_del[j] + g->ic_dur[j] && t >= g->ic_del[j]);
}

/* one POINT_PROCESS contribution through MechTemp::current_cpu
 * (mech_template.cuh:612-645): i1 = I(v+0.001), i0 = I(v) */
static void pp_add(double* rhs, double* d, int i, double i1, double i0, double area, int electrode) {
    double gg = (i1 - i0) / FD_EPS;
    gg *= 1.e2 / area;
    i0 *= 1.e2 / area;
    if (electrode) {
        rhs[i] += i0;
        d[i] -= gg;
    } else {
        rhs[i] -= i0;
        d[i] += gg;
    }
}

/* setup_tree_matrix_cpu, simulate.cpp:455-556, mechanisms in the exported
 * mechanism-list order (capacitance, pas, hh, IClamp, ExpSyn, Exp2Syn,
 * NetStim (no current), HalfGap, gapjunction_lr, gapjunction_noptr,
 * neuron_to_neuron_syn_lr). */
static void setup_tree_matrix(const hxo_group* g, hxo_state* s) {
    const int nn = g->nnode;
    double* v = s->v;
    double* rhs = s->rhs;
    double* d = s->d;
    for (int i = 0; i < nn; i++) {
        rhs[i] = 0.0;
        d[i] = 0.0;
    }
    /* pas */
    for (int j = 0; j < g->npas; j++) {
        int i = g->pas_node[j];
        double vv = v[i];
        double gg = g->pas_g[j] * ((vv + FD_EPS) - g->pas_e[j]);
        double r = g->pas_g[j] * (vv - g->pas_e[j]);
        gg = (gg - r) / FD_EPS;
        rhs[i] -= r;
        d[i] += gg;
    }
    /* hh */
    for (int j = 0; j < g->nhh; j++) {
        int i = g->hh_node[j];
        double vv = v[i];
        double gg = hh_current(vv + FD_EPS, g->hh_gnabar[j], g->hh_gkbar[j], g->hh_gl[j], s->m[j], s->h[j], s->n[j],
                               g->hh_ena[j], g->hh_ek[j], g->hh_el[j], NULL, NULL);
        double r = hh_current(vv, g->hh_gnabar[j], g->hh_gkbar[j], g->hh_gl[j], s->m[j], s->h[j], s->n[j],
                              g->hh_ena[j], g->hh_ek[j], g->hh_el[j], NULL, NULL);
        gg = (gg - r) / FD_EPS;
        rhs[i] -= r;
        d[i] += gg;
    }
    /* IClamp: POINT_PROCESS + ELECTRODE_CURRENT (mech_template.cuh:627-640) */
    for (int j = 0; j < g->nic; j++) {
        int i = g->ic_node[j];
        double cur = iclamp_on(g, j, s->t) ? g->ic_amp[j] : 0.0;
        pp_add(rhs, d, i, cur, cur, g->area[i], 1);
    }
    const hxo_net* N = g->net;
    if (N) {
        /* ExpSyn: i = g (v - e) (expsyn.cpp:92-121) */
        for (int j = 0; j < N->nexp; j++) {
            int i = N->exp_node[j];
            double gs = s->sB[j], e = N->exp_e[j];
            pp_add(rhs, d, i, gs * (v[i] + FD_EPS - e), gs * (v[i] - e), g->area[i], 0);
        }
        /* Exp2Syn: i = (B - A)(v - e) */
        for (int q = 0; q < N->nexp2; q++) {
            int j = N->nexp + q, i = N->exp2_node[q];
            double gs = s->sB[j] - s->sA[j], e = N->exp2_e[q];
            pp_add(rhs, d, i, gs * ((v[i] + FD_EPS) - e), gs * (v[i] - e), g->area[i], 0);
        }
        /* HalfGap: i = (vgap - v) g, electrode current */
        for (int j = 0; j < N->nhg; j++) {
            int i = N->hg_node[j];
            double vg = s->vgap[j], gg = N->hg_g[j];
            pp_add(rhs, d, i, (vg - (v[i] + FD_EPS)) * gg, (vg - v[i]) * gg, g->area[i], 1);
        }
        /* gapjunction_lr: i = w (g (v - vpre)) */
        for (int j = 0; j < N->ngj; j++) {
            int i = N->gj_node[j];
            double vp = v[N->gj_pre[j]], gg = N->gj_g[j], w = N->gj_w[j];
            pp_add(rhs, d, i, w * (gg * ((v[i] + FD_EPS) - vp)), w * (gg * (v[i] - vp)), g->area[i], 0);
        }
        /* gapjunction_noptr: i = weight (v - vpre) (worm-mech/gapjunction_noptr.cu:33-36) */
        for (int j = 0; j < N->ngn; j++) {
            int i = N->gn_node[j];
            double vp = s->vpre_np[j], ww = N->gn_w[j];
            pp_add(rhs, d, i, ww * ((v[i] + FD_EPS) - vp), ww * (v[i] - vp), g->area[i], 0);
        }
        /* neuron_to_neuron_syn_lr: i = |w| (g s (v - erev)) */
        for (int j = 0; j < N->ngr; j++) {
            int i = N->gr_node[j];
            double aw = fabs(N->gr_w[j]), gs = s->gr_g[j] * s->gr_s[j], er = s->gr_erev[j];
            pp_add(rhs, d, i, aw * (gs * ((v[i] + FD_EPS) - er)), aw * (gs * (v[i] - er)), g->area[i], 0);
        }
    }
    /* library mechanisms (types after the network mechanisms) */
    hxo_lib_current(g, s->lib, v, rhs, d);
    /* cap_jacob_cpu, capac.cpp:68-78 with cj = 1/dt */
    {
        double cj = 1.0 / g->dt;
        double cfac = 0.001 * cj;
        for (int i = 0; i < nn; i++) d[i] += cfac * g->cm[i];
    }
    for (int i = g->ncell; i < nn; i++) {
        int p = g->parent[i];
        double dv = v[p] - v[i];
        rhs[i] -= g->b[i] * dv;
        rhs[p] += g->a[i] * dv;
    }
    for (int i = g->ncell; i < nn; i++) {
        d[i] -= g->b[i];
        d[g->parent[i]] -= g->a[i];
    }
}

/* solve_serial, simulate.cpp:558-581 */
static void solve_serial(const hxo_group* g, double* d, double* rhs) {
    const int nn = g->nnode;
    for (int i = nn - 1; i >= g->ncell; i--) {
        int p = g->parent[i];
        double pp = g->a[i] / d[i];
        d[p] -= pp * g->b[i];
        rhs[p] -= pp * rhs[i];
    }
    for (int i = 0; i < g->ncell; i++) rhs[i] /= d[i];
    for (int i = g->ncell; i < nn; i++) {
        rhs[i] -= g->b[i] * rhs[g->parent[i]];
        rhs[i] /= d[i];
    }
}

/* transposed solve: same elimination order with the off-diagonals swapped */
static void solve_serial_T(const hxo_group* g, double* d, double* rhs) {
    const int nn = g->nnode;
    for (int i = nn - 1; i >= g->ncell; i--) {
        int p = g->parent[i];
        double pp = g->b[i] / d[i];
        d[p] -= pp * g->a[i];
        rhs[p] -= pp * rhs[i];
    }
    for (int i = 0; i < g->ncell; i++) rhs[i] /= d[i];
    for (int i = g->ncell; i < nn; i++) {
        rhs[i] -= g->a[i] * rhs[g->parent[i]];
        rhs[i] /= d[i];
    }
}

/* nonvint_cpu, simulate.cpp:784-852: states at the updated v */
static void nonvint(const hxo_group* g, hxo_state* s) {
    const double dt = g->dt;
    hxo_lib_state_ion(g, s->lib, s->v); /* mech_write_state_ion_list first */
    hxo_lib_state(g, s->lib, s->v);
    for (int j = 0; j < g->nhh; j++) {
        hh_rates_t r;
        hh_rates(s->v[g->hh_node[j]], g->celsius, &r);
        s->m[j] = gate_step(s->m[j], r.minf, r.mtau, dt);
        s->h[j] = gate_step(s->h[j], r.hinf, r.htau, dt);
        s->n[j] = gate_step(s->n[j], r.ninf, r.ntau, dt);
    }
    const hxo_net* N = g->net;
    if (!N) return;
    for (int j = 0; j < N->nexp; j++) { /* expsyn.cpp:125-134 */
        double tau = N->exp_tau[j];
        s->sB[j] = s->sB[j] + (1. - exp(dt * ((-1.0) / tau))) * (-(0.0) / ((-1.0) / tau) - s->sB[j]);
    }
    for (int q = 0; q < N->nexp2; q++) { /* exp2syn_temp.cuh:51-58 */
        int j = N->nexp + q;
        double tau1 = s->s_tau1[j], tau2 = N->exp2_tau2[q];
        double A = s->sA[j], B = s->sB[j];
        s->sA[j] = A + (1.0 - exp(dt * (-1.0 / tau1))) * (-0.0 / (-1.0 / tau1) - A);
        s->sB[j] = B + (1.0 - exp(dt * (-1.0 / tau2))) * (-0.0 / (-1.0 / tau2) - B);
    }
    for (int j = 0; j < N->ngr; j++) { /* neuron_to_neuron_syn_lr.cu:126-145 (s_ds does not feed back) */
        double inf = gr_inf(N, j, s->v[N->gr_pre[j]]);
        double tau = (1.0 - inf) / s->gr_k[j];
        double E = exp(-dt / tau);
        s->gr_s[j] = inf + (s->gr_s[j] - inf) * E;
    }
}

/* fadvance_cpu, simulate.cpp:410-442 */
static void fadvance(const hxo_group* g, hxo_state* s) {
    spike_deliver(g, s);
    s->t += 0.5 * g->dt;
    setup_tree_matrix(g, s);
    solve_serial(g, s->d, s->rhs);
    for (int i = 0; i < g->nnode; i++) s->v[i] += s->rhs[i];
    if (g->net) gap_transfer(g->net, s, s->v);
    s->t += 0.5 * g->dt;
    nonvint(g, s);
}

static void record(const hxo_group* g, const hxo_state* s, int nprobe, const int* probe, double* row) {
    (void)g;
    for (int p = 0; p < nprobe; p++) row[p] = s->v[probe[p]];
}

int hxo_forward(const hxo_group* g, double v_init, int nstep, int nprobe, const int* probe, double* trace,
                double* v_final, double* m_final, double* h_final, double* n_final) {
    hxo_state s;
    if (g->net) g->net->nspike = g->net->ns_nspike = 0;
    if (state_alloc(g, &s)) {
        state_free(&s);
        return -1;
    }
    finitialize(g, &s, v_init);
    if (trace) record(g, &s, nprobe, probe, trace);
    for (int k = 0; k < nstep; k++) {
        fadvance(g, &s);
        if (trace) record(g, &s, nprobe, probe, trace + (size_t)(k + 1) * nprobe);
    }
    if (v_final) memcpy(v_final, s.v, sizeof(double) * g->nnode);
    if (m_final && g->nhh) memcpy(m_final, s.m, sizeof(double) * g->nhh);
    if (h_final && g->nhh) memcpy(h_final, s.h, sizeof(double) * g->nhh);
    if (n_final && g->nhh) memcpy(n_final, s.n, sizeof(double) * g->nhh);
    state_free(&s);
    return 0;
}

int hxo_forward_lib(const hxo_group* g, double v_init, int nstep, int nprobe, const int* probe, double* trace,
                    double* lib_final, int nlib_final) {
    hxo_state s;
    if (g->net) g->net->nspike = g->net->ns_nspike = 0;
    if (state_alloc(g, &s)) {
        state_free(&s);
        return -1;
    }
    finitialize(g, &s, v_init);
    if (trace) record(g, &s, nprobe, probe, trace);
    for (int k = 0; k < nstep; k++) {
        fadvance(g, &s);
        if (trace) record(g, &s, nprobe, probe, trace + (size_t)(k + 1) * nprobe);
    }
    int rc = lib_final ? hxo_lib_final(g, s.lib, lib_final, nlib_final) : 0;
    state_free(&s);
    return rc < 0 ? rc : 0;
}

/* ---------------------------------------------------------------- adjoint */
static void zero_if(double* p, int n) {
    if (p && n > 0) memset(p, 0, sizeof(double) * (size_t)n);
}

#define GADD(arr, j, x) \
    do {                \
        if (gr && gr->arr) gr->arr[j] += (x); \
    } while (0)

static _Thread_local double g_last_reverse_s = 0.0;

double hxo_last_reverse_seconds(void) { return g_last_reverse_s; }

int hxo_adjoint(const hxo_group* g, double v_init, int nstep, int nprobe, const int* probe, const double* dLdv,
                double* trace, hxo_grads* gr) {
    if (g->lib) return -2; /* library mechanisms: gradients are checked by finite differences */
    const int nn = g->nnode, nh = g->nhh;
    hxo_net* N = g->net;
    const int nsyn = N ? N->nexp + N->nexp2 : 0, ngr = N ? N->ngr : 0;
    const size_t nh1 = nh > 0 ? (size_t)nh : 1, ns1 = nsyn > 0 ? (size_t)nsyn : 1, ng1 = ngr > 0 ? (size_t)ngr : 1;
    const size_t T1 = (size_t)(nstep + 1);
    double* tv = (double*)malloc(sizeof(double) * (size_t)nn * T1);
    double* tm = (double*)malloc(sizeof(double) * nh1 * T1);
    double* th = (double*)malloc(sizeof(double) * nh1 * T1);
    double* tn = (double*)malloc(sizeof(double) * nh1 * T1);
    double* tA = (double*)malloc(sizeof(double) * ns1 * T1);
    double* tB = (double*)malloc(sizeof(double) * ns1 * T1);
    double* tS = (double*)malloc(sizeof(double) * ng1 * T1);
    double* tmid = (double*)malloc(sizeof(double) * T1);
    int* ev_off = (int*)calloc(T1 + 1, sizeof(int));
    double* lv = (double*)calloc((size_t)nn, sizeof(double));
    double* mu = (double*)calloc((size_t)nn, sizeof(double));
    double* w = (double*)calloc((size_t)nn, sizeof(double));
    double* dd = (double*)calloc((size_t)nn, sizeof(double));
    double* lm = (double*)calloc(nh1, sizeof(double));
    double* lh = (double*)calloc(nh1, sizeof(double));
    double* ln = (double*)calloc(nh1, sizeof(double));
    double* lA = (double*)calloc(ns1, sizeof(double));
    double* lB = (double*)calloc(ns1, sizeof(double));
    double* lS = (double*)calloc(ng1, sizeof(double));
    hxo_state s;
    int rc = -1;
    memset(&s, 0, sizeof(s));
    if (!tv || !tm || !th || !tn || !tA || !tB || !tS || !tmid || !ev_off || !lv || !mu || !w || !dd || !lm || !lh ||
        !ln || !lA || !lB || !lS)
        goto done;
    if (N) N->nspike = N->ns_nspike = 0;
    if (state_alloc(g, &s)) goto done;

    /* ---- forward with a full tape: state at the start of every step, the
     * synapse states after that step's deliveries, and the delivery list */
    s.rec_step = 0;
    finitialize(g, &s, v_init);
    if (trace) record(g, &s, nprobe, probe, trace);
    for (int k = 0; k < nstep; k++) {
        s.rec_step = k;
        spike_deliver(g, &s);
        memcpy(tv + (size_t)k * nn, s.v, sizeof(double) * nn);
        if (nh) {
            memcpy(tm + (size_t)k * nh, s.m, sizeof(double) * nh);
            memcpy(th + (size_t)k * nh, s.h, sizeof(double) * nh);
            memcpy(tn + (size_t)k * nh, s.n, sizeof(double) * nh);
        }
        if (nsyn) {
            memcpy(tA + (size_t)k * nsyn, s.sA, sizeof(double) * nsyn);
            memcpy(tB + (size_t)k * nsyn, s.sB, sizeof(double) * nsyn);
        }
        if (ngr) memcpy(tS + (size_t)k * ngr, s.gr_s, sizeof(double) * ngr);
        tmid[k] = s.t + 0.5 * g->dt;
        /* the rest of fadvance (spike delivery done above) */
        s.t += 0.5 * g->dt;
        setup_tree_matrix(g, &s);
        solve_serial(g, s.d, s.rhs);
        for (int i = 0; i < nn; i++) s.v[i] += s.rhs[i];
        if (N) gap_transfer(N, &s, s.v);
        s.t += 0.5 * g->dt;
        nonvint(g, &s);
        if (trace) record(g, &s, nprobe, probe, trace + (size_t)(k + 1) * nprobe);
    }
    memcpy(tv + (size_t)nstep * nn, s.v, sizeof(double) * nn);
    /* the reverse sweep's own wall time starts here (hxo_last_reverse_seconds) */
    struct timespec t_rev0;
    clock_gettime(CLOCK_MONOTONIC, &t_rev0);
    /* deliveries grouped by step (recorded in step order) */
    for (int e = 0; e < s.nev; e++) ev_off[s.ev[2 * e] + 1]++;
    for (int k = 0; k < nstep + 1; k++) ev_off[k + 1] += ev_off[k];

    if (gr) {
        zero_if(gr->hh_gnabar, nh);
        zero_if(gr->hh_gkbar, nh);
        zero_if(gr->hh_gl, nh);
        zero_if(gr->hh_el, nh);
        zero_if(gr->pas_g, g->npas);
        zero_if(gr->pas_e, g->npas);
        zero_if(gr->cm, nn);
        zero_if(gr->ic_amp, g->nic);
        if (N) {
            zero_if(gr->exp_w, N->nexp);
            zero_if(gr->exp_e, N->nexp);
            zero_if(gr->exp2_w, N->nexp2);
            zero_if(gr->exp2_e, N->nexp2);
            zero_if(gr->hg_g, N->nhg);
            zero_if(gr->gj_g, N->ngj);
            zero_if(gr->gj_w, N->ngj);
            zero_if(gr->gr_w, N->ngr);
            zero_if(gr->gn_w, N->ngn);
        }
    }
    const double dt = g->dt;
    const double cfac = 0.001 * (1.0 / dt);

    /* ---- reverse sweep */
    for (int k = nstep - 1; k >= 0; k--) {
        const double* vk = tv + (size_t)k * nn;
        const double* vk1 = tv + (size_t)(k + 1) * nn;
        const double* mk = tm + (size_t)k * nh;
        const double* hk = th + (size_t)k * nh;
        const double* nk = tn + (size_t)k * nh;
        /* loss on the recorded v after step k (trace row k+1) */
        for (int p = 0; p < nprobe; p++) lv[probe[p]] += dLdv[(size_t)(k + 1) * nprobe + p];
        /* state VJP at v' = v_{k+1}: x' = E x + (1-E) inf, E = exp(-dt/tau) */
        memcpy(mu, lv, sizeof(double) * nn);
        for (int j = 0; j < nh; j++) {
            int i = g->hh_node[j];
            double vp = vk1[i];
            hh_rates_t r;
            hh_drates_t dr;
            hh_rates(vp, g->celsius, &r);
            hh_drates(vp, g->celsius, &dr);
            double inf[3] = {r.minf, r.hinf, r.ninf};
            double tau[3] = {r.mtau, r.htau, r.ntau};
            double x[3] = {mk[j], hk[j], nk[j]};
            double* lx[3] = {&lm[j], &lh[j], &ln[j]};
            for (int q = 0; q < 3; q++) {
                double E = exp(dt * (-1.0 / tau[q]));
                double dnew_dv = (1.0 - E) * dr.dinf[q] + (inf[q] - x[q]) * E * dt * dr.q10 * dr.ds[q];
                mu[i] += *lx[q] * dnew_dv;
                *lx[q] *= E;
            }
        }
        if (N) {
            /* synapse decay x' = x + c (0 - x): dx'/dx = 1 - c */
            for (int j = 0; j < N->nexp; j++) lB[j] *= 1.0 - (1. - exp(dt * ((-1.0) / N->exp_tau[j])));
            for (int q = 0; q < N->nexp2; q++) {
                int j = N->nexp + q;
                lA[j] *= 1.0 - (1.0 - exp(dt * (-1.0 / s.s_tau1[j])));
                lB[j] *= 1.0 - (1.0 - exp(dt * (-1.0 / N->exp2_tau2[q])));
            }
            /* graded synapse: s' = inf + (s - inf) E, inf, E functions of vpre_{k+1} */
            for (int j = 0; j < ngr; j++) {
                int pre = N->gr_pre[j];
                double inf = gr_inf(N, j, vk1[pre]);
                double tau = (1.0 - inf) / s.gr_k[j];
                double E = exp(-dt / tau);
                double dinf = inf * (1.0 - inf) / N->gr_delta[j];
                double dE = (E == 0.0) ? 0.0 : E * (dt / (tau * tau)) * (-dinf / s.gr_k[j]);
                double sk = tS[(size_t)k * ngr + j];
                mu[pre] += lS[j] * (dinf * (1.0 - E) + (sk - inf) * dE);
                lS[j] *= E;
            }
        }
        /* recompute the step-k diagonal d (same assembly as the forward) */
        s.t = tmid[k];
        memcpy(s.v, vk, sizeof(double) * nn);
        if (nh) {
            memcpy(s.m, mk, sizeof(double) * nh);
            memcpy(s.h, hk, sizeof(double) * nh);
            memcpy(s.n, nk, sizeof(double) * nh);
        }
        if (nsyn) {
            memcpy(s.sA, tA + (size_t)k * nsyn, sizeof(double) * nsyn);
            memcpy(s.sB, tB + (size_t)k * nsyn, sizeof(double) * nsyn);
        }
        if (ngr) memcpy(s.gr_s, tS + (size_t)k * ngr, sizeof(double) * ngr);
        if (N) gap_transfer(N, &s, vk);
        setup_tree_matrix(g, &s);
        memcpy(dd, s.d, sizeof(double) * nn);
        /* w = M_k^{-T} mu */
        memcpy(w, mu, sizeof(double) * nn);
        solve_serial_T(g, dd, w);
        /* VJPs of rhs and d w.r.t. v_k, states and parameters */
        memcpy(lv, mu, sizeof(double) * nn); /* v_{k+1} = v_k + dv */
        for (int j = 0; j < g->npas; j++) {
            int i = g->pas_node[j];
            double ld = -w[i] * (vk1[i] - vk[i]);
            double gp = g->pas_g[j];
            GADD(pas_g, j, ld - w[i] * (vk[i] - g->pas_e[j]));
            GADD(pas_e, j, w[i] * gp);
            lv[i] += -w[i] * gp;
        }
        for (int j = 0; j < nh; j++) {
            int i = g->hh_node[j];
            double ld = -w[i] * (vk1[i] - vk[i]);
            double m = mk[j], h = hk[j], n = nk[j];
            double gnabar = g->hh_gnabar[j], gkbar = g->hh_gkbar[j], gl = g->hh_gl[j];
            double ena_t = ld - w[i] * (vk[i] - g->hh_ena[j]);
            double ek_t = ld - w[i] * (vk[i] - g->hh_ek[j]);
            double el_t = ld - w[i] * (vk[i] - g->hh_el[j]);
            double m3h = m * m * m * h, n4 = n * n * n * n;
            GADD(hh_gnabar, j, m3h * ena_t);
            GADD(hh_gkbar, j, n4 * ek_t);
            GADD(hh_gl, j, el_t);
            GADD(hh_el, j, w[i] * gl);
            lm[j] += 3.0 * gnabar * m * m * h * ena_t;
            lh[j] += gnabar * m * m * m * ena_t;
            ln[j] += 4.0 * gkbar * n * n * n * ek_t;
            lv[i] += -w[i] * (gnabar * m3h + gkbar * n4 + gl);
        }
        for (int j = 0; j < g->nic; j++) {
            int i = g->ic_node[j];
            if (iclamp_on(g, j, tmid[k])) GADD(ic_amp, j, w[i] * (1.e2 / g->area[i]));
        }
        if (N) {
            for (int j = 0; j < nsyn; j++) {
                int i = j < N->nexp ? N->exp_node[j] : N->exp2_node[j - N->nexp];
                double e = j < N->nexp ? N->exp_e[j] : N->exp2_e[j - N->nexp];
                double sa = 1.e2 / g->area[i];
                double G = s.sB[j] - s.sA[j];
                double ld = -w[i] * (vk1[i] - vk[i]);
                double lG = sa * (ld - w[i] * (vk[i] - e));
                lB[j] += lG;
                lA[j] -= lG;
                if (j < N->nexp) GADD(exp_e, j, w[i] * sa * G);
                else GADD(exp2_e, j - N->nexp, w[i] * sa * G);
                lv[i] += -w[i] * sa * G;
            }
            for (int e = ev_off[k]; e < ev_off[k + 1]; e++) {
                int j = s.ev[2 * e + 1];
                if (j < N->nexp) GADD(exp_w, j, lB[j]);
                else GADD(exp2_w, j - N->nexp, s.s_factor[j] * lA[j] + s.s_factor[j] * lB[j]);
            }
            for (int j = 0; j < N->nhg; j++) {
                int i = N->hg_node[j], q = N->hg_src[j];
                double sa = 1.e2 / g->area[i], gg = N->hg_g[j];
                double ld = -w[i] * (vk1[i] - vk[i]);
                GADD(hg_g, j, w[i] * sa * (vk[q] - vk[i]) + ld * sa);
                lv[i] += -w[i] * sa * gg;
                lv[q] += w[i] * sa * gg;
            }
            for (int j = 0; j < N->ngj; j++) {
                int i = N->gj_node[j], q = N->gj_pre[j];
                double sa = 1.e2 / g->area[i], gg = N->gj_g[j], ww = N->gj_w[j];
                double ld = -w[i] * (vk1[i] - vk[i]);
                double dv = vk[i] - vk[q];
                GADD(gj_w, j, -w[i] * sa * gg * dv + ld * sa * gg);
                GADD(gj_g, j, -w[i] * sa * ww * dv + ld * sa * ww);
                lv[i] += -w[i] * sa * ww * gg;
                lv[q] += w[i] * sa * ww * gg;
            }
            for (int j = 0; j < N->ngn; j++) {
                int i = N->gn_node[j], q = N->gn_src[j];
                double sa = 1.e2 / g->area[i], ww = N->gn_w[j];
                double ld = -w[i] * (vk1[i] - vk[i]);
                GADD(gn_w, j, -w[i] * sa * (vk[i] - vk[q]) + ld * sa);
                lv[i] += -w[i] * sa * ww;
                lv[q] += w[i] * sa * ww;
            }
            for (int j = 0; j < ngr; j++) {
                int i = N->gr_node[j];
                double sa = 1.e2 / g->area[i], W = N->gr_w[j], aw = fabs(W), gg = s.gr_g[j], er = s.gr_erev[j];
                double sk = tS[(size_t)k * ngr + j];
                double ld = -w[i] * (vk1[i] - vk[i]);
                double dvr = vk[i] - er;
                lS[j] += -w[i] * sa * aw * gg * dvr + ld * sa * aw * gg;
                double sgn = (W > 0) - (W < 0);
                GADD(gr_w, j, sgn * (-w[i] * sa * gg * sk * dvr + ld * sa * gg * sk));
                lv[i] += -w[i] * sa * aw * gg * sk;
            }
        }
        if (gr && gr->cm)
            for (int i = 0; i < nn; i++) gr->cm[i] += -w[i] * (vk1[i] - vk[i]) * cfac;
        for (int i = g->ncell; i < nn; i++) {
            int p = g->parent[i];
            lv[i] += g->b[i] * w[i] - g->a[i] * w[p];
            lv[p] += g->a[i] * w[p] - g->b[i] * w[i];
        }
    }
    {
        struct timespec t_rev1;
        clock_gettime(CLOCK_MONOTONIC, &t_rev1);
        g_last_reverse_s = (double)(t_rev1.tv_sec - t_rev0.tv_sec) + 1e-9 * (double)(t_rev1.tv_nsec - t_rev0.tv_nsec);
    }
    rc = 0;
done:
    state_free(&s);
    free(tv);
    free(tm);
    free(th);
    free(tn);
    free(tA);
    free(tB);
    free(tS);
    free(tmid);
    free(ev_off);
    free(lv);
    free(mu);
    free(w);
    free(dd);
    free(lm);
    free(lh);
    free(ln);
    free(lA);
    free(lB);
    free(lS);
    return rc;
}
