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
 * and the discrete adjoint of that step sequence (no reference counterpart).
 */
#include "hx_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define FD_EPS 0.001 /* mech_template.cuh:616,626 */

/* ---------------------------------------------------------------- hh */
/* hh_templated.cu:76-85 */
static double vtrap(double x, double y) {
    if (fabs(x / y) < 1e-6) return y * (1 - x / y / 2);
    return x / (exp(x / y) - 1);
}
/* d vtrap / dx, derivative of the branch vtrap() takes */
static double dvtrap(double x, double y) {
    if (fabs(x / y) < 1e-6) return -0.5;
    double e = exp(x / y);
    double em1 = e - 1;
    return (em1 - (x / y) * e) / (em1 * em1);
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

/* ---------------------------------------------------------------- state */
typedef struct {
    double* v;
    double* rhs;
    double* d;
    double* m;
    double* h;
    double* n;
    double t;
} hxo_state;

static int state_alloc(const hxo_group* g, hxo_state* s) {
    memset(s, 0, sizeof(*s));
    s->v = (double*)calloc((size_t)g->nnode, sizeof(double));
    s->rhs = (double*)calloc((size_t)g->nnode, sizeof(double));
    s->d = (double*)calloc((size_t)g->nnode, sizeof(double));
    size_t nh = g->nhh > 0 ? (size_t)g->nhh : 1;
    s->m = (double*)calloc(nh, sizeof(double));
    s->h = (double*)calloc(nh, sizeof(double));
    s->n = (double*)calloc(nh, sizeof(double));
    return (s->v && s->rhs && s->d && s->m && s->h && s->n) ? 0 : -1;
}

static void state_free(hxo_state* s) {
    free(s->v);
    free(s->rhs);
    free(s->d);
    free(s->m);
    free(s->h);
    free(s->n);
}

/* finitialize_cpu, simulate.cpp:271-339: v = v_init, mech INITIAL in
 * mech_current_list order (hh: gates at steady state of v). */
static void finitialize(const hxo_group* g, hxo_state* s, double v_init) {
    s->t = 0;
    for (int i = 0; i < g->nnode; i++) s->v[i] = v_init;
    for (int j = 0; j < g->nhh; j++) {
        hh_rates_t r;
        hh_rates(s->v[g->hh_node[j]], g->celsius, &r);
        s->m[j] = r.minf;
        s->h[j] = r.hinf;
        s->n[j] = r.ninf;
    }
}

static int iclamp_on(const hxo_group* g, int j, double t) {
    return (t < g->ic_del[j] + g->ic_dur[j] && t >= g->ic_del[j]);
}

/* setup_tree_matrix_cpu, simulate.cpp:455-556, mechanisms in CoreNEURON order
 * (capacitance, pas, hh, IClamp). */
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
        double gg = (cur - cur) / FD_EPS;
        double r = cur;
        double nd_area = g->area[i];
        gg *= 1.e2 / nd_area;
        r *= 1.e2 / nd_area;
        rhs[i] += r;
        d[i] -= gg;
    }
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

/* nonvint_cpu, simulate.cpp:784-852: hh state at the updated v */
static void nonvint(const hxo_group* g, hxo_state* s) {
    for (int j = 0; j < g->nhh; j++) {
        hh_rates_t r;
        hh_rates(s->v[g->hh_node[j]], g->celsius, &r);
        s->m[j] = gate_step(s->m[j], r.minf, r.mtau, g->dt);
        s->h[j] = gate_step(s->h[j], r.hinf, r.htau, g->dt);
        s->n[j] = gate_step(s->n[j], r.ninf, r.ntau, g->dt);
    }
}

/* fadvance_cpu, simulate.cpp:410-442 */
static void fadvance(const hxo_group* g, hxo_state* s) {
    s->t += 0.5 * g->dt;
    setup_tree_matrix(g, s);
    solve_serial(g, s->d, s->rhs);
    for (int i = 0; i < g->nnode; i++) s->v[i] += s->rhs[i];
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
    if (state_alloc(g, &s)) return -1;
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

/* ---------------------------------------------------------------- adjoint */
static void zero_if(double* p, int n) {
    if (p && n > 0) memset(p, 0, sizeof(double) * (size_t)n);
}

int hxo_adjoint(const hxo_group* g, double v_init, int nstep, int nprobe, const int* probe, const double* dLdv,
                double* trace, hxo_grads* gr) {
    const int nn = g->nnode, nh = g->nhh;
    const size_t nh1 = nh > 0 ? (size_t)nh : 1;
    double* tv = (double*)malloc(sizeof(double) * (size_t)nn * (size_t)(nstep + 1));
    double* tm = (double*)malloc(sizeof(double) * nh1 * (size_t)(nstep + 1));
    double* th = (double*)malloc(sizeof(double) * nh1 * (size_t)(nstep + 1));
    double* tn = (double*)malloc(sizeof(double) * nh1 * (size_t)(nstep + 1));
    double* tmid = (double*)malloc(sizeof(double) * (size_t)(nstep + 1));
    double* lv = (double*)calloc((size_t)nn, sizeof(double));
    double* mu = (double*)calloc((size_t)nn, sizeof(double));
    double* w = (double*)calloc((size_t)nn, sizeof(double));
    double* dd = (double*)calloc((size_t)nn, sizeof(double));
    double* lm = (double*)calloc(nh1, sizeof(double));
    double* lh = (double*)calloc(nh1, sizeof(double));
    double* ln = (double*)calloc(nh1, sizeof(double));
    hxo_state s;
    int rc = -1;
    if (!tv || !tm || !th || !tn || !tmid || !lv || !mu || !w || !dd || !lm || !lh || !ln) goto done;
    if (state_alloc(g, &s)) goto done;

    /* ---- forward with a full tape: state at the start of every step */
    finitialize(g, &s, v_init);
    if (trace) record(g, &s, nprobe, probe, trace);
    for (int k = 0; k < nstep; k++) {
        memcpy(tv + (size_t)k * nn, s.v, sizeof(double) * nn);
        if (nh) {
            memcpy(tm + (size_t)k * nh, s.m, sizeof(double) * nh);
            memcpy(th + (size_t)k * nh, s.h, sizeof(double) * nh);
            memcpy(tn + (size_t)k * nh, s.n, sizeof(double) * nh);
        }
        tmid[k] = s.t + 0.5 * g->dt;
        fadvance(g, &s);
        if (trace) record(g, &s, nprobe, probe, trace + (size_t)(k + 1) * nprobe);
    }
    memcpy(tv + (size_t)nstep * nn, s.v, sizeof(double) * nn);

    if (gr) {
        zero_if(gr->hh_gnabar, nh);
        zero_if(gr->hh_gkbar, nh);
        zero_if(gr->hh_gl, nh);
        zero_if(gr->hh_el, nh);
        zero_if(gr->pas_g, g->npas);
        zero_if(gr->pas_e, g->npas);
        zero_if(gr->cm, nn);
        zero_if(gr->ic_amp, g->nic);
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
        /* recompute the step-k diagonal d (same assembly as the forward) */
        s.t = tmid[k];
        memcpy(s.v, vk, sizeof(double) * nn);
        if (nh) {
            memcpy(s.m, mk, sizeof(double) * nh);
            memcpy(s.h, hk, sizeof(double) * nh);
            memcpy(s.n, nk, sizeof(double) * nh);
        }
        setup_tree_matrix(g, &s);
        memcpy(dd, s.d, sizeof(double) * nn);
        /* w = M_k^{-T} mu */
        memcpy(w, mu, sizeof(double) * nn);
        solve_serial_T(g, dd, w);
        /* VJPs of rhs and d w.r.t. v_k, gates and parameters */
        memcpy(lv, mu, sizeof(double) * nn); /* v_{k+1} = v_k + dv */
        for (int j = 0; j < g->npas; j++) {
            int i = g->pas_node[j];
            double ld = -w[i] * (vk1[i] - vk[i]);
            double gp = g->pas_g[j];
            if (gr && gr->pas_g) gr->pas_g[j] += ld - w[i] * (vk[i] - g->pas_e[j]);
            if (gr && gr->pas_e) gr->pas_e[j] += w[i] * gp;
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
            if (gr && gr->hh_gnabar) gr->hh_gnabar[j] += m3h * ena_t;
            if (gr && gr->hh_gkbar) gr->hh_gkbar[j] += n4 * ek_t;
            if (gr && gr->hh_gl) gr->hh_gl[j] += el_t;
            if (gr && gr->hh_el) gr->hh_el[j] += w[i] * gl;
            lm[j] += 3.0 * gnabar * m * m * h * ena_t;
            lh[j] += gnabar * m * m * m * ena_t;
            ln[j] += 4.0 * gkbar * n * n * n * ek_t;
            lv[i] += -w[i] * (gnabar * m3h + gkbar * n4 + gl);
        }
        for (int j = 0; j < g->nic; j++) {
            int i = g->ic_node[j];
            if (gr && gr->ic_amp && iclamp_on(g, j, tmid[k])) gr->ic_amp[j] += w[i] * (1.e2 / g->area[i]);
        }
        if (gr && gr->cm)
            for (int i = 0; i < nn; i++) gr->cm[i] += -w[i] * (vk1[i] - vk[i]) * cfac;
        for (int i = g->ncell; i < nn; i++) {
            int p = g->parent[i];
            lv[i] += g->b[i] * w[i] - g->a[i] * w[p];
            lv[p] += g->a[i] * w[p] - g->b[i] * w[i];
        }
    }
    rc = 0;
    state_free(&s);
done:
    free(tv);
    free(tm);
    free(th);
    free(tn);
    free(tmid);
    free(lv);
    free(mu);
    free(w);
    free(dd);
    free(lm);
    free(lh);
    free(ln);
    return rc;
}
