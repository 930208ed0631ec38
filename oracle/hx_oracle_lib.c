/*
 * hx_oracle_lib.c -- TEST INFRASTRUCTURE ONLY (see hx_oracle.h).
 *
 * The library mechanisms of the CPU oracle, restated in plain C in the
 * expression order of the reference's own files:
 *   ions (erev, Nernst, current reset)   src/mech/eion.cuh:38-56, 155-197
 *   CaDynamics_E2                        src/mech/user-mech/CaDynamics_E2.cu:78-137
 *   Ca_HVA                               src/mech/user-mech/CA_HVA.cu (vtrap, rates,
 *                                        current, state)
 *   Ca_LVAst                             src/mech/user-mech/Ca_LVAst.cu
 *   Im                                   src/mech/user-mech/Im.cu
 *   K_Pst, K_Tst                         src/mech/user-mech/K_Pst.cu, K_Tst.cu
 *   NaTg                                 src/mech/user-mech/NaTg.cu:78-160
 *   Nap_Et2                              src/mech/user-mech/Nap_Et2.cu
 *   SK_E2                                src/mech/user-mech/SK_E2.cu:70-132
 *   SKv3_1                               src/mech/user-mech/SKv3_1.cu
 *   hd_la (GLOBALs ehd .. qtl, celsius)  src/mech/user-mech/hd_la.cu:86-124
 *   km_la (GLOBALs Ra, Rb, tha, qa, tadj) src/mech/user-mech/km_la.cu:97-145
 *   kca_la (GLOBALs Ra, Rb, caix, tadj)  src/mech/user-mech/kca_la.cu:100-145
 *   it2_la (GLOBALs vshift .. wh2)       src/mech/user-mech/it2_la.cu:111-170
 *   kdr_la                               src/mech/user-mech/kdr_la.cu:67-118
 *   sca_la (GLOBALs vshift, tadj)        src/mech/user-mech/sca_la.cu:95-160
 *   Ca                                   src/mech/user-mech/Ca.cu
 *   shl1_lr, kvs1_lr, irk_lr, egl36_lr,  src/mech/worm-lr-mech/<name>.cu (setparames,
 *   shk1_lr, egl2_lr, cca1_lr, egl19_lr, current, state): i = w ik_tmp; the LRDS
 *   unc2_lr (calcium: i into ica),
 *   kcnl_lr (gate from cai), nca_lr (no gate),
 *   kqt3_lr (k_ion's ek; mf, ms start at 0)
 *                                        shadow gates (m_dm, ...) never reach v and
 *                                        are not carried
 *   cainternm_lr                         src/mech/worm-lr-mech/cainternm_lr.cu (Newton
 *                                        solve of the implicit calcium update)
 *   shl1, kvs1, irk, egl36, shk1, egl2,  src/mech/worm-mech/<name>.cu: the worm-lr
 *   cca1, egl19, unc2 (calcium: i into
 *   ica, erev 60 mV)
 *                                        gates with the kinetics hard-coded in
 *                                        setparames (kvs1: GLOBALs), current
 *                                        gb ... (v + 80), x + (1 - exp(-dt / tau))
 *                                        (inf - x) (kvs1: exp(dt (-1 / tau)))
 * through MechTemp's finite-difference current (mech_template.cuh:589-648)
 * and the state phase order of nonvint_cpu (simulate.cpp:784-852: mechanisms
 * that write an ion in their state update first, then the others in type
 * order).  Mechanism types follow the network mechanisms, in the order of the
 * hxo_lib tables.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "hx_oracle.h"
#include "hx_oracle_lib.h"

#define FD_EPS 0.001

static const int NPAR[HXO_LIB_NTYPE] = {1, 1, 4, 4, 1, 1, 1, 1, 1, 5, 1, 2, 1, 11, 6, 5, 16, 1, 5, 1,
                                        22, 16, 12, 9, 15, 10, 16, 29, 19, 6, 3, 29, 4,
                                        1, 13, 1, 1, 1, 1, 1, 1, 1};
static const int NST[HXO_LIB_NTYPE] = {0, 0, 0, 0, 2, 2, 1, 2, 2, 2, 2, 1, 1, 1, 1, 1, 2, 1, 2, 2,
                                       3, 2, 1, 3, 2, 1, 2, 2, 2, 1, 0, 4, 0,
                                       3, 2, 1, 3, 2, 1, 2, 2, 2};

struct hxo_libstate {
    double* st[HXO_LIB_NTYPE]; /* n x NST per table */
    double *cai, *eca, *ica;   /* per ca_ion instance */
    double *ena, *ek;          /* per na_ion / k_ion instance */
    int *na_of, *k_of, *ca_of; /* node -> ion instance, -1 if none */
};

/* units.h:18-24 (2018 CODATA) and eion.cuh:38-56 */
static const double kFaraday = 1.602176634e-19 * 6.02214076e+23;
static const double kGas = 1.380649e-23 * 6.02214076e+23;

static double ktf(double celsius) { return 1000. * kGas * (celsius + 273.15) / kFaraday; }

static double nernst(double ci, double co, double z, double celsius) {
    if (z == 0) return 0.;
    if (ci <= 0.) return 1e6;
    if (co <= 0.) return -1e6;
    return ktf(celsius) / z * log(co / ci);
}

static double qt23(void) { return pow(2.3, ((34.0 - 21.0) / 10.0)); }

/* cnexp update of NaTg, Nap_Et2, SKv3_1, SK_E2, Im, K_Pst, K_Tst, Ca_LVAst */
static double cnexp(double x, double inf, double tau, double dt) {
    return x + (1.0 - exp(dt * (-1.0 / tau))) * (-(inf / tau) / (-1.0 / tau) - x);
}

/* ------------------------------------------------------------------ rates */
static void natg_rates(double v, const double* p, double r[4]) {
    const double qt = qt23();
    const double vshifth = p[1], vshiftm = p[2], slopeh = p[3], slopem = p[4];
    double v_m = v;
    if (v_m == -38.0) v_m = v_m + 0.0001;
    const double mA = (0.182 * (v_m - (-38.0 + vshiftm))) / (1.0 - exp(-(v_m - (-38.0 + vshiftm)) / slopem));
    const double mB = (0.124 * (-v_m + (-38.0 + vshiftm))) / (1.0 - exp(-(-v_m + (-38.0 + vshiftm)) / slopem));
    r[1] = (1.0 / (mA + mB)) / qt;
    r[0] = mA / (mA + mB);
    double v_h = v;
    if (v_h == -66.0) v_h = v_h + 0.0001;
    const double hA = (-0.015 * (v_h - (-66.0 + vshifth))) / (1.0 - exp((v_h - (-66.0 + vshifth)) / slopeh));
    const double hB = (-0.015 * (-v_h + (-66.0 + vshifth))) / (1.0 - exp((-v_h + (-66.0 + vshifth)) / slopeh));
    r[3] = (1.0 / (hA + hB)) / qt;
    r[2] = hA / (hA + hB);
}

static void nap_rates(double v, double r[4]) {
    const double qt = qt23();
    r[0] = 1.0 / (1.0 + exp((v - (-52.6)) / (-4.6)));
    double v_m = v;
    if (v_m == -38.0) v_m = v_m + 0.0001;
    const double mA = (0.182 * (v_m - (-38.0))) / (1.0 - exp(-(v_m - (-38.0)) / 6.0));
    const double mB = (0.124 * (-v_m - 38.0)) / (1.0 - exp(-(-v_m - 38.0) / 6.0));
    r[1] = 6.0 * (1.0 / (mA + mB)) / qt;
    double v_h1 = v;
    if (v_h1 == -17.0) v_h1 = v_h1 + 0.0001;
    double v_h2 = v;
    if (v_h2 == -64.4) v_h2 = v_h2 + 0.0001;
    r[2] = 1.0 / (1.0 + exp((v - (-48.8)) / 10.0));
    const double hA = -2.88e-6 * (v_h1 + 17.0) / (1.0 - exp((v_h1 + 17.0) / 4.63));
    const double hB = 6.94e-6 * (v_h2 + 64.4) / (1.0 - exp(-(v_h2 + 64.4) / 2.63));
    r[3] = (1.0 / (hA + hB)) / qt;
}

static void kpst_rates(double v_param, double r[4]) {
    const double qt = qt23();
    const double v = v_param + 10.0;
    r[0] = (1.0 / (1.0 + exp(-(v + 1.0) / 12.0)));
    if (v < -50.0)
        r[1] = (1.25 + 175.03 * exp(-v * (-0.026))) / qt;
    else
        r[1] = ((1.25 + 13.0 * exp(-v * 0.026))) / qt;
    r[2] = 1.0 / (1.0 + exp(-(v + 54.0) / (-11.0)));
    r[3] = (360.0 + (1010.0 + 24.0 * (v + 55.0)) * exp(-pow(((v + 75.0) / 48.0), 2.0))) / qt;
}

static void ktst_rates(double v_param, double r[4]) {
    const double qt = qt23();
    const double v = v_param + 10.0;
    r[0] = 1.0 / (1.0 + exp(-(v + 0.0) / 19.0));
    r[1] = (0.34 + 0.92 * exp(-pow(((v + 71.0) / 59.0), 2.0))) / qt;
    r[2] = 1.0 / (1.0 + exp(-(v + 66.0) / (-10.0)));
    r[3] = (8.0 + 49.0 * exp(-pow(((v + 73.0) / 23.0), 2.0))) / qt;
}

static void calva_rates(double v_param, double r[4]) {
    const double qt = qt23();
    const double v = v_param + 10.0;
    r[0] = 1.0 / (1.0 + exp((v - (-30.0)) / (-6.0)));
    r[1] = (5.0 + 20.0 / (1.0 + exp((v - (-25.0)) / 5.0))) / qt;
    r[2] = 1.0 / (1.0 + exp((v - (-80.0)) / 6.4));
    r[3] = (20.0 + 50.0 / (1.0 + exp((v - (-40.0)) / 7.0))) / qt;
}

static double cahva_vtrap(double x, double y) {
    if (fabs(x / y) < 1e-6) return y * (1.0 - x / y / 2.0);
    return x / (exp(x / y) - 1.0);
}

static void cahva_rates(double v, double r[4]) {
    const double mA = 0.055 * cahva_vtrap(-27.0 - v, 3.8);
    const double mB = 0.94 * exp((-75.0 - v) / 17.0);
    r[0] = mA / (mA + mB);
    r[1] = 1.0 / (mA + mB);
    const double hA = 0.000457 * exp((-13.0 - v) / 50.0);
    const double hB = 0.0065 / (exp((-v - 15.0) / 28.0) + 1.0);
    r[2] = hA / (hA + hB);
    r[3] = 1.0 / (hA + hB);
}

static void im_rates(double v, double r[2]) {
    const double qt = qt23();
    const double mA = 3.3e-3 * exp(2.5 * 0.04 * (v - (-35.0)));
    const double mB = 3.3e-3 * exp(-2.5 * 0.04 * (v - (-35.0)));
    r[0] = mA / (mA + mB);
    r[1] = (1.0 / (mA + mB)) / qt;
}

static void skv31_rates(double v, double r[2]) {
    r[0] = 1.0 / (1.0 + exp((v - 18.700) / (-9.700)));
    r[1] = 0.2 * 20.0 / (1.0 + exp((v - (-46.560)) / (-44.140)));
}

/* hd_la.cu:86-104: p = ghdbar, vhalfl, tau, ehd, kl, vhalft, a0t, zetat, gmt, q10, qtl */
static void hdla_rate(double v, const double* p, double celsius, double r[2]) {
    const double vhalfl = p[1], tau = p[2], kl = p[4], vhalft = p[5], a0t = p[6], zetat = p[7], gmt = p[8];
    const double q10 = p[9], qtl = p[10];
    double a, qt;
    qt = pow(q10, ((celsius - 33.0) / 10.0));
    a = exp(0.0378 * zetat * (v - vhalft));
    r[0] = 1.0 / (1.0 + exp(-(v - vhalfl) / kl));
    r[1] = tau * exp(0.0378 * zetat * gmt * (v - vhalft)) / (qtl * qt * a0t * (1.0 + a));
}

/* km_la.cu:97-115: p = gbar, Ra, Rb, tha, qa, tadj; r = ninf, ntau, nexp */
static void kmla_trates(double v, const double* p, double dt, double r[3]) {
    const double Ra = p[1], Rb = p[2], tha = p[3], qa = p[4], tadj = p[5];
    const double a = Ra * (v - tha) / (1.0 - exp(-(v - tha) / qa));
    const double b = -Rb * (v - tha) / (1.0 - exp((v - tha) / qa));
    r[1] = 1.0 / (a + b);
    r[0] = a * r[1];
    const double tinc = -dt * tadj;
    r[2] = 1.0 - exp(tinc / r[1]);
}

/* kca_la.cu:100-110: p = gbar, Ra, Rb, caix, tadj; r = ninf, ntau, nexp */
static void kcala_rates(double cai, const double* p, double dt, double r[3]) {
    const double Ra = p[1], Rb = p[2], caix = p[3], tadj = p[4];
    const double a = Ra * pow(cai, caix);
    const double b = Rb;
    r[1] = 1.0 / (a + b);
    r[0] = a * r[1];
    const double tinc = -dt * tadj;
    r[2] = 1.0 - exp(tinc / r[1]);
}

/* it2_la.cu:111-130 at v_ = v + vshift: r = minf, mexp, hinf, hexp */
static void it2la_trates(double v_, const double* p, double dt, double r[4]) {
    const double v12m = p[2], vwm = p[3], v12h = p[4], vwh = p[5], am = p[6], ah = p[7], vm1 = p[8], vm2 = p[9];
    const double vh1 = p[10], vh2 = p[11], wm1 = p[12], wm2 = p[13], wh1 = p[14], wh2 = p[15];
    const double minf = 1.0 / (1.0 + exp(-(v_ + v12m) / vwm));
    const double hinf = 1.0 / (1.0 + exp((v_ + v12h) / vwh));
    const double mtau = (am + 1.0 / (exp((v_ + vm1) / wm1) + exp(-(v_ + vm2) / wm2)));
    const double htau = (ah + 1.0 / (exp((v_ + vh1) / wh1) + exp(-(v_ + vh2) / wh2)));
    const double tinc = -dt;
    r[0] = minf;
    r[1] = 1.0 - exp(tinc / mtau);
    r[2] = hinf;
    r[3] = 1.0 - exp(tinc / htau);
}

/* kdr_la.cu:67-77 (settables): r = minf, mtau */
static void kdrla_settables(double v, double r[2]) {
    r[0] = 1.0 / (1.0 + exp((-v - 29.5) / 10.0));
    if (v < -10.0)
        r[1] = 0.25 + 4.35 * exp((v + 10.0) / 10.0);
    else
        r[1] = 0.25 + 4.35 * exp((-v - 10.0) / 10.0);
}

/* sca_la.cu:95-125 at vm = v + vshift: p = gbar, inactF, actF, vshift, tadj;
 * r = minf, mexp, hinf, hexp */
static void scala_trates(double vm, const double* p, double dt, double r[4]) {
    const double inactF = p[1], actF = p[2], tadj = p[4];
    double a, b;
    a = 0.055 * (-27.0 - vm) / (exp((-27.0 - vm) / 3.8) - 1.0) / actF;
    b = 0.94 * exp((-75.0 - vm) / 17.0) / actF;
    const double mtau = 1.0 / (a + b);
    const double minf = a * mtau;
    a = 0.000457 * exp((-13.0 - vm) / 50.0) / inactF;
    b = 0.0065 / (exp((-vm - 15.0) / 28.0) + 1.0) / inactF;
    const double htau = 1.0 / (a + b);
    const double hinf = a * htau;
    const double tinc = -dt * tadj;
    r[0] = minf;
    r[1] = 1.0 - exp(tinc / mtau);
    r[2] = hinf;
    r[3] = 1.0 - exp(tinc / htau);
}

/* Ca.cu rates (volt == -27 moved by 1e-4); r = mInf, mTau, hInf, hTau */
static void ca_rates(double volt, double r[4]) {
    if (volt == -27.0) volt = volt + 0.0001;
    const double mA = (0.055 * (-27.0 - volt)) / (exp((-27.0 - volt) / 3.8) - 1.0);
    const double mB = (0.94 * exp((-75.0 - volt) / 17.0));
    r[0] = mA / (mA + mB);
    r[1] = 1.0 / (mA + mB);
    const double hA = (0.000457 * exp((-13.0 - volt) / 50.0));
    const double hB = (0.0065 / (exp((-volt - 15.0) / 28.0) + 1.0));
    r[2] = hA / (hA + hB);
    r[3] = 1.0 / (hA + hB);
}

/* worm-lr setparames at v: r = inf0, tau0, inf1, tau1, inf2, tau2 (the
 * time constants the cnexp update uses).  g = the GLOBALs (p + 4). */
static void worm_gates(int t, double v, const double* g, double r[8]) {
    switch (t) {
        case HXO_SHL1_LR: { /* vhm ka vhh ki atm btm ctm dtm etm ftm athf bthf cthf dthf aths bths cths dths */
            const double minf = 1.0 / (1.0 + exp(-(v - g[0]) / g[1]));
            const double hfinf = 1.0 / (1.0 + exp((v - g[2]) / g[3]));
            const double hsinf = 1.0 / (1.0 + exp((v - g[2]) / g[3]));
            const double tm = g[4] / (exp(-(v - g[5]) / g[6]) + exp((v - g[7]) / g[8])) + g[9];
            const double thf = g[10] / (1.0 + exp((v - g[11]) / g[12])) + g[13];
            const double ths = g[14] / (1.0 + exp((v - g[15]) / g[16])) + g[17];
            r[0] = minf; r[1] = tm * 0.4;
            r[2] = hfinf; r[3] = thf * 0.08;
            r[4] = hsinf; r[5] = ths * 0.3;
            break;
        }
        case HXO_KVS1_LR: { /* vhm ka vhh ki atm btm ctm dtm ath bth cth dth */
            r[0] = 1.0 / (1.0 + exp(-(v - g[0]) / g[1]));
            r[2] = 1.0 / (1.0 + exp((v - g[2]) / g[3]));
            r[1] = g[4] / (1.0 + exp((v - g[5]) / g[6])) + g[7];
            r[3] = g[8] / (1.0 + exp((v - g[9]) / g[10])) + g[11];
            break;
        }
        case HXO_IRK_LR: { /* vhm ka atm btm ctm dtm etm ftm */
            r[0] = 1.0 / (1.0 + exp((v - g[0]) / g[1]));
            r[1] = g[2] / (exp(-(v - g[3]) / g[4]) + exp((v - g[5]) / g[6])) + g[7];
            break;
        }
        case HXO_EGL36_LR: { /* vhm ka atms atmm atmf */
            r[0] = 1.0 / (1.0 + exp(-(v - g[0]) / g[1]));
            r[2] = 1.0 / (1.0 + exp(-(v - g[0]) / g[1]));
            r[4] = 1.0 / (1.0 + exp(-(v - g[0]) / g[1]));
            r[1] = g[4]; /* tmf = atmf */
            r[3] = g[3]; /* tmm = atmm */
            r[5] = g[2]; /* tms = atms */
            break;
        }
        case HXO_SHK1_LR: { /* vhm ka vhh ki atm btm ctm dtm etm ftm ath */
            r[0] = 1.0 / (1.0 + exp(-(v - g[0]) / g[1]));
            r[2] = 1.0 / (1.0 + exp((v - g[2]) / g[3]));
            r[1] = g[4] / (exp(-(v - g[5]) / g[6]) + exp((v - g[7]) / g[8])) + g[9];
            r[3] = g[10];
            break;
        }
        case HXO_EGL2_LR: { /* vhm ka atm btm ctm dtm */
            r[0] = 1.0 / (1.0 + exp(-(v - g[0]) / g[1]));
            r[1] = g[2] / (1.0 + exp((v - g[3]) / g[4])) + g[5];
            break;
        }
        case HXO_CCA1_LR: { /* vhm ka vhh ki atm btm ctm dtm ath bth cth dth */
            r[0] = 1.0 / (1.0 + exp(-(v - g[0]) / g[1]));
            r[2] = 1.0 / (1.0 + exp((v - g[2]) / g[3]));
            r[1] = g[4] / (1.0 + exp(-(v - g[5]) / g[6])) + g[7];
            r[3] = g[8] / (1.0 + exp((v - g[9]) / g[10])) + g[11];
            break;
        }
        case HXO_EGL19_LR: { /* vhm ka vhh ki vhhb kib ahinf bhinf chinf dhinf atm btm ctm dtm etm ftm gtm
                                ath bth cth dth eth fth gth hth */
            r[0] = 1.0 / (1.0 + exp(-(v - g[0]) / g[1]));
            r[2] = (g[6] / (1.0 + exp(-(v - g[2]) / g[3])) + g[7]) * (g[8] / (1.0 + exp((v - g[4]) / g[5])) + g[9]);
            r[1] = g[10] * exp(-pow((v - g[11]) / g[12], 2.0)) + g[13] * exp(-pow((v - g[14]) / g[15], 2.0)) + g[16];
            r[3] = g[17] * ((g[18] / (1.0 + exp((v - g[19]) / g[20]))) + (g[21] / (1.0 + exp((v - g[22]) / g[23]))) +
                            g[24]);
            break;
        }
        case HXO_UNC2_LR: { /* vhm ka vhh ki atm btm ctm dtm etm ath bth cth dth eth fth */
            r[0] = 1.0 / (1.0 + exp(-(v - g[0]) / g[1]));
            r[2] = 1.0 / (1.0 + exp((v - g[2]) / g[3]));
            r[1] = g[4] / (exp(-(v - g[5]) / g[6]) + exp((v - g[5]) / g[7])) + g[8];
            r[3] = g[9] / (1.0 + exp(-(v - g[10]) / g[11])) + g[12] / (1.0 + exp((v - g[13]) / g[14]));
            break;
        }
        case HXO_KQT3_LR: { /* vhm ka vhw kiw aw bw vhs kis as bs atmf btmf ctmf atms btms ctms dtms etms ftms
                               gtms atw btw ctw dtw ats; gates mf, ms (both minf), ww, s */
            const double minf = 1.0 / (1.0 + exp(-(v - g[0]) / g[1]));
            r[0] = minf;
            r[1] = g[10] / (1.0 + pow((v + g[11]) / g[12], 2.0));
            r[2] = minf;
            r[3] = g[13] + g[14] / (1.0 + pow(10.0, -g[15] * (g[16] - v))) +
                   g[17] / (1.0 + pow(10.0, -g[18] * (g[19] + v)));
            r[4] = g[4] + g[5] / (1.0 + exp((v - g[2]) / g[3]));
            r[5] = g[20] + g[21] / (1.0 + pow((v - g[22]) / g[23], 2.0));
            r[6] = g[8] + g[9] / (1.0 + exp((v - g[6]) / g[7]));
            r[7] = g[24];
            break;
        }
    }
}

/* worm-mech channels: the worm-lr type whose gates they share and their
 * kinetics constants (setparames' locals, in the worm-lr GLOBAL order) */
static int worm_lr_of(int t) {
    switch (t) {
        case HXO_SHL1: return HXO_SHL1_LR;
        case HXO_KVS1: return HXO_KVS1_LR;
        case HXO_IRK: return HXO_IRK_LR;
        case HXO_EGL36: return HXO_EGL36_LR;
        case HXO_SHK1: return HXO_SHK1_LR;
        case HXO_EGL2: return HXO_EGL2_LR;
        case HXO_CCA1: return HXO_CCA1_LR;
        case HXO_EGL19: return HXO_EGL19_LR;
        case HXO_UNC2: return HXO_UNC2_LR;
    }
    return -1;
}
static int worm_mech_ca(int t) { return t == HXO_CCA1 || t == HXO_EGL19 || t == HXO_UNC2; }
static const double kShl1K[18] = {11.2, 14.1, -33.1, 8.3, 13.8, -17.5, 12.9, -3.7, 6.5,
                                  1.9, 539.2, -28.2, 4.9, 27.3, 8422.0, -37.7, 6.4, 118.9};
static const double kIrkK[8] = {-82.0, 13.0, 17.1, -17.8, 20.3, -43.4, 11.2, 3.8};
static const double kEgl36K[5] = {63.0, 28.5, 355.0, 63.0, 13.0};
static const double kShk1K[11] = {20.4, 7.7, -7.0, 5.8, 26.6, -33.7, 15.8, -33.7, 15.4, 2.0, 1400.0};
static const double kEgl2K[6] = {-6.9, 14.9, 1845.8, -122.6, 13.8, 1517.74};
static const double kCca1K[12] = {-43.32, 7.6, -58.0, 7.0, 40.0, -62.5, -12.6, 0.7, 280.0, -60.7, 8.5, 19.8};
static const double kEgl19K[25] = {5.6, 7.5, 24.9, 12.0, -20.5, 8.1, 1.43, 0.14, 5.96, 0.60, 2.9, 5.2, 6.0,
                                   1.9, 1.4, 30.0, 2.3, 0.4, 44.6, -23.0, 5.0, 36.4, 28.7, 3.7, 43.1};
static const double kUnc2K[15] = {-12.2, 4.0, -52.5, 5.6, 1.5, -8.2, 9.1, 15.4, 0.1, 83.8, 52.9, -3.5, 72.1, 23.9, -3.6};
static const double* worm_consts(int t, const double* p) {
    switch (t) {
        case HXO_SHL1: return kShl1K;
        case HXO_KVS1: return p + 1; /* GLOBALs vhm_kvs1 .. dth_kvs1 */
        case HXO_IRK: return kIrkK;
        case HXO_EGL36: return kEgl36K;
        case HXO_SHK1: return kShk1K;
        case HXO_EGL2: return kEgl2K;
        case HXO_CCA1: return kCca1K;
        case HXO_EGL19: return kEgl19K;
        case HXO_UNC2: return kUnc2K;
    }
    return NULL;
}

static int is_worm(int t) { return (t >= HXO_SHL1_LR && t <= HXO_NCA_LR) || t == HXO_KQT3_LR; }

static double sk_zinf(double ca) {
    double ca_safe = ca;
    if (ca_safe < 1e-7) ca_safe = ca_safe + 1e-07;
    return 1.0 / (1.0 + pow((0.00043 / ca_safe), 4.8));
}

/* ------------------------------------------------------------------ current */
/* I(v) of one channel instance (the value current_single_node returns) */
static double chan_current(int t, double v, const double* p, const double* s, double erev) {
    switch (t) {
        case HXO_CA_HVA: {
            const double g = p[0] * s[0] * s[0] * s[1];
            return g * (v - erev);
        }
        case HXO_CA_LVAST:
        case HXO_K_PST:
            return p[0] * s[0] * s[0] * s[1] * (v - erev);
        case HXO_K_TST:
            return p[0] * pow(s[0], 4.0) * s[1] * (v - erev);
        case HXO_NATG:
        case HXO_NAP_ET2:
            return p[0] * s[0] * s[0] * s[0] * s[1] * (v - erev);
        case HXO_IM:
        case HXO_SKV3_1:
        case HXO_SK_E2:
            return p[0] * s[0] * (v - erev);
        case HXO_HD_LA: { /* ghd = ghdbar l; i = ghd (v - ehd) */
            const double ghd = p[0] * s[0];
            return ghd * (v - erev);
        }
        case HXO_KM_LA: { /* gk = tadj gbar n; ik = 1e-4 gk (v - ek) */
            const double gk = p[5] * p[0] * s[0];
            return (1e-4) * gk * (v - erev);
        }
        case HXO_KCA_LA: {
            const double gk = p[4] * p[0] * s[0];
            return (1e-4) * gk * (v - erev);
        }
        case HXO_IT2_LA: {
            const double gca = p[0] * s[0] * s[0] * s[1];
            return gca * (v - erev);
        }
        case HXO_KDR_LA: {
            const double m_4 = s[0] * s[0] * s[0] * s[0];
            return p[0] * m_4 * (v - erev);
        }
        case HXO_SCA_LA: {
            const double gca = p[4] * p[0] * s[0] * s[0] * s[1];
            return (1e-4) * gca * (v - erev);
        }
        case HXO_CA: {
            const double gCa = p[0] * s[0] * s[0] * s[1];
            return gCa * (v - erev);
        }
        /* worm-lr: p = w, gb, ek_tmp, ...; ik_tmp = gb ... (v - ek_tmp), i = w ik_tmp */
        case HXO_SHL1_LR: {
            const double ik_tmp = p[1] * s[0] * s[0] * s[0] * (0.7 * s[1] + 0.3 * s[2]) * (v - erev);
            return p[0] * ik_tmp;
        }
        case HXO_KVS1_LR:
        case HXO_SHK1_LR: {
            const double ik_tmp = p[1] * s[0] * s[1] * (v - erev);
            return p[0] * ik_tmp;
        }
        case HXO_IRK_LR:
        case HXO_EGL2_LR: {
            const double ik_tmp = p[1] * s[0] * (v - erev);
            return p[0] * ik_tmp;
        }
        case HXO_EGL36_LR: {
            const double ik_tmp = p[1] * (0.33 * s[0] + 0.36 * s[1] + 0.39 * s[2]) * (v - erev);
            return p[0] * ik_tmp;
        }
        case HXO_CCA1_LR: {
            const double ica_tmp = p[1] * s[0] * s[0] * s[1] * (v - erev);
            return p[0] * ica_tmp;
        }
        case HXO_EGL19_LR:
        case HXO_UNC2_LR: {
            const double ica_tmp = p[1] * s[0] * s[1] * (v - erev);
            return p[0] * ica_tmp;
        }
        case HXO_KCNL_LR: {
            const double ik_tmp = p[1] * s[0] * (v - erev);
            return p[0] * ik_tmp;
        }
        case HXO_NCA_LR: {
            const double ina_tmp = p[1] * (v - erev);
            return p[0] * ina_tmp;
        }
        case HXO_KQT3_LR: {
            const double ik_tmp = p[1] * (0.3 * s[0] + 0.7 * s[1]) * s[2] * s[3] * (v - erev);
            return p[0] * ik_tmp;
        }
        /* worm-mech: gb ... (v + 80.0), erev = -80 (v - (-80) == v + 80 exactly) */
        case HXO_SHL1:
            return p[0] * s[0] * s[0] * s[0] * (0.7 * s[1] + 0.3 * s[2]) * (v - erev);
        case HXO_KVS1:
        case HXO_SHK1:
            return p[0] * s[0] * s[1] * (v - erev);
        case HXO_IRK:
        case HXO_EGL2:
            return p[0] * s[0] * (v - erev);
        case HXO_EGL36:
            return p[0] * (0.33 * s[0] + 0.36 * s[1] + 0.39 * s[2]) * (v - erev);
        case HXO_CCA1: /* gb m m h (v - 60.0) */
            return p[0] * s[0] * s[0] * s[1] * (v - erev);
        case HXO_EGL19:
        case HXO_UNC2:
            return p[0] * s[0] * s[1] * (v - erev);
        default:
            return 0.0;
    }
}

/* 0: na, 1: k, 2: ca (the ion whose erev a channel reads and current it writes),
 * 3: none (hd_la: its own reversal potential ehd, no ion current), 4: its own
 * reversal potential ek_tmp (the worm-lr channels; their k current is not read;
 * kqt3_lr reads k_ion's ek), 5: hard-coded (the worm-mech channels: -80 mV,
 * the calcium ones 60 mV) */
static int chan_ion(int t) {
    if (t == HXO_KQT3_LR) return 1;
    if (worm_lr_of(t) >= 0) return 5;
    if (is_worm(t)) return 4;
    switch (t) {
        case HXO_HD_LA:
            return 3;
        case HXO_NATG:
        case HXO_NAP_ET2:
            return 0;
        case HXO_CA_HVA:
        case HXO_CA_LVAST:
        case HXO_IT2_LA:
        case HXO_SCA_LA:
        case HXO_CA:
            return 2;
        default:
            return 1;
    }
}

/* ------------------------------------------------------------------ lifecycle */
int hxo_lib_alloc(const hxo_group* g, struct hxo_libstate** out) {
    *out = NULL;
    if (!g->lib) return 0;
    struct hxo_libstate* L = (struct hxo_libstate*)calloc(1, sizeof(*L));
    if (!L) return -1;
    *out = L;
    const hxo_lib* lib = g->lib;
    for (int t = 0; t < HXO_LIB_NTYPE; t++) {
        L->st[t] = (double*)calloc((size_t)(lib->t[t].n * NST[t] + 1), sizeof(double));
        if (!L->st[t]) return -1;
    }
    const int nca = lib->t[HXO_CA_ION].n + 1;
    L->cai = (double*)calloc((size_t)nca, sizeof(double));
    L->eca = (double*)calloc((size_t)nca, sizeof(double));
    L->ica = (double*)calloc((size_t)nca, sizeof(double));
    L->ena = (double*)calloc((size_t)lib->t[HXO_NA_ION].n + 1, sizeof(double));
    L->ek = (double*)calloc((size_t)lib->t[HXO_K_ION].n + 1, sizeof(double));
    L->na_of = (int*)malloc(sizeof(int) * (size_t)g->nnode);
    L->k_of = (int*)malloc(sizeof(int) * (size_t)g->nnode);
    L->ca_of = (int*)malloc(sizeof(int) * (size_t)g->nnode);
    if (!(L->cai && L->eca && L->ica && L->ena && L->ek && L->na_of && L->k_of && L->ca_of)) return -1;
    for (int i = 0; i < g->nnode; i++) L->na_of[i] = L->k_of[i] = L->ca_of[i] = -1;
    for (int j = 0; j < lib->t[HXO_NA_ION].n; j++) L->na_of[lib->t[HXO_NA_ION].node[j]] = j;
    for (int j = 0; j < lib->t[HXO_K_ION].n; j++) L->k_of[lib->t[HXO_K_ION].node[j]] = j;
    for (int j = 0; j < lib->t[HXO_CA_ION].n; j++) L->ca_of[lib->t[HXO_CA_ION].node[j]] = j;
    return 0;
}

void hxo_lib_free(struct hxo_libstate* L) {
    if (!L) return;
    for (int t = 0; t < HXO_LIB_NTYPE; t++) free(L->st[t]);
    free(L->cai);
    free(L->eca);
    free(L->ica);
    free(L->ena);
    free(L->ek);
    free(L->na_of);
    free(L->k_of);
    free(L->ca_of);
    free(L);
}

/* erev / concentration an instance at node i reads */
static double ion_erev(const struct hxo_libstate* L, int ion, int i) {
    if (ion == 0) return L->ena[L->na_of[i]];
    if (ion == 1) return L->ek[L->k_of[i]];
    return L->eca[L->ca_of[i]];
}

/* finitialize: INITIAL blocks in type order (ions first; iontype flags:
 * na / k 0, ca 040|0100 when nernst else 0, eion.cuh:170-186) */
void hxo_lib_init(const hxo_group* g, struct hxo_libstate* L, const double* v) {
    if (!L) return;
    const hxo_lib* lib = g->lib;
    for (int j = 0; j < lib->t[HXO_NA_ION].n; j++) L->ena[j] = lib->t[HXO_NA_ION].par[j];
    for (int j = 0; j < lib->t[HXO_K_ION].n; j++) L->ek[j] = lib->t[HXO_K_ION].par[j];
    for (int j = 0; j < lib->t[HXO_CA_ION].n; j++) {
        const double* p = lib->t[HXO_CA_ION].par + 4 * j;
        L->cai[j] = p[0];
        L->eca[j] = p[3] != 0.0 ? nernst(p[0], p[1], 2.0, g->celsius) : p[2];
        L->ica[j] = 0.0;
    }
    for (int t = HXO_CA_HVA; t < HXO_LIB_NTYPE; t++) {
        const hxo_lib_table* T = &lib->t[t];
        for (int j = 0; j < T->n; j++) {
            const int i = T->node[j];
            const double* p = T->par + NPAR[t] * j;
            double* s = L->st[t] + NST[t] * j;
            double r[4] = {0.0, 0.0, 0.0, 0.0};
            switch (t) {
                case HXO_CA_HVA: cahva_rates(v[i], r); break;
                case HXO_CA_LVAST: calva_rates(v[i], r); break;
                case HXO_K_PST: kpst_rates(v[i], r); break;
                case HXO_K_TST: ktst_rates(v[i], r); break;
                case HXO_NATG: natg_rates(v[i], p, r); break;
                case HXO_NAP_ET2: nap_rates(v[i], r); break;
                case HXO_IM: im_rates(v[i], r); break;
                case HXO_SKV3_1: skv31_rates(v[i], r); break;
                case HXO_SK_E2: r[0] = sk_zinf(L->cai[L->ca_of[i]]); break;
                case HXO_HD_LA: hdla_rate(v[i], p, g->celsius, r); break;
                case HXO_KM_LA: kmla_trates(v[i], p, g->dt, r); break;
                case HXO_KCA_LA: kcala_rates(L->cai[L->ca_of[i]], p, g->dt, r); break;
                case HXO_IT2_LA: it2la_trates(v[i] + p[1], p, g->dt, r); break;
                case HXO_KDR_LA: kdrla_settables(v[i], r); r[0] = 0.0; break; /* m = minf; m = 0.0 */
                case HXO_SCA_LA: scala_trates(v[i] + p[3], p, g->dt, r); break;
                case HXO_CA: ca_rates(v[i], r); break;
            }
            if (t == HXO_KCNL_LR) { /* minf = cai / (kca + cai) */
                const double cai = L->cai[L->ca_of[i]];
                s[0] = cai / (p[3] + cai);
                continue;
            }
            if (t == HXO_NCA_LR || t == HXO_CAINTERNM_LR) continue; /* no INITIAL of a state */
            if (worm_lr_of(t) >= 0) { /* every gate at its steady state */
                double wr[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                worm_gates(worm_lr_of(t), v[i], worm_consts(t, p), wr);
                for (int q = 0; q < NST[t]; q++) s[q] = wr[2 * q];
                continue;
            }
            if (is_worm(t)) { /* every gate at its steady state (kqt3_lr: mf = ms = 0) */
                double wr[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                worm_gates(t, v[i], p + 4, wr);
                for (int q = 0; q < NST[t]; q++) s[q] = (t == HXO_KQT3_LR && q < 2) ? 0.0 : wr[2 * q];
                continue;
            }
            s[0] = r[0];
            if (NST[t] == 2) s[1] = r[2];
        }
    }
}

/* current phase: ion mechanisms (cur = 0, Nernst erev) then the channels in
 * type order, each through the FD conductance of MechTemp::current_cpu */
void hxo_lib_current(const hxo_group* g, struct hxo_libstate* L, const double* v, double* rhs, double* d) {
    if (!L) return;
    const hxo_lib* lib = g->lib;
    for (int j = 0; j < lib->t[HXO_CA_ION].n; j++) {
        const double* p = lib->t[HXO_CA_ION].par + 4 * j;
        L->ica[j] = 0.0;
        if (p[3] != 0.0) L->eca[j] = nernst(L->cai[j], p[1], 2.0, g->celsius);
    }
    for (int t = HXO_CA_HVA; t < HXO_LIB_NTYPE; t++) {
        const hxo_lib_table* T = &lib->t[t];
        const int ion = chan_ion(t);
        if (t == HXO_CAINTERNM_LR) continue; /* no current */
        for (int j = 0; j < T->n; j++) {
            const int i = T->node[j];
            const double* p = T->par + NPAR[t] * j;
            const double* s = L->st[t] + NST[t] * j;
            const double e = ion == 3   ? p[3]
                             : ion == 5 ? (worm_mech_ca(t) ? 60.0 : -80.0)
                             : t == HXO_KCNL_LR ? p[5]
                             : ion == 4 ? p[2]
                                        : ion_erev(L, ion, i);
            double gg = chan_current(t, v[i] + 0.001, p, s, e);
            const double r = chan_current(t, v[i], p, s, e);
            if (ion == 2 || (t >= HXO_CCA1_LR && t <= HXO_UNC2_LR) || worm_mech_ca(t))
                L->ica[L->ca_of[i]] += r; /* worm-lr calcium: i into ica */
            gg = (gg - r) / FD_EPS;
            rhs[i] -= r;
            d[i] += gg;
        }
    }
}

/* state phase, part 1: mechanisms that write an ion in their state update
 * (CaDynamics_E2, then cainternm_lr), in type order */
void hxo_lib_state_ion(const hxo_group* g, struct hxo_libstate* L, const double* v) {
    if (!L) return;
    const hxo_lib_table* T = &g->lib->t[HXO_CADYN];
    const double dt = g->dt;
    for (int j = 0; j < T->n; j++) {
        const int c = L->ca_of[T->node[j]];
        const double* p = T->par + 4 * j;
        const double FARADAY = 96485.3321233100184;
        const double gamma_val = p[0], decay_val = p[1], depth_val = p[2], minCai_val = p[3];
        const double ica_val = L->ica[c], cai_val = L->cai[c];
        const double drive_ica = -(10000.0) * (ica_val * gamma_val) / (2.0 * FARADAY * depth_val);
        const double exp_factor = exp(dt * (-1.0 / decay_val));
        const double steady_term = -(drive_ica - (-minCai_val) / decay_val) / (-1.0 / decay_val);
        L->cai[c] = cai_val + (1.0 - exp_factor) * (steady_term - cai_val);
    }
    /* cainternm_lr.cu state_single_node: Newton iterations on
     * F(c) = (-c + alpha(c) dt + cai_old) / dt, alpha = -f ica 1e6 / (2 F vcell)
     * - (c - caeq) / tca below 60 mV, -(c - caeq) / tca above; p = vcell, f,
     * tca, caeq */
    const hxo_lib_table* C = &g->lib->t[HXO_CAINTERNM_LR];
    for (int j = 0; j < C->n; j++) {
        const int i = C->node[j], c = L->ca_of[i];
        const double* p = C->par + 4 * j;
        const double FARADAY = 96485.0;
        const double ica = L->ica[c], old_cai = L->cai[c];
        double current_cai = old_cai;
        for (int iter = 0; iter < 50; iter++) {
            double alpha_val;
            if (v[i] <= 60.0)
                alpha_val = (-p[1] * ica * pow(10.0, 6.0) / (2.0 * FARADAY * p[0])) - ((current_cai - p[3]) / p[2]);
            else
                alpha_val = -(current_cai - p[3]) / p[2];
            const double F = (-current_cai + alpha_val * dt + old_cai) / dt;
            const double dalpha_dcai = -1.0 / p[2];
            const double J = (-1.0 + dalpha_dcai * dt) / dt;
            const double delta = F / J;
            current_cai -= delta;
            const double change = (fabs(old_cai) > 1e-8) ? fabs(delta / old_cai) : fabs(delta);
            if (change <= 1e-6 && fabs(F) <= 1e-8) break;
        }
        L->cai[c] = current_cai;
    }
}

/* state phase, part 2: the channels in type order at the updated v */
void hxo_lib_state(const hxo_group* g, struct hxo_libstate* L, const double* v) {
    if (!L) return;
    const hxo_lib* lib = g->lib;
    const double dt = g->dt;
    for (int t = HXO_CA_HVA; t < HXO_LIB_NTYPE; t++) {
        const hxo_lib_table* T = &lib->t[t];
        for (int j = 0; j < T->n; j++) {
            const int i = T->node[j];
            const double* p = T->par + NPAR[t] * j;
            double* s = L->st[t] + NST[t] * j;
            double r[4] = {0.0, 0.0, 0.0, 0.0};
            if (t == HXO_CA_HVA) {
                cahva_rates(v[i], r);
                s[0] = s[0] + (1.0 - exp(-dt / r[1])) * (r[0] - s[0]);
                s[1] = s[1] + (1.0 - exp(-dt / r[3])) * (r[2] - s[1]);
                continue;
            }
            if (t == HXO_SK_E2) {
                const double zTau = p[1];
                s[0] = cnexp(s[0], sk_zinf(L->cai[L->ca_of[i]]), zTau, dt);
                continue;
            }
            if (t == HXO_HD_LA) {
                hdla_rate(v[i], p, g->celsius, r);
                s[0] = s[0] + (1.0 - exp(-dt / r[1])) * (r[0] - s[0]);
                continue;
            }
            if (t == HXO_KM_LA) {
                kmla_trates(v[i], p, dt, r);
                s[0] = s[0] + r[2] * (r[0] - s[0]);
                continue;
            }
            if (t == HXO_KCA_LA) {
                kcala_rates(L->cai[L->ca_of[i]], p, dt, r);
                s[0] = s[0] + r[2] * (r[0] - s[0]);
                continue;
            }
            if (t == HXO_IT2_LA) {
                it2la_trates(v[i] + p[1], p, dt, r);
                s[0] = s[0] + r[1] * (r[0] - s[0]);
                s[1] = s[1] + r[3] * (r[2] - s[1]);
                continue;
            }
            if (t == HXO_KCNL_LR) { /* at the state phase's cai; tm = a */
                const double cai = L->cai[L->ca_of[i]];
                const double inf = cai / (p[3] + cai), tau = p[4];
                s[0] = s[0] + (1.0 - exp(dt * ((-1.0) / tau))) * (-(inf / tau) / ((-1.0) / tau) - s[0]);
                continue;
            }
            if (t == HXO_NCA_LR || t == HXO_CAINTERNM_LR) continue; /* no STATE of its own */
            if (worm_lr_of(t) >= 0) {
                double wr[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                worm_gates(worm_lr_of(t), v[i], worm_consts(t, p), wr);
                for (int q = 0; q < NST[t]; q++) {
                    const double inf = wr[2 * q], tau = wr[2 * q + 1];
                    if (t == HXO_KVS1)
                        s[q] = s[q] + (1.0 - exp(dt * (-1.0 / tau))) * (inf - s[q]);
                    else
                        s[q] = s[q] + (1.0 - exp(-dt / tau)) * (inf - s[q]);
                }
                continue;
            }
            if (is_worm(t)) { /* x + (1 - exp(dt ((-1) / tau))) (-(inf / tau) / ((-1) / tau) - x) */
                double wr[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                worm_gates(t, v[i], p + 4, wr);
                for (int q = 0; q < NST[t]; q++) {
                    const double inf = wr[2 * q], tau = wr[2 * q + 1];
                    s[q] = s[q] + (1.0 - exp(dt * ((-1.0) / tau))) * (-(inf / tau) / ((-1.0) / tau) - s[q]);
                }
                continue;
            }
            if (t == HXO_SCA_LA) {
                scala_trates(v[i] + p[3], p, dt, r);
                s[0] = s[0] + r[1] * (r[0] - s[0]);
                s[1] = s[1] + r[3] * (r[2] - s[1]);
                continue;
            }
            if (t == HXO_CA) {
                ca_rates(v[i], r);
                s[0] = s[0] + (1.0 - exp(-dt / r[1])) * (r[0] - s[0]);
                s[1] = s[1] + (1.0 - exp(-dt / r[3])) * (r[2] - s[1]);
                continue;
            }
            if (t == HXO_KDR_LA) {
                kdrla_settables(v[i], r);
                s[0] = s[0] + (1.0 - exp(-dt / r[1])) * (r[0] - s[0]);
                continue;
            }
            switch (t) {
                case HXO_CA_LVAST: calva_rates(v[i], r); break;
                case HXO_K_PST: kpst_rates(v[i], r); break;
                case HXO_K_TST: ktst_rates(v[i], r); break;
                case HXO_NATG: natg_rates(v[i], p, r); break;
                case HXO_NAP_ET2: nap_rates(v[i], r); break;
                case HXO_IM: im_rates(v[i], r); break;
                case HXO_SKV3_1: skv31_rates(v[i], r); break;
            }
            s[0] = cnexp(s[0], r[0], r[1], dt);
            if (NST[t] == 2) s[1] = cnexp(s[1], r[2], r[3], dt);
        }
    }
}

int hxo_lib_final(const hxo_group* g, const struct hxo_libstate* L, double* out, int cap) {
    if (!L) return 0;
    int k = 0;
    for (int t = 0; t < HXO_LIB_NTYPE; t++) {
        const int n = g->lib->t[t].n;
        if (t == HXO_CA_ION) {
            if (k + n > cap) return -2;
            memcpy(out + k, L->cai, sizeof(double) * (size_t)n);
            k += n;
        } else if (NST[t]) {
            if (k + n * NST[t] > cap) return -2;
            memcpy(out + k, L->st[t], sizeof(double) * (size_t)(n * NST[t]));
            k += n * NST[t];
        }
    }
    return k;
}
