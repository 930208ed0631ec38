// hx_mech.cuh -- device mechanism math (fp64) for the fused step kernels.
//
// hh follows src/mech/user-mech/hh_templated.cu:76-164 with the algebra of the
// cnexp update written without its redundant divisions: the reference's
//   m += (1 - exp(dt*(-1/mtau))) * ((minf/mtau)/(1/mtau) - m),  mtau = 1/(q10*(a+b))
// is computed as
//   m += (1 - exp(-dt*q10*(a+b))) * (minf - m).
// The six exponentials of the rate functions all have arguments linear in v
// with slopes 1/10, 1/18, 1/20, 1/80, so they are integer powers of one
// exponential z = exp(-(v+65)/720) times constants:
//   exp(-(v+65)/18) = z^40, exp(-(v+65)/20) = z^36, exp(-(v+65)/80) = z^9,
//   exp(-(v+40)/10) = z^72 e^2.5, exp(-(v+55)/10) = z^72 e, exp(-(v+35)/10) = z^72 e^3,
// and quotients use a Newton reciprocal.  These forms equal
// the reference's mathematically and differ by rounding only (a few 1e-14
// relative in the rates); parity is checked against the reference-order CPU
// oracle.
// The finite-difference conductance of MechTemp::current
// (mech_template.cuh:615-626) is kept: it is what the reference integrates.
#pragma once

#include <cuda_runtime.h>

namespace hx {

constexpr double kFdEps = 0.001;  // mech_template.cuh:616 and :626
constexpr double kInvFdEps = 1000.0;

// Branch-free reciprocal of a nonzero normal x (either sign): hardware
// estimate refined by two Newton-Raphson steps r <- r + r*(1 - x*r) (quadratic
// convergence from the ~2^-23 estimate to below double rounding).
__device__ __forceinline__ double rcp_nz(double x) {
    double r;
    asm("rcp.approx.ftz.f64 %0, %1;" : "=d"(r) : "d"(x));
    double e = __fma_rn(-x, r, 1.0);
    r = __fma_rn(r, e, r);
    e = __fma_rn(-x, r, 1.0);
    r = __fma_rn(r, e, r);
    return r;
}

// Steady states and rate sums (k = q10*(alpha+beta) = 1/tau) of m, h, n.
struct HHRates {
    double inf[3], k[3];
};

// e^2.5, e^3, e: the offsets of the vtrap / beta_h exponentials against z^72
constexpr double kE25 = 12.182493960703473;
constexpr double kE3 = 20.085536923187668;
constexpr double kE1 = 2.718281828459045;

// powers of z = exp(-(v+65)/720) used by the rates
struct ZPow {
    double z9, z36, z40, z72;
};

__device__ __forceinline__ ZPow zpow(double v) {
    const double z = exp(-(v + 65.0) * (1.0 / 720.0));
    const double z2 = z * z, z4 = z2 * z2, z8 = z4 * z4, z9 = z8 * z;
    const double z18 = z9 * z9, z36 = z18 * z18;
    return ZPow{z9, z36, z36 * z4, z36 * z36};
}

// Below this |u| = |x/10| the vtrap forms take exp(u) from a direct exp
// instead of the z powers (whose ~72 ulp would dominate exp(u) - 1 there), and
// the derivative's numerator from its series.
constexpr double kVtrapNear = 0.05;

// vtrap(x, 10) = x / (exp(x/10) - 1) with exp(x/10) given; the reference's
// small-argument branch (hh_templated.cu:76-85) is kept
__device__ __forceinline__ double vtrap10_e(double x, double ex) {
    const double u = x * 0.1;
    if (fabs(u) < 1e-6) return 10.0 * (1 - u * 0.5);
    if (fabs(u) < kVtrapNear) ex = exp(u);
    return x * rcp_nz(ex - 1);
}

// (exp(u) - 1 - u exp(u)) = -sum_{n>=2} (n-1) u^n / n!, for |u| < kVtrapNear
// (terms to n = 11: below double rounding there), free of the cancellation
// of the direct difference
__device__ __forceinline__ double vtrap_num_series(double u) {
    double t = 10.0 / 39916800.0;                 // n = 11: (n-1)/n!, Horner in u down to n = 2
    t = t * u + 9.0 / 3628800.0;                  // n = 10
    t = t * u + 8.0 / 362880.0;                   // n = 9
    t = t * u + 7.0 / 40320.0;                    // n = 8
    t = t * u + 6.0 / 5040.0;                     // n = 7
    t = t * u + 5.0 / 720.0;                      // n = 6
    t = t * u + 4.0 / 120.0;                      // n = 5
    t = t * u + 3.0 / 24.0;                       // n = 4
    t = t * u + 2.0 / 6.0;                        // n = 3
    t = t * u + 1.0 / 2.0;                        // n = 2
    return -(u * u) * t;
}

__device__ __forceinline__ void hh_rates(double v, double q10, HHRates& r) {
    const ZPow Z = zpow(v);
    double al, be, s;
    al = 0.1 * vtrap10_e(-(v + 40), Z.z72 * kE25);
    be = 4 * Z.z40;
    s = al + be;
    r.inf[0] = al * rcp_nz(s);
    r.k[0] = q10 * s;
    al = 0.07 * Z.z36;
    be = rcp_nz(Z.z72 * kE3 + 1);
    s = al + be;
    r.inf[1] = al * rcp_nz(s);
    r.k[1] = q10 * s;
    al = 0.01 * vtrap10_e(-(v + 55), Z.z72 * kE1);
    be = 0.125 * Z.z9;
    s = al + be;
    r.inf[2] = al * rcp_nz(s);
    r.k[2] = q10 * s;
}

// vtrap10 and its derivative in x, exp(x/10) given
__device__ __forceinline__ void vtrap10_d_e(double x, double ex, double& f, double& df) {
    const double u = x * 0.1;
    if (fabs(u) < 1e-6) {
        f = 10.0 * (1 - u * 0.5);
        df = -0.5;
    } else if (fabs(u) < kVtrapNear) {
        ex = exp(u);
        f = x * rcp_nz(ex - 1);
        const double r = rcp_nz(expm1(u));
        df = vtrap_num_series(u) * (r * r);
    } else {
        const double em1 = ex - 1;
        const double r = rcp_nz(em1);
        f = x * r;
        df = (em1 - u * ex) * (r * r);
    }
}

// Rates plus d inf/dv and d(alpha+beta)/dv.
struct HHRatesD {
    double inf[3], k[3], dinf[3], ds[3];
};

__device__ __forceinline__ void hh_rates_d(double v, double q10, HHRatesD& r) {
    const ZPow Z = zpow(v);
    double al, be, dal, dbe, s, f, df, rs;
    vtrap10_d_e(-(v + 40), Z.z72 * kE25, f, df);
    al = 0.1 * f;
    dal = -0.1 * df;
    be = 4 * Z.z40;
    dbe = be * (-1.0 / 18);
    s = al + be;
    rs = rcp_nz(s);
    r.inf[0] = al * rs;
    r.k[0] = q10 * s;
    r.dinf[0] = (dal * be - al * dbe) * (rs * rs);
    r.ds[0] = dal + dbe;
    al = 0.07 * Z.z36;
    dal = al * (-1.0 / 20);
    {
        const double u = Z.z72 * kE3;
        be = rcp_nz(u + 1);
        dbe = u * 0.1 * (be * be);
    }
    s = al + be;
    rs = rcp_nz(s);
    r.inf[1] = al * rs;
    r.k[1] = q10 * s;
    r.dinf[1] = (dal * be - al * dbe) * (rs * rs);
    r.ds[1] = dal + dbe;
    vtrap10_d_e(-(v + 55), Z.z72 * kE1, f, df);
    al = 0.01 * f;
    dal = -0.01 * df;
    be = 0.125 * Z.z9;
    dbe = be * (-1.0 / 80);
    s = al + be;
    rs = rcp_nz(s);
    r.inf[2] = al * rs;
    r.k[2] = q10 * s;
    r.dinf[2] = (dal * be - al * dbe) * (rs * rs);
    r.ds[2] = dal + dbe;
}

// hh_templated.cu:125-135
__device__ __forceinline__ double hh_current(double v, double gnabar, double gkbar, double gl, double m, double h,
                                             double n, double ena, double ek, double el) {
    double gna = gnabar * m * m * m * h;
    double ina = gna * (v - ena);
    double gk = gkbar * n * n * n * n;
    double ik = gk * (v - ek);
    double il = gl * (v - el);
    return ina + ik + il;
}

// cnexp: x' = x + (1 - exp(-dt k)) (inf - x)
__device__ __forceinline__ double gate_step(double x, double inf, double k, double dt) {
    return x + (1.0 - exp(-dt * k)) * (inf - x);
}

}  // namespace hx
