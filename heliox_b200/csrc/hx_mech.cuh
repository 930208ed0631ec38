// hx_mech.cuh -- device mechanism math (fp64) for the fused step kernels.
//
// hh follows src/mech/user-mech/hh_templated.cu:76-164 with the algebra of the
// cnexp update written without its redundant divisions: the reference's
//   m += (1 - exp(dt*(-1/mtau))) * ((minf/mtau)/(1/mtau) - m),  mtau = 1/(q10*(a+b))
// is computed as
//   m += (1 - exp(-dt*q10*(a+b))) * (minf - m),
// and divisions by the constants 10, 18, 20, 80 are multiplications by their
// reciprocals.  These forms equal the reference's mathematically and differ by
// rounding only (parity is checked against the reference-order CPU oracle).
// The finite-difference conductance of MechTemp::current
// (mech_template.cuh:615-626) is kept: it is what the reference integrates.
#pragma once

#include <cuda_runtime.h>

namespace hx {

constexpr double kFdEps = 0.001;  // mech_template.cuh:616 and :626
constexpr double kInvFdEps = 1000.0;

// Branch-free reciprocal for positive normal x: hardware estimate refined by
// two Newton-Raphson steps r <- r + r*(1 - x*r) (quadratic convergence from the
// ~2^-23 estimate to below double rounding).
__device__ __forceinline__ double rcp_pos(double x) {
    double r;
    asm("rcp.approx.ftz.f64 %0, %1;" : "=d"(r) : "d"(x));
    double e = __fma_rn(-x, r, 1.0);
    r = __fma_rn(r, e, r);
    e = __fma_rn(-x, r, 1.0);
    r = __fma_rn(r, e, r);
    return r;
}

// vtrap(x, 10) of hh_templated.cu:76-85 and its derivative in x.
__device__ __forceinline__ double vtrap10(double x) {
    const double u = x * 0.1;
    if (fabs(u) < 1e-6) return 10.0 * (1 - u * 0.5);
    return x / (exp(u) - 1);
}

__device__ __forceinline__ void vtrap10_d(double x, double& f, double& df) {
    const double u = x * 0.1;
    if (fabs(u) < 1e-6) {
        f = 10.0 * (1 - u * 0.5);
        df = -0.5;
    } else {
        const double e = exp(u);
        const double em1 = e - 1;
        const double r = 1.0 / em1;
        f = x * r;
        df = (em1 - u * e) * (r * r);
    }
}

// Steady states and rate sums (k = q10*(alpha+beta) = 1/tau) of m, h, n.
struct HHRates {
    double inf[3], k[3];
};

__device__ __forceinline__ void hh_rates(double v, double q10, HHRates& r) {
    double al, be, s;
    al = 0.1 * vtrap10(-(v + 40));
    be = 4 * exp(-(v + 65) * (1.0 / 18));
    s = al + be;
    r.inf[0] = al / s;
    r.k[0] = q10 * s;
    al = 0.07 * exp(-(v + 65) * (1.0 / 20));
    be = 1.0 / (exp(-(v + 35) * 0.1) + 1);
    s = al + be;
    r.inf[1] = al / s;
    r.k[1] = q10 * s;
    al = 0.01 * vtrap10(-(v + 55));
    be = 0.125 * exp(-(v + 65) * (1.0 / 80));
    s = al + be;
    r.inf[2] = al / s;
    r.k[2] = q10 * s;
}

// Rates plus d inf/dv and d(alpha+beta)/dv (shared exponentials).
struct HHRatesD {
    double inf[3], k[3], dinf[3], ds[3];
};

__device__ __forceinline__ void hh_rates_d(double v, double q10, HHRatesD& r) {
    double al, be, dal, dbe, s, f, df, rs;
    vtrap10_d(-(v + 40), f, df);
    al = 0.1 * f;
    dal = -0.1 * df;
    be = 4 * exp(-(v + 65) * (1.0 / 18));
    dbe = be * (-1.0 / 18);
    s = al + be;
    rs = 1.0 / s;
    r.inf[0] = al * rs;
    r.k[0] = q10 * s;
    r.dinf[0] = (dal * be - al * dbe) * (rs * rs);
    r.ds[0] = dal + dbe;
    al = 0.07 * exp(-(v + 65) * (1.0 / 20));
    dal = al * (-1.0 / 20);
    {
        const double u = exp(-(v + 35) * 0.1);
        be = 1.0 / (u + 1);
        dbe = u * 0.1 * (be * be);
    }
    s = al + be;
    rs = 1.0 / s;
    r.inf[1] = al * rs;
    r.k[1] = q10 * s;
    r.dinf[1] = (dal * be - al * dbe) * (rs * rs);
    r.ds[1] = dal + dbe;
    vtrap10_d(-(v + 55), f, df);
    al = 0.01 * f;
    dal = -0.01 * df;
    be = 0.125 * exp(-(v + 65) * (1.0 / 80));
    dbe = be * (-1.0 / 80);
    s = al + be;
    rs = 1.0 / s;
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
