// hx_mech.cuh -- device mechanism math (fp64) for the fused step kernels.
//
// Expression order follows the reference mechanisms so that, compiled without
// FMA contraction (--fmad=false, the GPU analogue of the reference CPU build's
// -ffp-contract=off, CMakeLists.txt:26-31), everything except the libm/CUDA
// transcendental calls rounds exactly as the reference CPU path does.
#pragma once

#include <cuda_runtime.h>

namespace hx {

constexpr double kFdEps = 0.001;  // mech_template.cuh:616 and :626

// ---- hh: src/mech/user-mech/hh_templated.cu:76-164
__device__ __forceinline__ double vtrap(double x, double y) {
    if (fabs(x / y) < 1e-6) return y * (1 - x / y / 2);
    return x / (exp(x / y) - 1);
}

struct HHRates {
    double minf, mtau, hinf, htau, ninf, ntau;
};

// hh_templated.cu:87-109 (q10 = pow(3, (celsius-6.3)/10) computed once on the host)
__device__ __forceinline__ void hh_rates(double v, double q10, HHRates& r) {
    double alpha, beta, sum;
    alpha = 0.1 * vtrap(-(v + 40), 10);
    beta = 4 * exp(-(v + 65) / 18);
    sum = alpha + beta;
    r.mtau = 1.0 / (q10 * sum);
    r.minf = alpha / sum;
    alpha = 0.07 * exp(-(v + 65) / 20);
    beta = 1.0 / (exp(-(v + 35) / 10) + 1);
    sum = alpha + beta;
    r.htau = 1.0 / (q10 * sum);
    r.hinf = alpha / sum;
    alpha = 0.01 * vtrap(-(v + 55), 10);
    beta = 0.125 * exp(-(v + 65) / 80);
    sum = alpha + beta;
    r.ntau = 1.0 / (q10 * sum);
    r.ninf = alpha / sum;
}

// Rates plus the derivatives the state VJP needs, sharing the exponentials:
// per gate q: inf, tau, d inf/dv and d(alpha+beta)/dv.
struct HHRatesD {
    double inf[3], tau[3], dinf[3], ds[3];
};

__device__ __forceinline__ void vtrap_d(double x, double y, double& f, double& df) {
    if (fabs(x / y) < 1e-6) {
        f = y * (1 - x / y / 2);
        df = -0.5;
    } else {
        double e = exp(x / y);
        double em1 = e - 1;
        f = x / em1;
        df = (em1 - (x / y) * e) / (em1 * em1);
    }
}

__device__ __forceinline__ void hh_rates_d(double v, double q10, HHRatesD& r) {
    double al, be, dal, dbe, s, f, df;
    // m
    vtrap_d(-(v + 40), 10, f, df);
    al = 0.1 * f;
    dal = -0.1 * df;
    be = 4 * exp(-(v + 65) / 18);
    dbe = -be / 18;
    s = al + be;
    r.tau[0] = 1.0 / (q10 * s);
    r.inf[0] = al / s;
    r.dinf[0] = (dal * be - al * dbe) / (s * s);
    r.ds[0] = dal + dbe;
    // h
    al = 0.07 * exp(-(v + 65) / 20);
    dal = -al / 20;
    {
        double u = exp(-(v + 35) / 10);
        be = 1.0 / (u + 1);
        dbe = u / (10 * (u + 1) * (u + 1));
    }
    s = al + be;
    r.tau[1] = 1.0 / (q10 * s);
    r.inf[1] = al / s;
    r.dinf[1] = (dal * be - al * dbe) / (s * s);
    r.ds[1] = dal + dbe;
    // n
    vtrap_d(-(v + 55), 10, f, df);
    al = 0.01 * f;
    dal = -0.01 * df;
    be = 0.125 * exp(-(v + 65) / 80);
    dbe = -be / 80;
    s = al + be;
    r.tau[2] = 1.0 / (q10 * s);
    r.inf[2] = al / s;
    r.dinf[2] = (dal * be - al * dbe) / (s * s);
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

// hh_templated.cu:161-163 (cnexp)
__device__ __forceinline__ double gate_step(double x, double inf, double tau, double dt) {
    return x + (1.0 - exp(dt * (-1.0 / tau))) * ((inf / tau) / (1.0 / tau) - x);
}

}  // namespace hx
