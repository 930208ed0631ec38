// hx_lib.cuh -- library mechanisms for the fused step kernels: the ions and
// the user-mech channel set, each written once as a template over its scalar
// type.  With double it is the forward; with the forward-mode dual numbers
// below it yields the exact partial derivatives the adjoint needs, so a
// mechanism added in this form gets its vector-Jacobian products without
// hand-derived code.
//
// Every formula keeps the operation order of the reference's mechanism
// (src/mech/user-mech/<name>.cu, cited per mechanism) and goes through the
// MechTemp contract (src/mech/mech_template.cuh:589-767): current
// I(v + 0.001) and I(v), conductance (I1 - I0) / 0.001, rhs -= I0, d += g,
// the ion current accumulated from the I(v) call; state updates at the new
// voltage, mechanisms that write an ion in their state update (CaDynamics_E2)
// first (nonvint_cpu, src/simulate.cpp:784-852).  Ions follow
// src/mech/eion.cuh: erev read from the instance (iontype 0) or recomputed by
// the Nernst equation from cai / cao at finitialize and at the start of every
// current phase (iontype 040 | 0100).
//
// The kernels are compiled with --fmad=false, so the primal part of a dual
// evaluation is bit-identical to the double evaluation of the same template.
#pragma once

#include <cuda_runtime.h>

#include "hx_dev.hpp"
#include "hx_mech.cuh"

namespace hx {
namespace lib {

#define HXD __host__ __device__ __forceinline__

// ------------------------------------------------------------ dual numbers
template <int N>
struct Dual {
    double v;
    double d[N];
    HXD Dual() {}
    HXD Dual(double x) : v(x) {
#pragma unroll
        for (int i = 0; i < N; ++i) d[i] = 0.0;
    }
    HXD static Dual var(double x, int k) {
        Dual r(x);
        r.d[k] = 1.0;
        return r;
    }
};

HXD double val(double x) { return x; }
template <int N>
HXD double val(const Dual<N>& x) {
    return x.v;
}

template <int N>
HXD Dual<N> operator+(const Dual<N>& a, const Dual<N>& b) {
    Dual<N> r;
    r.v = a.v + b.v;
#pragma unroll
    for (int i = 0; i < N; ++i) r.d[i] = a.d[i] + b.d[i];
    return r;
}
template <int N>
HXD Dual<N> operator+(const Dual<N>& a, double b) {
    Dual<N> r = a;
    r.v = a.v + b;
    return r;
}
template <int N>
HXD Dual<N> operator+(double a, const Dual<N>& b) {
    Dual<N> r = b;
    r.v = a + b.v;
    return r;
}
template <int N>
HXD Dual<N> operator-(const Dual<N>& a) {
    Dual<N> r;
    r.v = -a.v;
#pragma unroll
    for (int i = 0; i < N; ++i) r.d[i] = -a.d[i];
    return r;
}
template <int N>
HXD Dual<N> operator-(const Dual<N>& a, const Dual<N>& b) {
    Dual<N> r;
    r.v = a.v - b.v;
#pragma unroll
    for (int i = 0; i < N; ++i) r.d[i] = a.d[i] - b.d[i];
    return r;
}
template <int N>
HXD Dual<N> operator-(const Dual<N>& a, double b) {
    Dual<N> r = a;
    r.v = a.v - b;
    return r;
}
template <int N>
HXD Dual<N> operator-(double a, const Dual<N>& b) {
    Dual<N> r;
    r.v = a - b.v;
#pragma unroll
    for (int i = 0; i < N; ++i) r.d[i] = -b.d[i];
    return r;
}
template <int N>
HXD Dual<N> operator*(const Dual<N>& a, const Dual<N>& b) {
    Dual<N> r;
    r.v = a.v * b.v;
#pragma unroll
    for (int i = 0; i < N; ++i) r.d[i] = a.d[i] * b.v + a.v * b.d[i];
    return r;
}
template <int N>
HXD Dual<N> operator*(const Dual<N>& a, double b) {
    Dual<N> r;
    r.v = a.v * b;
#pragma unroll
    for (int i = 0; i < N; ++i) r.d[i] = a.d[i] * b;
    return r;
}
template <int N>
HXD Dual<N> operator*(double a, const Dual<N>& b) {
    Dual<N> r;
    r.v = a * b.v;
#pragma unroll
    for (int i = 0; i < N; ++i) r.d[i] = a * b.d[i];
    return r;
}
template <int N>
HXD Dual<N> operator/(const Dual<N>& a, const Dual<N>& b) {
    Dual<N> r;
    r.v = a.v / b.v;
    const double ib = 1.0 / b.v;
#pragma unroll
    for (int i = 0; i < N; ++i) r.d[i] = (a.d[i] - r.v * b.d[i]) * ib;
    return r;
}
template <int N>
HXD Dual<N> operator/(const Dual<N>& a, double b) {
    Dual<N> r;
    r.v = a.v / b;
#pragma unroll
    for (int i = 0; i < N; ++i) r.d[i] = a.d[i] / b;
    return r;
}
template <int N>
HXD Dual<N> operator/(double a, const Dual<N>& b) {
    Dual<N> r;
    r.v = a / b.v;
    const double s = -r.v / b.v;
#pragma unroll
    for (int i = 0; i < N; ++i) r.d[i] = s * b.d[i];
    return r;
}
template <int N>
HXD Dual<N> exp(const Dual<N>& a) {
    Dual<N> r;
    r.v = ::exp(a.v);
#pragma unroll
    for (int i = 0; i < N; ++i) r.d[i] = r.v * a.d[i];
    return r;
}
template <int N>
HXD Dual<N> log(const Dual<N>& a) {
    Dual<N> r;
    r.v = ::log(a.v);
    const double ia = 1.0 / a.v;
#pragma unroll
    for (int i = 0; i < N; ++i) r.d[i] = a.d[i] * ia;
    return r;
}
template <int N>
HXD Dual<N> pow(const Dual<N>& a, double c) {
    Dual<N> r;
    r.v = ::pow(a.v, c);
    const double s = c * ::pow(a.v, c - 1.0);
#pragma unroll
    for (int i = 0; i < N; ++i) r.d[i] = s * a.d[i];
    return r;
}
template <int N>
HXD Dual<N> exp10(const Dual<N>& a) {  // 10^a, d/da = ln(10) 10^a
    Dual<N> r;
    r.v = ::exp10(a.v);
    const double s = 2.302585092994045684 * r.v;
#pragma unroll
    for (int i = 0; i < N; ++i) r.d[i] = s * a.d[i];
    return r;
}
HXD double exp10(double x) { return ::exp10(x); }
HXD double exp(double x) { return ::exp(x); }
HXD double log(double x) { return ::log(x); }
HXD double pow(double x, double c) { return ::pow(x, c); }

// ------------------------------------------------------------ shared forms
// The device forms below are the reference's formulas with its divisions
// replaced by a Newton reciprocal (rcp_nz, hx_mech.cuh) or a multiplication
// by a constant's reciprocal, reciprocal pairs exp(x), exp(-x) taken from one
// exponential, and the cnexp update without its redundant divisions:
//   x + (1 - exp(dt (-1/tau))) (-(inf/tau) / (-1/tau) - x)
//     = x + (1 - exp(-dt / tau)) (inf - x).
// They equal the reference's formulas mathematically and differ by rounding
// only; oracle/hx_oracle_lib.c keeps the reference's exact operation order,
// and the GPU path is checked against it within the voltage tolerance.
__device__ __forceinline__ double rcp(double x) { return rcp_nz(x); }
template <int N>
__device__ __forceinline__ Dual<N> rcp(const Dual<N>& a) {
    Dual<N> r;
    r.v = rcp_nz(a.v);
    const double s = -r.v * r.v;
#pragma unroll
    for (int i = 0; i < N; ++i) r.d[i] = s * a.d[i];
    return r;
}

template <class T>
__device__ __forceinline__ T cnexp(const T& x, const T& inf, const T& tau, double dt) {
    return x + (1.0 - exp(-dt * rcp(tau))) * (inf - x);
}

// 1 / pow(2.3, (34 - 21) / 10): the channels' temperature factor (their rates
// divide by qt = 2.952882641412121...)
constexpr double kIqt = 1.0 / 0x1.79f80ef2e5449p+1;

// Nernst potential of a divalent ion (eion.cuh:38-56 with z = 2)
template <class T>
__device__ __forceinline__ T nernst2(const T& ci, double co, double ktf) {
    if (val(ci) <= 0.) return T(1e6);
    if (co <= 0.) return T(-1e6);
    return (ktf * 0.5) * log(co * rcp(ci));
}

// ------------------------------------------------------------ channels
// Each channel: kS gates, kP trainable parameters (the density gbar), the
// ion it reads erev of and writes its current to (0 Na, 1 K, 2 Ca; 3 none:
// a nonspecific current with the reversal potential fix[kErevFix]), kCai when
// its gates depend on cai.  cur(v, s, p, f, e) is the value
// current_single_node returns; gates(v, f, cai, r) gives every gate's steady
// state and time constant (r[2j], r[2j+1]).  The reference's STATE blocks of
// these channels are all the cnexp update of each gate toward its steady
// state, and their INITIAL blocks set each gate to it (chan_state,
// chan_init below).

// NaTg.cu:78-160.  exp(-(-v + c)/slope) = 1 / exp(-(v - c)/slope).
struct NaTg {
    static constexpr int kS = 2, kP = 1, kIon = 0;
    static constexpr bool kCai = false;
    static constexpr int kErevFix = 0;  // kIon 3: erev is fix[kErevFix]
    template <class T>
    __device__ static void rates(const T& v, const double* f, T r[4]) {
        const double vshifth = f[0], vshiftm = f[1], slopeh = f[2], slopem = f[3];
        T v_m = v;
        if (val(v_m) == -38.0) v_m = v_m + 0.0001;
        const T xm = v_m - (-38.0 + vshiftm);
        const T em = exp(-xm * rcp(slopem));
        const T mA = (0.182 * xm) * rcp(1.0 - em);
        const T mB = (0.124 * (-xm)) * rcp(1.0 - rcp(em));
        const T rm = rcp(mA + mB);
        r[1] = rm * kIqt;
        r[0] = mA * rm;
        T v_h = v;
        if (val(v_h) == -66.0) v_h = v_h + 0.0001;
        const T xh = v_h - (-66.0 + vshifth);
        const T eh = exp(xh * rcp(slopeh));
        const T hA = (-0.015 * xh) * rcp(1.0 - eh);
        const T hB = (-0.015 * (-xh)) * rcp(1.0 - rcp(eh));
        const T rh = rcp(hA + hB);
        r[3] = rh * kIqt;
        r[2] = hA * rh;
    }
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double*, const T& e) {
        return p[0] * s[0] * s[0] * s[0] * s[1] * (v - e);
    }
    template <class T>
    __device__ static void gates(const T& v, const double* f, const T&, T* r) {
        rates(v, f, r);
    }
};

// Nap_Et2.cu.  exp(-(-v - 38)/6) = 1 / exp(-(v + 38)/6).
struct NapEt2 {
    static constexpr int kS = 2, kP = 1, kIon = 0;
    static constexpr bool kCai = false;
    static constexpr int kErevFix = 0;  // kIon 3: erev is fix[kErevFix]
    template <class T>
    __device__ static void rates(const T& v, T r[4]) {
        r[0] = rcp(1.0 + exp((v - (-52.6)) * (1.0 / -4.6)));
        T v_m = v;
        if (val(v_m) == -38.0) v_m = v_m + 0.0001;
        const T xm = v_m - (-38.0);
        const T em = exp(-xm * (1.0 / 6.0));
        const T mA = (0.182 * xm) * rcp(1.0 - em);
        const T mB = (0.124 * (-xm)) * rcp(1.0 - rcp(em));
        r[1] = (6.0 * kIqt) * rcp(mA + mB);
        T v_h1 = v;
        if (val(v_h1) == -17.0) v_h1 = v_h1 + 0.0001;
        T v_h2 = v;
        if (val(v_h2) == -64.4) v_h2 = v_h2 + 0.0001;
        r[2] = rcp(1.0 + exp((v - (-48.8)) * 0.1));
        const T hA = (-2.88e-6 * (v_h1 + 17.0)) * rcp(1.0 - exp((v_h1 + 17.0) * (1.0 / 4.63)));
        const T hB = (6.94e-6 * (v_h2 + 64.4)) * rcp(1.0 - exp(-(v_h2 + 64.4) * (1.0 / 2.63)));
        r[3] = rcp(hA + hB) * kIqt;
    }
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double*, const T& e) {
        return p[0] * s[0] * s[0] * s[0] * s[1] * (v - e);
    }
    template <class T>
    __device__ static void gates(const T& v, const double*, const T&, T* r) {
        rates(v, r);
    }
};

// K_Pst.cu
struct KPst {
    static constexpr int kS = 2, kP = 1, kIon = 1;
    static constexpr bool kCai = false;
    static constexpr int kErevFix = 0;  // kIon 3: erev is fix[kErevFix]
    template <class T>
    __device__ static void rates(const T& v_param, T r[4]) {
        const T v = v_param + 10.0;
        r[0] = rcp(1.0 + exp(-(v + 1.0) * (1.0 / 12.0)));
        if (val(v) < -50.0)
            r[1] = (1.25 + 175.03 * exp(v * 0.026)) * kIqt;
        else
            r[1] = (1.25 + 13.0 * exp(-v * 0.026)) * kIqt;
        r[2] = rcp(1.0 + exp((v + 54.0) * (1.0 / 11.0)));
        const T y = (v + 75.0) * (1.0 / 48.0);
        r[3] = (360.0 + (1010.0 + 24.0 * (v + 55.0)) * exp(-(y * y))) * kIqt;
    }
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double*, const T& e) {
        return p[0] * s[0] * s[0] * s[1] * (v - e);
    }
    template <class T>
    __device__ static void gates(const T& v, const double*, const T&, T* r) {
        rates(v, r);
    }
};

// K_Tst.cu (m^4 as two squarings)
struct KTst {
    static constexpr int kS = 2, kP = 1, kIon = 1;
    static constexpr bool kCai = false;
    static constexpr int kErevFix = 0;  // kIon 3: erev is fix[kErevFix]
    template <class T>
    __device__ static void rates(const T& v_param, T r[4]) {
        const T v = v_param + 10.0;
        r[0] = rcp(1.0 + exp(-v * (1.0 / 19.0)));
        const T y1 = (v + 71.0) * (1.0 / 59.0);
        r[1] = (0.34 + 0.92 * exp(-(y1 * y1))) * kIqt;
        r[2] = rcp(1.0 + exp((v + 66.0) * 0.1));
        const T y2 = (v + 73.0) * (1.0 / 23.0);
        r[3] = (8.0 + 49.0 * exp(-(y2 * y2))) * kIqt;
    }
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double*, const T& e) {
        const T m2 = s[0] * s[0];
        return p[0] * (m2 * m2) * s[1] * (v - e);
    }
    template <class T>
    __device__ static void gates(const T& v, const double*, const T&, T* r) {
        rates(v, r);
    }
};

// Ca_LVAst.cu
struct CaLVAst {
    static constexpr int kS = 2, kP = 1, kIon = 2;
    static constexpr bool kCai = false;
    static constexpr int kErevFix = 0;  // kIon 3: erev is fix[kErevFix]
    template <class T>
    __device__ static void rates(const T& v_param, T r[4]) {
        const T v = v_param + 10.0;
        r[0] = rcp(1.0 + exp((v - (-30.0)) * (1.0 / -6.0)));
        r[1] = (5.0 + 20.0 * rcp(1.0 + exp((v - (-25.0)) * 0.2))) * kIqt;
        r[2] = rcp(1.0 + exp((v - (-80.0)) * (1.0 / 6.4)));
        r[3] = (20.0 + 50.0 * rcp(1.0 + exp((v - (-40.0)) * (1.0 / 7.0)))) * kIqt;
    }
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double*, const T& e) {
        return p[0] * s[0] * s[0] * s[1] * (v - e);
    }
    template <class T>
    __device__ static void gates(const T& v, const double*, const T&, T* r) {
        rates(v, r);
    }
};

// CA_HVA.cu (vtrap, rates, ca_hva_cal_current, state_single_node)
struct CaHVA {
    static constexpr int kS = 2, kP = 1, kIon = 2;
    static constexpr bool kCai = false;
    static constexpr int kErevFix = 0;  // kIon 3: erev is fix[kErevFix]
    template <class T>
    __device__ static T vtrap38(const T& x) {  // vtrap(x, 3.8)
        const T u = x * (1.0 / 3.8);
        if (fabs(val(u)) < 1e-6) return 3.8 * (1.0 - u * 0.5);
        return x * rcp(exp(u) - 1.0);
    }
    template <class T>
    __device__ static void rates(const T& v, T r[4]) {
        const T mA = 0.055 * vtrap38(-27.0 - v);
        const T mB = 0.94 * exp((-75.0 - v) * (1.0 / 17.0));
        const T rm = rcp(mA + mB);
        r[0] = mA * rm;
        r[1] = rm;
        const T hA = 0.000457 * exp((-13.0 - v) * 0.02);
        const T hB = 0.0065 * rcp(exp((-v - 15.0) * (1.0 / 28.0)) + 1.0);
        const T rh = rcp(hA + hB);
        r[2] = hA * rh;
        r[3] = rh;
    }
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double*, const T& e) {
        const T g = p[0] * s[0] * s[0] * s[1];
        return g * (v - e);
    }
    template <class T>
    __device__ static void gates(const T& v, const double*, const T&, T* r) {
        rates(v, r);
    }
};

// Im.cu.  exp(-0.1 (v + 35)) = 1 / exp(0.1 (v + 35)).
struct Im {
    static constexpr int kS = 1, kP = 1, kIon = 1;
    static constexpr bool kCai = false;
    static constexpr int kErevFix = 0;  // kIon 3: erev is fix[kErevFix]
    template <class T>
    __device__ static void rates(const T& v, T r[2]) {
        const T e = exp((2.5 * 0.04) * (v - (-35.0)));
        const T mA = 3.3e-3 * e;
        const T mB = 3.3e-3 * rcp(e);
        const T rs = rcp(mA + mB);
        r[0] = mA * rs;
        r[1] = rs * kIqt;
    }
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double*, const T& e) {
        return p[0] * s[0] * (v - e);
    }
    template <class T>
    __device__ static void gates(const T& v, const double*, const T&, T* r) {
        rates(v, r);
    }
};

// SKv3_1.cu
struct SKv31 {
    static constexpr int kS = 1, kP = 1, kIon = 1;
    static constexpr bool kCai = false;
    static constexpr int kErevFix = 0;  // kIon 3: erev is fix[kErevFix]
    template <class T>
    __device__ static void rates(const T& v, T r[2]) {
        r[0] = rcp(1.0 + exp((v - 18.700) * (1.0 / -9.700)));
        r[1] = (0.2 * 20.0) * rcp(1.0 + exp((v - (-46.560)) * (1.0 / -44.140)));
    }
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double*, const T& e) {
        return p[0] * s[0] * (v - e);
    }
    template <class T>
    __device__ static void gates(const T& v, const double*, const T&, T* r) {
        rates(v, r);
    }
};

// SK_E2.cu:70-132 (zTau: the mechanism's GLOBAL, f[0])
struct SKE2 {
    static constexpr int kS = 1, kP = 1, kIon = 1;
    static constexpr bool kCai = true;
    static constexpr int kErevFix = 0;  // kIon 3: erev is fix[kErevFix]
    template <class T>
    __device__ static T zinf(const T& ca) {
        T ca_safe = ca;
        if (val(ca_safe) < 1e-7) ca_safe = ca_safe + 1e-07;
        return rcp(1.0 + pow(0.00043 * rcp(ca_safe), 4.8));
    }
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double*, const T& e) {
        return p[0] * s[0] * (v - e);
    }
    template <class T>
    __device__ static void gates(const T&, const double* f, const T& cai, T* r) {
        r[0] = zinf(cai);
        r[1] = T(f[0]);
    }
};

// hd_la.cu:86-124 (Ih, a nonspecific current with the GLOBAL reversal
// potential ehd).  f: vhalfl, tau, ehd, kl, vhalft, a0t, zetat, gmt, c with
// c = qtl q10^((celsius - 33)/10) a0t from the load.
struct HdLa {
    static constexpr int kS = 1, kP = 1, kIon = 3;
    static constexpr bool kCai = false;
    static constexpr int kErevFix = 2;
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double*, const T& e) {
        const T ghd = p[0] * s[0];
        return ghd * (v - e);
    }
    template <class T>
    __device__ static void gates(const T& v, const double* f, const T&, T* r) {
        const double vhalfl = f[0], tau = f[1], kl = f[3], vhalft = f[4], zetat = f[6], gmt = f[7], c = f[8];
        const T x = v - vhalft;
        const T a = exp((0.0378 * zetat) * x);
        r[0] = rcp(1.0 + exp(-(v - vhalfl) * rcp(kl)));
        r[1] = (tau * exp(((0.0378 * zetat) * gmt) * x)) * rcp(c * (1.0 + a));
    }
};

// km_la.cu:97-145 (gbar in pS/um2; GLOBALs Ra, Rb, tha, qa, tadj).  The
// update x + nexp (inf - x), nexp = 1 - exp(-dt tadj / ntau), is the cnexp
// form with tau = ntau / tadj; exp((v - tha)/qa) = 1 / exp(-(v - tha)/qa).
struct KmLa {
    static constexpr int kS = 1, kP = 1, kIon = 1;
    static constexpr bool kCai = false;
    static constexpr int kErevFix = 0;
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double* f, const T& e) {
        const T gk = f[4] * p[0] * s[0];
        return (1e-4 * gk) * (v - e);
    }
    template <class T>
    __device__ static void gates(const T& v, const double* f, const T&, T* r) {
        const double Ra = f[0], Rb = f[1], tha = f[2], qa = f[3], tadj = f[4];
        const T x = v - tha;
        const T em = exp(-x * rcp(qa));
        const T a = (Ra * x) * rcp(1.0 - em);
        const T b = (-Rb * x) * rcp(1.0 - rcp(em));
        const T rs = rcp(a + b);
        r[0] = a * rs;
        r[1] = rs * rcp(tadj);
    }
};

// kca_la.cu:100-145 (gbar in pS/um2; GLOBALs Ra, Rb, caix, tadj): the gate
// depends on cai only; nexp = 1 - exp(-dt tadj / ntau) is the cnexp form with
// tau = ntau / tadj.
struct KcaLa {
    static constexpr int kS = 1, kP = 1, kIon = 1;
    static constexpr bool kCai = true;
    static constexpr int kErevFix = 0;
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double* f, const T& e) {
        const T gk = f[3] * p[0] * s[0];
        return (1e-4 * gk) * (v - e);
    }
    template <class T>
    __device__ static void gates(const T&, const double* f, const T& cai, T* r) {
        const double Ra = f[0], Rb = f[1], caix = f[2], tadj = f[3];
        const T a = Ra * pow(cai, caix);
        const T rs = rcp(a + Rb);
        r[0] = a * rs;
        r[1] = rs * rcp(tadj);
    }
};

// it2_la.cu:111-170 (T-type calcium; GLOBALs vshift .. wh2), gates at
// v + vshift with mexp = 1 - exp(-dt / mtau).
struct It2La {
    static constexpr int kS = 2, kP = 1, kIon = 2;
    static constexpr bool kCai = false;
    static constexpr int kErevFix = 0;
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double*, const T& e) {
        const T gca = p[0] * s[0] * s[0] * s[1];
        return gca * (v - e);
    }
    template <class T>
    __device__ static void gates(const T& v, const double* f, const T&, T* r) {
        const T u = v + f[0];
        r[0] = rcp(1.0 + exp(-(u + f[1]) * rcp(f[2])));
        r[1] = f[5] + rcp(exp((u + f[7]) * rcp(f[11])) + exp(-(u + f[8]) * rcp(f[12])));
        r[2] = rcp(1.0 + exp((u + f[3]) * rcp(f[4])));
        r[3] = f[6] + rcp(exp((u + f[9]) * rcp(f[13])) + exp(-(u + f[10]) * rcp(f[14])));
    }
};

// kdr_la.cu:67-118 (its INITIAL sets m to minf and then to 0)
struct KdrLa {
    static constexpr int kS = 1, kP = 1, kIon = 1;
    static constexpr bool kCai = false;
    static constexpr int kErevFix = 0;
    static constexpr unsigned kInitZero = 1u;  // bit j: gate j starts at 0
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double*, const T& e) {
        const T m2 = s[0] * s[0];
        return p[0] * (m2 * m2) * (v - e);
    }
    template <class T>
    __device__ static void gates(const T& v, const double*, const T&, T* r) {
        r[0] = rcp(1.0 + exp((-v - 29.5) * 0.1));
        if (val(v) < -10.0)
            r[1] = 0.25 + 4.35 * exp((v + 10.0) * 0.1);
        else
            r[1] = 0.25 + 4.35 * exp((-v - 10.0) * 0.1);
    }
};

// sca_la.cu:95-160 (gbar in pS/um2; RANGE inactF, actF; GLOBALs vshift,
// tadj): gates at v + vshift, mexp = 1 - exp(-dt tadj / mtau) (the cnexp
// form with tau = mtau / tadj).
struct ScaLa {
    static constexpr int kS = 2, kP = 1, kIon = 2;
    static constexpr bool kCai = false;
    static constexpr int kErevFix = 0;
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double* f, const T& e) {
        const T gca = f[3] * p[0] * s[0] * s[0] * s[1];
        return (1e-4 * gca) * (v - e);
    }
    template <class T>
    __device__ static void gates(const T& v, const double* f, const T&, T* r) {
        const double ia = rcp(f[1]), ii = rcp(f[0]), it = rcp(f[3]);
        const T vm = v + f[2];
        const T x = -27.0 - vm;
        const T a = (0.055 * x) * rcp(exp(x * (1.0 / 3.8)) - 1.0) * ia;
        const T b = (0.94 * exp((-75.0 - vm) * (1.0 / 17.0))) * ia;
        const T rm = rcp(a + b);
        r[0] = a * rm;
        r[1] = rm * it;
        const T a2 = (0.000457 * exp((-13.0 - vm) * 0.02)) * ii;
        const T b2 = (0.0065 * rcp(exp((-vm - 15.0) * (1.0 / 28.0)) + 1.0)) * ii;
        const T rh = rcp(a2 + b2);
        r[2] = a2 * rh;
        r[3] = rh * it;
    }
};

// Ca.cu (the high-voltage calcium current without CA_HVA's vtrap: v = -27
// is moved by 1e-4)
struct CaPlain {
    static constexpr int kS = 2, kP = 1, kIon = 2;
    static constexpr bool kCai = false;
    static constexpr int kErevFix = 0;
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double*, const T& e) {
        const T g = p[0] * s[0] * s[0] * s[1];
        return g * (v - e);
    }
    template <class T>
    __device__ static void gates(const T& v0, const double*, const T&, T* r) {
        T v = v0;
        if (val(v) == -27.0) v = v + 0.0001;
        const T x = -27.0 - v;
        const T mA = (0.055 * x) * rcp(exp(x * (1.0 / 3.8)) - 1.0);
        const T mB = 0.94 * exp((-75.0 - v) * (1.0 / 17.0));
        const T rm = rcp(mA + mB);
        r[0] = mA * rm;
        r[1] = rm;
        const T hA = 0.000457 * exp((-13.0 - v) * 0.02);
        const T hB = 0.0065 * rcp(exp((-v - 15.0) * (1.0 / 28.0)) + 1.0);
        const T rh = rcp(hA + hB);
        r[2] = hA * rh;
        r[3] = rh;
    }
};

// worm-lr channels (src/mech/worm-lr-mech/<name>.cu): current
// w (gb gates (v - ek_tmp)) with the trainable weight w = p[0]; f = gb, ek_tmp,
// dv, then the kinetics GLOBALs g[] in the mechanism's order; steady states
// and time constants from setparames at v (the LRDS shadow gates of the
// reference, advanced at v + dv, never reach v and are not carried).
struct WormBase {
    static constexpr int kP = 1, kIon = 3;
    static constexpr bool kCai = false;
    static constexpr int kErevFix = 1;
};
template <class T>
__device__ __forceinline__ T sig_up(const T& v, double vh, double k) {  // 1 / (1 + exp(-(v - vh) / k))
    return rcp(1.0 + exp(-(v - vh) * rcp(k)));
}
template <class T>
__device__ __forceinline__ T sig_dn(const T& v, double vh, double k) {  // 1 / (1 + exp((v - vh) / k))
    return rcp(1.0 + exp((v - vh) * rcp(k)));
}
template <class T>  // a / (exp(-(v - b)/c) + exp((v - d)/e)) + f
__device__ __forceinline__ T bell(const T& v, double a, double b, double c, double d, double e, double f) {
    return a * rcp(exp(-(v - b) * rcp(c)) + exp((v - d) * rcp(e))) + f;
}
struct Shl1Lr : WormBase {  // shl1_lr.cu
    static constexpr int kS = 3;
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double* f, const T& e) {
        return p[0] * (f[0] * s[0] * s[0] * s[0] * (0.7 * s[1] + 0.3 * s[2]) * (v - e));
    }
    template <class T>
    __device__ static void gates(const T& v, const double* f, const T&, T* r) {
        const double* g = f + 3;
        const T hinf = sig_dn(v, g[2], g[3]);
        r[0] = sig_up(v, g[0], g[1]);
        r[1] = bell(v, g[4], g[5], g[6], g[7], g[8], g[9]) * 0.4;
        r[2] = hinf;
        r[3] = (g[10] * sig_dn(v, g[11], g[12]) + g[13]) * 0.08;
        r[4] = hinf;
        r[5] = (g[14] * sig_dn(v, g[15], g[16]) + g[17]) * 0.3;
    }
};
struct Kvs1Lr : WormBase {  // kvs1_lr.cu
    static constexpr int kS = 2;
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double* f, const T& e) {
        return p[0] * (f[0] * s[0] * s[1] * (v - e));
    }
    template <class T>
    __device__ static void gates(const T& v, const double* f, const T&, T* r) {
        const double* g = f + 3;
        r[0] = sig_up(v, g[0], g[1]);
        r[1] = g[4] * sig_dn(v, g[5], g[6]) + g[7];
        r[2] = sig_dn(v, g[2], g[3]);
        r[3] = g[8] * sig_dn(v, g[9], g[10]) + g[11];
    }
};
struct IrkLr : WormBase {  // irk_lr.cu
    static constexpr int kS = 1;
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double* f, const T& e) {
        return p[0] * (f[0] * s[0] * (v - e));
    }
    template <class T>
    __device__ static void gates(const T& v, const double* f, const T&, T* r) {
        const double* g = f + 3;
        r[0] = sig_dn(v, g[0], g[1]);
        r[1] = bell(v, g[2], g[3], g[4], g[5], g[6], g[7]);
    }
};
struct Egl36Lr : WormBase {  // egl36_lr.cu: time constants atmf, atmm, atms
    static constexpr int kS = 3;
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double* f, const T& e) {
        return p[0] * (f[0] * (0.33 * s[0] + 0.36 * s[1] + 0.39 * s[2]) * (v - e));
    }
    template <class T>
    __device__ static void gates(const T& v, const double* f, const T&, T* r) {
        const double* g = f + 3;
        const T inf = sig_up(v, g[0], g[1]);
        r[0] = inf;
        r[1] = T(g[4]);
        r[2] = inf;
        r[3] = T(g[3]);
        r[4] = inf;
        r[5] = T(g[2]);
    }
};
struct Shk1Lr : WormBase {  // shk1_lr.cu
    static constexpr int kS = 2;
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double* f, const T& e) {
        return p[0] * (f[0] * s[0] * s[1] * (v - e));
    }
    template <class T>
    __device__ static void gates(const T& v, const double* f, const T&, T* r) {
        const double* g = f + 3;
        r[0] = sig_up(v, g[0], g[1]);
        r[1] = bell(v, g[4], g[5], g[6], g[7], g[8], g[9]);
        r[2] = sig_dn(v, g[2], g[3]);
        r[3] = T(g[10]);
    }
};
struct Egl2Lr : WormBase {  // egl2_lr.cu
    static constexpr int kS = 1;
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double* f, const T& e) {
        return p[0] * (f[0] * s[0] * (v - e));
    }
    template <class T>
    __device__ static void gates(const T& v, const double* f, const T&, T* r) {
        const double* g = f + 3;
        r[0] = sig_up(v, g[0], g[1]);
        r[1] = g[2] * sig_dn(v, g[3], g[4]) + g[5];
    }
};

// worm-lr calcium channels: their own eca_tmp, the current w i_tmp goes into
// the node's calcium current (ica)
struct WormCaBase : WormBase {
    static constexpr int kIonCur = 2;
};
struct Cca1Lr : WormCaBase {  // cca1_lr.cu (nrn_current_like, setparames)
    static constexpr int kS = 2;
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double* f, const T& e) {
        return p[0] * (f[0] * s[0] * s[0] * s[1] * (v - e));
    }
    template <class T>
    __device__ static void gates(const T& v, const double* f, const T&, T* r) {
        const double* g = f + 3;
        r[0] = sig_up(v, g[0], g[1]);
        r[1] = g[4] * sig_up(v, g[5], g[6]) + g[7];
        r[2] = sig_dn(v, g[2], g[3]);
        r[3] = g[8] * sig_dn(v, g[9], g[10]) + g[11];
    }
};
struct Egl19Lr : WormCaBase {  // egl19_lr.cu
    static constexpr int kS = 2;
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double* f, const T& e) {
        return p[0] * (f[0] * s[0] * s[1] * (v - e));
    }
    template <class T>
    __device__ static void gates(const T& v, const double* f, const T&, T* r) {
        const double* g = f + 3;
        r[0] = sig_up(v, g[0], g[1]);
        r[2] = (g[6] * sig_up(v, g[2], g[3]) + g[7]) * (g[8] * sig_dn(v, g[4], g[5]) + g[9]);
        const T y1 = (v - g[11]) * rcp(g[12]), y2 = (v - g[14]) * rcp(g[15]);
        r[1] = g[10] * exp(-(y1 * y1)) + g[13] * exp(-(y2 * y2)) + g[16];
        r[3] = g[17] * (g[18] * sig_dn(v, g[19], g[20]) + g[21] * sig_dn(v, g[22], g[23]) + g[24]);
    }
};
struct Unc2Lr : WormCaBase {  // unc2_lr.cu
    static constexpr int kS = 2;
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double* f, const T& e) {
        return p[0] * (f[0] * s[0] * s[1] * (v - e));
    }
    template <class T>
    __device__ static void gates(const T& v, const double* f, const T&, T* r) {
        const double* g = f + 3;
        r[0] = sig_up(v, g[0], g[1]);
        r[2] = sig_dn(v, g[2], g[3]);
        r[1] = bell(v, g[4], g[5], g[6], g[5], g[7], g[8]);
        r[3] = g[9] * sig_up(v, g[10], g[11]) + g[12] * sig_dn(v, g[13], g[14]);
    }
};

struct KcnlLr : WormBase {  // kcnl_lr.cu: f = gb, dv, kca, a, ek_tmp (GLOBALs kca, a, ek_tmp)
    static constexpr int kS = 1;
    static constexpr bool kCai = true;
    static constexpr int kErevFix = 4;
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double* f, const T& e) {
        return p[0] * (f[0] * s[0] * (v - e));
    }
    template <class T>
    __device__ static void gates(const T&, const double* f, const T& cai, T* r) {
        r[0] = cai * rcp(f[2] + cai);
        r[1] = T(f[3]);
    }
};
struct NcaLr : WormBase {  // nca_lr.cu: a weighted leak, f = gb, ena_tmp
    static constexpr int kS = 0;
    template <class T>
    __device__ static T cur(const T& v, const T*, const T* p, const double* f, const T& e) {
        return p[0] * (f[0] * (v - e));
    }
    template <class T>
    __device__ static void gates(const T&, const double*, const T&, T*) {}
};
// kqt3_lr.cu: w (gb (0.3 mf + 0.7 ms) ww s (v - ek)) with k_ion's ek; f = gb,
// ek_tmp (not read), dv, then the GLOBALs vhm ka vhw kiw aw bw vhs kis as bs
// atmf btmf ctmf atms btms ctms dtms etms ftms gtms atw btw ctw dtw ats; its
// INITIAL starts mf and ms at 0
struct Kqt3Lr : WormBase {
    static constexpr int kS = 4;
    static constexpr int kIon = 1;
    static constexpr unsigned kInitZero = 3u;
    template <class T>
    __device__ static T cur(const T& v, const T* s, const T* p, const double* f, const T& e) {
        return p[0] * (f[0] * (0.3 * s[0] + 0.7 * s[1]) * s[2] * s[3] * (v - e));
    }
    template <class T>
    __device__ static void gates(const T& v, const double* f, const T&, T* r) {
        const double* g = f + 3;
        const T minf = sig_up(v, g[0], g[1]);
        const T uf = (v + g[11]) * rcp(g[12]);
        const T uw = (v - g[22]) * rcp(g[23]);
        r[0] = minf;
        r[1] = g[10] * rcp(1.0 + uf * uf);
        r[2] = minf;
        r[3] = g[13] + g[14] * rcp(1.0 + exp10(-g[15] * (g[16] - v))) + g[17] * rcp(1.0 + exp10(-g[18] * (g[19] + v)));
        r[4] = g[4] + g[5] * sig_dn(v, g[2], g[3]);
        r[5] = g[20] + g[21] * rcp(1.0 + uw * uw);
        r[6] = g[8] + g[9] * sig_dn(v, g[6], g[7]);
        r[7] = T(g[24]);
    }
};

// worm-mech channels (src/mech/worm-mech/<name>.cu): the worm-lr sibling's
// gates and current with p[0] = gb (trainable) and the fixed vector 1, -80
// (their hard-coded reversal potential: gb ... (v + 80)), 0, then the
// kinetics constants of their setparames (kvs1: its GLOBALs)
struct Shl1 : Shl1Lr {};
struct Kvs1 : Kvs1Lr {};
struct Irk : IrkLr {};
struct Egl36 : Egl36Lr {};
struct Shk1 : Shk1Lr {};
struct Egl2 : Egl2Lr {};
struct Cca1 : Cca1Lr {};  // calcium (current into ica): erev 60, gb ... (v - 60)
struct Egl19 : Egl19Lr {};
struct Unc2 : Unc2Lr {};

// cainternm_lr.cu state_single_node: the calcium update c = cai_old + dt
// alpha(c), alpha = -f ica 1e6 / (2 F vcell) - (c - caeq) / tca at or below
// 60 mV (the drive term drops above), solved by the reference's Newton
// iterations (F = 96485; f = f, tca, caeq).  alpha is linear in c, so the
// iterations land on the closed form (cai_old + dt (A + caeq / tca)) /
// (1 + dt / tca) up to rounding; the adjoint differentiates that form.
__device__ __forceinline__ double caint_newton(double old_cai, double ica, double vcell, const double* f, double v,
                                               double dt) {
    const double fr = f[0], tca = f[1], caeq = f[2];
    double c = old_cai;
    for (int it = 0; it < 50; ++it) {
        const double alpha = v <= 60.0 ? (-fr * ica * 1e6 / (2.0 * 96485.0 * vcell)) - ((c - caeq) / tca)
                                       : -(c - caeq) / tca;
        const double F = (-c + alpha * dt + old_cai) / dt;
        const double J = (-1.0 + (-1.0 / tca) * dt) / dt;
        const double delta = F / J;
        c -= delta;
        const double change = fabs(old_cai) > 1e-8 ? fabs(delta / old_cai) : fabs(delta);
        if (change <= 1e-6 && fabs(F) <= 1e-8) break;
    }
    return c;
}
template <class T>
__device__ __forceinline__ T caint_closed(const T& old_cai, const T& ica, const T& vcell, const double* f, double v,
                                          double dt) {
    const double tca = f[1], caeq = f[2];
    const T a = v <= 60.0 ? (-f[0] * 1e6 / (2.0 * 96485.0)) * ica * rcp(vcell) : T(0.0);
    return (old_cai + dt * (a + caeq / tca)) * (1.0 / (1.0 + dt / tca));
}

// the ion whose current a channel writes: kIonCur when it names one, else its
// erev ion (0 Na, 1 K, 2 Ca; none for own-erev channels)
template <class M, class = void>
struct IonCur {
    static constexpr int value = M::kIon <= 2 ? M::kIon : -1;
};
template <class M>
struct IonCur<M, decltype((void)M::kIonCur)> {
    static constexpr int value = M::kIonCur;
};

// CaDynamics_E2.cu:101-137: cai' from cai and the step's calcium current.
// The reference's steady term -(drive - (-minCai)/decay) / (-1/decay)
// equals drive decay + minCai.
template <class T>
__device__ __forceinline__ T cadyn(const T& cai, const T& ica, const T& gamma, const T& decay, const T& depth,
                                   const T& minCai, double dt) {
    const double FARADAY = 96485.3321233100184;
    const T drive_ica = (-10000.0 * (ica * gamma)) * rcp((2.0 * FARADAY) * depth);
    const T exp_factor = exp(-dt * rcp(decay));
    const T steady_term = drive_ica * decay + minCai;
    return cai + (1.0 - exp_factor) * (steady_term - cai);
}

// ------------------------------------------------------------ type table
enum LibType : int {
    kNaIon = 0, kKIon, kCaIon, kCaDyn, kCaHVA, kCaLVAst, kIm, kKPst, kKTst, kNaTg, kNapEt2, kSKE2, kSKv31, kHdLa,
    kKmLa, kKcaLa, kIt2La, kKdrLa, kScaLa, kCaPlain, kShl1Lr, kKvs1Lr, kIrkLr, kEgl36Lr, kShk1Lr, kEgl2Lr, kCca1Lr,
    kEgl19Lr, kUnc2Lr, kKcnlLr, kNcaLr, kKqt3Lr, kCainternmLr, kShl1, kKvs1, kIrk, kEgl36, kShk1, kEgl2, kCca1,
    kEgl19, kUnc2, kNType
};
static_assert(kNType <= 64, "the per-node type mask (DevLib::mask) holds one bit per type");
// first trainable kind of each type, relative to HX_P_CADYN_GAMMA (-1: none)
__host__ __device__ constexpr int kind0(int t) {
    return t < kCaDyn ? -1 : t == kCaDyn ? 0 : t + 0;
}
// states per entry / fixed parameters per entry / trainable parameters per instance
__host__ __device__ constexpr int nstate(int t) {
    return t == kCaIon ? 1
           : (t == kNcaLr || t == kCainternmLr) ? 0
           : t == kKqt3Lr ? 4
           : (t == kShl1Lr || t == kEgl36Lr || t == kShl1 || t == kEgl36) ? 3
           : (t == kIm || t == kSKE2 || t == kSKv31 || t == kHdLa || t == kKmLa || t == kKcaLa || t == kKdrLa ||
              t == kIrkLr || t == kEgl2Lr || t == kKcnlLr || t == kIrk || t == kEgl2)
               ? 1
           : t >= kCaHVA ? 2
                         : 0;
}
__host__ __device__ constexpr int nfix(int t) {
    return (t == kNaIon || t == kKIon) ? 1 : t == kCaIon ? 4 : t == kNaTg ? 4 : t == kSKE2 ? 1 : t == kHdLa ? 9
           : t == kKmLa ? 5 : t == kKcaLa ? 4 : t == kIt2La ? 15 : t == kScaLa ? 4 : t == kShl1Lr ? 21
           : t == kKvs1Lr ? 15 : t == kIrkLr ? 11 : t == kEgl36Lr ? 8 : t == kShk1Lr ? 14 : t == kEgl2Lr ? 9
           : t == kCca1Lr ? 15 : t == kEgl19Lr ? 28 : t == kUnc2Lr ? 18 : t == kKcnlLr ? 5 : t == kNcaLr ? 2
           : t == kKqt3Lr ? 28 : t == kCainternmLr ? 3 : t == kShl1 ? 21 : t == kKvs1 ? 15 : t == kIrk ? 11
           : t == kEgl36 ? 8 : t == kShk1 ? 14 : t == kEgl2 ? 9 : t == kCca1 ? 15 : t == kEgl19 ? 28
           : t == kUnc2 ? 18 : 0;
}
__host__ __device__ constexpr int ntrain(int t) { return t < kCaDyn ? 0 : t == kCaDyn ? 4 : 1; }

#define HX_LIB_CHANNELS(X) \
    X(kCaHVA, CaHVA)       \
    X(kCaLVAst, CaLVAst)   \
    X(kIm, Im)             \
    X(kKPst, KPst)         \
    X(kKTst, KTst)         \
    X(kNaTg, NaTg)         \
    X(kNapEt2, NapEt2)     \
    X(kSKE2, SKE2)         \
    X(kSKv31, SKv31)       \
    X(kHdLa, HdLa)         \
    X(kKmLa, KmLa)         \
    X(kKcaLa, KcaLa)       \
    X(kIt2La, It2La)       \
    X(kKdrLa, KdrLa)       \
    X(kScaLa, ScaLa)       \
    X(kCaPlain, CaPlain)   \
    X(kShl1Lr, Shl1Lr)     \
    X(kKvs1Lr, Kvs1Lr)     \
    X(kIrkLr, IrkLr)       \
    X(kEgl36Lr, Egl36Lr)   \
    X(kShk1Lr, Shk1Lr)     \
    X(kEgl2Lr, Egl2Lr)     \
    X(kCca1Lr, Cca1Lr)     \
    X(kEgl19Lr, Egl19Lr)   \
    X(kUnc2Lr, Unc2Lr)     \
    X(kKcnlLr, KcnlLr)     \
    X(kNcaLr, NcaLr)       \
    X(kKqt3Lr, Kqt3Lr)     \
    X(kShl1, Shl1)         \
    X(kKvs1, Kvs1)         \
    X(kIrk, Irk)           \
    X(kEgl36, Egl36)       \
    X(kShk1, Shk1)         \
    X(kEgl2, Egl2)         \
    X(kCca1, Cca1)         \
    X(kEgl19, Egl19)       \
    X(kUnc2, Unc2)

// ------------------------------------------------------------ drivers
// one channel's forward contribution; returns I(v) (the ion current)
template <class M>
__device__ __forceinline__ double fwd_cur(double v, const double* s, const double* p, const double* f, double e,
                                          double& r, double& dd) {
    double gg = M::template cur<double>(v + kFdEps, s, p, f, e);
    const double i0 = M::template cur<double>(v, s, p, f, e);
    gg = (gg - i0) / kFdEps;
    r -= i0;
    dd += gg;
    return i0;
}

// Adjoint of one channel's part of step k: Phi = -w I(v) + ld (I(v+eps) -
// I(v))/eps + li I(v) (w: adjoint of rhs, ld: of d, li: of the ion current).
// Returns dPhi/dv, adds dPhi/ds to ls, dPhi/dp to gp and dPhi/de to le.
template <class M>
__device__ __forceinline__ double vjp_cur(double v, const double* s, const double* p, const double* f, double e,
                                          double w, double ld, double li, double* ls, double* gp, double& le) {
    constexpr int N = 2 + M::kS + M::kP;
    using D = Dual<N>;
    D ds[M::kS + 1], dp[M::kP];
#pragma unroll
    for (int i = 0; i < M::kS; ++i) ds[i] = D::var(s[i], 1 + i);
#pragma unroll
    for (int i = 0; i < M::kP; ++i) dp[i] = D::var(p[i], 1 + M::kS + i);
    const D dv = D::var(v, 0), de = D::var(e, N - 1);
    const D i1 = M::template cur<D>(dv + kFdEps, ds, dp, f, de);
    const D i0 = M::template cur<D>(dv, ds, dp, f, de);
    double gr[N];
#pragma unroll
    for (int k = 0; k < N; ++k) gr[k] = (li - w) * i0.d[k] + ld * ((i1.d[k] - i0.d[k]) / kFdEps);
#pragma unroll
    for (int i = 0; i < M::kS; ++i) ls[i] += gr[1 + i];
#pragma unroll
    for (int i = 0; i < M::kP; ++i) gp[i] += gr[1 + M::kS + i];
    le += gr[N - 1];
    return gr[0];
}

// A channel's state phase: each gate x' = x + (1 - exp(-dt/tau)) (inf - x)
template <class M>
__device__ __forceinline__ void chan_state(double v, double dt, double* s, const double* f, double cai) {
    double r[2 * M::kS + 1];
    M::template gates<double>(v, f, cai, r);
#pragma unroll
    for (int j = 0; j < M::kS; ++j) s[j] = cnexp(s[j], r[2 * j], r[2 * j + 1], dt);
}

// INITIAL: every gate at its steady state, except the gates of the bit mask
// kInitZero at 0 (kdr_la: m; kqt3_lr: mf, ms)
template <class M, class = void>
struct InitZero {
    static constexpr unsigned value = 0u;
};
template <class M>
struct InitZero<M, decltype((void)M::kInitZero)> {
    static constexpr unsigned value = M::kInitZero;
};
template <class M>
__device__ __forceinline__ void chan_init(double v, double* s, const double* f, double cai) {
    double r[2 * M::kS + 1];
    M::template gates<double>(v, f, cai, r);
#pragma unroll
    for (int j = 0; j < M::kS; ++j) s[j] = ((InitZero<M>::value >> j) & 1u) ? 0.0 : r[2 * j];
}

// Adjoint of one channel's state update s_{k+1} = F(v_{k+1}, s_k[, cai_{k+1}]):
// lam holds dL/ds_{k+1} on entry and dL/ds_k on return (d x'/d x = exp(-dt/tau));
// returns dL/dv_{k+1} and adds dL/dcai_{k+1} to lcai.  The gates' steady
// states and time constants depend on v (and cai) only, so they are
// evaluated with one or two dual lanes.
template <class M>
__device__ __forceinline__ double vjp_state(double v1, double dt, const double* s, const double* f, double cai,
                                            double* lam, double& lcai) {
    constexpr int N = M::kCai ? 2 : 1;
    using D = Dual<N>;
    const D dv = D::var(v1, 0);
    const D dc = M::kCai ? D::var(cai, N - 1) : D(cai);
    D r[2 * M::kS + 1];
    M::template gates<D>(dv, f, dc, r);
    double mu = 0.0;
#pragma unroll
    for (int j = 0; j < M::kS; ++j) {
        const D E = exp(-dt * rcp(r[2 * j + 1]));
        const double x = s[j];
        const D y = x + (1.0 - E) * (r[2 * j] - x);
        const double l = lam[j];
        mu += l * y.d[0];
        if (M::kCai) lcai += l * y.d[N - 1];
        lam[j] = l * E.v;
    }
    return mu;
}

__device__ __forceinline__ int entry_type(int code) { return code >> 24; }
__device__ __forceinline__ int entry_inst(int code) { return code & 0xFFFFFF; }

// calcium reversal potential of a ca_ion entry (f: cai0, cao, eca, nernst)
__device__ __forceinline__ double ca_erev(double cai, const double* f, double ktf) {
    return f[3] != 0.0 ? nernst2(cai, f[1], ktf) : f[2];
}

// Current phase of GPU node gi at voltage v with the states X (the flat
// state array of the step): adds the channels' rhs / d contributions in type
// order and returns the node's calcium current.
__device__ __forceinline__ double lib_current(const DevLib& L, int gi, double v, const double* X, double& r,
                                              double& dd) {
    const int e0 = __ldg(L.node_off + gi), e1 = __ldg(L.node_off + gi + 1);
    double ena = 0.0, ek = 0.0, eca = 0.0, ica = 0.0;
    for (int e = e0; e < e1; ++e) {
        const int code = __ldg(L.ent + e), t = entry_type(code), inst = entry_inst(code);
        const double* s = X + __ldg(L.ent_st + e);
        const double* f = L.fix + __ldg(L.ent_fix + e);
        switch (t) {
            case kNaIon:
                ena = __ldg(f);
                break;
            case kKIon:
                ek = __ldg(f);
                break;
            case kCaIon:
                eca = ca_erev(s[0], f, L.ktf);
                break;
#define HX_LIB_FWD(T_, M_)                                                          \
    case T_: {                                                                      \
        const double p[1] = {__ldg(L.prm[kind0(T_)] + inst)};                       \
        const double e_ = M_::kIon == 0 ? ena : M_::kIon == 1 ? ek : M_::kIon == 2 ? eca : __ldg(f + M_::kErevFix); \
        const double i0 = fwd_cur<M_>(v, s, p, f, e_, r, dd);                       \
        if (IonCur<M_>::value == 2) ica += i0;                                      \
    } break;
                HX_LIB_CHANNELS(HX_LIB_FWD)
#undef HX_LIB_FWD
            default:
                break;
        }
    }
    return ica;
}

// State phase of the nodes [i0, i1) of a cell that this thread owns (i0 +
// tl, step nt), mechanism type by mechanism type: the calcium dynamics
// (CaDynamics_E2 or cainternm_lr) first (from
// the step's calcium current L.nica), then the channels in type order at the
// new voltage -- per node the reference's order (nonvint_cpu), and each pass
// runs one mechanism's code over all the thread's nodes (shorter live
// ranges: the forward kernel's spills drop from ~1 KB to under 100 B a
// thread).  sv: the new voltages, pb: the pack's first GPU node.
template <int T, class M>
__device__ __forceinline__ void lib_state_type(const DevLib& L, int pb, int i0, int i1, int tl, int nt,
                                               const double* sv) {
    for (int i = i0 + tl; i < i1; i += nt) {
        const int gi = pb + i;
        const unsigned long long m = __ldg(L.mask + gi);
        if (!(m & (1ull << T))) continue;
        const int e0 = __ldg(L.node_off + gi);
        const int e = e0 + __popcll(m & ((1ull << T) - 1ull));
        double cai = 0.0;
        if (M::kCai) cai = L.st[__ldg(L.ent_st + e0 + __popcll(m & ((1ull << kCaIon) - 1ull)))];
        chan_state<M>(sv[i], L.dt, L.st + __ldg(L.ent_st + e), L.fix + __ldg(L.ent_fix + e), cai);
    }
}

__device__ __forceinline__ void lib_state_cell(const DevLib& L, int pb, int i0, int i1, int tl, int nt,
                                               const double* sv) {
    for (int i = i0 + tl; i < i1; i += nt) {
        const int gi = pb + i;
        const unsigned long long m = __ldg(L.mask + gi);
        if (m & (1ull << kCaDyn)) {
            const int e = __ldg(L.node_off + gi) + __popcll(m & ((1ull << kCaDyn) - 1ull));
            const int inst = entry_inst(__ldg(L.ent + e));
            double* cai = L.st + __ldg(L.ent_st + e - 1);  // the node's ca_ion entry precedes CaDynamics_E2
            *cai = cadyn<double>(*cai, L.nica[gi], __ldg(L.prm[0] + inst), __ldg(L.prm[1] + inst),
                                 __ldg(L.prm[2] + inst), __ldg(L.prm[3] + inst), L.dt);
        } else if (m & (1ull << kCainternmLr)) {
            const int e0 = __ldg(L.node_off + gi);
            const int e = e0 + __popcll(m & ((1ull << kCainternmLr) - 1ull));
            const int inst = entry_inst(__ldg(L.ent + e));
            double* cai = L.st + __ldg(L.ent_st + e0 + __popcll(m & ((1ull << kCaIon) - 1ull)));
            *cai = caint_newton(*cai, L.nica[gi], __ldg(L.prm[kind0(kCainternmLr)] + inst), L.fix + __ldg(L.ent_fix + e),
                                sv[i], L.dt);
        }
    }
#define HX_LIB_STT(T_, M_) lib_state_type<T_, M_>(L, pb, i0, i1, tl, nt, sv);
    HX_LIB_CHANNELS(HX_LIB_STT)
#undef HX_LIB_STT
}

// finitialize of GPU node gi at v: ca_ion's initial cai, the channels' INITIAL
// blocks in type order.
__device__ __forceinline__ void lib_init(const DevLib& L, int gi, double v) {
    const int e0 = L.node_off[gi], e1 = L.node_off[gi + 1];
    double cai = 0.0;
    for (int e = e0; e < e1; ++e) {
        const int t = entry_type(L.ent[e]);
        double* s = L.st + L.ent_st[e];
        const double* f = L.fix + L.ent_fix[e];
        switch (t) {
            case kCaIon:
                cai = f[0];
                s[0] = cai;
                break;
#define HX_LIB_INIT(T_, M_)       \
    case T_:                      \
        chan_init<M_>(v, s, f, cai);   \
        break;
                HX_LIB_CHANNELS(HX_LIB_INIT)
#undef HX_LIB_INIT
            default:
                break;
        }
    }
}

// Adjoint of the state phase of step k at GPU node gi: v1 = v_{k+1}, Xk / Xk1
// the states at the start of steps k / k+1, ica the step's calcium current.
// L.lam holds dL/dX_{k+1} on entry; on return the state-phase part of
// dL/dX_k, and L.nlica[gi] the adjoint of ica.  Returns dL/dv_{k+1} through
// the state updates.
__device__ __forceinline__ double lib_state_adj(const DevLib& L, int gi, double v1, const double* Xk,
                                                const double* Xk1, double ica) {
    const int e0 = __ldg(L.node_off + gi), e1 = __ldg(L.node_off + gi + 1);
    if (e0 == e1) return 0.0;
    int cs = -1;
    for (int e = e0; e < e1 && e < e0 + 3; ++e)
        if (entry_type(__ldg(L.ent + e)) == kCaIon) cs = __ldg(L.ent_st + e);
    const double cai1 = cs >= 0 ? Xk1[cs] : 0.0;
    double* lam = L.lam;
    double mu = 0.0, lcai1 = 0.0;
    bool dyn = false;
    int ci = -1;  // the cainternm_lr entry: last in type order, applied first in the state phase
    for (int e = e1 - 1; e >= e0; --e) {
        const int code = __ldg(L.ent + e), t = entry_type(code), inst = entry_inst(code);
        const int so = __ldg(L.ent_st + e);
        const double* f = L.fix + __ldg(L.ent_fix + e);
        switch (t) {
#define HX_LIB_SADJ(T_, M_)                                                 \
    case T_:                                                                \
        mu += vjp_state<M_>(v1, L.dt, Xk + so, f, cai1, lam + so, lcai1);  \
        break;
            HX_LIB_CHANNELS(HX_LIB_SADJ)
#undef HX_LIB_SADJ
            case kCaDyn: {
                dyn = true;
                using D = Dual<6>;
                const double lt = lam[cs] + lcai1;
                const D out = cadyn<D>(D::var(Xk[cs], 0), D::var(ica, 1), D::var(__ldg(L.prm[0] + inst), 2),
                                       D::var(__ldg(L.prm[1] + inst), 3), D::var(__ldg(L.prm[2] + inst), 4),
                                       D::var(__ldg(L.prm[3] + inst), 5), L.dt);
                lam[cs] = lt * out.d[0];
                L.nlica[gi] = lt * out.d[1];
#pragma unroll
                for (int j = 0; j < 4; ++j) L.grad[j][inst] += lt * out.d[2 + j];
            } break;
            case kCainternmLr:
                dyn = true;
                ci = e;
                break;
            case kCaIon:
                if (!dyn) {  // no calcium dynamics: cai_{k+1} = cai_k
                    lam[cs] += lcai1;
                    L.nlica[gi] = 0.0;
                }
                break;
            default:
                break;
        }
    }
    if (ci >= 0) {  // after every reader of cai_{k+1} has added to lcai1
        using D = Dual<3>;
        const int inst = entry_inst(__ldg(L.ent + ci));
        const double lt = lam[cs] + lcai1;
        const D out = caint_closed<D>(D::var(Xk[cs], 0), D::var(ica, 1),
                                      D::var(__ldg(L.prm[kind0(kCainternmLr)] + inst), 2),
                                      L.fix + __ldg(L.ent_fix + ci), v1, L.dt);
        lam[cs] = lt * out.d[0];
        L.nlica[gi] = lt * out.d[1];
        L.grad[kind0(kCainternmLr)][inst] += lt * out.d[2];
    }
    return mu;
}

// Adjoint of the current phase of step k at GPU node gi (v_k = v, states Xk)
// with w = dL/drhs_k, ld = dL/dd_k: adds dL/dX_k to L.lam and the parameter
// gradients; returns dL/dv_k through the library currents.
__device__ __forceinline__ double lib_current_adj(const DevLib& L, int gi, double v, const double* Xk, double w,
                                                  double ld) {
    const int e0 = __ldg(L.node_off + gi), e1 = __ldg(L.node_off + gi + 1);
    if (e0 == e1) return 0.0;
    double* lam = L.lam;
    double ena = 0.0, ek = 0.0, eca = 0.0, lica = 0.0, leca = 0.0, lv = 0.0;
    int cs = -1;
    const double* fca = nullptr;
    for (int e = e0; e < e1; ++e) {
        const int code = __ldg(L.ent + e), t = entry_type(code), inst = entry_inst(code);
        const int so = __ldg(L.ent_st + e);
        const double* f = L.fix + __ldg(L.ent_fix + e);
        switch (t) {
            case kNaIon:
                ena = __ldg(f);
                break;
            case kKIon:
                ek = __ldg(f);
                break;
            case kCaIon:
                cs = so;
                fca = f;
                eca = ca_erev(Xk[so], f, L.ktf);
                lica = L.nlica[gi];
                break;
#define HX_LIB_CADJ(T_, M_)                                                                    \
    case T_: {                                                                                 \
        const double p[1] = {__ldg(L.prm[kind0(T_)] + inst)};                                  \
        const double e_ = M_::kIon == 0 ? ena : M_::kIon == 1 ? ek : M_::kIon == 2 ? eca : __ldg(f + M_::kErevFix); \
        double gp[1] = {0.0}, le = 0.0;                                                        \
        lv += vjp_cur<M_>(v, Xk + so, p, f, e_, w, ld, IonCur<M_>::value == 2 ? lica : 0.0, lam + so, \
                          gp, le);                                                             \
        L.grad[kind0(T_)][inst] += gp[0];                                                      \
        if (M_::kIon == 2) leca += le;                                                         \
    } break;
                HX_LIB_CHANNELS(HX_LIB_CADJ)
#undef HX_LIB_CADJ
            default:
                break;
        }
    }
    if (cs >= 0 && fca[3] != 0.0 && Xk[cs] > 0.0 && fca[1] > 0.0)  // eca = ktf/2 log(cao/cai)
        lam[cs] += leca * (-(L.ktf / 2.0) / Xk[cs]);
    return lv;
}

#undef HXD

}  // namespace lib
}  // namespace hx
