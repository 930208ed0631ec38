// hx_kernels.cu -- fused per-timestep kernels for sm_100a (fp64).
//
// One CTA owns one cell pack for a whole window of timesteps: voltages, the
// Hines matrix (d, rhs), the axial coefficients and the hh gates stay in shared
// memory across steps; only the forward tape, the recorded probes and the
// mechanism parameters (L2-resident) touch global memory inside the loop.
//
// Forward step (reference: Simulate::fadvance_cpu, src/simulate.cpp:410-442):
//   A  node-parallel: mechanism currents with the finite-difference
//      conductance (mech_template.cuh:589-648), capacitance jacobian
//      (capac.cpp:68-78) and the axial terms (simulate.cpp:542-555) gathered
//      per node in the order the reference's scatter loop applies them;
//   B  Hines solve, one thread per unbranched chain, levels deepest-first then
//      root-first (solve_serial, simulate.cpp:558-581, reproduced bit for bit);
//   C  v += dv (update_cpu, simulate.cpp:759-770), then the hh cnexp state
//      update at the new voltage (nonvint_cpu, simulate.cpp:784-852).
// Backward step: the transpose of the above, in reverse (no reference
// counterpart; the reference's only gradient is the LRDS replay).
#include <cuda_runtime.h>

#include "hx_dev.hpp"
#include "hx_kernels.hpp"
#include "hx_mech.cuh"

namespace hx {

// ------------------------------------------------------------------ init
__global__ void init_state_kernel(DevGroup G, DevState S, double v_init) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < G.nnode) S.v[i] = v_init;
    if (i < G.nhh) {
        HHRates r;
        hh_rates(v_init, G.q10, r);  // hh INITIAL: gates at steady state (hh_templated.cu:111-122)
        S.m[i] = r.minf;
        S.h[i] = r.hinf;
        S.n[i] = r.ninf;
    }
}

// ------------------------------------------------------------------ Hines (shared memory)
// Triangularise + back-substitute the pack's tree system.  A = coefficient
// eliminating a child into its parent, U = coupling of a node to its parent
// (forward: A=a, U=b; transposed system: A=b, U=a).
__device__ __forceinline__ void hines_smem(const DevGroup& G, int p, const double* __restrict__ A,
                                           const double* __restrict__ U, double* __restrict__ d,
                                           double* __restrict__ rhs) {
    const int bb = G.pack_br_off[p];
    const int* lo = G.level_br_off + G.pack_lvl_off[p];
    const int nlev = G.pack_nlev[p];
    for (int L = nlev - 1; L >= 0; --L) {
        const int b0 = lo[L], b1 = lo[L + 1];
        for (int br = b0 + (int)threadIdx.x; br < b1; br += blockDim.x) {
            const int gb = bb + br;
            const int h = G.br_head[gb], e = G.br_end[gb];
            double de = d[e], re = rhs[e];
            // child branches fold into the branch end in descending reference index
            for (int k = G.br_child_off[gb]; k < G.br_child_off[gb + 1]; ++k) {
                const int c = G.br_child[k];
                const double f = A[c] / d[c];
                de = de - f * U[c];
                re = re - f * rhs[c];
            }
            for (int j = e; j > h; --j) {
                d[j] = de;
                rhs[j] = re;
                const double f = A[j] / de;
                de = d[j - 1] - f * U[j];
                re = rhs[j - 1] - f * re;
            }
            d[h] = de;
            rhs[h] = re;
        }
        __syncthreads();
    }
    for (int L = 0; L < nlev; ++L) {
        const int b0 = lo[L], b1 = lo[L + 1];
        for (int br = b0 + (int)threadIdx.x; br < b1; br += blockDim.x) {
            const int gb = bb + br;
            const int h = G.br_head[gb], e = G.br_end[gb];
            const int par = G.br_parent[gb];
            double x = rhs[h];
            if (par >= 0) x = x - U[h] * rhs[par];
            x = x / d[h];
            rhs[h] = x;
            for (int j = h + 1; j <= e; ++j) {
                x = (rhs[j] - U[j] * x) / d[j];
                rhs[j] = x;
            }
        }
        __syncthreads();
    }
}

// ------------------------------------------------------------------ assembly
// rhs/d of node i (pack-local) in the reference's accumulation order:
// pas, hh, IClamp (CoreNEURON type order), capacitance jacobian, axial terms.
template <bool kRhs>
__device__ __forceinline__ void assemble(const DevGroup& G, int nb, int hb, int i, const double* __restrict__ sv,
                                         const double* __restrict__ sa, const double* __restrict__ sb, int jh,
                                         double m, double h, double n, double tmid, double& r_out, double& d_out) {
    const int gi = nb + i;
    const double vi = sv[i];
    double r = 0.0, dd = 0.0;
    const int jp = G.node_pas[gi];
    if (jp >= 0) {  // pas_templated.cu:27-31 through MechTemp::current (FD conductance)
        const double g = G.pas_g[jp], e = G.pas_e[jp];
        double g1 = g * ((vi + kFdEps) - e);
        const double i0 = g * (vi - e);
        g1 = (g1 - i0) / kFdEps;
        r -= i0;
        dd += g1;
    }
    if (jh >= 0) {  // hh_templated.cu:137-149
        const int gj = hb + jh;
        const double gnabar = G.hh_gnabar[gj], gkbar = G.hh_gkbar[gj], gl = G.hh_gl[gj];
        const double ena = G.hh_ena[gj], ek = G.hh_ek[gj], el = G.hh_el[gj];
        double g1 = hh_current(vi + kFdEps, gnabar, gkbar, gl, m, h, n, ena, ek, el);
        const double i0 = hh_current(vi, gnabar, gkbar, gl, m, h, n, ena, ek, el);
        g1 = (g1 - i0) / kFdEps;
        r -= i0;
        dd += g1;
    }
    for (int k = G.node_ic_off[gi]; k < G.node_ic_off[gi + 1]; ++k) {  // iclamp_templated.cu:35-45, electrode
        const int j = G.node_ic[k];
        const double del = G.ic_del[j], dur = G.ic_dur[j];
        const double cur = (tmid < del + dur && tmid >= del) ? G.ic_amp[j] : 0.0;
        double g1 = (cur - cur) / kFdEps;
        double i0 = cur;
        const double s = 1.e2 / G.area[gi];
        g1 *= s;
        i0 *= s;
        r += i0;
        dd -= g1;
    }
    dd += G.cfac * G.cm[gi];
    const int par = G.node_parent[gi];
    const int c0 = G.node_child_off[gi], c1 = G.node_child_off[gi + 1];
    if (kRhs) {
        if (par >= 0) {
            const double dv = sv[par] - vi;
            r -= sb[i] * dv;
        }
        for (int k = c0; k < c1; ++k) {
            const int c = G.node_child[k];
            const double dv = vi - sv[c];
            r += sa[c] * dv;
        }
    }
    if (par >= 0) dd -= sb[i];
    for (int k = c0; k < c1; ++k) dd -= sa[G.node_child[k]];
    r_out = r;
    d_out = dd;
}

// ------------------------------------------------------------------ forward
__global__ void __launch_bounds__(kThreads) fwd_kernel(DevGroup G, DevState S, DevTape T, int write_tape,
                                                        DevProbe P, double* __restrict__ trace,
                                                        const double* __restrict__ tmid, int k0, int k1) {
    extern __shared__ double smem[];
    const int p = blockIdx.x;
    const int tid = threadIdx.x, nt = blockDim.x;
    const int nb = G.pack_node_off[p], n = G.pack_node_off[p + 1] - nb;
    const int hb = G.pack_hh_off[p], nh = G.pack_hh_off[p + 1] - hb;
    double* sv = smem;
    double* srhs = sv + G.smem_n;
    double* sd = srhs + G.smem_n;
    double* sa = sd + G.smem_n;
    double* sb = sa + G.smem_n;
    double* sgm = sb + G.smem_n;
    double* sgh = sgm + G.smem_nh;
    double* sgn = sgh + G.smem_nh;
    for (int i = tid; i < n; i += nt) {
        sv[i] = S.v[nb + i];
        sa[i] = G.a[nb + i];
        sb[i] = G.b[nb + i];
    }
    for (int j = tid; j < nh; j += nt) {
        sgm[j] = S.m[hb + j];
        sgh[j] = S.h[hb + j];
        sgn[j] = S.n[hb + j];
    }
    const int q0 = P.pack_off[p], q1 = P.pack_off[p + 1];
    __syncthreads();
    if (k0 == 0 && trace)
        for (int q = q0 + tid; q < q1; q += nt) trace[P.slot[q]] = sv[P.local[q]];
    for (int k = k0; k < k1; ++k) {
        if (write_tape) {
            const size_t row = (size_t)(k - T.k_base);
            double* tv = T.v + row * (size_t)G.nnode + nb;
            for (int i = tid; i < n; i += nt) tv[i] = sv[i];
            const size_t ho = row * (size_t)G.nhh + hb;
            for (int j = tid; j < nh; j += nt) {
                T.m[ho + j] = sgm[j];
                T.h[ho + j] = sgh[j];
                T.n[ho + j] = sgn[j];
            }
        }
        const double tm = tmid[k];
        // A: assembly
        for (int i = tid; i < n; i += nt) {
            const int jh = G.node_hh[nb + i];
            double gm = 0.0, gh = 0.0, gn = 0.0;
            if (jh >= 0) {
                gm = sgm[jh];
                gh = sgh[jh];
                gn = sgn[jh];
            }
            double r, dd;
            assemble<true>(G, nb, hb, i, sv, sa, sb, jh, gm, gh, gn, tm, r, dd);
            srhs[i] = r;
            sd[i] = dd;
        }
        __syncthreads();
        // B: Hines solve (rhs := dv)
        hines_smem(G, p, sa, sb, sd, srhs);
        // C: update + states
        for (int i = tid; i < n; i += nt) {
            const double vn = sv[i] + srhs[i];
            sv[i] = vn;
            const int jh = G.node_hh[nb + i];
            if (jh >= 0) {
                HHRates r;
                hh_rates(vn, G.q10, r);
                sgm[jh] = gate_step(sgm[jh], r.minf, r.mtau, G.dt);
                sgh[jh] = gate_step(sgh[jh], r.hinf, r.htau, G.dt);
                sgn[jh] = gate_step(sgn[jh], r.ninf, r.ntau, G.dt);
            }
        }
        __syncthreads();
        if (trace)
            for (int q = q0 + tid; q < q1; q += nt) trace[(size_t)(k + 1) * P.nprobe + P.slot[q]] = sv[P.local[q]];
    }
    if (write_tape) {
        double* tv = T.v + (size_t)(k1 - T.k_base) * (size_t)G.nnode + nb;
        for (int i = tid; i < n; i += nt) tv[i] = sv[i];
    }
    for (int i = tid; i < n; i += nt) S.v[nb + i] = sv[i];
    for (int j = tid; j < nh; j += nt) {
        S.m[hb + j] = sgm[j];
        S.h[hb + j] = sgh[j];
        S.n[hb + j] = sgn[j];
    }
}

// ------------------------------------------------------------------ backward
// Reverse sweep over steps [k_lo, k_hi).  Per step k, with lv = dL/dv_{k+1}
// and lm/lh/ln = dL/d(gates_{k+1}):
//   S  gates_{k+1} = E*gates_k + (1-E)*inf(v_{k+1}):  mu = lv + sum lg*dgate'/dv',
//      lg *= E;
//   A  recompute the diagonal d_k (FD conductances at v_k, gates_k);
//   B  w = M_k^{-T} mu (Hines with a and b swapped);
//   V  lambda_d = -w*dv; VJPs of rhs_k and d_k into lv (dL/dv_k), the gate
//      adjoints and the per-instance parameter gradients.
__global__ void __launch_bounds__(kThreads) bwd_kernel(DevGroup G, DevTape T, DevAdj A, DevGrad GR, DevProbe P,
                                                        const double* __restrict__ dLdv,
                                                        const double* __restrict__ tmid, int k_hi, int k_lo) {
    extern __shared__ double smem[];
    const int p = blockIdx.x;
    const int tid = threadIdx.x, nt = blockDim.x;
    const int nb = G.pack_node_off[p], n = G.pack_node_off[p + 1] - nb;
    const int hb = G.pack_hh_off[p], nh = G.pack_hh_off[p + 1] - hb;
    double* slv = smem;
    double* sw = slv + G.smem_n;
    double* sd = sw + G.smem_n;
    double* svk = sd + G.smem_n;
    double* svk1 = svk + G.smem_n;
    double* sa = svk1 + G.smem_n;
    double* sb = sa + G.smem_n;
    double* slm = sb + G.smem_n;
    double* slh = slm + G.smem_nh;
    double* sln = slh + G.smem_nh;
    const double dt = G.dt, q10 = G.q10;
    for (int i = tid; i < n; i += nt) {
        slv[i] = A.lv[nb + i];
        sa[i] = G.a[nb + i];
        sb[i] = G.b[nb + i];
        svk1[i] = T.v[(size_t)(k_hi - T.k_base) * (size_t)G.nnode + nb + i];
    }
    for (int j = tid; j < nh; j += nt) {
        slm[j] = A.lm[hb + j];
        slh[j] = A.lh[hb + j];
        sln[j] = A.ln[hb + j];
    }
    const int q0 = P.pack_off[p], q1 = P.pack_off[p + 1];
    __syncthreads();
    for (int k = k_hi - 1; k >= k_lo; --k) {
        const size_t row = (size_t)(k - T.k_base);
        const double* tv = T.v + row * (size_t)G.nnode + nb;
        const double* tgm = T.m + row * (size_t)G.nhh + hb;
        const double* tgh = T.h + row * (size_t)G.nhh + hb;
        const double* tgn = T.n + row * (size_t)G.nhh + hb;
        for (int i = tid; i < n; i += nt) svk[i] = tv[i];
        if (tid == 0)
            for (int q = q0; q < q1; ++q) slv[P.local[q]] += dLdv[(size_t)(k + 1) * P.nprobe + P.slot[q]];
        __syncthreads();
        const double tm = tmid[k];
        // S + A
        for (int i = tid; i < n; i += nt) {
            double mu = slv[i];
            const int jh = G.node_hh[nb + i];
            double gm = 0.0, gh = 0.0, gn = 0.0;
            if (jh >= 0) {
                gm = tgm[jh];
                gh = tgh[jh];
                gn = tgn[jh];
                HHRatesD R;
                hh_rates_d(svk1[i], q10, R);
                const double x[3] = {gm, gh, gn};
                double lam[3] = {slm[jh], slh[jh], sln[jh]};
#pragma unroll
                for (int q = 0; q < 3; ++q) {
                    const double E = exp(dt * (-1.0 / R.tau[q]));
                    const double dnew = (1.0 - E) * R.dinf[q] + (R.inf[q] - x[q]) * E * dt * q10 * R.ds[q];
                    mu += lam[q] * dnew;
                    lam[q] *= E;
                }
                slm[jh] = lam[0];
                slh[jh] = lam[1];
                sln[jh] = lam[2];
            }
            double r, dd;
            assemble<false>(G, nb, hb, i, svk, sa, sb, jh, gm, gh, gn, tm, r, dd);
            sd[i] = dd;
            sw[i] = mu;
            slv[i] = mu;
        }
        __syncthreads();
        // B: w = M^{-T} mu
        hines_smem(G, p, sb, sa, sd, sw);
        // V
        for (int i = tid; i < n; i += nt) {
            const int gi = nb + i;
            const double w = sw[i];
            const double vk = svk[i];
            const double ld = -w * (svk1[i] - vk);
            double lvn = slv[i];
            const int jp = G.node_pas[gi];
            if (jp >= 0) {
                const double g = G.pas_g[jp];
                GR.pas_g[jp] += ld - w * (vk - G.pas_e[jp]);
                GR.pas_e[jp] += w * g;
                lvn -= w * g;
            }
            const int jh = G.node_hh[gi];
            if (jh >= 0) {
                const int gj = hb + jh;
                const double m = tgm[jh], h = tgh[jh], nn = tgn[jh];
                const double gnabar = G.hh_gnabar[gj], gkbar = G.hh_gkbar[gj], gl = G.hh_gl[gj];
                const double t_na = ld - w * (vk - G.hh_ena[gj]);
                const double t_k = ld - w * (vk - G.hh_ek[gj]);
                const double t_l = ld - w * (vk - G.hh_el[gj]);
                const double m2h = m * m * h, n3 = nn * nn * nn;
                GR.hh_gnabar[gj] += m2h * m * t_na;
                GR.hh_gkbar[gj] += n3 * nn * t_k;
                GR.hh_gl[gj] += t_l;
                GR.hh_el[gj] += w * gl;
                slm[jh] += 3.0 * gnabar * m2h * t_na;
                slh[jh] += gnabar * m * m * m * t_na;
                sln[jh] += 4.0 * gkbar * n3 * t_k;
                lvn -= w * (gnabar * m2h * m + gkbar * n3 * nn + gl);
            }
            for (int k2 = G.node_ic_off[gi]; k2 < G.node_ic_off[gi + 1]; ++k2) {
                const int j = G.node_ic[k2];
                const double del = G.ic_del[j], dur = G.ic_dur[j];
                if (tm < del + dur && tm >= del) GR.ic_amp[j] += w * (1.e2 / G.area[gi]);
            }
            GR.cm[gi] += ld * G.cfac;
            const int par = G.node_parent[gi];
            if (par >= 0) lvn += sb[i] * w - sa[i] * sw[par];
            for (int k2 = G.node_child_off[gi]; k2 < G.node_child_off[gi + 1]; ++k2) {
                const int c = G.node_child[k2];
                lvn += sa[c] * w - sb[c] * sw[c];
            }
            slv[i] = lvn;
        }
        double* tmp = svk1;
        svk1 = svk;
        svk = tmp;
        __syncthreads();
    }
    for (int i = tid; i < n; i += nt) A.lv[nb + i] = slv[i];
    for (int j = tid; j < nh; j += nt) {
        A.lm[hb + j] = slm[j];
        A.lh[hb + j] = slh[j];
        A.ln[hb + j] = sln[j];
    }
}

// ------------------------------------------------------------------ small kernels
__global__ void gather_kernel(const double* __restrict__ src, const int* __restrict__ idx, double* __restrict__ dst,
                              int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = src[idx[i]];
}

__global__ void scatter_kernel(const double* __restrict__ src, const int* __restrict__ idx, double* __restrict__ dst,
                               int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[idx[i]] = src[i];
}

// out[c] = sum over entries e of column c (CSR, stable order) of scale[e]*grad[flat[e]]
__global__ void reduce_cols_kernel(const double* __restrict__ grad, const int* __restrict__ col_off,
                                   const int* __restrict__ flat, const float* __restrict__ scale,
                                   float* __restrict__ out, int ncol) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= ncol) return;
    double s = 0.0;
    for (int e = col_off[c]; e < col_off[c + 1]; ++e) s += (double)scale[e] * grad[flat[e]];
    out[c] = (float)s;
}

// ------------------------------------------------------------------ launchers
size_t fwd_smem_bytes(const DevGroup& G) { return sizeof(double) * (5 * (size_t)G.smem_n + 3 * (size_t)G.smem_nh); }
size_t bwd_smem_bytes(const DevGroup& G) { return sizeof(double) * (7 * (size_t)G.smem_n + 3 * (size_t)G.smem_nh); }

cudaError_t configure_kernels(size_t smem_fwd, size_t smem_bwd) {
    cudaError_t e = cudaFuncSetAttribute(fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_fwd);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bwd);
}

cudaError_t launch_init(const DevGroup& G, const DevState& S, double v_init, cudaStream_t st) {
    int n = G.nnode > G.nhh ? G.nnode : G.nhh;
    init_state_kernel<<<(n + 255) / 256, 256, 0, st>>>(G, S, v_init);
    return cudaGetLastError();
}

cudaError_t launch_fwd(const DevGroup& G, const DevState& S, const DevTape& T, int write_tape, const DevProbe& P,
                       double* trace, const double* tmid, int k0, int k1, cudaStream_t st) {
    fwd_kernel<<<G.npack, kThreads, fwd_smem_bytes(G), st>>>(G, S, T, write_tape, P, trace, tmid, k0, k1);
    return cudaGetLastError();
}

cudaError_t launch_bwd(const DevGroup& G, const DevTape& T, const DevAdj& A, const DevGrad& GR, const DevProbe& P,
                       const double* dLdv, const double* tmid, int k_hi, int k_lo, cudaStream_t st) {
    bwd_kernel<<<G.npack, kThreads, bwd_smem_bytes(G), st>>>(G, T, A, GR, P, dLdv, tmid, k_hi, k_lo);
    return cudaGetLastError();
}

cudaError_t launch_gather(const double* src, const int* idx, double* dst, int n, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    gather_kernel<<<(n + 255) / 256, 256, 0, st>>>(src, idx, dst, n);
    return cudaGetLastError();
}

cudaError_t launch_scatter(const double* src, const int* idx, double* dst, int n, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    scatter_kernel<<<(n + 255) / 256, 256, 0, st>>>(src, idx, dst, n);
    return cudaGetLastError();
}

cudaError_t launch_reduce_cols(const double* grad, const int* col_off, const int* flat, const float* scale,
                               float* out, int ncol, cudaStream_t st) {
    if (ncol <= 0) return cudaSuccess;
    reduce_cols_kernel<<<(ncol + 255) / 256, 256, 0, st>>>(grad, col_off, flat, scale, out, ncol);
    return cudaGetLastError();
}

}  // namespace hx
