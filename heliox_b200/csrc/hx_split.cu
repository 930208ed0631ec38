// hx_split.cu -- step kernels for one cell larger than a CTA (config 3 scale).
//
// The plan (hx_plan.cpp, split_cell) cuts the tree into a top part, solved by
// CTA 0, and subtrees packed into the other CTAs; each CTA keeps its nodes in
// shared memory exactly as the per-pack kernels do.  The tree solve of one
// step then runs in three stages: every subtree eliminates itself up to its
// root; CTA 0 folds the subtree roots into the top part, solves it and hands
// each subtree the solution at its root's parent; the subtrees back-substitute.
// The stages are ordered by grid barriers of a cooperative launch.  The
// forward overlaps stage 3 of step k with stage 1 of step k+1 (and CTA 0's
// whole step sits between the two barriers), so each step costs two barriers:
//
//   subtree CTAs:  ..tri(k) | B1 | B2 | back(k) update(k) tape/assemble/tri(k+1) | B1 ..
//   CTA 0:         ........ | B1 | assemble(k) tri back update | B2 | ........
//
// Values crossing CTAs: the eliminated diagonal / rhs of each subtree root
// (xd, xrhs), the solution at its parent (xx), the root's v (xv, for the
// parent's axial current) and the parent's v (xvp, for the root's).  The
// backward runs the same stages on the transposed system; CTA 0 applies the
// VJP of step k at the start of its next stage, once the subtrees have
// published w at their roots.
//
// Every barrier wait is bounded: a barrier that gives up sets *err, later
// barriers return at once and the kernels finish their loops without
// waiting; the host reports the error.
#include <cuda_runtime.h>

#include "hx_dev.hpp"
#include "hx_kernels.hpp"
#include "hx_mech.cuh"
#include "hx_step.cuh"

namespace hx {

// Grid barrier over the cooperative launch.  gen: the generation this CTA
// expects to see released (kept by thread 0).
__device__ __forceinline__ void grid_sync(const DevSplit& X, unsigned& gen) {
    __syncthreads();
    if (threadIdx.x == 0) {
        volatile unsigned* vgen = X.bar + 1;
        volatile int* verr = X.err;
        __threadfence();
        if (*verr == 0) {
            const unsigned arrived = atomicAdd(X.bar, 1u);
            if (arrived == (unsigned)X.nblocks - 1u) {
                atomicExch(X.bar, 0u);
                __threadfence();
                atomicAdd(X.bar + 1, 1u);
            } else {
                long long it = 0;
                while (*vgen == gen && *verr == 0) {
                    if (++it > X.spin_limit) {
                        atomicOr(X.err, 1);
                        break;
                    }
                    __nanosleep(100);
                }
            }
        }
        __threadfence();
        gen++;
    }
    __syncthreads();
}

// axial terms of a split cell: parent / children coded -(2 + subtree id)
// live in other CTAs (their v in xvp / xv, their a from global memory)
template <bool kRhs>
__device__ __forceinline__ void axial_split(const DevGroup& G, const Meta& M, const DevSplit& X, int i,
                                            const double* __restrict__ sv, const double* __restrict__ sa,
                                            const double* __restrict__ sb, double& r, double& dd) {
    const double vi = sv[i];
    const int par = M.par[i];
    if (par >= 0) {
        if (kRhs) r -= sb[i] * (sv[par] - vi);
        dd -= sb[i];
    } else if (par <= -2) {
        if (kRhs) r -= sb[i] * (X.xvp[-par - 2] - vi);
        dd -= sb[i];
    }
    const int c1 = M.cho[i + 1];
    for (int k = M.cho[i]; k < c1; ++k) {
        const int c = M.ch[k];
        if (c >= 0) {
            const double ac = sa[c];
            if (kRhs) r += ac * (vi - sv[c]);
            dd -= ac;
        } else {
            const int id = -c - 2;
            const double ac = __ldg(G.a + X.sub_root[id]);
            if (kRhs) r += ac * (vi - X.xv[id]);
            dd -= ac;
        }
    }
}

// Triangularisation of one cell group (as hines_cell) with coded children:
// a child in another CTA folds in with its published (xd, xrhs).
template <bool kTransposed>
__device__ __forceinline__ void tri_split(const DevGroup& G, const Meta& M, const Grp& g, const DevSplit& X,
                                          const double* __restrict__ sa, const double* __restrict__ sb,
                                          double* __restrict__ d, double* __restrict__ rhs) {
    const double* __restrict__ A = kTransposed ? sb : sa;
    const double* __restrict__ U = kTransposed ? sa : sb;
    const int* lo = M.lvl + g.lvl;
    for (int L = g.nlev - 1; L >= 0; --L) {
        const int b1 = lo[L + 1];
        for (int br = lo[L] + g.tl; br < b1; br += g.nt) {
            const int h = M.bh[br], e = M.be[br];
            double de = d[e], re = rhs[e];
            const int c1 = M.bco[br + 1];
            for (int k = M.bco[br]; k < c1; ++k) {
                const int c = M.bc[k];
                if (c >= 0) {
                    de = __fma_rn(-(A[c] * U[c]), d[c], de);
                    re = __fma_rn(-A[c], rhs[c], re);
                } else {
                    const int id = -c - 2, gr = X.sub_root[id];
                    const double Ac = kTransposed ? __ldg(G.b + gr) : __ldg(G.a + gr);
                    const double Uc = kTransposed ? __ldg(G.a + gr) : __ldg(G.b + gr);
                    de = __fma_rn(-(Ac * Uc), X.xd[id], de);
                    re = __fma_rn(-Ac, X.xrhs[id], re);
                }
            }
            double pp = de, qq = 1.0, yy = re;
            int j = e;
            for (; j - h >= kBlk; j -= kBlk) {
                tri_block<false>(d, rhs, A, U, j, kBlk, pp, qq, yy);
                const double s = rescale_pow2(pp);
                pp *= s;
                qq *= s;
                yy *= s;
            }
            if (j > h) tri_block<true>(d, rhs, A, U, j, j - h, pp, qq, yy);
            const double ip = rcp_nz(pp);
            d[h] = qq * ip;
            rhs[h] = yy * ip;
        }
        g.sync();
    }
}

// Back-substitution of one cell group; a root whose parent is in another CTA
// starts from the published solution there (xx).
template <bool kTransposed>
__device__ __forceinline__ void back_split(const Meta& M, const Grp& g, const DevSplit& X,
                                           const double* __restrict__ sa, const double* __restrict__ sb,
                                           const double* __restrict__ d, double* __restrict__ rhs) {
    const double* __restrict__ U = kTransposed ? sa : sb;
    const int* lo = M.lvl + g.lvl;
    for (int L = 0; L < g.nlev; ++L) {
        const int b1 = lo[L + 1];
        for (int br = lo[L] + g.tl; br < b1; br += g.nt) {
            const int h = M.bh[br], e = M.be[br];
            const int par = M.bp[br];
            double x = rhs[h];
            if (par >= 0)
                x = __fma_rn(-(U[h] * d[h]), rhs[par], x);
            else if (par <= -2)
                x = __fma_rn(-(U[h] * d[h]), X.xx[-par - 2], x);
            rhs[h] = x;
            int j = h + 1;
            for (; e - j + 1 >= kBlk; j += kBlk) back_block<false>(d, rhs, U, j, kBlk, x);
            if (j <= e) back_block<true>(d, rhs, U, j, e - j + 1, x);
        }
        g.sync();
    }
}

// ------------------------------------------------------------------ forward
__global__ void __launch_bounds__(kSplitThreads, 1) split_fwd_kernel(DevGroup G, DevState S, DevTape T, int write_tape,
                                                                 DevProbe P, double* __restrict__ trace,
                                                                 const double* __restrict__ tmid, int k0, int k1,
                                                                 DevSplit X) {
    extern __shared__ double smem[];
    const int p = blockIdx.x;
    const int N_ = G.smem_n;
    double* sv = smem;
    double* srhs = sv + N_;
    double* sd = srhs + N_;
    double* sa = sd + N_;
    double* sb = sa + N_;
    double* sgm = sb + N_;
    double* sgh = sgm + N_;
    double* sgn = sgh + N_;
    Meta M;
    Grp g;
    const bool active = setup_pack(G, p, reinterpret_cast<int*>(sgn + N_), M, g);
    const bool top = (p == 0);
    unsigned gen = 0;
    if (threadIdx.x == 0) gen = *(volatile unsigned*)(X.bar + 1);
    const int pb = G.pack_node_off[p];
    const int i0 = active ? g.nb : 0, i1 = active ? g.nb + g.n : 0;
    const int sub = top ? -1 : g.slot - 1;  // subtree id of a subtree group (one slot in pack 0)
    if (active) {
        for (int i = i0 + g.tl; i < i1; i += g.nt) {
            sv[i] = S.v[pb + i];
            sa[i] = G.a[pb + i];
            sb[i] = G.b[pb + i];
            sgm[i] = S.m[pb + i];
            sgh[i] = S.h[pb + i];
            sgn[i] = S.n[pb + i];
        }
        g.sync();
    }
    const int q0 = active ? P.slot_off[g.slot] : 0, q1 = active ? P.slot_off[g.slot + 1] : 0;
    auto trace_row = [&](int row) {
        if (!trace) return;
        for (int q = q0 + g.tl; q < q1; q += g.nt) trace[(size_t)row * P.nprobe + P.slot[q]] = sv[P.local[q]];
    };
    auto tape_row = [&](int k) {
        if (!write_tape) return;
        const size_t off = (size_t)(k - T.k_base) * (size_t)G.nnode + pb;
        for (int i = i0 + g.tl; i < i1; i += g.nt) {
            T.v[off + i] = sv[i];
            T.m[off + i] = sgm[i];
            T.h[off + i] = sgh[i];
            T.n[off + i] = sgn[i];
        }
    };
    auto assemble_all = [&](int k) {
        const double tm = tmid[k];
        for (int i = i0 + g.tl; i < i1; i += g.nt) {
            double r, dd;
            const int fl = M.flag[i];
            NodePar q;
            load_par(G, pb + i, fl, q);
            assemble<true, false, true>(G, M, pb, i, fl, q, sv[i], sv, sa, sb, sgm[i], sgh[i], sgn[i], tm, r, dd);
            axial_split<true>(G, M, X, i, sv, sa, sb, r, dd);
            srhs[i] = r;
            sd[i] = dd;
        }
        g.sync();
    };
    auto update_all = [&]() {
        for (int i = i0 + g.tl; i < i1; i += g.nt) {
            const double vn = sv[i] + srhs[i];
            sv[i] = vn;
            if (M.flag[i] & kHasHH) {
                HHRates r;
                hh_rates(vn, G.q10, r);
                sgm[i] = gate_step(sgm[i], r.inf[0], r.k[0], G.dt);
                sgh[i] = gate_step(sgh[i], r.inf[1], r.k[1], G.dt);
                sgn[i] = gate_step(sgn[i], r.inf[2], r.k[2], G.dt);
            }
        }
        g.sync();
    };
    // interface values of the initial state
    if (active) {
        if (top) {
            for (int id = g.tl; id < X.nsub; id += g.nt) X.xvp[id] = sv[X.sub_parent[id]];
        } else if (g.tl == 0) {
            X.xv[sub] = sv[i0];
        }
        if (k0 == 0) trace_row(0);
    }
    grid_sync(X, gen);
    if (!top && active && k0 < k1) {
        tape_row(k0);
        assemble_all(k0);
        tri_split<false>(G, M, g, X, sa, sb, sd, srhs);
        if (g.tl == 0) {
            X.xd[sub] = sd[i0];
            X.xrhs[sub] = srhs[i0];
        }
    }
    for (int k = k0; k < k1; ++k) {
        grid_sync(X, gen);  // B1: subtree roots eliminated for step k
        if (top && active) {
            tape_row(k);
            assemble_all(k);
            tri_split<false>(G, M, g, X, sa, sb, sd, srhs);
            back_split<false>(M, g, X, sa, sb, sd, srhs);
            for (int id = g.tl; id < X.nsub; id += g.nt) X.xx[id] = srhs[X.sub_parent[id]];
            update_all();
            for (int id = g.tl; id < X.nsub; id += g.nt) X.xvp[id] = sv[X.sub_parent[id]];
            trace_row(k + 1);
        }
        grid_sync(X, gen);  // B2: the top part is solved and updated
        if (!top && active) {
            back_split<false>(M, g, X, sa, sb, sd, srhs);
            update_all();
            if (g.tl == 0) X.xv[sub] = sv[i0];
            trace_row(k + 1);
            if (k + 1 < k1) {
                tape_row(k + 1);
                assemble_all(k + 1);
                tri_split<false>(G, M, g, X, sa, sb, sd, srhs);
                if (g.tl == 0) {
                    X.xd[sub] = sd[i0];
                    X.xrhs[sub] = srhs[i0];
                }
            }
        }
    }
    if (!active) return;
    if (write_tape) {
        const size_t off = (size_t)(k1 - T.k_base) * (size_t)G.nnode + pb;
        for (int i = i0 + g.tl; i < i1; i += g.nt) T.v[off + i] = sv[i];
    }
    for (int i = i0 + g.tl; i < i1; i += g.nt) {
        S.v[pb + i] = sv[i];
        S.m[pb + i] = sgm[i];
        S.h[pb + i] = sgh[i];
        S.n[pb + i] = sgn[i];
    }
}

// ------------------------------------------------------------------ backward
__global__ void __launch_bounds__(kSplitThreads, 1) split_bwd_kernel(DevGroup G, DevTape T, DevAdj Ad, DevGrad GR,
                                                                 DevProbe P, const double* __restrict__ dLdv,
                                                                 const double* __restrict__ tmid, int k_hi, int k_lo,
                                                                 DevSplit X) {
    extern __shared__ double smem[];
    const int p = blockIdx.x;
    const int N_ = G.smem_n;
    double* slv = smem;
    double* sw = slv + N_;
    double* sd = sw + N_;
    double* sa = sd + N_;
    double* sb = sa + N_;
    double* svk = sb + N_;
    double* svk1 = svk + N_;
    double* slm = svk1 + N_;
    double* slh = slm + N_;
    double* sln = slh + N_;
    Meta M;
    Grp g;
    const bool active = setup_pack(G, p, reinterpret_cast<int*>(sln + N_), M, g);
    const bool top = (p == 0);
    unsigned gen = 0;
    if (threadIdx.x == 0) gen = *(volatile unsigned*)(X.bar + 1);
    const int pb = G.pack_node_off[p];
    const int i0 = active ? g.nb : 0, i1 = active ? g.nb + g.n : 0;
    const int sub = top ? -1 : g.slot - 1;
    const double dt = G.dt, q10 = G.q10;
    if (active) {
        for (int i = i0 + g.tl; i < i1; i += g.nt) {
            slv[i] = Ad.lv[pb + i];
            sa[i] = G.a[pb + i];
            sb[i] = G.b[pb + i];
            slm[i] = Ad.lm[pb + i];
            slh[i] = Ad.lh[pb + i];
            sln[i] = Ad.ln[pb + i];
            svk1[i] = T.v[(size_t)(k_hi - T.k_base) * (size_t)G.nnode + pb + i];
        }
        g.sync();
    }
    const int q0 = active ? P.slot_off[g.slot] : 0, q1 = active ? P.slot_off[g.slot + 1] : 0;
    // lv += dL/dv_{k+1} at the probes, tape v_k into svk, S+A phase, transposed elimination
    auto stage1 = [&](int k) {
        const size_t off = (size_t)(k - T.k_base) * (size_t)G.nnode + pb;
        copy_in(svk, T.v + off, i0, i1, g);
        probe_inject(P, q0, q1, dLdv + (size_t)(k + 1) * P.nprobe, slv, g);
        g.sync();
        const double tm = tmid[k];
        for (int i = i0 + g.tl; i < i1; i += g.nt) {
            double mu = slv[i];
            const int fl = M.flag[i];
            double gm = 0.0, gh = 0.0, gn = 0.0;
            if (fl & kHasHH) {
                gm = T.m[off + i];
                gh = T.h[off + i];
                gn = T.n[off + i];
                HHRatesD R;
                hh_rates_d(svk1[i], q10, R);
                const double x[3] = {gm, gh, gn};
                double lam[3] = {slm[i], slh[i], sln[i]};
#pragma unroll
                for (int q = 0; q < 3; ++q) {
                    const double E = exp(-dt * R.k[q]);
                    const double dnew = (1.0 - E) * R.dinf[q] + (R.inf[q] - x[q]) * E * dt * q10 * R.ds[q];
                    mu += lam[q] * dnew;
                    lam[q] *= E;
                }
                slm[i] = lam[0];
                slh[i] = lam[1];
                sln[i] = lam[2];
            }
            NodePar q;
            load_par(G, pb + i, fl, q);
            double r, dd;
            assemble<false, false, true>(G, M, pb, i, fl, q, svk[i], svk, sa, sb, gm, gh, gn, tm, r, dd);
            axial_split<false>(G, M, X, i, svk, sa, sb, r, dd);
            sd[i] = dd;
            sw[i] = mu;
            slv[i] = mu;
        }
        g.sync();
        tri_split<true>(G, M, g, X, sa, sb, sd, sw);
    };
    // VJPs of step k (w in sw, v_k in svk, v_{k+1} in svk1); lv := dL/dv_k
    auto vjp = [&](int k) {
        const size_t off = (size_t)(k - T.k_base) * (size_t)G.nnode + pb;
        const double tm = tmid[k];
        for (int i = i0 + g.tl; i < i1; i += g.nt) {
            const int gi = pb + i;
            const int fl = M.flag[i];
            NodePar q;
            load_par(G, gi, fl, q);
            const double w = sw[i];
            const double vk = svk[i];
            const double ld = -w * (svk1[i] - vk);
            double lm = slm[i], lh = slh[i], ln = sln[i];
            double lvn = vjp_mech(G, GR, T, off, i, gi, fl, q, w, vk, ld, tm, slv[i], lm, lh, ln);
            if (fl & kHasHH) {
                slm[i] = lm;
                slh[i] = lh;
                sln[i] = ln;
            }
            const int par = M.par[i];
            if (par >= 0)
                lvn += sb[i] * w - sa[i] * sw[par];
            else if (par <= -2)
                lvn += sb[i] * w - sa[i] * X.xx[-par - 2];
            const int c1n = M.cho[i + 1];
            for (int k2 = M.cho[i]; k2 < c1n; ++k2) {
                const int c = M.ch[k2];
                if (c >= 0) {
                    lvn += sa[c] * w - sb[c] * sw[c];
                } else {
                    const int id = -c - 2, gr = X.sub_root[id];
                    lvn += __ldg(G.a + gr) * w - __ldg(G.b + gr) * X.xv[id];
                }
            }
            slv[i] = lvn;
        }
        double* tmp = svk1;
        svk1 = svk;
        svk = tmp;
        g.sync();
    };
    if (!top && active && k_lo < k_hi) {
        stage1(k_hi - 1);
        if (g.tl == 0) {
            X.xd[sub] = sd[i0];
            X.xrhs[sub] = sw[i0];
        }
    }
    grid_sync(X, gen);  // the interface arrays of the first stage are visible
    for (int k = k_hi - 1; k >= k_lo; --k) {
        grid_sync(X, gen);  // B1
        if (top && active) {
            if (k + 1 < k_hi) vjp(k + 1);
            stage1(k);
            back_split<true>(M, g, X, sa, sb, sd, sw);
            for (int id = g.tl; id < X.nsub; id += g.nt) X.xx[id] = sw[X.sub_parent[id]];
            g.sync();
        }
        grid_sync(X, gen);  // B2
        if (!top && active) {
            back_split<true>(M, g, X, sa, sb, sd, sw);
            if (g.tl == 0) X.xv[sub] = sw[i0];
            vjp(k);
            if (k > k_lo) {
                stage1(k - 1);
                if (g.tl == 0) {
                    X.xd[sub] = sd[i0];
                    X.xrhs[sub] = sw[i0];
                }
            }
        }
    }
    grid_sync(X, gen);  // the subtree roots' w of step k_lo is published
    if (top && active && k_lo < k_hi) vjp(k_lo);
    if (!active) return;
    for (int i = i0 + g.tl; i < i1; i += g.nt) {
        Ad.lv[pb + i] = slv[i];
        Ad.lm[pb + i] = slm[i];
        Ad.lh[pb + i] = slh[i];
        Ad.ln[pb + i] = sln[i];
    }
}

const void* split_fwd_kernel_ptr() { return (const void*)split_fwd_kernel; }
const void* split_bwd_kernel_ptr() { return (const void*)split_bwd_kernel; }

cudaError_t configure_split(size_t smem_fwd, size_t smem_bwd) {
    cudaError_t e = cudaFuncSetAttribute(split_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_fwd);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(split_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bwd);
}

cudaError_t launch_split_fwd(const DevGroup& G, const DevState& S, const DevTape& T, int write_tape, const DevProbe& P,
                             double* trace, const double* tmid, int k0, int k1, const DevSplit& X, cudaStream_t st) {
    DevGroup g = G;
    DevState s = S;
    DevTape t = T;
    DevProbe pr = P;
    DevSplit x = X;
    void* args[] = {&g, &s, &t, &write_tape, &pr, &trace, &tmid, &k0, &k1, &x};
    return cudaLaunchCooperativeKernel((const void*)split_fwd_kernel, dim3(G.npack), dim3(kSplitThreads), args,
                                       split_fwd_smem_bytes(G), st);
}

cudaError_t launch_split_bwd(const DevGroup& G, const DevTape& T, const DevAdj& A, const DevGrad& GR, const DevProbe& P,
                             const double* dLdv, const double* tmid, int k_hi, int k_lo, const DevSplit& X,
                             cudaStream_t st) {
    DevGroup g = G;
    DevTape t = T;
    DevAdj a = A;
    DevGrad gr = GR;
    DevProbe pr = P;
    DevSplit x = X;
    void* args[] = {&g, &t, &a, &gr, &pr, &dLdv, &tmid, &k_hi, &k_lo, &x};
    return cudaLaunchCooperativeKernel((const void*)split_bwd_kernel, dim3(G.npack), dim3(kSplitThreads), args,
                                       split_bwd_smem_bytes(G), st);
}

}  // namespace hx
