// hx_kernels.cu -- fused per-timestep kernels for sm_100a (fp64).
//
// One CTA owns one pack of whole cells for a launch's window of timesteps
// (one CTA per SM; the planner packs cells so that as few waves as the shared
// memory allows hold them).  Shared memory holds only what neighbouring nodes
// exchange: the Hines system (v, rhs, d, a, b in the forward; w, d, a, b in the
// reverse sweep), four doubles per branch segment for the reduced-tree solve
// and the pack's topology tables.  Gates, node adjoints, gradient
// accumulators, synapse states and parameters live in global memory (L2), each
// read and written only by the thread that owns the node.  Each cell is
// advanced by its own group of warps, synchronised by a named barrier, so the
// serial parts of one cell's Hines solve overlap the mechanism arithmetic of
// the other cells on the same SM.
//
// Forward step (reference: Simulate::fadvance_cpu, src/simulate.cpp:410-442):
//   A  node-parallel: the gates' cnexp update from v_k (nonvint_cpu,
//      simulate.cpp:784-852, applied one step late so the gates are read once
//      a step), mechanism currents with the finite-difference conductance
//      (mech_template.cuh:589-648), capacitance jacobian (capac.cpp:68-78)
//      and the axial terms (simulate.cpp:542-555) gathered per node in the
//      order the reference's scatter loop applies them;
//   B  Hines solve by segments (hines_rt, hx_step.cuh);
//   C  v += dv (update_cpu, simulate.cpp:759-770).
// Backward step: the transpose of the above, in reverse (no reference
// counterpart; the reference's only gradient is the LRDS replay).
#include <cuda_runtime.h>

#include "hx_dev.hpp"
#include "hx_kernels.hpp"
#include "hx_mech.cuh"
#include "hx_step.cuh"

namespace hx {

// ------------------------------------------------------------------ init
__global__ void init_state_kernel(DevGroup G, DevState S, double v_init) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= G.nnode) return;
    S.v[i] = v_init;
    double m = 0.0, h = 0.0, n = 0.0;
    if (G.node_flags[i] & kHasHH) {  // hh INITIAL: gates at steady state (hh_templated.cu:111-122)
        HHRates r;
        hh_rates(v_init, G.q10, r);
        m = r.inf[0];
        h = r.inf[1];
        n = r.inf[2];
    }
    S.m[i] = m;
    S.h[i] = h;
    S.n[i] = n;
}

// finitialize of the library mechanisms (after init_state_kernel)
__global__ void lib_init_kernel(DevLib L, int nnode, double v_init) {
    const int gi = blockIdx.x * blockDim.x + threadIdx.x;
    if (gi < nnode) lib::lib_init(L, gi, v_init);
}

// ------------------------------------------------------------------ forward
// kNet adds, per step: PreSyn threshold detection at the step's start
// (PreSyn::threshold_detect_cpu, presyn.cpp:133-177: a spike at t_k when
// v > threshold and the hysteresis flag is clear), delivery of the step's
// events from bucket k (net_receive: A += w*fA, B += w*fB; the reference's
// delivery condition deliver_time <= t + dt/2 is resolved into the bucket
// index when an event is routed), the network currents and the synapse /
// graded-synapse state updates.  In a coupled launch (gaps, graded
// synapses) partner voltages come from N.vpeer and v_{k+1} goes to N.vout,
// so that no CTA reads a value another CTA rewrites; a grid-synchronous
// coupled launch (N.gsync, cooperative) runs many steps, v_k in
// N.vbuf[k & 1], with one grid barrier after each step's v_{k+1} is stored.
//
// kLib adds the library mechanisms (hx_lib.cuh): their currents after the
// other mechanisms in phase A, their state updates in phase C, and their
// states in the tape (the cell's contiguous state range, row per step).
template <bool kNet, bool kLib = false, bool kCpl = false>
__global__ void __launch_bounds__(kThreads, 1) fwd_kernel(DevGroup G, DevState S, DevTape T, int write_tape,
                                                           DevProbe P, double* __restrict__ trace,
                                                           const double* __restrict__ tmid, int k0, int k1, DevNet N,
                                                           DevLib L) {
    extern __shared__ double smem[];
    const int p = blockIdx.x;
    const int N_ = G.smem_n;
    double* sv = smem;
    double* srhs = sv + N_;
    double* sd = srhs + N_;
    double* sa = sd + N_;
    double* sb = sa + N_;
    double* scd = sb + N_;  // per-segment contributions and couplings of hines_rt
    double* scr = scd + G.smem_br;
    double* sfe = scr + G.smem_br;
    double* sge = sfe + G.smem_br;
    double* send = sge + G.smem_br;
    Meta M;
    Grp g;
    if (!setup_pack(G, p, reinterpret_cast<int*>(send), M, g)) return;
    const int pb = G.pack_node_off[p];
    const int i0 = g.nb, i1 = g.nb + g.n;
    for (int i = i0 + g.tl; i < i1; i += g.nt) {
        sv[i] = S.v[pb + i];
        sa[i] = G.a[pb + i];
        sb[i] = G.b[pb + i];
    }
    // kNet: the cell's synapses [c0, c1) (global ids); their states N.sA/N.sB
    // are touched only by the thread that owns the synapse's node
    int c0 = 0, c1 = 0, psnode = -1, psflag = 0, gid = 0;
    double psthr = 0.0;
    if (kNet) {
        c0 = N.node_syn_off[pb + i0];
        c1 = N.node_syn_off[pb + i1];
        psnode = N.cs_ps_node[g.slot];
        if (psnode >= 0) {
            psflag = N.cs_ps_flag[g.slot];
            psthr = N.cs_ps_thr[g.slot];
            gid = N.cs_gid[g.slot];
        }
    }
    const int q0 = P.slot_off[g.slot], q1 = P.slot_off[g.slot + 1];
    int ls0 = 0, ls1 = 0;  // kLib: the cell's range of the flat state array
    if (kLib) {
        ls0 = L.ent_st[L.node_off[pb + i0]];
        ls1 = L.ent_st[L.node_off[pb + i1]];
    }
    // kNet: the event count of the next step's bucket, read one step ahead
    // (all buckets of the launch's steps are routed before the launch)
    int ev_next = (kNet && k0 < k1) ? N.ev_cnt[(size_t)k0 * N.npack + p] : 0;
    // grid-synchronous coupled launch: the CTA's active threads and barrier generation
    const bool gs = kCpl && N.gsync;
    int nact = 0;
    unsigned gen = 0;
    if (gs) {
        const int s1 = G.pack_slot_off[p + 1] - 1;
        nact = 32 * (G.cs_warp0[s1] + G.cs_nwarp[s1]);
        if (threadIdx.x == 0) gen = *(volatile unsigned*)(N.gbar + 1);
    }
    g.sync();
    if (k0 == 0 && trace)
        for (int q = q0 + g.tl; q < q1; q += g.nt) trace[P.slot[q]] = sv[P.local[q]];
    for (int k = k0; k < k1; ++k) {
        const double* vpeer = kCpl ? (gs ? N.vbuf + (size_t)(k & 1) * (size_t)G.nnode : N.vpeer) : nullptr;
        // tape rows are written with streaming stores (evict first) so that the
        // row stream does not push the per-node parameters out of L2
        const size_t toff = (size_t)(k - T.k_base) * (size_t)G.nnode + pb;
        if (write_tape)
            for (int i = i0 + g.tl; i < i1; i += g.nt) __stcs(T.v + toff + i, sv[i]);
        if (kLib && write_tape) {
            double* row = L.tape + (size_t)(k - L.k_base) * (size_t)L.nst;
            for (int j = ls0 + g.tl; j < ls1; j += g.nt) __stcs(row + j, L.st[j]);
        }
        if (kNet) {
            if (N.detect && g.tl == 0 && psnode >= 0) {
                const double pv = sv[psnode];
                if (pv > psthr && !psflag) {
                    const int q = atomicAdd(N.win_n, 1);
                    if (q < N.win_cap) N.win_spk[q] = make_int2(gid, k);
                    psflag = 1;
                } else if (pv <= psthr) {
                    psflag = 0;
                }
            }
            // the step's events of this pack: the owner of the synapse's node adds them
            const size_t b = (size_t)k * N.npack + p;
            const int cnt = min(ev_next, N.ev_cap);
            if (k + 1 < k1) ev_next = N.ev_cnt[b + N.npack];
            const int* ev = N.ev_syn + b * N.ev_cap;
            for (int e = 0; e < cnt; ++e) {
                const int j = ev[e];
                if (j >= c0 && j < c1 && (__ldg(N.syn_node + j) - pb - i0) % g.nt == g.tl) {
                    const double w = __ldg(N.syn_w + j);
                    N.sA[j] += w * __ldg(N.syn_fA + j);
                    N.sB[j] += w * __ldg(N.syn_fB + j);
                }
            }
        }
        const double tm = tmid[k];
        // A: gates of step k, tape row k, assembly.  The gates live in S.m/h/n;
        // their cnexp update from v_k is applied here, one step late, so that
        // they are read once per step together with the parameters (at the
        // launch's first step S holds the current gates already).
        SynNext nx;
        if (kNet) syn_next(G, N, M, pb, i0 + g.tl, i1, nx);
        for (int i = i0 + g.tl; i < i1; i += g.nt) {
            const int fl = M.flag[i];
            NodePar q;
            load_par(G, pb + i, fl, q);
            SynPre sp;
            if (kNet) {
                load_syn(N, nx, N.sA, N.sB, sp);
                syn_next(G, N, M, pb, i + g.nt, i1, nx);
            }
            double gm = 0.0, gh = 0.0, gn = 0.0;
            if (fl & kHasHH) {
                gm = S.m[pb + i];
                gh = S.h[pb + i];
                gn = S.n[pb + i];
            }
            const double vi = sv[i];
            if ((fl & kHasHH) && k > k0) {
                HHRates rt;
                hh_rates(vi, G.q10, rt);
                gm = gate_step(gm, rt.inf[0], rt.k[0], G.dt);
                gh = gate_step(gh, rt.inf[1], rt.k[1], G.dt);
                gn = gate_step(gn, rt.inf[2], rt.k[2], G.dt);
                S.m[pb + i] = gm;
                S.h[pb + i] = gh;
                S.n[pb + i] = gn;
            }
            if (write_tape && (fl & kHasHH)) {
                __stcs(T.m + toff + i, gm);
                __stcs(T.h + toff + i, gh);
                __stcs(T.n + toff + i, gn);
            }
            double r, dd;
            if (kNet) {
                const int gi = pb + i;
                if (kCpl && (fl & kHasCpl)) {  // graded synapses: s_k from s_{k-1} and vpre_k (deferred cnexp update)
                    const int r1 = __ldg(N.node_gr_off + gi + 1);
                    for (int j = __ldg(N.node_gr_off + gi); j < r1; ++j) {
                        double sj = N.gr_s[j];
                        if (write_tape && k == T.k_base) N.tS[(size_t)j] = sj;  // row 0: s_{k_base - 1}
                        if (k > 0) {
                            const double vpre = __ldcg(vpeer + __ldg(N.gr_pre + j));
                            const double inf = 1.0 / (1.0 + exp((__ldg(N.gr_vth + j) - vpre) / __ldg(N.gr_delta + j)));
                            const double tau = (1.0 - inf) / __ldg(N.gr_k + j);
                            sj = inf + (sj - inf) * exp(-G.dt / tau);
                            N.gr_s[j] = sj;
                        }
                        if (write_tape) N.tS[(size_t)(k - T.k_base + 1) * N.ngr + j] = sj;
                    }
                }
                if (kLib) {  // library channels after the network mechanisms (CoreNEURON type order)
                    double ica;
                    assemble<true, true, false, true, kCpl>(G, M, pb, i, fl, q, vi, sv, sa, sb, gm, gh, gn, tm, r, dd,
                                                            N, N.sA, N.sB, sp, N.gr_s, vpeer, &L, L.st, &ica);
                    L.nica[pb + i] = ica;
                } else {
                    assemble<true, true, false, false, kCpl>(G, M, pb, i, fl, q, vi, sv, sa, sb, gm, gh, gn, tm, r,
                                                             dd, N, N.sA, N.sB, sp, N.gr_s, vpeer);
                }
            } else if (kLib) {
                double ica;
                assemble<true, false, false, true>(G, M, pb, i, fl, q, vi, sv, sa, sb, gm, gh, gn, tm, r, dd, N,
                                                   nullptr, nullptr, SynPre{}, nullptr, nullptr, &L, L.st, &ica);
                L.nica[pb + i] = ica;
            } else {
                assemble<true>(G, M, pb, i, fl, q, vi, sv, sa, sb, gm, gh, gn, tm, r, dd);
            }
            srhs[i] = r;
            sd[i] = dd;
        }
        g.sync();
        // B: Hines solve (rhs := dv)
        hines_rt<false>(M, g, sa, sb, sd, srhs, scd, scr, sfe, sge);
        // C: v update (the gates follow in the next step's A, or below)
        for (int i = i0 + g.tl; i < i1; i += g.nt) sv[i] = sv[i] + srhs[i];
        if (kNet) {
            // the cell's synapses, coalesced over its threads (every owner's
            // reads of phase A are behind the barrier above; the next step's
            // deliveries behind the one below): states after this step's
            // deliveries into the tape, then the decay x + c (0 - x)
            // (expsyn.cpp:125-134, exp2syn_temp.cuh:51-58)
            const size_t toffs = (size_t)(k - T.k_base) * (size_t)N.nsyn;
            for (int j = c0 + g.tl; j < c1; j += g.nt) {
                const double A = N.sA[j], B = N.sB[j];
                if (N.tA) {
                    N.tA[toffs + j] = A;
                    N.tB[toffs + j] = B;
                }
                N.sA[j] = A + __ldg(N.syn_cA + j) * (0.0 - A);
                N.sB[j] = B + __ldg(N.syn_cB + j) * (0.0 - B);
            }
        }
        // library states at the new v, type by type over this thread's nodes
        if (kLib) lib::lib_state_cell(L, pb, i0, i1, g.tl, g.nt, sv);
        g.sync();
        if (trace)
            for (int q = q0 + g.tl; q < q1; q += g.nt) trace[(size_t)(k + 1) * P.nprobe + P.slot[q]] = sv[P.local[q]];
        if (gs) {  // v_{k+1} of the cell for every partner, then the step's grid barrier
            double* vn = N.vbuf + (size_t)((k + 1) & 1) * (size_t)G.nnode + pb;
            for (int i = i0 + g.tl; i < i1; i += g.nt) __stcg(vn + i, sv[i]);
            if (k + 1 < k1) grid_barrier(N.gbar, N.gerr, G.npack, N.gspin, nact, gen);
        }
    }
    if (write_tape) {
        const size_t off = (size_t)(k1 - T.k_base) * (size_t)G.nnode + pb;
        for (int i = i0 + g.tl; i < i1; i += g.nt) __stcs(T.v + off + i, sv[i]);
        if (kLib) {
            double* row = L.tape + (size_t)(k1 - L.k_base) * (size_t)L.nst;
            for (int j = ls0 + g.tl; j < ls1; j += g.nt) __stcs(row + j, L.st[j]);
        }
    }
    double* vdst = kCpl ? N.vout : S.v;
    for (int i = i0 + g.tl; i < i1; i += g.nt) {
        if (!gs) vdst[pb + i] = sv[i];  // (grid-synchronous: stored with the last step)
        if ((M.flag[i] & kHasHH) && k1 > k0) {  // gates of step k1 (the update the last step deferred)
            const double gm = S.m[pb + i], gh = S.h[pb + i], gn = S.n[pb + i];
            HHRates rt;
            hh_rates(sv[i], G.q10, rt);
            S.m[pb + i] = gate_step(gm, rt.inf[0], rt.k[0], G.dt);
            S.h[pb + i] = gate_step(gh, rt.inf[1], rt.k[1], G.dt);
            S.n[pb + i] = gate_step(gn, rt.inf[2], rt.k[2], G.dt);
        }
    }
    if (kNet && g.tl == 0 && psnode >= 0) N.cs_ps_flag[g.slot] = psflag;
}

// ------------------------------------------------------------------ backward
// Reverse sweep over steps [k_lo, k_hi).  Per step k, with lv = dL/dv_{k+1}
// and lm/lh/ln = dL/d(gates_{k+1}):
//   S  gates_{k+1} = E*gates_k + (1-E)*inf(v_{k+1}), E = exp(-dt k(v_{k+1})):
//      mu = lv + sum lg*dgate'/dv', lg *= E;  synapse states: lx *= 1 - c;
//   A  recompute the diagonal d_k (FD conductances at v_k, gates_k);
//   B  w = M_k^{-T} mu (Hines with a and b swapped);
//   V  lambda_d = -w*dv; VJPs of rhs_k and d_k into lv (dL/dv_k), the gate
//      and synapse adjoints and the per-node parameter gradients; then the
//      weight gradients of the step's events (A' = A + fA w, B' = B + fB w).
// The FD conductance expressions are differentiated as the functions of the
// parameters they are (for currents linear in v their v-derivative is 0).
// Coupled launches (one step): the dL/dv_k contributions of a gap or graded
// synapse to its partner node go through N.x_*_out and are gathered by the
// launch of step k-1 from N.x_*_in, in the fixed order of N.node_in.  A
// grid-synchronous coupled launch (N.gsync) runs many steps: step k writes
// N.xbuf[k & 1], step k-1 gathers it after the step's grid barrier.
// kLib: the library mechanisms' state-update adjoints join mu in S + A (their
// currents recomputed from the tape give d_k and the calcium current), the
// adjoints of their currents join dL/dv_k in V (hx_lib.cuh).
template <bool kNet, bool kLib = false, bool kCpl = false>
__global__ void __launch_bounds__(kThreads, 1) bwd_kernel(DevGroup G, DevTape T, DevAdj Ad, DevGrad GR, DevProbe P,
                                                           const double* __restrict__ dLdv,
                                                           const double* __restrict__ tmid, int k_hi, int k_lo,
                                                           DevNet N, DevLib L) {
    extern __shared__ double smem[];
    const int p = blockIdx.x;
    const int N_ = G.smem_n;
    // shared memory: the transposed system (w, d, a, b); the node adjoints
    // lv, lm, lh, ln stay in Ad and v_k, v_{k+1} are read from the tape, each
    // by the thread that owns the node
    double* sw = smem;
    double* sd = sw + N_;
    double* sa = sd + N_;
    double* sb = sa + N_;
    double* scd = sb + N_;  // per-segment contributions and couplings of hines_rt
    double* scr = scd + G.smem_br;
    double* sfe = scr + G.smem_br;
    double* sge = sfe + G.smem_br;
    double* send = sge + G.smem_br;
    Meta M;
    Grp g;
    if (!setup_pack(G, p, reinterpret_cast<int*>(send), M, g)) return;
    const int pb = G.pack_node_off[p];
    const int i0 = g.nb, i1 = g.nb + g.n;
    const double dt = G.dt, q10 = G.q10;
    double* __restrict__ lv = Ad.lv + pb;
    double* __restrict__ lmv = Ad.lm + pb;
    double* __restrict__ lhv = Ad.lh + pb;
    double* __restrict__ lnv = Ad.ln + pb;
    const bool gs = kCpl && N.gsync;
    // partner contributions to dL/dv_{k+1} written by step k+1 (its launch, or
    // its iteration of a grid-synchronous launch), in the fixed order of node_in
    auto gather_in = [&](const double* xhg, const double* xgj, const double* xgr) {
        for (int i = i0 + g.tl; i < i1; i += g.nt)
            if (M.flag[i] & kHasIn) {
                double l = lv[i];
                const int e1 = __ldg(N.node_in_off + pb + i + 1);
                for (int e = __ldg(N.node_in_off + pb + i); e < e1; ++e) {
                    const int code = __ldg(N.node_in + e), kind = code >> 28, inst = code & 0x0FFFFFFF;
                    l += __ldcg((kind == 0 ? xhg : kind == 1 ? xgj : xgr) + inst);
                }
                lv[i] = l;
            }
    };
    for (int i = i0 + g.tl; i < i1; i += g.nt) {
        sa[i] = G.a[pb + i];
        sb[i] = G.b[pb + i];
    }
    if (kCpl && !gs) gather_in(N.x_hg_in, N.x_gj_in, N.x_gr_in);
    int nact = 0;
    unsigned gen = 0;
    if (gs) {
        const int s1 = G.pack_slot_off[p + 1] - 1;
        nact = 32 * (G.cs_warp0[s1] + G.cs_nwarp[s1]);
        if (threadIdx.x == 0) gen = *(volatile unsigned*)(N.gbar + 1);
    }
    // kNet: the cell's synapses [c0, c1); their adjoints Ad.lA/Ad.lB and
    // gradients are touched only by the thread that owns the synapse's node
    int c0 = 0, c1 = 0;
    double* __restrict__ slA = Ad.lA;
    double* __restrict__ slB = Ad.lB;
    if (kNet) {
        c0 = N.node_syn_off[pb + i0];
        c1 = N.node_syn_off[pb + i1];
    }
    const int q0 = P.slot_off[g.slot], q1 = P.slot_off[g.slot + 1];
    g.sync();
    for (int k = k_hi - 1; k >= k_lo; --k) {
        const size_t off = (size_t)(k - T.k_base) * (size_t)G.nnode + pb;
        double *xo_hg = nullptr, *xo_gj = nullptr, *xo_gr = nullptr;
        if (kCpl) {
            if (gs) {
                const double* xi = N.xbuf + (size_t)((k + 1) & 1) * N.xstride;
                double* xo = N.xbuf + (size_t)(k & 1) * N.xstride;
                gather_in(xi, xi + N.nhg, xi + N.nhg + N.ngj);
                g.sync();
                xo_hg = xo;
                xo_gj = xo + N.nhg;
                xo_gr = xo + N.nhg + N.ngj;
            } else {
                xo_hg = N.x_hg_out;
                xo_gj = N.x_gj_out;
                xo_gr = N.x_gr_out;
            }
        }
        probe_inject(P, q0, q1, dLdv + (size_t)(k + 1) * P.nprobe, lv, g);
        g.sync();
        const double tm = tmid[k];
        const double* tA = kNet ? N.tA + (size_t)(k - T.k_base) * (size_t)N.nsyn : nullptr;
        const double* tB = kNet ? N.tB + (size_t)(k - T.k_base) * (size_t)N.nsyn : nullptr;
        const double* grs = kCpl ? N.tS + (size_t)(k - T.k_base + 1) * N.ngr : nullptr;
        const int ev_k = kNet ? N.ev_cnt[(size_t)k * N.npack + p] : 0;  // used at the step's end
        const double* vpeer = T.v + (size_t)(k - T.k_base) * (size_t)G.nnode;
        // S + A
        if (kNet)  // synapse-state adjoints through the decay (the cell's synapses, coalesced)
            for (int j = c0 + g.tl; j < c1; j += g.nt) {
                slA[j] *= 1.0 - __ldg(N.syn_cA + j);
                slB[j] *= 1.0 - __ldg(N.syn_cB + j);
            }
        SynNext nx;
        if (kNet) syn_next(G, N, M, pb, i0 + g.tl, i1, nx);
        for (int i = i0 + g.tl; i < i1; i += g.nt) {
            const int fl = M.flag[i];
            double mu = lv[i];
            const double vk = T.v[off + i];
            double gm = 0.0, gh = 0.0, gn = 0.0;
            if (fl & kHasHH) {
                gm = T.m[off + i];
                gh = T.h[off + i];
                gn = T.n[off + i];
                double lm = lmv[i], lh = lhv[i], ln = lnv[i];
                mu = gate_adj(T.v[off + G.nnode + i], q10, dt, gm, gh, gn, mu, lm, lh, ln);
                lmv[i] = lm;
                lhv[i] = lh;
                lnv[i] = ln;
            }
            // (parameters loaded after the rate chain: held across it they spill)
            NodePar q;
            load_par(G, pb + i, fl, q);
            double r, dd;
            if (kNet) {
                SynPre sp;
                load_syn(N, nx, tA, tB, sp);
                syn_next(G, N, M, pb, i + g.nt, i1, nx);
                if (kLib) {
                    const double* Xk = L.tape + (size_t)(k - L.k_base) * (size_t)L.nst;
                    double ica;
                    assemble<false, true, false, true, kCpl>(G, M, pb, i, fl, q, vk, nullptr, sa, sb, gm, gh, gn, tm,
                                                             r, dd, N, tA, tB, sp, grs, vpeer, &L, Xk, &ica);
                    mu += lib::lib_state_adj(L, pb + i, T.v[off + G.nnode + i], Xk, Xk + L.nst, ica);
                } else {
                    assemble<false, true, false, false, kCpl>(G, M, pb, i, fl, q, vk, nullptr, sa, sb, gm, gh, gn, tm,
                                                              r, dd, N, tA, tB, sp, grs, vpeer);
                }
            } else if (kLib) {
                const double* Xk = L.tape + (size_t)(k - L.k_base) * (size_t)L.nst;
                double ica;
                assemble<false, false, false, true>(G, M, pb, i, fl, q, vk, nullptr, sa, sb, gm, gh, gn, tm, r, dd,
                                                    N, nullptr, nullptr, SynPre{}, nullptr, nullptr, &L, Xk, &ica);
                mu += lib::lib_state_adj(L, pb + i, T.v[off + G.nnode + i], Xk, Xk + L.nst, ica);
            } else {
                assemble<false>(G, M, pb, i, fl, q, vk, nullptr, sa, sb, gm, gh, gn, tm, r, dd);
            }
            sd[i] = dd;
            sw[i] = mu;
            lv[i] = mu;
        }
        g.sync();
        // B: w = M^{-T} mu
        hines_rt<true>(M, g, sa, sb, sd, sw, scd, scr, sfe, sge);
        if (k > k_lo && g.tl < 4) {  // the next step's tape rows of the cell, into L2 (read after this phase)
            const double* row = (g.tl == 0 ? T.v : g.tl == 1 ? T.m : g.tl == 2 ? T.h : T.n) + off - G.nnode + i0;
            prefetch_l2(row, sizeof(double) * (size_t)(i1 - i0));
        }
        // V
        if (kNet) syn_next(G, N, M, pb, i0 + g.tl, i1, nx);
        for (int i = i0 + g.tl; i < i1; i += g.nt) {
            const int gi = pb + i;
            const int fl = M.flag[i];
            NodePar q;
            load_par(G, gi, fl, q);
            // the node's first synapse: tape states and reversal potential, and
            // its adjoints and e-gradient (read-modify-written below)
            SynPre sp;
            double la0 = 0.0, lb0 = 0.0, ge0 = 0.0;
            if (kNet) {
                load_syn(N, nx, tA, tB, sp);
                syn_next(G, N, M, pb, i + g.nt, i1, nx);
                if (sp.s0 < sp.s1) {
                    la0 = slA[sp.s0];
                    lb0 = slB[sp.s0];
                    if (!(GR.skip & (1u << HX_P_EXPSYN_E))) ge0 = GR.syn_e[sp.s0];
                }
            }
            const double w = sw[i];
            const double vk = T.v[off + i];
            // last read of row k+1 (streaming load); rows are read twice, once as
            // row k of their own step and once as row k+1 of the step below
            const double ld = -w * (__ldcs(T.v + off + G.nnode + i) - vk);
            const double lvn0 = lv[i];
            double lm = 0.0, lh = 0.0, ln = 0.0;
            if (fl & kHasHH) {
                lm = lmv[i];
                lh = lhv[i];
                ln = lnv[i];
            }
            double lvn = vjp_mech(G, GR, T, off, i, gi, fl, q, w, vk, ld, tm, lvn0, lm, lh, ln);
            if (kLib) lvn += lib::lib_current_adj(L, gi, vk, L.tape + (size_t)(k - L.k_base) * (size_t)L.nst, w, ld);
            if (fl & kHasHH) {
                lmv[i] = lm;
                lhv[i] = lh;
                lnv[i] = ln;
            }
            if (kNet && (fl & (kHasSyn | kHasCpl))) {
                const double sarea = sp.sarea;
                if (fl & kHasSyn) {
                    double Gs = sp.B0 - sp.A0, lG = sarea * (ld - w * (vk - sp.E0));
                    slB[sp.s0] = lb0 + lG;
                    slA[sp.s0] = la0 - lG;
                    const bool g_e = !(GR.skip & (1u << HX_P_EXPSYN_E));
                    if (g_e) GR.syn_e[sp.s0] = ge0 + w * sarea * Gs;
                    lvn -= w * sarea * Gs;
                    for (int j = sp.s0 + 1; j < sp.s1; ++j) {
                        Gs = tB[j] - tA[j];
                        lG = sarea * (ld - w * (vk - __ldg(N.syn_e + j)));
                        slB[j] += lG;
                        slA[j] -= lG;
                        if (g_e) GR.syn_e[j] += w * sarea * Gs;
                        lvn -= w * sarea * Gs;
                    }
                }
                if (kCpl && (fl & kHasCpl)) {
                    const int h1 = __ldg(N.node_hg_off + gi + 1);
                    for (int j = __ldg(N.node_hg_off + gi); j < h1; ++j) {
                        const int src = __ldg(N.hg_src + j);
                        const double gg = __ldg(N.hg_g + j);
                        if (!(GR.skip & (1u << HX_P_HALFGAP_G))) GR.hg_g[j] += w * sarea * (vpeer[src] - vk) + ld * sarea;
                        lvn -= w * sarea * gg;
                        __stcg(xo_hg + j, w * sarea * gg);
                    }
                    const int j1 = __ldg(N.node_gj_off + gi + 1);
                    for (int j = __ldg(N.node_gj_off + gi); j < j1; ++j) {
                        const int q = __ldg(N.gj_pre + j);
                        const double gg = __ldg(N.gj_g + j), ww = __ldg(N.gj_w + j), dv = vk - vpeer[q];
                        if (!(GR.skip & (1u << HX_P_GAPJ_W))) GR.gj_w[j] += -w * sarea * gg * dv + ld * sarea * gg;
                        if (!(GR.skip & (1u << HX_P_GAPJ_G))) GR.gj_g[j] += -w * sarea * ww * dv + ld * sarea * ww;
                        lvn -= w * sarea * ww * gg;
                        __stcg(xo_gj + j, w * sarea * ww * gg);
                    }
                    const int r1 = __ldg(N.node_gr_off + gi + 1);
                    for (int j = __ldg(N.node_gr_off + gi); j < r1; ++j) {
                        const double W = __ldg(N.gr_w + j), aw = fabs(W), gg = __ldg(N.gr_g + j);
                        const double er = __ldg(N.gr_erev + j), sk = grs[j], dvr = vk - er;
                        double ls = N.lS[j] - w * sarea * aw * gg * dvr + ld * sarea * aw * gg;
                        const double sgn = (double)((W > 0) - (W < 0));
                        if (!(GR.skip & (1u << HX_P_GRADED_W)))
                            GR.gr_w[j] += sgn * (-w * sarea * gg * sk * dvr + ld * sarea * gg * sk);
                        lvn -= w * sarea * aw * gg * sk;
                        // state map s_k = F(s_{k-1}, vpre_k): its vpre_k part goes to the
                        // presynaptic node (gathered by the launch of step k-1)
                        double x = 0.0;
                        if (k > 0) {
                            const double vpre = vpeer[__ldg(N.gr_pre + j)];
                            const double dl = __ldg(N.gr_delta + j), kk = __ldg(N.gr_k + j);
                            const double inf = 1.0 / (1.0 + exp((__ldg(N.gr_vth + j) - vpre) / dl));
                            const double tau = (1.0 - inf) / kk;
                            const double E = exp(-dt / tau);
                            const double dinf = inf * (1.0 - inf) / dl;
                            const double dE = (E == 0.0) ? 0.0 : E * (dt / (tau * tau)) * (-dinf / kk);
                            const double sprev = N.tS[(size_t)(k - T.k_base) * N.ngr + j];
                            x = ls * (dinf * (1.0 - E) + (sprev - inf) * dE);
                            ls *= E;
                        }
                        __stcg(xo_gr + j, x);
                        N.lS[j] = ls;
                    }
                }
            }
            const int par = M.par[i];
            if (par >= 0) lvn += sb[i] * w - sa[i] * sw[par];
            const int c1n = M.cho[i + 1];
            for (int k2 = M.cho[i]; k2 < c1n; ++k2) {
                const int c = M.ch[k2];
                lvn += sa[c] * w - sb[c] * sw[c];
            }
            lv[i] = lvn;
        }
        if (kNet && !(GR.skip & (1u << HX_P_EXPSYN_W))) {  // event weight gradients: dL/dw += fA lA' + fB lB' per delivery at step k (owner thread)
            const size_t b = (size_t)k * N.npack + p;
            const int cnt = min(ev_k, N.ev_cap);
            const int* ev = N.ev_syn + b * N.ev_cap;
            for (int e = 0; e < cnt; ++e) {
                const int j = ev[e];
                if (j >= c0 && j < c1 && (__ldg(N.syn_node + j) - pb - i0) % g.nt == g.tl)
                    GR.syn_w[j] += __ldg(N.syn_fA + j) * slA[j] + __ldg(N.syn_fB + j) * slB[j];
            }
        }
        g.sync();
        if (gs && k > k_lo) grid_barrier(N.gbar, N.gerr, G.npack, N.gspin, nact, gen);
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

// Soma-trace MSE objective: loss = mean over rows 1..nrow-1 and all columns of
// (trace - target)^2, dLdv = its gradient (row 0, the initial state, gets 0).
// Deterministic: fixed-size block partials, then one block sums them in order.
constexpr int kMseBlocks = 256;
__global__ void mse_grad_kernel(const double* __restrict__ tr, const double* __restrict__ tg, double* __restrict__ g,
                                double* __restrict__ partial, long long n, long long ncol, double scale) {
    __shared__ double red[256];
    double acc = 0.0;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        if (i < ncol) {
            g[i] = 0.0;
        } else {
            const double e = tr[i] - tg[i];
            g[i] = 2.0 * scale * e;
            acc += e * e;
        }
    }
    red[threadIdx.x] = acc;
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
        if ((int)threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
        __syncthreads();
    }
    if (threadIdx.x == 0) partial[blockIdx.x] = red[0];
}

__global__ void mse_final_kernel(const double* __restrict__ partial, double* __restrict__ loss, double scale) {
    __shared__ double red[kMseBlocks];
    red[threadIdx.x] = partial[threadIdx.x];
    __syncthreads();
    for (int s = kMseBlocks / 2; s > 0; s >>= 1) {
        if ((int)threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
        __syncthreads();
    }
    if (threadIdx.x == 0) *loss = red[0] * scale;
}

cudaError_t launch_mse(const double* trace, const double* target, double* dLdv, double* partial, double* loss,
                       int nrow, int ncol, cudaStream_t st) {
    const long long n = (long long)nrow * ncol;
    const double scale = (nrow > 1 && ncol > 0) ? 1.0 / ((double)(nrow - 1) * ncol) : 0.0;
    mse_grad_kernel<<<kMseBlocks, 256, 0, st>>>(trace, target, dLdv, partial, n, ncol, scale);
    mse_final_kernel<<<1, kMseBlocks, 0, st>>>(partial, loss, scale);
    return cudaGetLastError();
}

// Adam over external-gradient slots, one slot per registered parameter
// (reference: AdamOptimizer::step_cpu, src/optimizer/optimizer.cpp:351-397, with
// one weight per entry): g = grad*impedance*inv_record_steps, biased moments,
// bias correction with the host-computed powers, w -= lr*mhat/(sqrt(vhat)+eps),
// then the gradient slot is zeroed.
__global__ void adam_kernel(double* const* __restrict__ wbase, const int* __restrict__ kind,
                            const int* __restrict__ slot, double* __restrict__ grad, double* __restrict__ m,
                            double* __restrict__ v, int n, double lr, double impedance, double inv_record_steps,
                            double beta1, double beta2, double eps, double bc1, double bc2) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const double g = grad[i] * impedance * inv_record_steps;
    const double mi = beta1 * m[i] + (1.0 - beta1) * g;
    const double vi = beta2 * v[i] + (1.0 - beta2) * g * g;
    m[i] = mi;
    v[i] = vi;
    const double mh = mi / (1.0 - bc1);
    const double vh = vi / (1.0 - bc2);
    double* w = wbase[kind[i]] + slot[i];
    *w = *w - lr * mh / (sqrt(vh) + eps);
    grad[i] = 0.0;
}

cudaError_t launch_adam(double* const* wbase, const int* kind, const int* slot, double* grad, double* m, double* v,
                        int n, double lr, double impedance, double inv_record_steps, double beta1, double beta2,
                        double eps, double bc1, double bc2, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    adam_kernel<<<(n + 255) / 256, 256, 0, st>>>(wbase, kind, slot, grad, m, v, n, lr, impedance, inv_record_steps,
                                                 beta1, beta2, eps, bc1, bc2);
    return cudaGetLastError();
}

// grad[i] = src[flat[i]] * scale (adjoint gradients into optimizer slots)
__global__ void take_scaled_kernel(const double* __restrict__ src, const int* __restrict__ flat,
                                   double* __restrict__ dst, int n, double scale) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = src[flat[i]] * scale;
}

cudaError_t launch_take_scaled(const double* src, const int* flat, double* dst, int n, double scale, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    take_scaled_kernel<<<(n + 255) / 256, 256, 0, st>>>(src, flat, dst, n, scale);
    return cudaGetLastError();
}

__global__ void f32_to_f64_kernel(const float* __restrict__ a, double* __restrict__ b, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) b[i] = (double)a[i];
}

cudaError_t launch_f32_to_f64(const float* a, double* b, int n, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    f32_to_f64_kernel<<<(n + 255) / 256, 256, 0, st>>>(a, b, n);
    return cudaGetLastError();
}

// ------------------------------------------------------------------ launchers
size_t fwd_smem_bytes(const DevGroup& G) {
    return sizeof(double) * (5 * (size_t)G.smem_n + 4 * (size_t)G.smem_br) + meta_bytes(G);
}
size_t bwd_smem_bytes(const DevGroup& G) {
    return sizeof(double) * (4 * (size_t)G.smem_n + 4 * (size_t)G.smem_br) + meta_bytes(G);
}
// split-cell kernels (hx_split.cu) keep the gates / node adjoints in shared memory
size_t split_fwd_smem_bytes(const DevGroup& G) { return sizeof(double) * 8 * (size_t)G.smem_n + meta_bytes(G); }
size_t split_bwd_smem_bytes(const DevGroup& G) { return sizeof(double) * 10 * (size_t)G.smem_n + meta_bytes(G); }

cudaError_t configure_kernels(size_t smem_fwd, size_t smem_bwd, size_t smem_fwd_net, size_t smem_bwd_net) {
    cudaError_t e = cudaFuncSetAttribute(fwd_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_fwd);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(bwd_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bwd);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(fwd_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_fwd);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(bwd_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bwd);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(fwd_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_fwd_net);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(fwd_kernel<true, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem_fwd_net);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(bwd_kernel<true, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem_bwd_net);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(fwd_kernel<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_fwd_net);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(bwd_kernel<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bwd_net);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(fwd_kernel<true, true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem_fwd_net);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(bwd_kernel<true, true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem_bwd_net);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(bwd_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bwd_net);
}

const void* fwd_cpl_kernel_ptr(bool lib) {
    return lib ? (const void*)fwd_kernel<true, true, true> : (const void*)fwd_kernel<true, false, true>;
}
const void* bwd_cpl_kernel_ptr(bool lib) {
    return lib ? (const void*)bwd_kernel<true, true, true> : (const void*)bwd_kernel<true, false, true>;
}

cudaError_t launch_init(const DevGroup& G, const DevState& S, double v_init, cudaStream_t st) {
    init_state_kernel<<<(G.nnode + 255) / 256, 256, 0, st>>>(G, S, v_init);
    return cudaGetLastError();
}

cudaError_t launch_lib_init(const DevLib& L, int nnode, double v_init, cudaStream_t st) {
    if (nnode <= 0) return cudaSuccess;
    lib_init_kernel<<<(nnode + 255) / 256, 256, 0, st>>>(L, nnode, v_init);
    return cudaGetLastError();
}

cudaError_t launch_fwd(const DevGroup& G, const DevState& S, const DevTape& T, int write_tape, const DevProbe& P,
                       double* trace, const double* tmid, int k0, int k1, cudaStream_t st, const DevNet* N,
                       const DevLib* L) {
    if (N) {
        DevLib Lc{};
        if (L) {
            Lc = *L;
            Lc.k_base = T.k_base;
        }
        if (N->coupled && N->gsync) {  // every pack co-resident: one cooperative launch for the window
            DevGroup Gc = G;
            DevState Sc = S;
            DevTape Tc = T;
            DevProbe Pc = P;
            DevNet Nc = *N;
            void* args[] = {&Gc, &Sc, &Tc, &write_tape, &Pc, &trace, &tmid, &k0, &k1, &Nc, &Lc};
            const void* f = L ? (const void*)fwd_kernel<true, true, true> : (const void*)fwd_kernel<true, false, true>;
            return cudaLaunchCooperativeKernel(f, dim3(G.npack), dim3(kThreads), args, fwd_smem_bytes(G), st);
        }
        if (L) {  // library mechanisms in a network group
            if (N->coupled)
                fwd_kernel<true, true, true><<<G.npack, kThreads, fwd_smem_bytes(G), st>>>(G, S, T, write_tape, P, trace,
                                                                                       tmid, k0, k1, *N, Lc);
            else
                fwd_kernel<true, true><<<G.npack, kThreads, fwd_smem_bytes(G), st>>>(G, S, T, write_tape, P, trace, tmid,
                                                                                   k0, k1, *N, Lc);
            return cudaGetLastError();
        }
        if (N->coupled)
            fwd_kernel<true, false, true><<<G.npack, kThreads, fwd_smem_bytes(G), st>>>(G, S, T, write_tape, P, trace,
                                                                                   tmid, k0, k1, *N, DevLib{});
        else
            fwd_kernel<true><<<G.npack, kThreads, fwd_smem_bytes(G), st>>>(G, S, T, write_tape, P, trace,
                                                                                   tmid, k0, k1, *N, DevLib{});
    } else if (L) {
        DevLib Lk = *L;
        Lk.k_base = T.k_base;
        fwd_kernel<false, true><<<G.npack, kThreads, fwd_smem_bytes(G), st>>>(G, S, T, write_tape, P, trace,
                                                                                tmid, k0, k1, DevNet{}, Lk);
    } else {
        fwd_kernel<false><<<G.npack, kThreads, fwd_smem_bytes(G), st>>>(G, S, T, write_tape, P, trace, tmid, k0,
                                                                          k1, DevNet{}, DevLib{});
    }
    return cudaGetLastError();
}

cudaError_t launch_bwd(const DevGroup& G, const DevTape& T, const DevAdj& A, const DevGrad& GR, const DevProbe& P,
                       const double* dLdv, const double* tmid, int k_hi, int k_lo, cudaStream_t st, const DevNet* N,
                       const DevLib* L) {
    if (N) {
        DevLib Lc{};
        if (L) {
            Lc = *L;
            Lc.k_base = T.k_base;
        }
        if (N->coupled && N->gsync) {
            DevGroup Gc = G;
            DevTape Tc = T;
            DevAdj Ac = A;
            DevGrad GRc = GR;
            DevProbe Pc = P;
            DevNet Nc = *N;
            void* args[] = {&Gc, &Tc, &Ac, &GRc, &Pc, &dLdv, &tmid, &k_hi, &k_lo, &Nc, &Lc};
            const void* f = L ? (const void*)bwd_kernel<true, true, true> : (const void*)bwd_kernel<true, false, true>;
            return cudaLaunchCooperativeKernel(f, dim3(G.npack), dim3(kThreads), args, bwd_smem_bytes(G), st);
        }
        if (L) {
            if (N->coupled)
                bwd_kernel<true, true, true><<<G.npack, kThreads, bwd_smem_bytes(G), st>>>(G, T, A, GR, P, dLdv, tmid,
                                                                                       k_hi, k_lo, *N, Lc);
            else
                bwd_kernel<true, true><<<G.npack, kThreads, bwd_smem_bytes(G), st>>>(G, T, A, GR, P, dLdv, tmid, k_hi,
                                                                                   k_lo, *N, Lc);
            return cudaGetLastError();
        }
        if (N->coupled)
            bwd_kernel<true, false, true><<<G.npack, kThreads, bwd_smem_bytes(G), st>>>(G, T, A, GR, P, dLdv, tmid, k_hi,
                                                                                   k_lo, *N, DevLib{});
        else
            bwd_kernel<true><<<G.npack, kThreads, bwd_smem_bytes(G), st>>>(G, T, A, GR, P, dLdv, tmid, k_hi,
                                                                                   k_lo, *N, DevLib{});
    } else if (L) {
        DevLib Lk = *L;
        Lk.k_base = T.k_base;
        bwd_kernel<false, true><<<G.npack, kThreads, bwd_smem_bytes(G), st>>>(G, T, A, GR, P, dLdv, tmid, k_hi,
                                                                                k_lo, DevNet{}, Lk);
    } else {
        bwd_kernel<false><<<G.npack, kThreads, bwd_smem_bytes(G), st>>>(G, T, A, GR, P, dLdv, tmid, k_hi, k_lo,
                                                                          DevNet{}, DevLib{});
    }
    return cudaGetLastError();
}

// ---------------------------------------------------------------- network helpers
// Per-synapse constants (GPU order).  kind 0 ExpSyn: c_B = 1 - exp(dt*(-1/tau)),
// an event adds w to B (expsyn.cpp:125-149).  kind 1 Exp2Syn: tau1 clamped to
// [1e-9, 0.9999] tau2, factor = 1/(exp(-tp/tau2) - exp(-tp/tau1)) at the
// peak time tp, an event adds w*factor to A and B (exp2syn_temp.cuh:29-66).
__global__ void syn_prep_kernel(int n, const int* __restrict__ kind, const double* __restrict__ tau1,
                                const double* __restrict__ tau2, double dt, double* cA, double* cB, double* fA,
                                double* fB) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n) return;
    if (kind[j] == 0) {
        const double tau = tau2[j];
        cA[j] = 0.0;
        cB[j] = 1. - exp(dt * ((-1.0) / tau));
        fA[j] = 0.0;
        fB[j] = 1.0;
    } else {
        double t1 = tau1[j];
        const double t2 = tau2[j];
        if (t1 / t2 > 0.9999) t1 = 0.9999 * t2;
        if (t1 / t2 < 1e-9) t1 = t2 * 1e-9;
        const double tp = (t1 * t2) / (t2 - t1) * log(t2 / t1);
        const double f = 1.0 / (-exp(-tp / t1) + exp(-tp / t2));
        cA[j] = 1.0 - exp(dt * (-1.0 / t1));
        cB[j] = 1.0 - exp(dt * (-1.0 / t2));
        fA[j] = f;
        fB[j] = f;
    }
}

// finitialize of the network state: synapse states 0 (expsyn.cpp:76-83,
// exp2syn_temp.cuh:38-40); graded synapses s = inf(v_init) and the
// sign-of-w parameter set of their INITIAL block (neuron_to_neuron_syn_lr.cu:
// 102-118).
__global__ void init_net_kernel(int nsyn, double* sA, double* sB, int ngr, const double* __restrict__ gr_w,
                                const double* __restrict__ gr_vth, const double* __restrict__ gr_delta,
                                double* gr_g, double* gr_k, double* gr_erev, double* gr_s, double v_init) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j < nsyn) {
        sA[j] = 0.0;
        sB[j] = 0.0;
    }
    if (j < ngr) {
        gr_s[j] = 1.0 / (1.0 + exp((gr_vth[j] - v_init) / gr_delta[j]));
        const bool exc = gr_w[j] > 0.0;
        gr_g[j] = exc ? 4.9 : 2.0;
        gr_k[j] = exc ? 0.5 : 0.015000001;
        gr_erev[j] = exc ? 30.0 : -70.0;
    }
}

// Event routing: every spike (source gid, step j) reaches the local synapses
// of its source; the delivery step is the first k >= j with
// t_j + delay <= t_k + dt/2 (the reference's post_spike_receive condition,
// postsyn.cpp:43-61, applied at the start of every step).  The event goes to
// the bucket of (step, the synapse's pack), so a CTA reads only its own
// events.  Events before k_min (inside an already simulated window) set bit 1
// of *err, a full bucket bit 2; bucket counts keep counting past ev_cap so
// the needed size is known.
__global__ void route_kernel(const int2* __restrict__ spk, const int* __restrict__ nspk_dev, int nspk_max,
                             const int* __restrict__ src_off, const int* __restrict__ src_syn, int nsrc,
                             const double* __restrict__ delay, const double* __restrict__ tstart, int nstep,
                             double half_dt, int k_min, const int* __restrict__ syn_pack, int npack, int* ev_cnt,
                             int* ev_syn, int ev_cap, int* err) {
    const int n = nspk_dev ? min(*nspk_dev, nspk_max) : nspk_max;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int2 sp = spk[i];
        if (sp.x < 0 || sp.x >= nsrc || sp.y < 0 || sp.y >= nstep) continue;
        const double tj = tstart[sp.y];
        const int e1 = src_off[sp.x + 1];
        for (int e = src_off[sp.x]; e < e1; ++e) {
            const int syn = src_syn[e];
            const double td = tj + delay[syn];
            int lo = sp.y, hi = nstep;  // first k in [lo, hi) with td <= tstart[k] + half_dt, else hi
            while (lo < hi) {
                const int mid = (lo + hi) >> 1;
                if (td <= tstart[mid] + half_dt)
                    hi = mid;
                else
                    lo = mid + 1;
            }
            if (lo >= nstep) continue;
            if (lo < k_min) {
                atomicOr(err, 1);
                continue;
            }
            const size_t b = (size_t)lo * npack + __ldg(syn_pack + syn);
            const int c = atomicAdd(ev_cnt + b, 1);
            if (c < ev_cap)
                ev_syn[b * ev_cap + c] = syn;
            else
                atomicOr(err, 2);
        }
    }
}

// appends the window's spikes to the forward's spike log
__global__ void log_append_kernel(const int2* __restrict__ win, const int* __restrict__ win_n, int win_cap,
                                  int2* log, int* log_n, int log_cap, int* err, int* win_max) {
    const int n = min(*win_n, win_cap);
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        if (*win_n > win_cap) atomicOr(err, 4);
        atomicMax(win_max, *win_n);
    }
    const int base = *log_n;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        if (base + i < log_cap) log[base + i] = win[i];
}

__global__ void log_advance_kernel(const int* __restrict__ win_n, int win_cap, int* log_n) {
    *log_n += min(*win_n, win_cap);
}

// A rank's status after its last window: (error bits | extra, largest bucket
// count over the nstep buckets), (largest window spike count, 0).  One block;
// the ranks all-gather it.
__global__ void net_status_kernel(const int* __restrict__ err, const int* __restrict__ ev_cnt, int nstep,
                                  const int* __restrict__ win_max, int extra, int2* out) {
    __shared__ int red[256];
    int m = 0;
    for (int k = threadIdx.x; k < nstep; k += blockDim.x) m = max(m, ev_cnt[k]);
    red[threadIdx.x] = m;
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
        if ((int)threadIdx.x < s) red[threadIdx.x] = max(red[threadIdx.x], red[threadIdx.x + s]);
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        out[0] = make_int2(*err | extra, red[0]);
        out[1] = make_int2(*win_max, 0);
    }
}

// The library's reciprocal over an array (verification of rcp_nz against IEEE division)
__global__ void rcp_nz_kernel(const double* __restrict__ x, double* __restrict__ y, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = rcp_nz(x[i]);
}

cudaError_t launch_rcp_nz(const double* x, double* y, int n, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    rcp_nz_kernel<<<(n + 255) / 256, 256, 0, st>>>(x, y, n);
    return cudaGetLastError();
}

cudaError_t launch_net_status(const int* err, const int* ev_cnt, int nstep, const int* win_max, int extra, int2* out,
                              cudaStream_t st) {
    net_status_kernel<<<1, 256, 0, st>>>(err, ev_cnt, nstep, win_max, extra, out);
    return cudaGetLastError();
}

cudaError_t launch_syn_prep(int n, const int* kind, const double* tau1, const double* tau2, double dt, double* cA,
                            double* cB, double* fA, double* fB, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    syn_prep_kernel<<<(n + 255) / 256, 256, 0, st>>>(n, kind, tau1, tau2, dt, cA, cB, fA, fB);
    return cudaGetLastError();
}

cudaError_t launch_init_net(int nsyn, double* sA, double* sB, int ngr, const double* gr_w, const double* gr_vth,
                            const double* gr_delta, double* gr_g, double* gr_k, double* gr_erev, double* gr_s,
                            double v_init, cudaStream_t st) {
    const int n = nsyn > ngr ? nsyn : ngr;
    if (n <= 0) return cudaSuccess;
    init_net_kernel<<<(n + 255) / 256, 256, 0, st>>>(nsyn, sA, sB, ngr, gr_w, gr_vth, gr_delta, gr_g, gr_k, gr_erev,
                                                     gr_s, v_init);
    return cudaGetLastError();
}

cudaError_t launch_route(const int2* spk, const int* nspk_dev, int nspk_max, const int* src_off, const int* src_syn,
                         int nsrc, const double* delay, const double* tstart, int nstep, double half_dt, int k_min,
                         const int* syn_pack, int npack, int* ev_cnt, int* ev_syn, int ev_cap, int* err,
                         cudaStream_t st) {
    if (nspk_max <= 0) return cudaSuccess;
    int blocks = (nspk_max + 255) / 256;
    if (blocks > 4 * 148) blocks = 4 * 148;
    route_kernel<<<blocks, 256, 0, st>>>(spk, nspk_dev, nspk_max, src_off, src_syn, nsrc, delay, tstart, nstep,
                                         half_dt, k_min, syn_pack, npack, ev_cnt, ev_syn, ev_cap, err);
    return cudaGetLastError();
}

cudaError_t launch_log_append(const int2* win, const int* win_n, int win_cap, int2* log, int* log_n, int log_cap,
                              int* err, int* win_max, cudaStream_t st) {
    int blocks = (win_cap + 255) / 256;
    if (blocks > 148) blocks = 148;
    if (blocks < 1) blocks = 1;
    log_append_kernel<<<blocks, 256, 0, st>>>(win, win_n, win_cap, log, log_n, log_cap, err, win_max);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    log_advance_kernel<<<1, 1, 0, st>>>(win_n, win_cap, log_n);
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
