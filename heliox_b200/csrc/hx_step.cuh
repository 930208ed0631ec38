// hx_step.cuh -- device building blocks of the step kernels (shared by
// hx_kernels.cu and hx_split.cu): the cell-group layout in shared memory, the
// branch-level Hines solve and the per-node assembly of rhs/d.
#pragma once

#include <cuda_runtime.h>

#include "heliox_b200.h"
#include "hx_dev.hpp"
#include "hx_lib.cuh"
#include "hx_mech.cuh"

namespace hx {

// ------------------------------------------------------------------ Hines (shared memory)
// hines_cell (below) solves one cell's tree system in place: d (diagonal in,
// reciprocal of the eliminated diagonal out), rhs (right-hand side in, solution
// out).  sa/sb are the axial coefficients in shared memory; A eliminates a
// child into its parent and U couples a node to its parent (forward: A=a, U=b;
// transposed system: A=b, U=a).
//
// The reference eliminates with a division on every step of the chain
// (solve_serial, simulate.cpp:558-581).  Here the eliminated diagonal and rhs
// of an unbranched chain are carried in projective form (tri_block below), so
// the serial dependencies are FMAs only; exact power-of-two rescaling keeps
// p, q, y in range and the reciprocals are formed off the chains with a
// branch-free Newton reciprocal.  The back-substitution is one FMA per node.
__device__ __forceinline__ double rescale_pow2(double x) {
    // 2^-floor(log2 x) for positive normal x; exact
    const long long e = ((__double_as_longlong(x) >> 52) & 0x7FF);
    return __longlong_as_double((2046LL - e) << 52);
}

// Register-blocked chain kernels.  Every block loads up to kBlk nodes' operands
// from shared memory into registers before the dependent arithmetic and stores
// the results afterwards, so that no shared-memory load waits behind a store
// of the same array on the critical path.  cnt <= kBlk nodes are processed;
// callers pass kBlk for full blocks.
constexpr int kBlk = 4;

// tri_block: triangularisation of a chain from node j downwards in projective
// form.  With d'_k = p_k/q_k and the eliminated rhs r'_k = y_k/q_k:
//   p_{k-1} = d_{k-1} p_k - A_k U_k q_k,   q_{k-1} = p_k,
//   y_{k-1} = rhs_{k-1} p_k - A_k y_k     (one FMA on the y chain),
// two FMA chains without division.  For k = j .. j-cnt+1 it stores
// d[k] = 1/d'_k = q_k/p_k and rhs[k] = r'_k/d'_k = y_k/p_k (the reciprocal is
// off both chains) and leaves (p, q, y) of node j-cnt.
template <bool kGuard>
__device__ __forceinline__ void tri_block(double* __restrict__ d, double* __restrict__ rhs,
                                          const double* __restrict__ A, const double* __restrict__ U, int j, int cnt,
                                          double& pp, double& qq, double& yy) {
    double dl[kBlk], rl[kBlk], al[kBlk], cl[kBlk], pv[kBlk], qv[kBlk], yv[kBlk];
#pragma unroll
    for (int u = 0; u < kBlk; ++u) {
        if (!kGuard || u < cnt) {
            dl[u] = d[j - 1 - u];
            rl[u] = rhs[j - 1 - u];
            al[u] = A[j - u];
            cl[u] = al[u] * U[j - u];
        }
    }
#pragma unroll
    for (int u = 0; u < kBlk; ++u) {
        pv[u] = 1.0;
        if (!kGuard || u < cnt) {
            pv[u] = pp;
            qv[u] = qq;
            yv[u] = yy;
            const double pn = __fma_rn(dl[u], pp, -(cl[u] * qq));
            const double yn = __fma_rn(-al[u], yy, rl[u] * pp);
            qq = pp;
            pp = pn;
            yy = yn;
        }
    }
    // the block's reciprocals 1/p_u from one reciprocal of their product
    // (batch inversion); the block starts at p in [1, 2) (rescaled by the
    // caller), so the product of its four pivots' p stays far inside the
    // double range
    const double a1 = pv[0] * pv[1], a2 = a1 * pv[2], a3 = a2 * pv[3];
    double inv = rcp_nz(a3);
    double ip[kBlk];
    ip[3] = inv * a2;
    inv *= pv[3];
    ip[2] = inv * a1;
    inv *= pv[2];
    ip[1] = inv * pv[0];
    ip[0] = inv * pv[1];
#pragma unroll
    for (int u = 0; u < kBlk; ++u) {
        if (!kGuard || u < cnt) {
            d[j - u] = qv[u] * ip[u];
            rhs[j - u] = yv[u] * ip[u];
        }
    }
}

// back_block: x_k = rhs'_k/d'_k - (U_k/d'_k) x_{k-1} for k = j .. j+cnt-1
// (d holds 1/d'_k, rhs holds rhs'_k/d'_k); one FMA per node on the chain.
template <bool kGuard>
__device__ __forceinline__ void back_block(const double* __restrict__ d, double* __restrict__ rhs,
                                           const double* __restrict__ U, int j, int cnt, double& x) {
    double hl[kBlk], gl[kBlk];
#pragma unroll
    for (int u = 0; u < kBlk; ++u) {
        if (!kGuard || u < cnt) {
            hl[u] = U[j + u] * d[j + u];
            gl[u] = rhs[j + u];
        }
    }
#pragma unroll
    for (int u = 0; u < kBlk; ++u) {
        if (!kGuard || u < cnt) {
            x = __fma_rn(-hl[u], x, gl[u]);
            gl[u] = x;
        }
    }
#pragma unroll
    for (int u = 0; u < kBlk; ++u)
        if (!kGuard || u < cnt) rhs[j + u] = gl[u];
}

// ------------------------------------------------------------------ cell groups
// Shared-memory copies of the pack's topology and schedule.  Node tables are
// 16-bit (pack-local ids and offsets; a pack holds at most 32767 nodes) and the
// node flags 8-bit; the branch tables are ints.
struct Meta {
    short* par;           // node parent (pack-local), -1 for roots, -(2 + subtree) across CTAs
    unsigned char* flag;  // NodeFlag bits
    short* cho;           // node child offsets into ch (size n+1)
    short* ch;            // node children (pack-local), ascending reference index
    int* bh;    // branch head / end / head's parent (pack-local nodes)
    int* be;
    int* bp;
    int* bco;   // branch child offsets into bc (size nbr+1)
    int* bc;    // child-branch heads, descending reference index
    int* bcb;   // the same children as pack-local branch ids (-1: in another CTA)
    int* lvl;   // level tables of the pack's cells (pack-local branch ids)
};

// One cell and the warps of the CTA that own it.
struct Grp {
    int nb, n;       // pack-local first node, node count
    int tl, nt;      // thread index inside the group, group size
    int bar, nwarp;  // named barrier id (multi-warp groups)
    int lvl, nlev;   // offset of the cell's level table in Meta::lvl, levels
    int slot;        // global cell-slot index
    __device__ __forceinline__ void sync() const {
        if (nwarp == 1)
            __syncwarp();
        else
            asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(nt) : "memory");
    }
};

// Grid barrier of a grid-synchronous coupled launch over the CTA's active
// threads (nact: the pack's warps x 32; idle warps have returned): named
// barrier 15 (cell groups use 1..8), then thread 0 arrives at the grid
// counter and waits for the generation to move.  Every wait is bounded: a
// wait that gives up sets *err, and later barriers return at once (the
// launch then finishes its loop and the host reports the error).
__device__ __forceinline__ void grid_barrier(unsigned* bar, int* err, int nblocks, long long spin, int nact,
                                             unsigned& gen) {
    asm volatile("bar.sync 15, %0;" ::"r"(nact) : "memory");
    if (threadIdx.x == 0) {
        volatile unsigned* vgen = bar + 1;
        volatile int* verr = err;
        __threadfence();
        if (*verr == 0) {
            const unsigned arrived = atomicAdd(bar, 1u);
            if (arrived == (unsigned)nblocks - 1u) {
                atomicExch(bar, 0u);
                __threadfence();
                atomicAdd(bar + 1, 1u);
            } else {
                long long it = 0;
                while (*vgen == gen && *verr == 0) {
                    if (++it > spin) {
                        atomicOr(err, 1);
                        break;
                    }
                    __nanosleep(100);
                }
            }
        }
        __threadfence();
        gen++;
    }
    asm volatile("bar.sync 15, %0;" ::"r"(nact) : "memory");
}

// Bytes of the Meta tables in shared memory (a multiple of 16).
__host__ __device__ inline size_t meta_bytes(const DevGroup& G) {
    const size_t ints = 4 * (size_t)G.smem_br + 1 + 2 * (size_t)G.smem_bch + G.smem_lvl;
    const size_t shorts = 2 * (size_t)G.smem_n + 1 + G.smem_nch;
    const size_t b = 4 * ints + 2 * shorts + (size_t)G.smem_n;
    return (b + 15) & ~(size_t)15;
}

// Loads the pack's tables into shared memory (whole CTA), then returns the
// calling thread's cell group; false for warps the pack leaves idle.
__device__ __forceinline__ bool setup_pack(const DevGroup& G, int p, int* ibase, Meta& M, Grp& g) {
    const int tid = threadIdx.x, nt = blockDim.x;
    M.bh = ibase;
    M.be = M.bh + G.smem_br;
    M.bp = M.be + G.smem_br;
    M.bco = M.bp + G.smem_br;
    M.bc = M.bco + G.smem_br + 1;
    M.bcb = M.bc + G.smem_bch;
    M.lvl = M.bcb + G.smem_bch;
    M.par = reinterpret_cast<short*>(M.lvl + G.smem_lvl);
    M.cho = M.par + G.smem_n;
    M.ch = M.cho + G.smem_n + 1;
    M.flag = reinterpret_cast<unsigned char*>(M.ch + G.smem_nch);
    const int pb = G.pack_node_off[p], pn = G.pack_node_off[p + 1] - pb;
    const int nch0 = G.pack_nch_off[p], nch = G.pack_nch_off[p + 1] - nch0;
    const int br0 = G.pack_br_off[p], nbr = G.pack_br_off[p + 1] - br0;
    const int bc0 = G.pack_bch_off[p], nbc = G.pack_bch_off[p + 1] - bc0;
    const int s0 = G.pack_slot_off[p], s1 = G.pack_slot_off[p + 1];
    const int l0 = G.cs_lvl_off[s0], l1 = G.cs_lvl_off[s1 - 1] + G.cs_nlev[s1 - 1] + 1;
    for (int i = tid; i < pn; i += nt) {
        M.par[i] = (short)G.node_parent[pb + i];
        M.flag[i] = (unsigned char)G.node_flags[pb + i];
        M.cho[i] = (short)(G.node_child_off[pb + i] - nch0);
    }
    if (tid == 0) M.cho[pn] = (short)nch;
    for (int k = tid; k < nch; k += nt) M.ch[k] = (short)G.node_child[nch0 + k];
    for (int k = tid; k < nbr; k += nt) {
        M.bh[k] = G.br_head[br0 + k];
        M.be[k] = G.br_end[br0 + k];
        M.bp[k] = G.br_parent[br0 + k];
        M.bco[k] = G.br_child_off[br0 + k] - bc0;
    }
    if (tid == 0) M.bco[nbr] = nbc;
    for (int k = tid; k < nbc; k += nt) {
        M.bc[k] = G.br_child[bc0 + k];
        M.bcb[k] = G.br_child_br[bc0 + k];
    }
    for (int k = tid; k < l1 - l0; k += nt) M.lvl[k] = G.level_br_off[l0 + k];
    __syncthreads();
    const int w = tid >> 5;
    for (int s = s0; s < s1; ++s) {
        const int w0 = G.cs_warp0[s], nw = G.cs_nwarp[s];
        if (w >= w0 && w < w0 + nw) {
            g.nb = G.cs_node0[s];
            g.n = G.cs_nnode[s];
            g.tl = tid - 32 * w0;
            g.nt = 32 * nw;
            g.bar = G.cs_bar[s];
            g.slot = s;
            g.nwarp = nw;
            g.lvl = G.cs_lvl_off[s] - l0;
            g.nlev = G.cs_nlev[s];
            return true;
        }
    }
    return false;
}

// hines_rt: Hines solve of one cell's system by its warp group, in three
// phases over the cell's branch segments (a branch cut into pieces of at
// most kSegMax nodes; segments sorted by level, lo[L] .. lo[L+1] the segments
// of level L):
//  1. every segment eliminates its interior nodes h .. e-1 top-down, keeping
//     its head's parent P and its end e: d[k] := 1/D'_k on the interior, the
//     end's diagonal / rhs updated in place, the fill couplings P-e (fe in
//     P's row, ge in e's row) and the interior's contributions to P's
//     diagonal / rhs (dD, dR) kept per segment;
//  2. the tree of segment ends is solved level by level: an end folds in its
//     child segments' contributions cd, cr (their dD + fe ge / D_e, dR +
//     fe R_e / D_e), then x_e = R_e/D_e - (ge/D_e) x_P root-first;
//  3. every segment solves its interior from x_P and x_e (forward r'' sweep,
//     then back-substitution).
// Thread tl takes segments lo[0] + tl + m nt in phases 1 and 3 and the
// level's segments lo[L] + tl + m nt in phase 2, so a cell with more
// segments than threads (a large cell on one warp) keeps this form; every
// segment's arithmetic is the same whichever thread does it.  The serial
// depth is the longest segment twice (times the segments a thread carries)
// plus the number of levels, instead of the longest branch of every level.
// cd, cr, fe, ge: one double per segment of the pack each.  The elimination
// order differs from the reference's, so results agree to rounding (the CPU
// replay of this form is checked against solve_serial by hx_plan_check).
template <bool kTransposed>
__device__ __forceinline__ void hines_rt(const Meta& M, const Grp& g, const double* __restrict__ sa,
                                         const double* __restrict__ sb, double* __restrict__ d,
                                         double* __restrict__ rhs, double* __restrict__ cd, double* __restrict__ cr,
                                         double* __restrict__ fe, double* __restrict__ ge) {
    const double* __restrict__ A = kTransposed ? sb : sa;
    const double* __restrict__ U = kTransposed ? sa : sb;
    const int* lo = M.lvl + g.lvl;
    const int s_end = lo[g.nlev];
    for (int s = lo[0] + g.tl; s < s_end; s += g.nt) {
        const int h = M.bh[s], e = M.be[s];
        if (h == e) {
            fe[s] = A[h];
            ge[s] = U[h];
            cd[s] = 0.0;
            cr[s] = 0.0;
            continue;
        }
        double inv = rcp_nz(d[h]);
        double rp = rhs[h];
        double F = A[h], Gc = U[h];
        double dD = F * Gc * inv, dR = F * rp * inv;
        d[h] = inv;
        // interior nodes h+1 .. e-1 in register blocks: operands loaded
        // ahead of the dependent arithmetic, results stored after it
        int k = h + 1;
        for (; k + kBlk <= e; k += kBlk) {
            double uk[kBlk], ak[kBlk], dk[kBlk], rk[kBlk], iv[kBlk];
#pragma unroll
            for (int u = 0; u < kBlk; ++u) {
                uk[u] = U[k + u];
                ak[u] = A[k + u];
                dk[u] = d[k + u];
                rk[u] = rhs[k + u];
            }
#pragma unroll
            for (int u = 0; u < kBlk; ++u) {
                const double Dk = __fma_rn(-(uk[u] * ak[u]), inv, dk[u]);
                const double rn = __fma_rn(-(uk[u] * rp), inv, rk[u]);
                F = -(F * ak[u]) * inv;
                Gc = -(uk[u] * Gc) * inv;
                inv = rcp_nz(Dk);
                rp = rn;
                dD = __fma_rn(F * Gc, inv, dD);
                dR = __fma_rn(F * rp, inv, dR);
                iv[u] = inv;
            }
#pragma unroll
            for (int u = 0; u < kBlk; ++u) d[k + u] = iv[u];
        }
        for (; k < e; ++k) {
            const double Uk = U[k], Ak = A[k];
            const double Dk = __fma_rn(-(Uk * Ak), inv, d[k]);
            const double rk = __fma_rn(-(Uk * rp), inv, rhs[k]);
            F = -(F * Ak) * inv;
            Gc = -(Uk * Gc) * inv;
            inv = rcp_nz(Dk);
            rp = rk;
            dD = __fma_rn(F * Gc, inv, dD);
            dR = __fma_rn(F * rp, inv, dR);
            d[k] = inv;
        }
        const double Ue = U[e], Ae = A[e];
        d[e] = __fma_rn(-(Ue * Ae), inv, d[e]);
        rhs[e] = __fma_rn(-(Ue * rp), inv, rhs[e]);
        fe[s] = -(F * Ae) * inv;
        ge[s] = -(Ue * Gc) * inv;
        cd[s] = dD;
        cr[s] = dR;
    }
    g.sync();
    for (int L = g.nlev - 1; L >= 0; --L) {
        const int l1 = lo[L + 1];
        for (int s = lo[L] + g.tl; s < l1; s += g.nt) {
            const int e = M.be[s];
            double De = d[e], Re = rhs[e];
            const int c1 = M.bco[s + 1];
            for (int k = M.bco[s]; k < c1; ++k) {
                const int c = M.bcb[k];
                De -= cd[c];
                Re -= cr[c];
            }
            const double ie = rcp_nz(De);
            const double gv = Re * ie, he = ge[s] * ie;
            const double f = fe[s];
            cd[s] = __fma_rn(f, he, cd[s]);
            cr[s] = __fma_rn(f, gv, cr[s]);
            d[e] = he;
            rhs[e] = gv;
        }
        g.sync();
    }
    for (int L = 0; L < g.nlev; ++L) {
        const int l1 = lo[L + 1];
        for (int s = lo[L] + g.tl; s < l1; s += g.nt) {
            const int e = M.be[s], P = M.bp[s];
            double x = rhs[e];
            if (P >= 0) x = __fma_rn(-d[e], rhs[P], x);
            rhs[e] = x;
        }
        g.sync();
    }
    for (int s = lo[0] + g.tl; s < s_end; s += g.nt) {
        const int h = M.bh[s], e = M.be[s], P = M.bp[s];
        if (h >= e) continue;
        double t = rhs[h];
        if (P >= 0) t = __fma_rn(-U[h], rhs[P], t);
        t *= d[h];
        rhs[h] = t;
        int k = h + 1;
        for (; k + kBlk <= e; k += kBlk) {
            double cu[kBlk], rr[kBlk];
#pragma unroll
            for (int u = 0; u < kBlk; ++u) {
                const double ik = d[k + u];
                cu[u] = U[k + u] * ik;
                rr[u] = rhs[k + u] * ik;
            }
#pragma unroll
            for (int u = 0; u < kBlk; ++u) {
                t = __fma_rn(-cu[u], t, rr[u]);
                rr[u] = t;
            }
#pragma unroll
            for (int u = 0; u < kBlk; ++u) rhs[k + u] = rr[u];
        }
        for (; k < e; ++k) {
            const double ik = d[k];
            t = __fma_rn(-(U[k] * ik), t, rhs[k] * ik);
            rhs[k] = t;
        }
        double x = rhs[e];
        k = e - 1;
        for (; k - kBlk + 1 >= h; k -= kBlk) {
            double ca[kBlk], rr[kBlk];
#pragma unroll
            for (int u = 0; u < kBlk; ++u) {
                ca[u] = A[k - u + 1] * d[k - u];
                rr[u] = rhs[k - u];
            }
#pragma unroll
            for (int u = 0; u < kBlk; ++u) {
                x = __fma_rn(-ca[u], x, rr[u]);
                rr[u] = x;
            }
#pragma unroll
            for (int u = 0; u < kBlk; ++u) rhs[k - u] = rr[u];
        }
        for (; k >= h; --k) {
            x = __fma_rn(-(A[k + 1] * d[k]), x, rhs[k]);
            rhs[k] = x;
        }
    }
    g.sync();
}

// ------------------------------------------------------------------ per-step I/O
// dst[i] = src[i] for the group's nodes i = i0 + tl + j*nt, four loads in flight
// per thread before the stores.
__device__ __forceinline__ void copy_in(double* __restrict__ dst, const double* __restrict__ src, int i0, int i1,
                                        const Grp& g) {
    for (int i = i0 + g.tl; i < i1; i += 4 * g.nt) {
        double x[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int j = i + u * g.nt;
            x[u] = j < i1 ? src[j] : 0.0;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int j = i + u * g.nt;
            if (j < i1) dst[j] = x[u];
        }
    }
}

// L2 prefetch hint for the 16-byte-aligned part of [p, p + bytes) (one bulk
// instruction; never touches bytes outside the range).
__device__ __forceinline__ void prefetch_l2(const void* p, size_t bytes) {
    const unsigned long long a = ((unsigned long long)p + 15ull) & ~15ull;
    const unsigned long long e = ((unsigned long long)p + bytes) & ~15ull;
    if (e > a)
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"((unsigned)(e - a)) : "memory");
}

// lv[l] += dL/dv at the group's probes (row of dLdv): probes [q0, q1) are
// sorted by node, so each node's run is summed in probe order by one thread.
__device__ __forceinline__ void probe_inject(const DevProbe& P, int q0, int q1, const double* __restrict__ row,
                                             double* lv, const Grp& g) {
    for (int q = q0 + g.tl; q < q1; q += g.nt) {
        const int l = P.local[q];
        if (q > q0 && P.local[q - 1] == l) continue;
        double s = lv[l];
        for (int r = q; r < q1 && P.local[r] == l; ++r) s += row[P.slot[r]];
        lv[l] = s;
    }
    __threadfence_block();
}

// ------------------------------------------------------------------ assembly
// One point-process contribution through MechTemp::current
// (mech_template.cuh:612-645): i1 = I(v+0.001), i0 = I(v), scaled by
// sarea = 1e2/area (the node's quotient, computed once per node and step).
__device__ __forceinline__ void pp_add(double i1, double i0, double sarea, bool electrode, double& r, double& dd) {
    double gg = (i1 - i0) * kInvFdEps;
    gg *= sarea;
    i0 *= sarea;
    if (electrode) {
        r += i0;
        dd -= gg;
    } else {
        r -= i0;
        dd += gg;
    }
}

// Network currents of GPU node gi after IClamp, in the exported mechanism
// order: ExpSyn, Exp2Syn (expsyn.cpp:92-121, exp2syn_temp.cuh:45-49), HalfGap
// (HalfGap.cu:56-62, electrode), gapjunction_lr (gapjunction_lr.cu:58-65),
// neuron_to_neuron_syn_lr (neuron_to_neuron_syn_lr.cu:120-127).  synA/synB are
// the cell's synapse states indexed from syn0; grs the graded states s_k.
// A node's synapse range and its first synapse's states and reversal
// potential, loaded at the top of a node iteration (load_syn, next to
// load_par) so that their latency overlaps the mechanism arithmetic instead of
// adding a dependent round trip where the current is assembled.
struct SynPre {
    int s0 = 0, s1 = 0;
    double A0 = 0.0, B0 = 0.0, E0 = 0.0, sarea = 1.0;
};

// The synapse range of the node a thread takes next (pack-local node i, i >=
// i1: none), loaded one iteration ahead so that load_syn finds it ready.
struct SynNext {
    int s0 = 0, s1 = 0;
    double sarea = 1.0;  // 1e2 / the node's area (network nodes)
};

__device__ __forceinline__ void syn_next(const DevGroup& G, const DevNet& N, const Meta& M, int pb, int i, int i1,
                                         SynNext& nx) {
    nx.s0 = nx.s1 = 0;
    if (i >= i1) return;
    const int fl = M.flag[i];
    if (fl & kHasSyn) {
        nx.s0 = __ldg(N.node_syn_off + pb + i);
        nx.s1 = __ldg(N.node_syn_off + pb + i + 1);
    }
    if (fl & (kHasSyn | kHasCpl)) nx.sarea = 1.e2 / __ldg(G.area + pb + i);
}

__device__ __forceinline__ void load_syn(const DevNet& N, const SynNext& nx, const double* __restrict__ synA,
                                         const double* __restrict__ synB, SynPre& sp) {
    sp.s0 = nx.s0;
    sp.s1 = nx.s1;
    sp.sarea = nx.sarea;
    if (sp.s0 < sp.s1) {
        sp.A0 = synA[sp.s0];
        sp.B0 = synB[sp.s0];
        sp.E0 = __ldg(N.syn_e + sp.s0);
    }
}

template <bool kCpl>
__device__ __forceinline__ void assemble_net(const DevGroup& G, const DevNet& N, int gi, int fl, double vi,
                                             const double* __restrict__ synA, const double* __restrict__ synB,
                                             const SynPre& sp, const double* grs,
                                             const double* __restrict__ vpeer, double& r, double& dd) {
    if (!(fl & (kHasSyn | kHasCpl))) return;
    const double sarea = sp.sarea;
    if (fl & kHasSyn) {
        double gs = sp.B0 - sp.A0, e = sp.E0;
        pp_add(gs * ((vi + kFdEps) - e), gs * (vi - e), sarea, false, r, dd);
        for (int j = sp.s0 + 1; j < sp.s1; ++j) {
            gs = synB[j] - synA[j];
            e = __ldg(N.syn_e + j);
            pp_add(gs * ((vi + kFdEps) - e), gs * (vi - e), sarea, false, r, dd);
        }
    }
    if (!kCpl || !(fl & kHasCpl)) return;
    const int h1 = __ldg(N.node_hg_off + gi + 1);
    for (int j = __ldg(N.node_hg_off + gi); j < h1; ++j) {
        // partner voltages with L2-coherent loads: a grid-synchronous launch
        // rewrites vpeer's buffer between steps
        const double vg = __ldcg(vpeer + __ldg(N.hg_src + j)), g = __ldg(N.hg_g + j);
        pp_add((vg - (vi + kFdEps)) * g, (vg - vi) * g, sarea, true, r, dd);
    }
    const int j1 = __ldg(N.node_gj_off + gi + 1);
    for (int j = __ldg(N.node_gj_off + gi); j < j1; ++j) {
        const double vp = __ldcg(vpeer + __ldg(N.gj_pre + j)), g = __ldg(N.gj_g + j), w = __ldg(N.gj_w + j);
        pp_add(w * (g * ((vi + kFdEps) - vp)), w * (g * (vi - vp)), sarea, false, r, dd);
    }
    const int r1 = __ldg(N.node_gr_off + gi + 1);
    for (int j = __ldg(N.node_gr_off + gi); j < r1; ++j) {
        const double aw = fabs(__ldg(N.gr_w + j)), gs = __ldg(N.gr_g + j) * grs[j], er = __ldg(N.gr_erev + j);
        pp_add(aw * (gs * ((vi + kFdEps) - er)), aw * (gs * (vi - er)), sarea, false, r, dd);
    }
}

// Per-node mechanism parameters.  The loops over nodes load them for one node
// with load_par at the top of an iteration, ahead of the arithmetic and of any
// store, so that the global loads of an iteration are in flight together
// rather than one round trip per mechanism.
struct NodePar {
    double pas_g, pas_e;
    double gnabar, gkbar, gl, ena, ek, el;
    double cm;
    int ic0, ic1;  // the node's IClamp range in node_ic
};

__device__ __forceinline__ void load_par(const DevGroup& G, int gi, int fl, NodePar& q) {
    q.pas_g = q.pas_e = 0.0;
    q.gnabar = q.gkbar = q.gl = q.ena = q.ek = q.el = 0.0;
    if (fl & kHasPas) {
        q.pas_g = __ldg(G.pas_g + gi);
        q.pas_e = __ldg(G.pas_e + gi);
    }
    if (fl & kHasHH) {
        q.gnabar = __ldg(G.hh_gnabar + gi);
        q.gkbar = __ldg(G.hh_gkbar + gi);
        q.gl = __ldg(G.hh_gl + gi);
        q.ena = __ldg(G.hh_ena + gi);
        q.ek = __ldg(G.hh_ek + gi);
        q.el = __ldg(G.hh_el + gi);
    }
    q.cm = __ldg(G.cm + gi);
    q.ic0 = __ldg(G.node_ic_off + gi);
    q.ic1 = __ldg(G.node_ic_off + gi + 1);
}

// Adjoint of the gates' cnexp update gates_{k+1} = E gates_k + (1 - E) inf(v_{k+1}),
// E = exp(-dt k(v_{k+1})) (hh_templated.cu:151-164): returns mu plus the gates'
// v_{k+1}-derivatives weighted by their adjoints, and scales the adjoints by E.
__device__ __forceinline__ double gate_adj(double v1, double q10, double dt, double gm, double gh, double gn,
                                           double mu, double& lm, double& lh, double& ln) {
    HHRatesD R;
    hh_rates_d(v1, q10, R);
    const double x[3] = {gm, gh, gn};
    double lam[3] = {lm, lh, ln};
#pragma unroll
    for (int q = 0; q < 3; ++q) {
        const double E = exp(-dt * R.k[q]);
        const double dnew = (1.0 - E) * R.dinf[q] + (R.inf[q] - x[q]) * E * dt * q10 * R.ds[q];
        mu += lam[q] * dnew;
        lam[q] *= E;
    }
    lm = lam[0];
    lh = lam[1];
    ln = lam[2];
    return mu;
}

// Mechanism part of the VJP of step k at GPU node gi (pas, hh, IClamp,
// capacitance): w = (M^-T mu)_i, ld = -w (v_{k+1} - v_k).  Accumulates the
// parameter gradients, adds the gate adjoint increments to lm/lh/ln and
// returns lvn minus the node's own conductance terms.  The gradient
// accumulators and gates are loaded before the first store.
__device__ __forceinline__ double vjp_mech(const DevGroup& G, const DevGrad& GR, const DevTape& T, size_t off, int i,
                                           int gi, int fl, const NodePar& q, double w, double vk, double ld,
                                           double tm, double lvn, double& lm, double& lh, double& ln) {
    // accumulators the caller asked for (GR.skip clear), all loaded before the first store
    const unsigned sk = GR.skip;
    const bool g_pg = !(sk & (1u << HX_P_PAS_G)), g_pe = !(sk & (1u << HX_P_PAS_E));
    const bool g_na = !(sk & (1u << HX_P_HH_GNABAR)), g_k = !(sk & (1u << HX_P_HH_GKBAR));
    const bool g_l = !(sk & (1u << HX_P_HH_GL)), g_el = !(sk & (1u << HX_P_HH_EL));
    const bool g_cm = !(sk & (1u << HX_P_CM)), g_ic = !(sk & (1u << HX_P_IC_AMP));
    double m = 0.0, h = 0.0, nn = 0.0;
    double a_pg = 0.0, a_pe = 0.0, a_na = 0.0, a_k = 0.0, a_l = 0.0, a_el = 0.0, a_cm = 0.0;
    if (fl & kHasPas) {
        if (g_pg) a_pg = GR.pas_g[gi];
        if (g_pe) a_pe = GR.pas_e[gi];
    }
    if (fl & kHasHH) {
        // the gates' last read of their tape row (streaming loads)
        m = __ldcs(T.m + off + i);
        h = __ldcs(T.h + off + i);
        nn = __ldcs(T.n + off + i);
        if (g_na) a_na = GR.hh_gnabar[gi];
        if (g_k) a_k = GR.hh_gkbar[gi];
        if (g_l) a_l = GR.hh_gl[gi];
        if (g_el) a_el = GR.hh_el[gi];
    }
    if (g_cm) a_cm = GR.cm[gi];
    if (fl & kHasPas) {
        if (g_pg) GR.pas_g[gi] = a_pg + (ld - w * (vk - q.pas_e));
        if (g_pe) GR.pas_e[gi] = a_pe + w * q.pas_g;
        lvn -= w * q.pas_g;
    }
    if (fl & kHasHH) {
        const double t_na = ld - w * (vk - q.ena);
        const double t_k = ld - w * (vk - q.ek);
        const double t_l = ld - w * (vk - q.el);
        const double m2h = m * m * h, n3 = nn * nn * nn;
        if (g_na) GR.hh_gnabar[gi] = a_na + m2h * m * t_na;
        if (g_k) GR.hh_gkbar[gi] = a_k + n3 * nn * t_k;
        if (g_l) GR.hh_gl[gi] = a_l + t_l;
        if (g_el) GR.hh_el[gi] = a_el + w * q.gl;
        lm += 3.0 * q.gnabar * m2h * t_na;
        lh += q.gnabar * m * m * m * t_na;
        ln += 4.0 * q.gkbar * n3 * t_k;
        lvn -= w * (q.gnabar * m2h * m + q.gkbar * n3 * nn + q.gl);
    }
    if (g_ic)
        for (int k2 = q.ic0; k2 < q.ic1; ++k2) {
            const int j = __ldg(G.node_ic + k2);
            const double del = __ldg(G.ic_del + j), dur = __ldg(G.ic_dur + j);
            if (tm < del + dur && tm >= del) GR.ic_amp[j] += w * (1.e2 / __ldg(G.area + gi));
        }
    if (g_cm) GR.cm[gi] = a_cm + ld * G.cfac;
    return lvn;
}

// rhs/d of pack-local node i in the reference's accumulation order:
// pas, hh, IClamp (CoreNEURON type order), [network currents], [library
// channels; *ica receives the node's calcium current], capacitance
// jacobian, axial terms.  vi is the node's voltage; sv (neighbour voltages) is
// read only when kRhs.
template <bool kRhs, bool kNet = false, bool kSplitAxial = false, bool kLib = false, bool kCpl = false>
__device__ __forceinline__ void assemble(const DevGroup& G, const Meta& M, int pb, int i, int fl, const NodePar& q,
                                         double vi, const double* __restrict__ sv, const double* __restrict__ sa,
                                         const double* __restrict__ sb, double m, double h, double n, double tmid,
                                         double& r_out, double& d_out, const DevNet& N = DevNet{},
                                         const double* synA = nullptr, const double* synB = nullptr,
                                         const SynPre& sp = SynPre{}, const double* grs = nullptr,
                                         const double* vpeer = nullptr,
                                         const DevLib* L = nullptr, const double* X = nullptr,
                                         double* ica = nullptr) {
    const int gi = pb + i;
    double r = 0.0, dd = 0.0;
    if (fl & kHasPas) {  // pas_templated.cu:27-31 through MechTemp::current (FD conductance)
        double g1 = q.pas_g * ((vi + kFdEps) - q.pas_e);
        const double i0 = q.pas_g * (vi - q.pas_e);
        g1 = (g1 - i0) * kInvFdEps;
        r -= i0;
        dd += g1;
    }
    if (fl & kHasHH) {  // hh_templated.cu:137-149
        double g1 = hh_current(vi + kFdEps, q.gnabar, q.gkbar, q.gl, m, h, n, q.ena, q.ek, q.el);
        const double i0 = hh_current(vi, q.gnabar, q.gkbar, q.gl, m, h, n, q.ena, q.ek, q.el);
        g1 = (g1 - i0) * kInvFdEps;
        r -= i0;
        dd += g1;
    }
    for (int k = q.ic0; k < q.ic1; ++k) {  // iclamp_templated.cu:35-45, electrode
        const int j = __ldg(G.node_ic + k);
        const double del = __ldg(G.ic_del + j), dur = __ldg(G.ic_dur + j);
        const double cur = (tmid < del + dur && tmid >= del) ? __ldg(G.ic_amp + j) : 0.0;
        r += cur * (1.e2 / __ldg(G.area + gi));
    }
    if (kNet) assemble_net<kCpl>(G, N, gi, fl, vi, synA, synB, sp, grs, vpeer, r, dd);
    if (kLib) *ica = lib::lib_current(*L, gi, vi, X, r, dd);  // library types follow the network ones
    dd += G.cfac * q.cm;
    if (kSplitAxial) {  // parent / children may sit in other CTAs (a split cell)
        r_out = r;
        d_out = dd;
        return;
    }
    const int par = M.par[i];
    if (par >= 0) {
        if (kRhs) r -= sb[i] * (sv[par] - vi);
        dd -= sb[i];
    }
    const int c1 = M.cho[i + 1];
    for (int k = M.cho[i]; k < c1; ++k) {
        const int c = M.ch[k];
        const double ac = sa[c];
        if (kRhs) r += ac * (vi - sv[c]);
        dd -= ac;
    }
    r_out = r;
    d_out = dd;
}

}  // namespace hx
