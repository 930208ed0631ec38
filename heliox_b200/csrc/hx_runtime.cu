// hx_runtime.cu -- the C ABI (include/heliox_b200.h) over the plan and kernels.
//
// Owns device buffers (grow-only, reused across calls like the reference's
// LearnRuntime::ensure_buf, src/runtime_api/learn/LearnRuntime.cpp:877-895),
// the forward tape / checkpoint policy and the launch stream.  All work is
// enqueued on one stream; host-buffer entry points stage through pinned memory.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "heliox_b200.h"
#include "hx_ctx.hpp"
#include "hx_dev.hpp"
#include "hx_kernels.hpp"
#include "hx_plan.hpp"

int hx_fail(hx_ctx* c, const std::string& m) {
    if (c) c->err = m;
    return -1;
}
static int fail(hx_ctx* c, const std::string& m) { return hx_fail(c, m); }

#define HXC(call)                                                                                    \
    do {                                                                                             \
        cudaError_t _e = (call);                                                                     \
        if (_e != cudaSuccess) return fail(ctx, std::string(#call) + ": " + cudaGetErrorString(_e)); \
    } while (0)

static size_t kind_count(const hx_ctx* c, int kind) {
    const hx::Plan& P = c->P;
    switch (kind) {
        case HX_P_HH_GNABAR:
        case HX_P_HH_GKBAR:
        case HX_P_HH_GL:
        case HX_P_HH_EL:
            return (size_t)P.nhh;
        case HX_P_PAS_G:
        case HX_P_PAS_E:
            return (size_t)P.npas;
        case HX_P_CM:
            return (size_t)P.nnode;
        case HX_P_IC_AMP:
            return (size_t)P.nic;
        case HX_P_EXPSYN_W:
        case HX_P_EXPSYN_E:
            return (size_t)c->nexp;
        case HX_P_EXP2SYN_W:
        case HX_P_EXP2SYN_E:
            return (size_t)c->nexp2;
        case HX_P_HALFGAP_G:
            return (size_t)c->nhg;
        case HX_P_GAPJ_G:
        case HX_P_GAPJ_W:
            return (size_t)c->ngj_lr;
        case HX_P_GAPNP_W:
            return (size_t)c->ngnp;
        case HX_P_GRADED_W:
            return (size_t)c->ngr;
    }
    const int lt = hx_lib_type_of_kind(kind);
    if (lt >= 0) return (size_t)c->lib_n[lt];
    return 0;
}

// Device storage of a kind: node-indexed for density mechanisms and cm, per
// instance for IClamp and the network kinds.  ExpSyn and Exp2Syn share one
// array per variable (GPU synapse order), owned by the ExpSyn kind;
// gapjunction_lr and gapjunction_noptr share the gap arrays (noptr instances
// carry g = weight, w = 1), owned by the gapjunction_lr kinds.
static size_t kind_store(const hx_ctx* c, int kind) {
    switch (kind) {
        case HX_P_IC_AMP:
            return (size_t)c->P.nic;
        case HX_P_EXPSYN_W:
        case HX_P_EXPSYN_E:
            return (size_t)c->nsyn;
        case HX_P_EXP2SYN_W:
        case HX_P_EXP2SYN_E:
            return 0;
        case HX_P_HALFGAP_G:
            return (size_t)c->nhg;
        case HX_P_GAPJ_G:
        case HX_P_GAPJ_W:
            return (size_t)c->ngj;
        case HX_P_GAPNP_W:
            return 0;
        case HX_P_GRADED_W:
            return (size_t)c->ngr;
    }
    const int lt = hx_lib_type_of_kind(kind);
    if (lt >= 0) return (size_t)c->lib_n[lt];  // per instance, GPU instance order
    return (size_t)c->P.nnode;
}

static int store_kind(int kind) {
    return kind == HX_P_EXP2SYN_W   ? HX_P_EXPSYN_W
           : kind == HX_P_EXP2SYN_E ? HX_P_EXPSYN_E
           : kind == HX_P_GAPNP_W   ? HX_P_GAPJ_G
                                    : kind;
}
double* hx_kind_ptr(hx_ctx* c, int kind) { return c->prm[store_kind(kind)].p; }
size_t hx_grad_base(const hx_ctx* c, int kind) { return c->grad_off[store_kind(kind)]; }

// dynamic shared memory per CTA of the two step kernels for a plan (the
// split-cell kernels when the plan splits a cell)
static void plan_smem(const hx::Plan& P, size_t& fwd, size_t& bwd) {
    hx::DevGroup Gt{};
    Gt.smem_n = std::max(P.max_pack_nodes, 1);
    Gt.smem_br = P.max_pack_branches;
    Gt.smem_bch = P.max_pack_bch;
    Gt.smem_nch = P.max_pack_nch;
    Gt.smem_lvl = P.warps * (P.max_levels + 1);
    fwd = P.nsub > 0 ? hx::split_fwd_smem_bytes(Gt) : hx::fwd_smem_bytes(Gt);
    bwd = P.nsub > 0 ? hx::split_bwd_smem_bytes(Gt) : hx::bwd_smem_bytes(Gt);
}

static void fill_stats(const hx::Plan& P, hx_plan_stats* out) {
    out->npack = P.npack;
    out->max_pack_nodes = P.max_pack_nodes;
    out->max_pack_hh = P.max_pack_hh;
    out->max_levels = P.max_levels;
    out->max_crit_nodes = P.max_crit;
    out->nbranch = (int)P.br_head.size();
    out->imbalance = P.imbalance;
    out->nsub = P.nsub;
    out->est_max = P.est_max;
    out->est_mean = P.est_mean;
    plan_smem(P, out->smem_fwd, out->smem_bwd);
}

static std::vector<int> invert(const std::vector<int>& g2r, size_t n) {
    std::vector<int> r2g(std::max<size_t>(n, 1), 0);
    for (size_t i = 0; i < g2r.size(); i++) r2g[g2r[i]] = (int)i;
    return r2g;
}

extern "C" {

int hx_abi_version(void) { return HX_ABI_VERSION; }

int hx_create(hx_ctx** out, int device) {
    if (!out) return -1;
    *out = nullptr;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev <= 0) return -2;
    if (device < 0 || device >= ndev) return -3;
    hx_ctx* ctx = new hx_ctx();
    ctx->device = device;
    if (cudaSetDevice(device) != cudaSuccess || cudaStreamCreateWithFlags(&ctx->own, cudaStreamNonBlocking) != cudaSuccess) {
        delete ctx;
        return -4;
    }
    ctx->st = ctx->own;
    for (auto& e : ctx->ev) cudaEventCreate(&e);
    *out = ctx;
    return 0;
}

int hx_destroy(hx_ctx* ctx) {
    if (!ctx) return 0;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->st);
    for (auto& e : ctx->ev)
        if (e) cudaEventDestroy(e);
    for (cudaEvent_t e : ctx->kev)
        if (e) cudaEventDestroy(e);
    if (ctx->own) cudaStreamDestroy(ctx->own);
    for (AdamOpt* o : ctx->opts) delete o;
    delete ctx;
    return 0;
}

const char* hx_last_error(hx_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

int hx_set_stream(hx_ctx* ctx, void* stream) {
    if (!ctx) return -1;
    ctx->st = stream ? (cudaStream_t)stream : ctx->own;
    return 0;
}

int hx_set_pack_target(hx_ctx* ctx, int nodes_per_warp) {
    if (!ctx) return -1;
    if (nodes_per_warp < 0) return fail(ctx, "nodes_per_warp must be >= 0");
    ctx->pack_target = nodes_per_warp;
    return 0;
}

int hx_set_tape_budget(hx_ctx* ctx, size_t bytes) {
    if (!ctx) return -1;
    ctx->tape_budget = bytes;
    return 0;
}

int hx_set_split_barrier_limit(hx_ctx* ctx, long long sleeps) {
    if (!ctx) return -1;
    if (sleeps < 0) return fail(ctx, "barrier limit must be >= 0");
    ctx->split_spin_limit = sleeps ? sleeps : hx::kSplitSpinLimitDefault;
    ctx->X.spin_limit = ctx->split_spin_limit;
    ctx->N.gspin = ctx->split_spin_limit;
    return 0;
}

int hx_set_grad_kinds(hx_ctx* ctx, const int* kinds, int n) {
    if (!ctx) return -1;
    if (n <= 0) {
        ctx->grad_skip = 0;
        return 0;
    }
    if (!kinds) return fail(ctx, "null kinds");
    unsigned need = 0;
    for (int i = 0; i < n; i++) {
        if (kinds[i] < 0 || kinds[i] >= HX_P_COUNT) return fail(ctx, "bad parameter kind");
        const int sk = store_kind(kinds[i]);
        if (sk < 16) need |= 1u << sk;
    }
    ctx->grad_skip = ~need & 0xFFFFu;
    return 0;
}

int hx_set_grid_sync(hx_ctx* ctx, int enable) {
    if (!ctx) return -1;
    ctx->gsync_allowed = enable != 0;
    ctx->N.gsync = ctx->gsync_fit && ctx->gsync_allowed ? 1 : 0;
    return 0;
}

int hx_plan_check(const hx_group_desc* desc, int nodes_per_warp, hx_plan_stats* out, double* max_abs_diff,
                  double* pq_rel_diff) {
    return hx_plan_check_cap(desc, nodes_per_warp, 0, out, max_abs_diff, pq_rel_diff);
}

int hx_plan_check_cap(const hx_group_desc* desc, int nodes_per_warp, int max_pack_nodes, hx_plan_stats* out,
                      double* max_abs_diff, double* pq_rel_diff) {
    return hx_plan_check_sm(desc, nodes_per_warp, max_pack_nodes, 0, out, max_abs_diff, pq_rel_diff);
}

int hx_plan_check_sm(const hx_group_desc* desc, int nodes_per_warp, int max_pack_nodes, int nsm, hx_plan_stats* out,
                     double* max_abs_diff, double* pq_rel_diff) {
    if (!desc) return -1;
    hx::Plan P;
    // as hx_load_group: a single cell above the capacity is planned for the
    // split-cell kernels' CTA width
    const bool split = desc->ncell == 1 && max_pack_nodes > 0 && desc->nnode > max_pack_nodes;
    std::string e = hx::build_plan(*desc, nodes_per_warp, max_pack_nodes, P, nsm,
                                   split ? hx::kSplitThreads / 32 : hx::kWarpsPerCta);
    if (!e.empty()) {
        fprintf(stderr, "hx_plan_check: %s\n", e.c_str());
        return -2;
    }
    if (out) fill_stats(P, out);
    if (max_abs_diff || pq_rel_diff) {
        // seeded diagonally dominant system; serial solve in reference order vs planned schedule
        const int n = desc->nnode;
        std::mt19937_64 rng(12345);
        std::uniform_real_distribution<double> U(0.5, 1.5);
        double worst = 0.0, worst_pq = 0.0;
        for (int transposed = 0; transposed < 2; transposed++) {
            std::vector<double> d(n), r(n);
            for (int i = 0; i < n; i++) {
                d[i] = 40.0 * U(rng) + 10.0;
                r[i] = U(rng) - 1.0;
            }
            for (int i = desc->ncell; i < n; i++) {
                d[i] -= desc->b[i];
                d[desc->parent[i]] -= desc->a[i];
            }
            std::vector<double> ds = d, rs = r;
            const double* A = transposed ? desc->b : desc->a;
            const double* Uc = transposed ? desc->a : desc->b;
            for (int i = n - 1; i >= desc->ncell; i--) {
                int p = desc->parent[i];
                double f = A[i] / ds[i];
                ds[p] -= f * Uc[i];
                rs[p] -= f * rs[i];
            }
            for (int i = 0; i < desc->ncell; i++) rs[i] /= ds[i];
            for (int i = desc->ncell; i < n; i++) {
                rs[i] -= Uc[i] * rs[desc->parent[i]];
                rs[i] /= ds[i];
            }
            std::vector<double> ag(n), bg(n), dg(n), rg(n);
            for (int gi = 0; gi < n; gi++) {
                int ref = P.gpu2ref[gi];
                ag[gi] = desc->a[ref];
                bg[gi] = desc->b[ref];
                dg[gi] = d[ref];
                rg[gi] = r[ref];
            }
            std::vector<double> dq = dg, rq = rg, dt = dg, rt = rg;
            hx::planned_solve_cpu(P, ag.data(), bg.data(), dg.data(), rg.data(), transposed != 0);
            hx::planned_solve_pq_cpu(P, ag.data(), bg.data(), dq.data(), rq.data(), transposed != 0);
            if (P.nsub == 0) hx::planned_solve_rt_cpu(P, ag.data(), bg.data(), dt.data(), rt.data(), transposed != 0);
            double scale = 0.0;
            for (int gi = 0; gi < n; gi++) scale = std::max(scale, std::fabs(rs[gi]));
            for (int gi = 0; gi < n; gi++) {
                worst = std::max(worst, std::fabs(rg[gi] - rs[P.gpu2ref[gi]]));
                worst_pq = std::max(worst_pq, std::fabs(rq[gi] - rs[P.gpu2ref[gi]]) / scale);
                if (P.nsub == 0) worst_pq = std::max(worst_pq, std::fabs(rt[gi] - rs[P.gpu2ref[gi]]) / scale);
            }
        }
        if (max_abs_diff) *max_abs_diff = worst;
        if (pq_rel_diff) *pq_rel_diff = worst_pq;
    }
    return 0;
}

int hx_load_group(hx_ctx* ctx, const hx_group_desc* desc) {
    if (!ctx || !desc) return fail(ctx, "null argument");
    HXC(cudaSetDevice(ctx->device));
    ctx->loaded = false;
    ctx->captured = false;
    ctx->probe_key.clear();
    ctx->tmid_steps = -1;
    // per-CTA node capacity from the opt-in shared memory: the forward kernel
    // keeps 5 doubles per node (the backward 4) plus about 9 bytes of
    // topology tables and the per-segment arrays (network groups keep their
    // synapse states in global memory).  A single cell larger than that is
    // split across CTAs, whose kernels keep 10 doubles per node.  The plan is
    // checked against the exact table sizes and rebuilt with a capacity
    // smaller by its overshoot while it does not fit: the step kernels are
    // latency bound, so the nodes a wave of CTAs holds sets the throughput.
    int optin = 0, nsm = 0;
    HXC(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, ctx->device));
    HXC(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, ctx->device));
    int cap_nodes = (int)((optin - 1024) / (5 * sizeof(double) + 8));
    bool split_kernels = false;
    if (desc->ncell == 1 && desc->nnode > cap_nodes) {
        split_kernels = true;
        cap_nodes = (int)((optin - 4096) / (10 * sizeof(double) + 10));
    }
    cap_nodes = std::min(cap_nodes, 32767);  // 16-bit node tables
    const int warps = split_kernels ? hx::kSplitThreads / 32 : hx::kWarpsPerCta;
    std::string e = hx::build_plan(*desc, ctx->pack_target, cap_nodes, ctx->P, nsm, warps);
    if (!e.empty()) return fail(ctx, "invalid group: " + e);
    for (int shrink = 0; shrink < 200 && desc->nnode > 0; shrink++) {
        const hx::Plan& Pc = ctx->P;
        hx::DevGroup Gt{};
        Gt.smem_n = std::max(Pc.max_pack_nodes, 1);
        Gt.smem_br = Pc.max_pack_branches;
        Gt.smem_bch = Pc.max_pack_bch;
        Gt.smem_nch = Pc.max_pack_nch;
        Gt.smem_lvl = Pc.warps * (Pc.max_levels + 1);
        const size_t need = split_kernels ? std::max(hx::split_fwd_smem_bytes(Gt), hx::split_bwd_smem_bytes(Gt))
                                          : std::max(hx::fwd_smem_bytes(Gt), hx::bwd_smem_bytes(Gt));
        if (need <= (size_t)optin) break;
        // shrink by the overshoot (at least 0.2 %, at most 1.5 % a step)
        const double f = std::max(0.985, std::min(0.998, 0.999 * (double)optin / (double)need));
        cap_nodes = std::min(cap_nodes - 1, (int)(cap_nodes * f));
        e = hx::build_plan(*desc, ctx->pack_target, cap_nodes, ctx->P, nsm, warps);
        if (!e.empty()) return fail(ctx, "invalid group: " + e);
    }
    const hx::Plan& P = ctx->P;
    cudaStream_t st = ctx->st;
    const size_t nn = P.nnode, nc = P.nic;
    ctx->dt = desc->dt;
    ctx->celsius = desc->celsius;
    HXC(ctx->pack_node_off.upload(P.pack_node_off, st));
    HXC(ctx->pack_slot_off.upload(P.pack_slot_off, st));
    HXC(ctx->pack_br_off.upload(P.pack_br_off, st));
    HXC(ctx->pack_bch_off.upload(P.pack_bch_off, st));
    HXC(ctx->pack_nch_off.upload(P.pack_nch_off, st));
    HXC(ctx->cs_node0.upload(P.cs_node0, st));
    HXC(ctx->cs_nnode.upload(P.cs_nnode, st));
    HXC(ctx->cs_warp0.upload(P.cs_warp0, st));
    HXC(ctx->cs_nwarp.upload(P.cs_nwarp, st));
    HXC(ctx->cs_bar.upload(P.cs_bar, st));
    HXC(ctx->cs_lvl_off.upload(P.cs_lvl_off, st));
    HXC(ctx->cs_nlev.upload(P.cs_nlev, st));
    HXC(ctx->level_br_off.upload(P.level_br_off, st));
    HXC(ctx->br_head.upload(P.br_head, st));
    HXC(ctx->br_end.upload(P.br_end, st));
    HXC(ctx->br_parent.upload(P.br_parent, st));
    HXC(ctx->br_child_off.upload(P.br_child_off, st));
    HXC(ctx->br_child.upload(P.br_child, st));
    HXC(ctx->br_child_br.upload(P.br_child_br, st));
    HXC(ctx->node_parent.upload(P.node_parent, st));
    HXC(ctx->node_child_off.upload(P.node_child_off, st));
    HXC(ctx->node_child.upload(P.node_child, st));
    HXC(ctx->node_ic_off.upload(P.node_ic_off, st));
    HXC(ctx->node_ic.upload(P.node_ic, st));
    std::vector<int> flags(nn, 0);
    for (size_t gi = 0; gi < nn; gi++)
        flags[gi] = (P.node_pas[gi] >= 0 ? hx::kHasPas : 0) | (P.node_hh[gi] >= 0 ? hx::kHasHH : 0);
    {  // network instances on / partners of each node (indices are validated by hx_net_load)
        auto mark = [&](const int* node, int n, int bit) {
            for (int i = 0; node && i < n; i++)
                if (node[i] >= 0 && (size_t)node[i] < nn) flags[P.ref2gpu[node[i]]] |= bit;
        };
        mark(desc->expsyn_node, desc->nexpsyn, hx::kHasSyn);
        mark(desc->exp2syn_node, desc->nexp2syn, hx::kHasSyn);
        mark(desc->hg_node, desc->nhalfgap, hx::kHasCpl);
        mark(desc->gj_node, desc->ngapj, hx::kHasCpl);
        mark(desc->gn_node, desc->ngapnp, hx::kHasCpl);
        mark(desc->gr_node, desc->ngraded, hx::kHasCpl);
        mark(desc->hg_src, desc->nhalfgap, hx::kHasIn);
        mark(desc->gj_pre, desc->ngapj, hx::kHasIn);
        mark(desc->gn_src, desc->ngapnp, hx::kHasIn);
        mark(desc->gr_pre, desc->ngraded, hx::kHasIn);
    }
    HXC(ctx->node_flags.upload(flags, st));

    // network tables (instance orders, kinds 8.. maps, device arrays)
    if (hx_net_load(ctx, desc)) return -1;
    // reference instance -> device slot per kind (network kinds: hx_net_load)
    for (int k = 0; k < HX_P_EXPSYN_W; k++) {
        std::vector<int>& m = ctx->kmap_h[k];
        m.assign(std::max<size_t>(kind_count(ctx, k), 1), 0);
        const size_t cnt = kind_count(ctx, k);
        for (size_t r = 0; r < cnt; r++) {
            if (k <= HX_P_HH_EL)
                m[r] = P.ref2gpu[desc->hh_node[r]];
            else if (k <= HX_P_PAS_E)
                m[r] = P.ref2gpu[desc->pas_node[r]];
            else if (k == HX_P_CM)
                m[r] = P.ref2gpu[r];
        }
        if (k == HX_P_IC_AMP) {
            std::vector<int> inv = invert(P.ic_gpu2ref, P.nic);
            for (size_t r = 0; r < cnt; r++) m[r] = inv[r];
        }
        HXC(ctx->kmap[k].upload(m, st));
    }
    // library mechanism tables (kinds HX_P_CADYN_GAMMA..)
    if (hx_lib_load(ctx, desc)) return -1;
    // node-indexed copies of reference-ordered arrays
    auto node_arr = [&](const double* src) {
        std::vector<double> out(std::max<size_t>(nn, 1), 0.0);
        for (size_t gi = 0; gi < nn; gi++) out[gi] = src[P.gpu2ref[gi]];
        return out;
    };
    auto inst_arr = [&](int kind, const double* src) {  // density-mechanism instance values -> node slots
        std::vector<double> out(std::max<size_t>(kind_store(ctx, kind), 1), 0.0);
        const size_t cnt = kind_count(ctx, kind);
        for (size_t r = 0; r < cnt; r++) out[ctx->kmap_h[kind][r]] = src[r];
        return out;
    };
    HXC(ctx->a.upload(node_arr(desc->a), st));
    HXC(ctx->b.upload(node_arr(desc->b), st));
    HXC(ctx->area.upload(node_arr(desc->area), st));
    HXC(ctx->prm[HX_P_CM].upload(node_arr(desc->cm), st));
    HXC(ctx->prm[HX_P_HH_GNABAR].upload(inst_arr(HX_P_HH_GNABAR, desc->hh_gnabar), st));
    HXC(ctx->prm[HX_P_HH_GKBAR].upload(inst_arr(HX_P_HH_GKBAR, desc->hh_gkbar), st));
    HXC(ctx->prm[HX_P_HH_GL].upload(inst_arr(HX_P_HH_GL, desc->hh_gl), st));
    HXC(ctx->prm[HX_P_HH_EL].upload(inst_arr(HX_P_HH_EL, desc->hh_el), st));
    HXC(ctx->hh_ena.upload(inst_arr(HX_P_HH_GNABAR, desc->hh_ena), st));
    HXC(ctx->hh_ek.upload(inst_arr(HX_P_HH_GNABAR, desc->hh_ek), st));
    HXC(ctx->prm[HX_P_PAS_G].upload(inst_arr(HX_P_PAS_G, desc->pas_g), st));
    HXC(ctx->prm[HX_P_PAS_E].upload(inst_arr(HX_P_PAS_E, desc->pas_e), st));
    HXC(ctx->ic_del.upload(inst_arr(HX_P_IC_AMP, desc->ic_del), st));
    HXC(ctx->ic_dur.upload(inst_arr(HX_P_IC_AMP, desc->ic_dur), st));
    HXC(ctx->prm[HX_P_IC_AMP].upload(inst_arr(HX_P_IC_AMP, desc->ic_amp), st));

    HXC(ctx->sv.ensure(nn));
    HXC(ctx->sm.ensure(nn));
    HXC(ctx->sh.ensure(nn));
    HXC(ctx->sn.ensure(nn));
    HXC(ctx->lv.ensure(nn));
    HXC(ctx->lm.ensure(nn));
    HXC(ctx->lh.ensure(nn));
    HXC(ctx->ln.ensure(nn));
    ctx->grad_off[0] = 0;
    for (int k = 0; k < HX_P_COUNT; k++) ctx->grad_off[k + 1] = ctx->grad_off[k] + kind_store(ctx, k);
    HXC(ctx->grad.ensure(ctx->grad_off[HX_P_COUNT]));
    for (int k = 0; k < hx::kLibKinds; k++) ctx->L.grad[k] = ctx->grad.p + ctx->grad_off[HX_P_CADYN_GAMMA + k];
    // staging of per-kind gathers at grad_off[k]: kinds without storage of their
    // own (Exp2Syn, gapjunction_noptr) stage past their offset
    HXC(ctx->stage_dev.ensure(ctx->grad_off[HX_P_COUNT] + std::max({nn, (size_t)ctx->nsyn, (size_t)ctx->ngj})));

    hx::DevGroup& G = ctx->G;
    G = hx::DevGroup{};
    G.npack = P.npack;
    G.nnode = P.nnode;
    G.nic = P.nic;
    G.smem_n = std::max(P.max_pack_nodes, 1);
    G.smem_br = P.max_pack_branches;
    G.smem_bch = P.max_pack_bch;
    G.smem_nch = P.max_pack_nch;
    G.smem_lvl = P.warps * (P.max_levels + 1);
    G.pack_node_off = ctx->pack_node_off.p;
    G.pack_slot_off = ctx->pack_slot_off.p;
    G.pack_br_off = ctx->pack_br_off.p;
    G.pack_bch_off = ctx->pack_bch_off.p;
    G.pack_nch_off = ctx->pack_nch_off.p;
    G.cs_node0 = ctx->cs_node0.p;
    G.cs_nnode = ctx->cs_nnode.p;
    G.cs_warp0 = ctx->cs_warp0.p;
    G.cs_nwarp = ctx->cs_nwarp.p;
    G.cs_bar = ctx->cs_bar.p;
    G.cs_lvl_off = ctx->cs_lvl_off.p;
    G.cs_nlev = ctx->cs_nlev.p;
    G.level_br_off = ctx->level_br_off.p;
    G.br_head = ctx->br_head.p;
    G.br_end = ctx->br_end.p;
    G.br_parent = ctx->br_parent.p;
    G.br_child_off = ctx->br_child_off.p;
    G.br_child = ctx->br_child.p;
    G.br_child_br = ctx->br_child_br.p;
    G.node_parent = ctx->node_parent.p;
    G.node_child_off = ctx->node_child_off.p;
    G.node_child = ctx->node_child.p;
    G.node_flags = ctx->node_flags.p;
    G.node_ic_off = ctx->node_ic_off.p;
    G.node_ic = ctx->node_ic.p;
    G.a = ctx->a.p;
    G.b = ctx->b.p;
    G.cm = ctx->prm[HX_P_CM].p;
    G.area = ctx->area.p;
    G.hh_gnabar = ctx->prm[HX_P_HH_GNABAR].p;
    G.hh_gkbar = ctx->prm[HX_P_HH_GKBAR].p;
    G.hh_gl = ctx->prm[HX_P_HH_GL].p;
    G.hh_el = ctx->prm[HX_P_HH_EL].p;
    G.hh_ena = ctx->hh_ena.p;
    G.hh_ek = ctx->hh_ek.p;
    G.pas_g = ctx->prm[HX_P_PAS_G].p;
    G.pas_e = ctx->prm[HX_P_PAS_E].p;
    G.ic_del = ctx->ic_del.p;
    G.ic_dur = ctx->ic_dur.p;
    G.ic_amp = ctx->prm[HX_P_IC_AMP].p;
    G.dt = desc->dt;
    G.cfac = 0.001 * (1.0 / desc->dt);                  // capac.cpp:56,70 with cj = 1/dt
    G.q10 = std::pow(3.0, (desc->celsius - 6.3) / 10);  // hh_templated.cu:90
    ctx->split = P.nsub > 0;
    if (ctx->split && ctx->lib) return fail(ctx, "library mechanisms on a cell split across CTAs are not supported");
    size_t sf = ctx->split ? hx::split_fwd_smem_bytes(G) : hx::fwd_smem_bytes(G);
    size_t sb = ctx->split ? hx::split_bwd_smem_bytes(G) : hx::bwd_smem_bytes(G);
    size_t sfn = hx::fwd_smem_bytes(G), sbn = hx::bwd_smem_bytes(G);
    int maxsmem = 0;
    HXC(cudaDeviceGetAttribute(&maxsmem, cudaDevAttrMaxSharedMemoryPerBlockOptin, ctx->device));
    const size_t need = std::max(ctx->net ? std::max(sfn, sbn) : sb, sf);
    if (need > (size_t)maxsmem)
        return fail(ctx, "cell pack needs " + std::to_string(need) + " B shared memory (> " + std::to_string(maxsmem) +
                             "); lower the pack target or split the cell");
    HXC(hx::configure_kernels(std::min(hx::fwd_smem_bytes(G), (size_t)maxsmem),
                              std::min(hx::bwd_smem_bytes(G), (size_t)maxsmem), std::min(sfn, (size_t)maxsmem),
                              std::min(sbn, (size_t)maxsmem)));
    // coupled networks: grid-synchronous launches (many steps a launch, one
    // grid barrier a step) when every pack can be co-resident
    ctx->gsync_fit = false;
    if (ctx->coupled && !ctx->split) {
        int coop = 0, per_f = 0, per_b = 0;
        HXC(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, ctx->device));
        HXC(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_f, hx::fwd_cpl_kernel_ptr(ctx->lib), hx::kThreads,
                                                          std::min(sfn, (size_t)maxsmem)));
        HXC(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_b, hx::bwd_cpl_kernel_ptr(ctx->lib), hx::kThreads,
                                                          std::min(sbn, (size_t)maxsmem)));
        ctx->gsync_fit = coop && (long long)std::min(per_f, per_b) * nsm >= P.npack;
    }
    ctx->N.gsync = ctx->gsync_fit && ctx->gsync_allowed ? 1 : 0;
    if (ctx->split) {
        if (ctx->net) return fail(ctx, "a cell split across CTAs cannot carry network parts");
        HXC(hx::configure_split(sf, sb));
        int per_sm = 0, per_sm_b = 0;
        HXC(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, hx::split_fwd_kernel_ptr(), hx::kSplitThreads, sf));
        HXC(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm_b, hx::split_bwd_kernel_ptr(), hx::kSplitThreads, sb));
        if ((long long)std::min(per_sm, per_sm_b) * nsm < P.npack)
            return fail(ctx, "split cell needs " + std::to_string(P.npack) + " co-resident CTAs (have " +
                                 std::to_string(std::min(per_sm, per_sm_b) * nsm) + ")");
        HXC(ctx->sub_root.upload(P.sub_root, st));
        HXC(ctx->sub_parent.upload(P.sub_parent, st));
        for (auto* b : {&ctx->xd, &ctx->xrhs, &ctx->xx, &ctx->xv, &ctx->xvp}) HXC(b->ensure(P.nsub));
        HXC(ctx->split_bar.ensure(2));
        HXC(ctx->split_err.ensure(1));
        hx::DevSplit& X = ctx->X;
        X.nsub = P.nsub;
        X.nblocks = P.npack;
        X.sub_root = ctx->sub_root.p;
        X.sub_parent = ctx->sub_parent.p;
        X.xd = ctx->xd.p;
        X.xrhs = ctx->xrhs.p;
        X.xx = ctx->xx.p;
        X.xv = ctx->xv.p;
        X.xvp = ctx->xvp.p;
        X.bar = ctx->split_bar.p;
        X.err = ctx->split_err.p;
        X.spin_limit = ctx->split_spin_limit;
    }
    {
        std::vector<double*> ptrs(HX_P_COUNT);
        for (int k = 0; k < HX_P_COUNT; k++) ptrs[k] = hx_kind_ptr(ctx, k);
        HXC(ctx->prm_ptrs.upload(ptrs, st));
    }
    for (AdamOpt* o : ctx->opts) delete o;  // bindings refer to the previous group
    ctx->opts.clear();
    HXC(cudaStreamSynchronize(st));
    ctx->loaded = true;
    return 0;
}

int hx_get_plan_stats(hx_ctx* ctx, hx_plan_stats* out) {
    if (!ctx || !out) return -1;
    if (!ctx->loaded) return fail(ctx, "no group loaded");
    fill_stats(ctx->P, out);
    return 0;
}

int hx_set_param(hx_ctx* ctx, int kind, const double* values, int n) {
    if (!ctx || !values) return fail(ctx, "null argument");
    if (!ctx->loaded) return fail(ctx, "no group loaded");
    if (kind < 0 || kind >= HX_P_COUNT) return fail(ctx, "bad parameter kind");
    const size_t cnt = kind_count(ctx, kind);
    if ((size_t)n != cnt) return fail(ctx, "parameter count mismatch");
    if (!cnt) return 0;
    HXC(cudaSetDevice(ctx->device));
    // page-locked caller memory is copied directly; other memory goes through
    // the runtime's pinned staging buffer
    cudaPointerAttributes pa{};
    const bool pinned = cudaPointerGetAttributes(&pa, values) == cudaSuccess && pa.type == cudaMemoryTypeHost;
    if (!pinned) (void)cudaGetLastError();
    const double* src = values;
    if (!pinned) {
        HXC(ctx->pin.ensure(cnt * sizeof(double)));
        HXC(cudaStreamSynchronize(ctx->st));  // the pinned staging buffer may still be in flight
        memcpy(ctx->pin.p, values, cnt * sizeof(double));
        src = static_cast<const double*>(ctx->pin.p);
    }
    double* stage = ctx->stage_dev.p;
    HXC(cudaMemcpyAsync(stage, src, cnt * sizeof(double), cudaMemcpyHostToDevice, ctx->st));
    HXC(hx::launch_scatter(stage, ctx->kmap[kind].p, hx_kind_ptr(ctx, kind), (int)cnt, ctx->st));
    HXC(cudaStreamSynchronize(ctx->st));
    return 0;
}

int hx_get_param(hx_ctx* ctx, int kind, double* values, int n) {
    if (!ctx || !values) return fail(ctx, "null argument");
    if (!ctx->loaded) return fail(ctx, "no group loaded");
    if (kind < 0 || kind >= HX_P_COUNT) return fail(ctx, "bad parameter kind");
    const size_t cnt = kind_count(ctx, kind);
    if ((size_t)n != cnt) return fail(ctx, "parameter count mismatch");
    if (!cnt) return 0;
    HXC(cudaSetDevice(ctx->device));
    HXC(hx::launch_gather(hx_kind_ptr(ctx, kind), ctx->kmap[kind].p, ctx->stage_dev.p, (int)cnt, ctx->st));
    HXC(cudaMemcpyAsync(values, ctx->stage_dev.p, cnt * sizeof(double), cudaMemcpyDeviceToHost, ctx->st));
    HXC(cudaStreamSynchronize(ctx->st));
    return 0;
}

}  // extern "C"

// ---------------------------------------------------------------- capture / backward internals
int hx_setup_probes(hx_ctx* ctx, int nprobe, const int* probe_nodes) {
    if (nprobe < 0 || (nprobe > 0 && !probe_nodes)) return fail(ctx, "bad probe list");
    const hx::Plan& P = ctx->P;
    std::vector<int> key(probe_nodes, probe_nodes + nprobe);
    if (key == ctx->probe_key && ctx->pr_off.p) return 0;
    // cell slot of every GPU node
    const int nslot = (int)P.cs_node0.size();
    std::vector<int> node_slot(P.nnode, -1);
    for (int p = 0; p < P.npack; p++)
        for (int s = P.pack_slot_off[p]; s < P.pack_slot_off[p + 1]; s++)
            for (int l = P.cs_node0[s]; l < P.cs_node0[s] + P.cs_nnode[s]; l++) node_slot[P.pack_node_off[p] + l] = s;
    // per slot, sorted by (pack-local node, probe index): a node's probes form
    // one run, summed in probe order by one thread in the backward
    std::vector<std::vector<std::pair<int, int>>> per(nslot);
    for (int q = 0; q < nprobe; q++) {
        int r = probe_nodes[q];
        if (r < 0 || r >= P.nnode) return fail(ctx, "probe node out of range");
        int gi = P.ref2gpu[r];
        int pk = (int)(std::upper_bound(P.pack_node_off.begin(), P.pack_node_off.end(), gi) - P.pack_node_off.begin()) - 1;
        if (node_slot[gi] < 0) return fail(ctx, "probe node outside every cell slot");
        per[node_slot[gi]].push_back({gi - P.pack_node_off[pk], q});
    }
    std::vector<int> off(nslot + 1, 0), loc, slot;
    for (int s = 0; s < nslot; s++) {
        std::stable_sort(per[s].begin(), per[s].end(),
                         [](const std::pair<int, int>& x, const std::pair<int, int>& y) { return x.first < y.first; });
        for (auto& pr : per[s]) {
            loc.push_back(pr.first);
            slot.push_back(pr.second);
        }
        off[s + 1] = (int)loc.size();
    }
    if (loc.empty()) {
        loc.push_back(0);
        slot.push_back(0);
    }
    HXC(ctx->pr_off.upload(off, ctx->st));
    HXC(ctx->pr_local.upload(loc, ctx->st));
    HXC(ctx->pr_slot.upload(slot, ctx->st));
    ctx->probe_key = key;
    ctx->nprobe = nprobe;
    return 0;
}

hx::DevProbe hx_probe_view(hx_ctx* c) {
    hx::DevProbe p;
    p.slot_off = c->pr_off.p;
    p.local = c->pr_local.p;
    p.slot = c->pr_slot.p;
    p.nprobe = c->nprobe;
    return p;
}

int hx_setup_time(hx_ctx* ctx, int nstep) {
    // t accumulates in half steps exactly as Simulate::fadvance_cpu does
    // (simulate.cpp:417 and :774); IClamp sees the mid-step value.
    if (ctx->tmid_steps == nstep && ctx->tmid.p) return 0;
    std::vector<double> tm(std::max(nstep, 1)), ts(std::max(nstep, 1));
    double t = 0.0;
    for (int k = 0; k < nstep; k++) {
        ts[k] = t;
        t += 0.5 * ctx->dt;
        tm[k] = t;
        t += 0.5 * ctx->dt;
    }
    HXC(ctx->tmid.upload(tm, ctx->st));
    HXC(ctx->tstart.upload(ts, ctx->st));
    HXC(cudaStreamSynchronize(ctx->st));  // the source vector is pageable and goes out of scope
    ctx->tmid_steps = nstep;
    return 0;
}

static int plan_tape(hx_ctx* ctx, int nstep) {
    const size_t nn = ctx->P.nnode, nls = (size_t)ctx->lib_nst;
    const size_t per_step = (4 * nn + nls) * sizeof(double);  // v, m, h, n, library states
    size_t budget = ctx->tape_budget;
    if (!budget) {
        size_t fr = 0, tot = 0;
        HXC(cudaMemGetInfo(&fr, &tot));
        budget = (size_t)(0.6 * (double)(fr + 4 * ctx->tv.n * sizeof(double)));
    }
    const size_t full = per_step * (size_t)(nstep + 1);
    if (full <= budget) {
        ctx->full_tape = true;
        ctx->seg = nstep;
        ctx->nseg = 1;
        HXC(ctx->tv.ensure(nn * (size_t)(nstep + 1)));
        HXC(ctx->tm.ensure(nn * (size_t)(nstep + 1)));
        HXC(ctx->th.ensure(nn * (size_t)(nstep + 1)));
        HXC(ctx->tn.ensure(nn * (size_t)(nstep + 1)));
        if (ctx->lib) HXC(ctx->lib_tape.ensure(nls * (size_t)(nstep + 1)));
        return 0;
    }
    // checkpointed: segments of K steps; (K+1) tape rows + one checkpoint per segment within budget
    size_t K = (size_t)std::sqrt((double)nstep);
    if (K < 1) K = 1;
    while (K > 1 && (K + 1 + ((size_t)nstep + K - 1) / K) * per_step > budget) K /= 2;
    if ((K + 1 + ((size_t)nstep + K - 1) / K) * per_step > budget)
        return fail(ctx, "device memory too small for even a one-step tape");
    ctx->full_tape = false;
    ctx->seg = (int)K;
    ctx->nseg = (int)(((size_t)nstep + K - 1) / K);
    HXC(ctx->tv.ensure(nn * (K + 1)));
    HXC(ctx->tm.ensure(nn * (K + 1)));
    HXC(ctx->th.ensure(nn * (K + 1)));
    HXC(ctx->tn.ensure(nn * (K + 1)));
    HXC(ctx->ck.ensure(4 * nn * (size_t)ctx->nseg));
    if (ctx->lib) {
        HXC(ctx->lib_tape.ensure(nls * (K + 1)));
        HXC(ctx->lib_ck.ensure(nls * (size_t)ctx->nseg));
    }
    return 0;
}

static hx::DevState state_view(hx_ctx* c) { return hx::DevState{c->sv.p, c->sm.p, c->sh.p, c->sn.p}; }

static int copy_ck(hx_ctx* ctx, int s, bool save) {
    const size_t nn = ctx->P.nnode;
    double* base = ctx->ck.p + 4 * nn * (size_t)s;
    double* st[4] = {ctx->sv.p, ctx->sm.p, ctx->sh.p, ctx->sn.p};
    for (int k = 0; k < 4; k++) {
        if (save)
            HXC(cudaMemcpyAsync(base + k * nn, st[k], nn * 8, cudaMemcpyDeviceToDevice, ctx->st));
        else
            HXC(cudaMemcpyAsync(st[k], base + k * nn, nn * 8, cudaMemcpyDeviceToDevice, ctx->st));
    }
    if (ctx->lib && ctx->lib_nst) {
        const size_t nls = (size_t)ctx->lib_nst;
        double* lb = ctx->lib_ck.p + nls * (size_t)s;
        if (save)
            HXC(cudaMemcpyAsync(lb, ctx->lib_st.p, nls * 8, cudaMemcpyDeviceToDevice, ctx->st));
        else
            HXC(cudaMemcpyAsync(ctx->lib_st.p, lb, nls * 8, cudaMemcpyDeviceToDevice, ctx->st));
    }
    return 0;
}

int hx_kev_mark(hx_ctx* ctx, cudaStream_t st) {
    if (ctx->kev_n >= (int)ctx->kev.size()) {
        cudaEvent_t e = nullptr;
        HXC(cudaEventCreate(&e));
        ctx->kev.push_back(e);
    }
    HXC(cudaEventRecord(ctx->kev[ctx->kev_n], st));
    ctx->kev_n++;
    return 0;
}

// plain or split-cell kernels (the split ones reset their barrier state per launch)
static cudaError_t fwd_launch(hx_ctx* ctx, const hx::DevState& S, const hx::DevTape& T, int write_tape,
                              const hx::DevProbe& PV, double* trace, int k0, int k1) {
    if (!ctx->split) {
        if (!ctx->lib) return hx::launch_fwd(ctx->G, S, T, write_tape, PV, trace, ctx->tmid.p, k0, k1, ctx->st);
        hx::DevLib Lv = ctx->L;
        Lv.tape = ctx->lib_tape.p;
        return hx::launch_fwd(ctx->G, S, T, write_tape, PV, trace, ctx->tmid.p, k0, k1, ctx->st, nullptr, &Lv);
    }
    cudaError_t e = cudaMemsetAsync(ctx->split_bar.p, 0, 2 * sizeof(unsigned), ctx->st);
    if (e != cudaSuccess) return e;
    return hx::launch_split_fwd(ctx->G, S, T, write_tape, PV, trace, ctx->tmid.p, k0, k1, ctx->X, ctx->st);
}

static cudaError_t bwd_launch(hx_ctx* ctx, const hx::DevTape& T, const hx::DevAdj& A, const hx::DevGrad& GR,
                              const hx::DevProbe& PV, const double* dLdv, int k_hi, int k_lo) {
    if (!ctx->split) {
        if (!ctx->lib) return hx::launch_bwd(ctx->G, T, A, GR, PV, dLdv, ctx->tmid.p, k_hi, k_lo, ctx->st);
        hx::DevLib Lv = ctx->L;
        Lv.tape = ctx->lib_tape.p;
        return hx::launch_bwd(ctx->G, T, A, GR, PV, dLdv, ctx->tmid.p, k_hi, k_lo, ctx->st, nullptr, &Lv);
    }
    cudaError_t e = cudaMemsetAsync(ctx->split_bar.p, 0, 2 * sizeof(unsigned), ctx->st);
    if (e != cudaSuccess) return e;
    return hx::launch_split_bwd(ctx->G, T, A, GR, PV, dLdv, ctx->tmid.p, k_hi, k_lo, ctx->X, ctx->st);
}

// a split-cell grid barrier that gave up waiting (the results are then invalid)
static int check_split(hx_ctx* ctx) {
    if (!ctx->split) return 0;
    int err = 0;
    HXC(cudaMemcpyAsync(&err, ctx->split_err.p, 4, cudaMemcpyDeviceToHost, ctx->st));
    HXC(cudaStreamSynchronize(ctx->st));
    if (err) return fail(ctx, "a grid barrier of the split-cell kernels timed out");
    return 0;
}

static int run_forward(hx_ctx* ctx, int nstep, double v_init, int nprobe, const int* probe, double* trace_dev,
                       bool capture) {
    if (!ctx->loaded) return fail(ctx, "no group loaded");
    if (nstep < 0) return fail(ctx, "nstep must be >= 0");
    HXC(cudaSetDevice(ctx->device));
    if (hx_setup_probes(ctx, nprobe, probe)) return -1;
    if (hx_setup_time(ctx, nstep)) return -1;
    if (ctx->net) return hx_net_forward(ctx, nstep, v_init, trace_dev, capture);
    hx::DevTape T{nullptr, nullptr, nullptr, nullptr, 0};
    if (capture) {
        if (plan_tape(ctx, nstep)) return -1;
        T = hx::DevTape{ctx->tv.p, ctx->tm.p, ctx->th.p, ctx->tn.p, 0};
    }
    hx::DevState S = state_view(ctx);
    hx::DevProbe PV = hx_probe_view(ctx);
    HXC(hx::launch_init(ctx->G, S, v_init, ctx->st));
    if (ctx->lib) HXC(hx::launch_lib_init(ctx->L, (int)ctx->P.nnode, v_init, ctx->st));
    if (ctx->split) HXC(cudaMemsetAsync(ctx->split_err.p, 0, 4, ctx->st));
    HXC(cudaEventRecord(ctx->ev[0], ctx->st));
    int launches = 0;
    if (!capture || ctx->full_tape) {
        HXC(fwd_launch(ctx, S, T, capture ? 1 : 0, PV, trace_dev, 0, nstep));
        launches = 1;
    } else {
        for (int s = 0; s < ctx->nseg; s++) {
            if (copy_ck(ctx, s, true)) return -1;
            int k0 = s * ctx->seg, k1 = std::min(nstep, k0 + ctx->seg);
            HXC(fwd_launch(ctx, S, T, 0, PV, trace_dev, k0, k1));
            launches++;
        }
    }
    HXC(cudaEventRecord(ctx->ev[1], ctx->st));
    if (check_split(ctx)) return -1;
    ctx->launches[0] = launches;
    ctx->captured = capture;
    ctx->nstep = nstep;
    return 0;
}

static int run_backward(hx_ctx* ctx, const double* dLdv_dev) {
    if (!ctx->loaded) return fail(ctx, "no group loaded");
    if (!ctx->captured) return fail(ctx, "hx_backward needs a preceding hx_forward_capture");
    HXC(cudaSetDevice(ctx->device));
    if (ctx->net) return hx_net_backward(ctx, dLdv_dev);
    const size_t nn = ctx->P.nnode;
    HXC(cudaMemsetAsync(ctx->lv.p, 0, nn * 8, ctx->st));
    HXC(cudaMemsetAsync(ctx->lm.p, 0, nn * 8, ctx->st));
    HXC(cudaMemsetAsync(ctx->lh.p, 0, nn * 8, ctx->st));
    HXC(cudaMemsetAsync(ctx->ln.p, 0, nn * 8, ctx->st));
    HXC(cudaMemsetAsync(ctx->grad.p, 0, ctx->grad_off[HX_P_COUNT] * 8, ctx->st));
    if (ctx->lib && ctx->lib_nst) HXC(cudaMemsetAsync(ctx->lib_lam.p, 0, (size_t)ctx->lib_nst * 8, ctx->st));
    hx::DevAdj A{ctx->lv.p, ctx->lm.p, ctx->lh.p, ctx->ln.p};
    double* g = ctx->grad.p;
    hx::DevGrad GR{g + ctx->grad_off[HX_P_HH_GNABAR], g + ctx->grad_off[HX_P_HH_GKBAR], g + ctx->grad_off[HX_P_HH_GL],
                   g + ctx->grad_off[HX_P_HH_EL],     g + ctx->grad_off[HX_P_PAS_G],   g + ctx->grad_off[HX_P_PAS_E],
                   g + ctx->grad_off[HX_P_CM],        g + ctx->grad_off[HX_P_IC_AMP]};
    GR.skip = ctx->grad_skip;
    hx::DevProbe PV = hx_probe_view(ctx);
    hx::DevState S = state_view(ctx);
    if (ctx->split) HXC(cudaMemsetAsync(ctx->split_err.p, 0, 4, ctx->st));
    HXC(cudaEventRecord(ctx->ev[2], ctx->st));
    ctx->kev_n = 0;
    int launches = 0;
    if (ctx->full_tape) {
        hx::DevTape T{ctx->tv.p, ctx->tm.p, ctx->th.p, ctx->tn.p, 0};
        if (hx_kev_mark(ctx, ctx->st)) return -1;
        HXC(bwd_launch(ctx, T, A, GR, PV, dLdv_dev, ctx->nstep, 0));
        if (hx_kev_mark(ctx, ctx->st)) return -1;
        launches = 1;
    } else {
        for (int s = ctx->nseg - 1; s >= 0; s--) {
            int k0 = s * ctx->seg, k1 = std::min(ctx->nstep, k0 + ctx->seg);
            if (copy_ck(ctx, s, false)) return -1;
            hx::DevTape T{ctx->tv.p, ctx->tm.p, ctx->th.p, ctx->tn.p, k0};
            HXC(fwd_launch(ctx, S, T, 1, PV, nullptr, k0, k1));
            if (hx_kev_mark(ctx, ctx->st)) return -1;
            HXC(bwd_launch(ctx, T, A, GR, PV, dLdv_dev, k1, k0));
            if (hx_kev_mark(ctx, ctx->st)) return -1;
            launches += 2;
        }
    }
    HXC(cudaEventRecord(ctx->ev[3], ctx->st));
    if (check_split(ctx)) return -1;
    ctx->launches[1] = launches;
    return 0;
}

// per-kind gradients in reference instance order into device buffers
static int gather_grads_dev(hx_ctx* ctx, double* const* grads_dev) {
    if (!grads_dev) return 0;
    for (int k = 0; k < HX_P_COUNT; k++) {
        if (!grads_dev[k]) continue;
        const size_t cnt = kind_count(ctx, k);
        HXC(hx::launch_gather(ctx->grad.p + hx_grad_base(ctx, k), ctx->kmap[k].p, grads_dev[k], (int)cnt, ctx->st));
    }
    return 0;
}

extern "C" {

int hx_simulate(hx_ctx* ctx, int nstep, double v_init, int nprobe, const int* probe_nodes, double* trace) {
    if (!ctx) return -1;
    const size_t tn = (size_t)(nstep + 1) * (size_t)nprobe;
    HXC(ctx->trace_dev.ensure(tn));
    if (run_forward(ctx, nstep, v_init, nprobe, probe_nodes, ctx->trace_dev.p, false)) return -1;
    if (trace && tn) HXC(cudaMemcpyAsync(trace, ctx->trace_dev.p, tn * 8, cudaMemcpyDeviceToHost, ctx->st));
    HXC(cudaStreamSynchronize(ctx->st));
    return 0;
}

int hx_forward_capture(hx_ctx* ctx, int nstep, double v_init, int nprobe, const int* probe_nodes, double* trace) {
    if (!ctx) return -1;
    const size_t tn = (size_t)(nstep + 1) * (size_t)nprobe;
    HXC(ctx->trace_dev.ensure(tn));
    if (run_forward(ctx, nstep, v_init, nprobe, probe_nodes, ctx->trace_dev.p, true)) return -1;
    if (trace && tn) HXC(cudaMemcpyAsync(trace, ctx->trace_dev.p, tn * 8, cudaMemcpyDeviceToHost, ctx->st));
    HXC(cudaStreamSynchronize(ctx->st));
    return 0;
}

int hx_forward_capture_dev(hx_ctx* ctx, int nstep, double v_init, int nprobe, const int* probe_nodes,
                           double* trace_dev) {
    if (!ctx) return -1;
    return run_forward(ctx, nstep, v_init, nprobe, probe_nodes, trace_dev, true);
}

int hx_backward(hx_ctx* ctx, const double* dLdv, double* const* grads) {
    if (!ctx || !dLdv) return fail(ctx, "null argument");
    if (!ctx->captured) return fail(ctx, "hx_backward needs a preceding hx_forward_capture");
    const size_t tn = (size_t)(ctx->nstep + 1) * (size_t)ctx->nprobe;
    HXC(ctx->dLdv_dev.ensure(tn));
    if (tn) HXC(cudaMemcpyAsync(ctx->dLdv_dev.p, dLdv, tn * 8, cudaMemcpyHostToDevice, ctx->st));
    if (run_backward(ctx, ctx->dLdv_dev.p)) return -1;
    if (grads) {
        for (int k = 0; k < HX_P_COUNT; k++) {
            if (!grads[k]) continue;
            const size_t cnt = kind_count(ctx, k);
            if (!cnt) continue;
            double* sd = ctx->stage_dev.p + ctx->grad_off[k];
            HXC(hx::launch_gather(ctx->grad.p + hx_grad_base(ctx, k), ctx->kmap[k].p, sd, (int)cnt, ctx->st));
            HXC(cudaMemcpyAsync(grads[k], sd, cnt * 8, cudaMemcpyDeviceToHost, ctx->st));
        }
    }
    HXC(cudaStreamSynchronize(ctx->st));
    return 0;
}

int hx_backward_dev(hx_ctx* ctx, const double* dLdv_dev, double* const* grads_dev) {
    if (!ctx || !dLdv_dev) return fail(ctx, "null argument");
    if (run_backward(ctx, dLdv_dev)) return -1;
    return gather_grads_dev(ctx, grads_dev);
}

int hx_reduce_grads_f32(hx_ctx* ctx, int n, const int* kind, const int* index, const int32_t* dest,
                        const float* scale, float* out, int n_out) {
    if (!ctx || n < 0 || n_out < 0 || (n && (!kind || !index || !dest || !scale)) || (n_out && !out))
        return fail(ctx, "bad argument");
    if (!ctx->captured) return fail(ctx, "hx_reduce_grads_f32 needs a preceding backward");
    HXC(cudaSetDevice(ctx->device));
    std::vector<int> cnt(n_out + 1, 0);
    for (int e = 0; e < n; e++) {
        if (dest[e] < 0 || dest[e] >= n_out) return fail(ctx, "dest out of range");
        if (kind[e] < 0 || kind[e] >= HX_P_COUNT) return fail(ctx, "bad kind");
        if (index[e] < 0 || (size_t)index[e] >= kind_count(ctx, kind[e])) return fail(ctx, "index out of range");
        cnt[dest[e] + 1]++;
    }
    for (int c = 0; c < n_out; c++) cnt[c + 1] += cnt[c];
    // entries grouped by destination column, stable in input order; each entry
    // points at (offset of its kind) + (device slot of its reference instance)
    std::vector<int> flat(std::max(n, 1)), fill(cnt.begin(), cnt.end() - 1);
    std::vector<float> sc(std::max(n, 1));
    for (int e = 0; e < n; e++) {
        const int pos = fill[dest[e]]++;
        flat[pos] = (int)hx_grad_base(ctx, kind[e]) + ctx->kmap_h[kind[e]][index[e]];
        sc[pos] = scale[e];
    }
    HXC(ctx->red_off.upload(cnt, ctx->st));
    HXC(ctx->red_flat.upload(flat, ctx->st));
    HXC(ctx->red_scale.upload(sc, ctx->st));
    HXC(ctx->red_out.ensure(n_out));
    HXC(hx::launch_reduce_cols(ctx->grad.p, ctx->red_off.p, ctx->red_flat.p, ctx->red_scale.p, ctx->red_out.p, n_out,
                               ctx->st));
    if (n_out) HXC(cudaMemcpyAsync(out, ctx->red_out.p, (size_t)n_out * 4, cudaMemcpyDeviceToHost, ctx->st));
    HXC(cudaStreamSynchronize(ctx->st));
    return 0;
}

int hx_simulate_and_adjoint_into(hx_ctx* ctx, const float* dLtdv, int nstep, int n_output, const int32_t* poutput,
                                 int N, float* dw_out_n, float* dx, int n_param, const int* kind, const int* index,
                                 const int32_t* dest, const float* scale, double v_init, double grad_scale,
                                 double grad_l2norm_threshold, int clip_strategy) {
    if (!ctx || nstep < 0 || n_output < 0 || N < 0 || n_param < 0 || (n_output && (!dLtdv || !poutput)) ||
        (N && !dw_out_n))
        return fail(ctx, "bad argument");
    if (dx) return fail(ctx, "input gradients (dx) are not produced by the exact adjoint entry; pass NULL");
    if (clip_strategy != 0 && !(grad_l2norm_threshold > 0.0)) return fail(ctx, "invalid grad_l2norm_threshold");
    std::vector<int> probes(poutput, poutput + n_output);
    if (hx_forward_capture(ctx, nstep, v_init, n_output, probes.data(), nullptr)) return -1;
    // dL/d(trace): row 0 (the initial state) carries no loss; row t+1 of the
    // trace is row t of dLtdv
    std::vector<double> dl((size_t)(nstep + 1) * (size_t)n_output, 0.0);
    for (size_t e = 0; e < (size_t)nstep * (size_t)n_output; e++) dl[(size_t)n_output + e] = (double)dLtdv[e];
    if (hx_backward(ctx, dl.data(), nullptr)) return -1;
    if (hx_reduce_grads_f32(ctx, n_param, kind, index, dest, scale, dw_out_n, N)) return -1;
    double ss = 0.0;
    for (int c = 0; c < N; c++) {
        dw_out_n[c] = (float)((double)dw_out_n[c] * grad_scale);
        ss += (double)dw_out_n[c] * (double)dw_out_n[c];
    }
    const double l2 = std::sqrt(ss);
    if (clip_strategy != 0 && std::isfinite(l2) && l2 > grad_l2norm_threshold) {
        const double f = grad_l2norm_threshold / l2;
        for (int c = 0; c < N; c++) dw_out_n[c] = (float)((double)dw_out_n[c] * f);
    }
    return 0;
}

int hx_mse_loss_grad_dev(hx_ctx* ctx, const double* trace_dev, const double* target_dev, int nrow, int ncol,
                         double* dLdv_dev, double* loss_dev) {
    if (!ctx || !trace_dev || !target_dev || !dLdv_dev || !loss_dev || nrow < 1 || ncol < 0)
        return fail(ctx, "bad argument");
    HXC(cudaSetDevice(ctx->device));
    HXC(ctx->mse_partial.ensure(hx::kMsePartials));
    HXC(hx::launch_mse(trace_dev, target_dev, dLdv_dev, ctx->mse_partial.p, loss_dev, nrow, ncol, ctx->st));
    return 0;
}

int hx_rcp_nz_dev(const double* x_dev, double* y_dev, int n, void* stream) {
    if ((n > 0 && (!x_dev || !y_dev)) || n < 0) return -1;
    if (hx::launch_rcp_nz(x_dev, y_dev, n, (cudaStream_t)stream) != cudaSuccess) return -3;
    return 0;
}

int hx_last_kernel_ms(hx_ctx* ctx, int which, double* ms, int* launches) {
    if (!ctx || which < 0 || which > 2) return -1;
    if (which == 2) {  // the reverse kernel's launches alone
        double sum = 0.0;
        if (ctx->kev_n >= 2) HXC(cudaEventSynchronize(ctx->kev[ctx->kev_n - 1]));
        for (int i = 0; i + 1 < ctx->kev_n; i += 2) {
            float f = 0.f;
            HXC(cudaEventElapsedTime(&f, ctx->kev[i], ctx->kev[i + 1]));
            sum += f;
        }
        if (ms) *ms = sum;
        if (launches) *launches = ctx->kev_n / 2;
        return 0;
    }
    HXC(cudaEventSynchronize(ctx->ev[which * 2 + 1]));
    float f = 0.f;
    HXC(cudaEventElapsedTime(&f, ctx->ev[which * 2], ctx->ev[which * 2 + 1]));
    if (ms) *ms = f;
    if (launches) *launches = ctx->launches[which];
    return 0;
}

}  // extern "C"

// ---------------------------------------------------------------- optimizer
static AdamOpt* get_opt(hx_ctx* ctx, int id) {
    if (!ctx || id < 0 || id >= (int)ctx->opts.size() || !ctx->opts[id]) return nullptr;
    return ctx->opts[id];
}

extern "C" {

int hx_opt_create_adam(hx_ctx* ctx, double beta1, double beta2, double eps) {
    if (!ctx) return -1;
    if (!ctx->loaded) return fail(ctx, "no group loaded");
    if (!(beta1 >= 0 && beta1 < 1) || !(beta2 >= 0 && beta2 < 1) || !(eps > 0)) return fail(ctx, "bad Adam hyperparameters");
    AdamOpt* o = new AdamOpt();
    o->beta1 = beta1;
    o->beta2 = beta2;
    o->eps = eps;
    ctx->opts.push_back(o);
    return (int)ctx->opts.size() - 1;
}

int hx_opt_add_params(hx_ctx* ctx, int opt, int n, const int* kind, const int* index, double impedance) {
    AdamOpt* o = get_opt(ctx, opt);
    if (!o) return fail(ctx, "bad optimizer id");
    if (n <= 0 || !kind || !index) return fail(ctx, "empty parameter list");
    if (!(impedance > 0)) return fail(ctx, "impedance must be positive");
    HXC(cudaSetDevice(ctx->device));
    std::vector<int> kv(n), sv(n), fv(n);
    for (int i = 0; i < n; i++) {
        if (kind[i] < 0 || kind[i] >= HX_P_COUNT) return fail(ctx, "bad parameter kind");
        if (index[i] < 0 || (size_t)index[i] >= kind_count(ctx, kind[i])) return fail(ctx, "parameter index out of range");
        kv[i] = kind[i];
        sv[i] = ctx->kmap_h[kind[i]][index[i]];
        fv[i] = (int)hx_grad_base(ctx, kind[i]) + sv[i];
    }
    o->kind_h = kv;
    o->ref_h.assign(index, index + n);
    o->n = n;
    o->impedance = impedance;
    o->step = 0;
    HXC(o->kind.upload(kv, ctx->st));
    HXC(o->slot.upload(sv, ctx->st));
    HXC(o->flat.upload(fv, ctx->st));
    HXC(o->grad.ensure(n));
    HXC(o->m.ensure(n));
    HXC(o->v.ensure(n));
    HXC(o->f32.ensure(n));
    HXC(cudaMemsetAsync(o->grad.p, 0, n * 8, ctx->st));
    HXC(cudaMemsetAsync(o->m.p, 0, n * 8, ctx->st));
    HXC(cudaMemsetAsync(o->v.p, 0, n * 8, ctx->st));
    HXC(cudaStreamSynchronize(ctx->st));
    return 0;
}

int hx_opt_set_grads_f32(hx_ctx* ctx, int opt, const float* grads, int n) {
    AdamOpt* o = get_opt(ctx, opt);
    if (!o || !grads) return fail(ctx, "bad argument");
    if (n != o->n) return fail(ctx, "gradient count mismatch");
    HXC(cudaSetDevice(ctx->device));
    HXC(cudaMemcpyAsync(o->f32.p, grads, (size_t)n * 4, cudaMemcpyHostToDevice, ctx->st));
    HXC(hx::launch_f32_to_f64(o->f32.p, o->grad.p, n, ctx->st));
    HXC(cudaStreamSynchronize(ctx->st));
    return 0;
}

int hx_opt_grads_from_backward(hx_ctx* ctx, int opt, double scale) {
    AdamOpt* o = get_opt(ctx, opt);
    if (!o) return fail(ctx, "bad optimizer id");
    if (!ctx->captured) return fail(ctx, "no backward to take gradients from");
    HXC(cudaSetDevice(ctx->device));
    HXC(hx::launch_take_scaled(ctx->grad.p, o->flat.p, o->grad.p, o->n, scale, ctx->st));
    return 0;
}

int hx_opt_grad_buffer(hx_ctx* ctx, int opt, double** dev_ptr, int* n) {
    AdamOpt* o = get_opt(ctx, opt);
    if (!o || !dev_ptr || !n) return fail(ctx, "bad argument");
    *dev_ptr = o->grad.p;
    *n = o->n;
    return 0;
}

int hx_opt_set_allreduce(hx_ctx* ctx, int opt, hx_allreduce_fn fn, void* user) {
    AdamOpt* o = get_opt(ctx, opt);
    if (!o) return fail(ctx, "bad optimizer id");
    o->allreduce = fn;
    o->allreduce_user = user;
    return 0;
}

int hx_opt_step(hx_ctx* ctx, int opt, double lr, double inv_record_steps) {
    AdamOpt* o = get_opt(ctx, opt);
    if (!o) return fail(ctx, "bad optimizer id");
    HXC(cudaSetDevice(ctx->device));
    // data-parallel replicas: sum the slot gradients over ranks on the launch
    // stream, ordered after the kernels that wrote them and before Adam
    if (o->allreduce && o->allreduce(o->allreduce_user, o->grad.p, o->n, (void*)ctx->st) != 0)
        return fail(ctx, "gradient all-reduce callback failed");
    o->step++;
    const double bc1 = std::pow(o->beta1, (double)o->step);
    const double bc2 = std::pow(o->beta2, (double)o->step);
    HXC(hx::launch_adam(ctx->prm_ptrs.p, o->kind.p, o->slot.p, o->grad.p, o->m.p, o->v.p, o->n, lr,
                        o->impedance, inv_record_steps, o->beta1, o->beta2, o->eps, bc1, bc2, ctx->st));
    return 0;
}

int hx_opt_get_adam_state(hx_ctx* ctx, int opt, long long* step, double* m, double* v, int n, double* hyper3) {
    AdamOpt* o = get_opt(ctx, opt);
    if (!o) return fail(ctx, "bad optimizer id");
    if (n != o->n) return fail(ctx, "state size mismatch");
    HXC(cudaSetDevice(ctx->device));
    if (step) *step = o->step;
    if (m) HXC(cudaMemcpyAsync(m, o->m.p, (size_t)n * 8, cudaMemcpyDeviceToHost, ctx->st));
    if (v) HXC(cudaMemcpyAsync(v, o->v.p, (size_t)n * 8, cudaMemcpyDeviceToHost, ctx->st));
    HXC(cudaStreamSynchronize(ctx->st));
    if (hyper3) {
        hyper3[0] = o->beta1;
        hyper3[1] = o->beta2;
        hyper3[2] = o->eps;
    }
    return 0;
}

int hx_opt_set_adam_state(hx_ctx* ctx, int opt, long long step, const double* m, const double* v, int n,
                          const double* hyper3) {
    AdamOpt* o = get_opt(ctx, opt);
    if (!o || !m || !v) return fail(ctx, "bad argument");
    if (n != o->n) return fail(ctx, "state size mismatch");
    if (step < 0) return fail(ctx, "negative step count");
    HXC(cudaSetDevice(ctx->device));
    o->step = step;
    HXC(cudaMemcpyAsync(o->m.p, m, (size_t)n * 8, cudaMemcpyHostToDevice, ctx->st));
    HXC(cudaMemcpyAsync(o->v.p, v, (size_t)n * 8, cudaMemcpyHostToDevice, ctx->st));
    HXC(cudaStreamSynchronize(ctx->st));
    if (hyper3) {
        o->beta1 = hyper3[0];
        o->beta2 = hyper3[1];
        o->eps = hyper3[2];
    }
    return 0;
}

int hx_opt_reset(hx_ctx* ctx, int opt) {
    AdamOpt* o = get_opt(ctx, opt);
    if (!o) return fail(ctx, "bad optimizer id");
    HXC(cudaSetDevice(ctx->device));
    o->step = 0;
    if (o->n) {
        HXC(cudaMemsetAsync(o->m.p, 0, (size_t)o->n * 8, ctx->st));
        HXC(cudaMemsetAsync(o->v.p, 0, (size_t)o->n * 8, ctx->st));
        HXC(cudaMemsetAsync(o->grad.p, 0, (size_t)o->n * 8, ctx->st));
    }
    HXC(cudaStreamSynchronize(ctx->st));
    return 0;
}

}  // extern "C"
