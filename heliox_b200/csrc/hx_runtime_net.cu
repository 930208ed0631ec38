// hx_runtime_net.cu -- network groups: synapses, spikes, NetStims, gaps and
// graded synapses (the kNet instantiation of the step kernels).
//
// Forward of an event network: windows of W steps, W no longer than the
// shortest NetCon delay (in steps), so that every event produced inside a
// window is delivered in a later one.  After each window the window's spikes
// are appended to the spike log, optionally all-gathered across ranks through
// the caller's exchange hook, and routed into per-step event buckets.  NetStim
// trains do not depend on any voltage: they are generated on the host once
// per forward length (hx_netstim.cpp) and routed before the first window.
// Groups coupled by gap junctions or graded synapses exchange partner
// voltages every step through a ping-pong buffer: a window is one
// cooperative launch with a grid barrier per step when every pack can be
// co-resident, else one launch per step.  Library mechanisms may sit in
// network groups (the kNet + kLib instantiations).
//
// Backward: the event schedule of the forward is held fixed; the reverse
// sweep reads the synapse states after each step's deliveries from the tape
// and adds the weight gradient of every delivery.  Checkpointed segments are
// replayed without detection (events come from the buckets).
#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "heliox_b200.h"
#include "hx_ctx.hpp"
#include "hx_kernels.hpp"
#include "hx_netstim.hpp"

#define HXC(call)                                                                                       \
    do {                                                                                                \
        cudaError_t _e = (call);                                                                        \
        if (_e != cudaSuccess) return hx_fail(ctx, std::string(#call) + ": " + cudaGetErrorString(_e)); \
    } while (0)

namespace {

// instance order of one network mechanism on the GPU: by GPU node, then the
// reference order (ExpSyn before Exp2Syn for synapses)
struct Ord {
    int gnode, kord, ref;
    bool operator<(const Ord& o) const {
        if (gnode != o.gnode) return gnode < o.gnode;
        if (kord != o.kord) return kord < o.kord;
        return ref < o.ref;
    }
};

std::vector<int> csr_by_node(const std::vector<Ord>& v, int nn) {
    std::vector<int> off(nn + 1, 0);
    for (const Ord& o : v) off[o.gnode + 1]++;
    for (int i = 0; i < nn; i++) off[i + 1] += off[i];
    return off;
}

int window_from_delay(double dmin, double dt) {
    // smallest delivery lag (steps) of a delay: t_j + d <= t_k + dt/2 first holds
    // near k - j = (d - dt/2)/dt; one step of margin absorbs the rounding of t
    const double lag = std::floor((dmin - 0.5 * dt) / dt) - 1.0;
    return lag < 1.0 ? 1 : (int)std::min(lag, 1.0e6);
}

}  // namespace

constexpr int kFreeWindow = 256;

int hx_net_load(hx_ctx* ctx, const hx_group_desc* d) {
    const hx::Plan& P = ctx->P;
    cudaStream_t st = ctx->st;
    const int nn = P.nnode;
    ctx->nexp = std::max(d->nexpsyn, 0);
    ctx->nexp2 = std::max(d->nexp2syn, 0);
    ctx->nsyn = ctx->nexp + ctx->nexp2;
    ctx->nstim = std::max(d->nnetstim, 0);
    ctx->nhg = std::max(d->nhalfgap, 0);
    ctx->ngj_lr = std::max(d->ngapj, 0);
    ctx->ngnp = std::max(d->ngapnp, 0);
    ctx->ngj = ctx->ngj_lr + ctx->ngnp;
    ctx->ngr = std::max(d->ngraded, 0);
    ctx->gid_base = d->gid_base;
    ctx->nsrc_cells = d->nsrc_cells > 0 ? d->nsrc_cells : d->ncell;
    ctx->nsrc = ctx->nsrc_cells + ctx->nstim;
    ctx->coupled = ctx->nhg || ctx->ngj || ctx->ngr;
    ctx->net = ctx->nsyn || ctx->nstim || ctx->coupled || d->ps_thresh;
    ctx->ns_steps = -1;
    ctx->N = hx::DevNet{};
    for (int k = HX_P_EXPSYN_W; k < HX_P_COUNT; k++) {
        ctx->kmap_h[k].assign(1, 0);
    }
    if (!ctx->net) {
        for (int k = HX_P_EXPSYN_W; k < HX_P_COUNT; k++) HXC(ctx->kmap[k].upload(ctx->kmap_h[k], st));
        return 0;
    }
    if (ctx->gid_base < 0 || ctx->gid_base + d->ncell > ctx->nsrc_cells)
        return hx_fail(ctx, "gid_base + ncell exceeds nsrc_cells");
    auto bad_node = [&](const int* a, int n) {
        for (int i = 0; i < n; i++)
            if (a[i] < 0 || a[i] >= nn) return true;
        return false;
    };
    if (bad_node(d->expsyn_node, ctx->nexp) || bad_node(d->exp2syn_node, ctx->nexp2) ||
        bad_node(d->hg_node, ctx->nhg) || bad_node(d->hg_src, ctx->nhg) || bad_node(d->gj_node, ctx->ngj_lr) ||
        bad_node(d->gj_pre, ctx->ngj_lr) || bad_node(d->gn_node, ctx->ngnp) || bad_node(d->gn_src, ctx->ngnp) ||
        bad_node(d->gr_node, ctx->ngr) || bad_node(d->gr_pre, ctx->ngr))
        return hx_fail(ctx, "network node index out of range");
    // ---- exponential synapses
    std::vector<Ord> so;
    so.reserve(ctx->nsyn);
    double dmin = 1e300;
    for (int kord = 0; kord < 2; kord++) {
        const int n = kord ? ctx->nexp2 : ctx->nexp;
        const int* node = kord ? d->exp2syn_node : d->expsyn_node;
        const int* src = kord ? d->exp2syn_src : d->expsyn_src;
        const double* dl = kord ? d->exp2syn_delay : d->expsyn_delay;
        const double* t2 = kord ? d->exp2syn_tau2 : d->expsyn_tau;
        for (int i = 0; i < n; i++) {
            if (src[i] < 0 || src[i] >= ctx->nsrc) return hx_fail(ctx, "NetCon source out of range");
            if (!(dl[i] >= d->dt)) return hx_fail(ctx, "NetCon delays must be at least dt");
            if (!(t2[i] > 0)) return hx_fail(ctx, "synapse time constants must be positive");
            dmin = std::min(dmin, dl[i]);
            so.push_back(Ord{P.ref2gpu[node[i]], kord, i});
        }
    }
    std::sort(so.begin(), so.end());
    const int ns = ctx->nsyn;
    std::vector<int> kind(std::max(ns, 1), 0);
    std::vector<double> e(std::max(ns, 1), 0.0), w(std::max(ns, 1), 0.0), dl(std::max(ns, 1), 0.0),
        t1(std::max(ns, 1), 0.0), t2(std::max(ns, 1), 0.0);
    ctx->kmap_h[HX_P_EXPSYN_W].assign(std::max(ctx->nexp, 1), 0);
    ctx->kmap_h[HX_P_EXP2SYN_W].assign(std::max(ctx->nexp2, 1), 0);
    std::vector<std::vector<int>> by_src(ctx->nsrc);
    for (int j = 0; j < ns; j++) {
        const Ord& o = so[j];
        kind[j] = o.kord;
        if (o.kord == 0) {
            e[j] = d->expsyn_e[o.ref];
            w[j] = d->expsyn_weight[o.ref];
            dl[j] = d->expsyn_delay[o.ref];
            t2[j] = d->expsyn_tau[o.ref];
            ctx->kmap_h[HX_P_EXPSYN_W][o.ref] = j;
            by_src[d->expsyn_src[o.ref]].push_back(j);
        } else {
            e[j] = d->exp2syn_e[o.ref];
            w[j] = d->exp2syn_weight[o.ref];
            dl[j] = d->exp2syn_delay[o.ref];
            t1[j] = d->exp2syn_tau1[o.ref];
            t2[j] = d->exp2syn_tau2[o.ref];
            ctx->kmap_h[HX_P_EXP2SYN_W][o.ref] = j;
            by_src[d->exp2syn_src[o.ref]].push_back(j);
        }
    }
    ctx->kmap_h[HX_P_EXPSYN_E] = ctx->kmap_h[HX_P_EXPSYN_W];
    ctx->kmap_h[HX_P_EXP2SYN_E] = ctx->kmap_h[HX_P_EXP2SYN_W];
    std::vector<int> nso = csr_by_node(so, nn), pso(P.npack + 1);
    for (int p = 0; p <= P.npack; p++) pso[p] = nso[P.pack_node_off[p]];
    // node and pack of every synapse (delivery by the node's owner thread,
    // events bucketed per pack)
    std::vector<int> snode(std::max(ns, 1), 0), spack(std::max(ns, 1), 0);
    for (int j = 0; j < ns; j++) snode[j] = so[j].gnode;
    for (int p = 0; p < P.npack; p++)
        for (int j = pso[p]; j < pso[p + 1]; j++) spack[j] = p;
    std::vector<int> soff(ctx->nsrc + 1, 0), slist;
    for (int s = 0; s < ctx->nsrc; s++) {
        soff[s + 1] = soff[s] + (int)by_src[s].size();
        slist.insert(slist.end(), by_src[s].begin(), by_src[s].end());
    }
    if (slist.empty()) slist.push_back(0);
    HXC(ctx->node_syn_off.upload(nso, st));
    HXC(ctx->pack_syn_off.upload(pso, st));
    HXC(ctx->syn_node.upload(snode, st));
    HXC(ctx->syn_pack.upload(spack, st));
    HXC(ctx->syn_kind.upload(kind, st));
    HXC(ctx->prm[HX_P_EXPSYN_E].upload(e, st));
    HXC(ctx->prm[HX_P_EXPSYN_W].upload(w, st));
    HXC(ctx->syn_delay.upload(dl, st));
    HXC(ctx->syn_tau1.upload(t1, st));
    HXC(ctx->syn_tau2.upload(t2, st));
    HXC(ctx->src_off.upload(soff, st));
    HXC(ctx->src_syn.upload(slist, st));
    for (auto* b : {&ctx->syn_cA, &ctx->syn_cB, &ctx->syn_fA, &ctx->syn_fB, &ctx->sA, &ctx->sB, &ctx->lA, &ctx->lB})
        HXC(b->ensure(std::max(ns, 1)));
    HXC(hx::launch_syn_prep(ns, ctx->syn_kind.p, ctx->syn_tau1.p, ctx->syn_tau2.p, d->dt, ctx->syn_cA.p,
                            ctx->syn_cB.p, ctx->syn_fA.p, ctx->syn_fB.p, st));
    // ---- PreSyn per cell slot (root node of the cell)
    const int ncs = (int)P.cs_node0.size();
    std::vector<int> psn(std::max(ncs, 1), -1), gid(std::max(ncs, 1), 0);
    std::vector<double> thr(std::max(ncs, 1), 10.0);
    for (int p = 0; p < P.npack; p++)
        for (int s = P.pack_slot_off[p]; s < P.pack_slot_off[p + 1]; s++) {
            const int cell = P.cs_cell[s];
            psn[s] = P.ref2gpu[cell] - P.pack_node_off[p];
            gid[s] = ctx->gid_base + cell;
            thr[s] = d->ps_thresh ? d->ps_thresh[cell] : 10.0;
        }
    HXC(ctx->cs_ps_node.upload(psn, st));
    HXC(ctx->cs_gid.upload(gid, st));
    HXC(ctx->cs_ps_thr.upload(thr, st));
    HXC(ctx->cs_ps_flag.ensure(std::max(ncs, 1)));
    // ---- gaps and graded synapses
    auto order = [&](int n, const int* node) {
        std::vector<Ord> v(n);
        for (int i = 0; i < n; i++) v[i] = Ord{P.ref2gpu[node[i]], 0, i};
        std::sort(v.begin(), v.end());
        return v;
    };
    std::vector<Ord> ho = order(ctx->nhg, d->hg_node), ro = order(ctx->ngr, d->gr_node);
    // gapjunction_lr and gapjunction_noptr instances in one array: by node,
    // then mechanism (the reference's current order on a node), then instance
    std::vector<Ord> jo;
    jo.reserve(ctx->ngj);
    for (int i = 0; i < ctx->ngj_lr; i++) jo.push_back(Ord{P.ref2gpu[d->gj_node[i]], 0, i});
    for (int i = 0; i < ctx->ngnp; i++) jo.push_back(Ord{P.ref2gpu[d->gn_node[i]], 1, i});
    std::sort(jo.begin(), jo.end());
    auto gather_d = [](const std::vector<Ord>& v, const double* a) {
        std::vector<double> out(std::max<size_t>(v.size(), 1), 0.0);
        for (size_t i = 0; i < v.size(); i++) out[i] = a[v[i].ref];
        return out;
    };
    auto partner = [&](const std::vector<Ord>& v, const int* a) {
        std::vector<int> out(std::max<size_t>(v.size(), 1), 0);
        for (size_t i = 0; i < v.size(); i++) out[i] = P.ref2gpu[a[v[i].ref]];
        return out;
    };
    auto kmap_of = [](const std::vector<Ord>& v) {
        std::vector<int> m(std::max<size_t>(v.size(), 1), 0);
        for (size_t i = 0; i < v.size(); i++) m[v[i].ref] = (int)i;
        return m;
    };
    HXC(ctx->node_hg_off.upload(csr_by_node(ho, nn), st));
    HXC(ctx->node_gj_off.upload(csr_by_node(jo, nn), st));
    HXC(ctx->node_gr_off.upload(csr_by_node(ro, nn), st));
    std::vector<int> hs = partner(ho, d->hg_src), rp = partner(ro, d->gr_pre);
    std::vector<int> jp(std::max<size_t>(jo.size(), 1), 0);
    std::vector<double> jg(std::max<size_t>(jo.size(), 1), 0.0), jw(std::max<size_t>(jo.size(), 1), 0.0);
    std::vector<int> jmap_lr(std::max(ctx->ngj_lr, 1), 0), jmap_np(std::max(ctx->ngnp, 1), 0);
    for (size_t q = 0; q < jo.size(); q++) {
        const int r = jo[q].ref;
        if (jo[q].kord == 0) {
            jp[q] = P.ref2gpu[d->gj_pre[r]];
            jg[q] = d->gj_g[r];
            jw[q] = d->gj_w[r];
            jmap_lr[r] = (int)q;
        } else {  // i = weight (v - vpre) is w (g (v - vpre)) with g = weight, w = 1, bit for bit
            jp[q] = P.ref2gpu[d->gn_src[r]];
            jg[q] = d->gn_weight[r];
            jw[q] = 1.0;
            jmap_np[r] = (int)q;
        }
    }
    HXC(ctx->hg_src.upload(hs, st));
    HXC(ctx->gj_pre.upload(jp, st));
    HXC(ctx->gr_pre.upload(rp, st));
    HXC(ctx->prm[HX_P_HALFGAP_G].upload(gather_d(ho, d->hg_g), st));
    HXC(ctx->prm[HX_P_GAPJ_G].upload(jg, st));
    HXC(ctx->prm[HX_P_GAPJ_W].upload(jw, st));
    HXC(ctx->prm[HX_P_GRADED_W].upload(gather_d(ro, d->gr_w), st));
    HXC(ctx->gr_delta.upload(gather_d(ro, d->gr_delta), st));
    HXC(ctx->gr_vth.upload(gather_d(ro, d->gr_vth), st));
    for (auto* b : {&ctx->gr_g, &ctx->gr_k, &ctx->gr_erev, &ctx->gr_s, &ctx->lS}) HXC(b->ensure(std::max(ctx->ngr, 1)));
    ctx->kmap_h[HX_P_HALFGAP_G] = kmap_of(ho);
    ctx->kmap_h[HX_P_GAPJ_G] = jmap_lr;
    ctx->kmap_h[HX_P_GAPJ_W] = jmap_lr;
    ctx->kmap_h[HX_P_GAPNP_W] = jmap_np;
    ctx->kmap_h[HX_P_GRADED_W] = kmap_of(ro);
    // incoming partner contributions per node: (kind << 28 | instance), kind-major
    {
        std::vector<std::vector<int>> in(nn);
        for (int i = 0; i < ctx->nhg; i++) in[hs[i]].push_back((0 << 28) | i);
        for (int i = 0; i < ctx->ngj; i++) in[jp[i]].push_back((1 << 28) | i);
        for (int i = 0; i < ctx->ngr; i++) in[rp[i]].push_back((2 << 28) | i);
        std::vector<int> off(nn + 1, 0), lst;
        for (int q = 0; q < nn; q++) {
            off[q + 1] = off[q] + (int)in[q].size();
            lst.insert(lst.end(), in[q].begin(), in[q].end());
        }
        if (lst.empty()) lst.push_back(0);
        HXC(ctx->node_in_off.upload(off, st));
        HXC(ctx->node_in.upload(lst, st));
    }
    const size_t nx = (size_t)ctx->nhg + ctx->ngj + ctx->ngr;
    if (ctx->coupled) {
        HXC(ctx->vbuf.ensure(2 * (size_t)nn));
        HXC(ctx->xbuf.ensure(2 * std::max<size_t>(nx, 1)));
    }
    for (int k = HX_P_EXPSYN_W; k < HX_P_COUNT; k++) HXC(ctx->kmap[k].upload(ctx->kmap_h[k], st));
    HXC(ctx->dev_err.ensure(1));
    HXC(ctx->win_n.ensure(1));
    HXC(ctx->log_n.ensure(1));
    // ---- NetStims (host generator input) and the window
    ctx->ns_interval.assign(d->ns_interval ? d->ns_interval : nullptr, d->ns_interval ? d->ns_interval + ctx->nstim : nullptr);
    ctx->ns_number.assign(d->ns_number ? d->ns_number : nullptr, d->ns_number ? d->ns_number + ctx->nstim : nullptr);
    ctx->ns_start.assign(d->ns_start ? d->ns_start : nullptr, d->ns_start ? d->ns_start + ctx->nstim : nullptr);
    ctx->ns_noise.assign(d->ns_noise ? d->ns_noise : nullptr, d->ns_noise ? d->ns_noise + ctx->nstim : nullptr);
    if (ctx->nstim && (ctx->ns_interval.size() != (size_t)ctx->nstim || ctx->ns_number.size() != (size_t)ctx->nstim ||
                       ctx->ns_start.size() != (size_t)ctx->nstim || ctx->ns_noise.size() != (size_t)ctx->nstim))
        return hx_fail(ctx, "NetStim table incomplete");
    ctx->ns_rng = d->netstim_rng;
    ctx->dmin = ns ? dmin : 0.0;
    // coupled groups without grid-synchronous launches take one step per
    // window (net_window); without events the window is free and kept at
    // kFreeWindow steps, so that checkpoint segments (multiples of the
    // window) can stay near sqrt(nstep)
    ctx->window = ns ? window_from_delay(dmin, d->dt) : kFreeWindow;
    ctx->ck_net_stride = 2 * (size_t)ns + (size_t)ctx->ngr;

    hx::DevNet& N = ctx->N;
    N.nsyn = ns;
    N.npack = P.npack;
    N.syn_node = ctx->syn_node.p;
    N.node_syn_off = ctx->node_syn_off.p;
    N.pack_syn_off = ctx->pack_syn_off.p;
    N.syn_e = ctx->prm[HX_P_EXPSYN_E].p;
    N.syn_w = ctx->prm[HX_P_EXPSYN_W].p;
    N.syn_cA = ctx->syn_cA.p;
    N.syn_cB = ctx->syn_cB.p;
    N.syn_fA = ctx->syn_fA.p;
    N.syn_fB = ctx->syn_fB.p;
    N.sA = ctx->sA.p;
    N.sB = ctx->sB.p;
    N.cs_ps_node = ctx->cs_ps_node.p;
    N.cs_gid = ctx->cs_gid.p;
    N.cs_ps_thr = ctx->cs_ps_thr.p;
    N.cs_ps_flag = ctx->cs_ps_flag.p;
    N.win_n = ctx->win_n.p;
    N.node_hg_off = ctx->node_hg_off.p;
    N.hg_src = ctx->hg_src.p;
    N.hg_g = ctx->prm[HX_P_HALFGAP_G].p;
    N.node_gj_off = ctx->node_gj_off.p;
    N.gj_pre = ctx->gj_pre.p;
    N.gj_g = ctx->prm[HX_P_GAPJ_G].p;
    N.gj_w = ctx->prm[HX_P_GAPJ_W].p;
    N.node_gr_off = ctx->node_gr_off.p;
    N.gr_pre = ctx->gr_pre.p;
    N.gr_w = ctx->prm[HX_P_GRADED_W].p;
    N.gr_g = ctx->gr_g.p;
    N.gr_k = ctx->gr_k.p;
    N.gr_erev = ctx->gr_erev.p;
    N.gr_delta = ctx->gr_delta.p;
    N.gr_vth = ctx->gr_vth.p;
    N.ngr = ctx->ngr;
    N.gr_s = ctx->gr_s.p;
    N.lS = ctx->lS.p;
    N.coupled = ctx->coupled ? 1 : 0;
    N.node_in_off = ctx->node_in_off.p;
    N.node_in = ctx->node_in.p;
    N.nhg = ctx->nhg;
    N.ngj = ctx->ngj;
    N.vbuf = ctx->vbuf.p;
    N.xbuf = ctx->xbuf.p;
    N.xstride = std::max<size_t>((size_t)ctx->nhg + ctx->ngj + ctx->ngr, 1);
    if (ctx->coupled) {
        HXC(ctx->gs_bar.ensure(2));
        HXC(ctx->gs_err.ensure(1));
        HXC(cudaMemsetAsync(ctx->gs_err.p, 0, 4, st));
    }
    N.gbar = ctx->gs_bar.p;
    N.gerr = ctx->gs_err.p;
    N.gspin = ctx->split_spin_limit;
    N.gsync = 0;  // set at load once the packs' co-residency is known
    return 0;
}

// ---------------------------------------------------------------- forward
static int net_window(const hx_ctx* c, int nstep) {
    int W = c->window_user > 0 ? c->window_user : c->window;
    if (c->coupled && !c->N.gsync) W = 1;
    return std::max(1, std::min(W, std::max(nstep, 1)));
}

// one checkpoint: v, m, h, n, then synapse A, B and graded s (library
// states in lib_ck)
static int net_ck(hx_ctx* ctx, int s, bool save, double* vsrc) {
    if (ctx->lib && ctx->lib_nst) {
        const size_t nls = (size_t)ctx->lib_nst;
        double* lb = ctx->lib_ck.p + nls * (size_t)s;
        if (save)
            HXC(cudaMemcpyAsync(lb, ctx->lib_st.p, nls * 8, cudaMemcpyDeviceToDevice, ctx->st));
        else
            HXC(cudaMemcpyAsync(ctx->lib_st.p, lb, nls * 8, cudaMemcpyDeviceToDevice, ctx->st));
    }
    const size_t nn = ctx->P.nnode;
    const size_t stride = 4 * nn + ctx->ck_net_stride;
    double* base = ctx->ck.p + stride * (size_t)s;
    double* st[7] = {vsrc, ctx->sm.p, ctx->sh.p, ctx->sn.p, ctx->sA.p, ctx->sB.p, ctx->gr_s.p};
    const size_t len[7] = {nn, nn, nn, nn, (size_t)ctx->nsyn, (size_t)ctx->nsyn, (size_t)ctx->ngr};
    size_t off = 0;
    for (int k = 0; k < 7; k++) {
        if (len[k]) {
            if (save)
                HXC(cudaMemcpyAsync(base + off, st[k], len[k] * 8, cudaMemcpyDeviceToDevice, ctx->st));
            else
                HXC(cudaMemcpyAsync(st[k], base + off, len[k] * 8, cudaMemcpyDeviceToDevice, ctx->st));
        }
        off += len[k];
    }
    return 0;
}

// W: the forward window; a free window (no synapses, no window set by the
// caller) follows the checkpoint segment instead
static int net_plan_tape(hx_ctx* ctx, int nstep, int& W) {
    const size_t nn = ctx->P.nnode, ns = ctx->nsyn, ng = ctx->ngr, nls = ctx->lib ? (size_t)ctx->lib_nst : 0;
    const size_t per_step = (4 * nn + 2 * ns + ng + nls) * sizeof(double);
    size_t budget = ctx->tape_budget;
    if (!budget) {
        size_t fr = 0, tot = 0;
        HXC(cudaMemGetInfo(&fr, &tot));
        budget = (size_t)(0.6 * (double)(fr + (4 * ctx->tv.n + 2 * ctx->tA.n + ctx->tS.n + ctx->ck.n) * sizeof(double)));
    }
    auto alloc = [&](size_t rows, size_t ckn) -> int {
        HXC(ctx->tv.ensure(nn * rows));
        HXC(ctx->tm.ensure(nn * rows));
        HXC(ctx->th.ensure(nn * rows));
        HXC(ctx->tn.ensure(nn * rows));
        HXC(ctx->tA.ensure(std::max<size_t>(ns * rows, 1)));
        HXC(ctx->tB.ensure(std::max<size_t>(ns * rows, 1)));
        HXC(ctx->tS.ensure(std::max<size_t>(ng * (rows + 1), 1)));
        if (nls) HXC(ctx->lib_tape.ensure(nls * rows));
        if (ckn) HXC(ctx->ck.ensure((4 * nn + ctx->ck_net_stride) * ckn));
        if (ckn && nls) HXC(ctx->lib_ck.ensure(nls * ckn));
        return 0;
    };
    if (per_step * (size_t)(nstep + 2) <= budget) {
        ctx->full_tape = true;
        ctx->seg = nstep;
        ctx->nseg = 1;
        return alloc((size_t)nstep + 1, 0);
    }
    // segments of K steps, K a multiple of the window
    // (ranks that exchange windows keep the one window they agreed on)
    const bool free_window = ctx->nsyn == 0 && ctx->window_user <= 0 && !(ctx->exchange && ctx->nranks > 1);
    if (free_window) W = 1;
    size_t K = (size_t)std::sqrt((double)nstep);
    K = std::max<size_t>(W, (K + W - 1) / W * W);
    while (K > (size_t)W && (K + 2 + ((size_t)nstep + K - 1) / K) * per_step > budget) K -= W;
    if (free_window) W = (int)K;
    if ((K + 2 + ((size_t)nstep + K - 1) / K) * per_step > budget)
        return hx_fail(ctx, "device memory too small for the network tape");
    ctx->full_tape = false;
    ctx->seg = (int)K;
    ctx->nseg = (int)(((size_t)nstep + K - 1) / K);
    return alloc(K + 1, (size_t)ctx->nseg);
}

static int net_netstim(hx_ctx* ctx, int nstep) {
    if (!ctx->nstim) {
        ctx->ns_count = 0;
        return 0;
    }
    if (ctx->ns_steps == nstep) return 0;
    std::vector<double> ts(std::max(nstep, 1));
    double t = 0.0;
    for (int k = 0; k < nstep; k++) {
        ts[k] = t;
        t += 0.5 * ctx->dt;
        t += 0.5 * ctx->dt;
    }
    hx::NetStimTable tab;
    tab.n = ctx->nstim;
    tab.interval = ctx->ns_interval.data();
    tab.number = ctx->ns_number.data();
    tab.start = ctx->ns_start.data();
    tab.noise = ctx->ns_noise.data();
    tab.rng_mode = ctx->ns_rng;
    std::vector<int> id, step;
    hx::netstim_trains(tab, ts, ctx->dt, nstep, id, step);
    std::vector<int2> spk(std::max<size_t>(id.size(), 1));
    for (size_t i = 0; i < id.size(); i++) spk[i] = make_int2(ctx->nsrc_cells + id[i], step[i]);
    HXC(ctx->ns_spk.upload(spk, ctx->st));
    HXC(cudaStreamSynchronize(ctx->st));
    ctx->ns_count = (int)id.size();
    ctx->ns_steps = nstep;
    return 0;
}

int hx_net_forward(hx_ctx* ctx, int nstep, double v_init, double* trace_dev, bool capture) {
    cudaStream_t st = ctx->st;
    const hx::Plan& P = ctx->P;
    const size_t nn = P.nnode;
    int W = net_window(ctx, nstep);
    const int ncell = (int)P.cs_node0.size();
    // Several ranks exchange window spikes: every rank takes the same
    // collective steps whatever happens locally.  A host-side failure on one
    // rank does not end its loop early (its peers would wait in the next
    // all-gather): it stops launching work, keeps exchanging (a send buffer
    // of padding), and reports the failure in the status word all ranks
    // all-gather after the last window; every rank then returns the same
    // outcome, and a bucket overflow anywhere reruns the forward on all ranks
    // with the largest bucket need.  Only a rank that cannot hold the
    // exchange buffers, or whose exchange itself fails, returns at once (the
    // process group's timeout then ends the peers' collective).
    const bool multi = ctx->exchange && ctx->nranks > 1;
    // window spike buffer: one rank alone holds its bound (a PreSyn fires at
    // most every other step); ranks that exchange send buffers of the agreed
    // size win_cap_cur (most windows carry far fewer spikes than the bound),
    // grown on every rank alike when one overflows
    int own_cap = 0;  // (W is final after the tape plan below)
    const size_t nbucket = (size_t)std::max(nstep, 1) * (size_t)std::max(P.npack, 1);  // (step, pack) event buckets
    if (multi) {
        HXC(ctx->st_send.ensure(2));
        HXC(ctx->st_recv.ensure(2 * (size_t)ctx->nranks));
    }
    HXC(ctx->win_max.ensure(1));
    auto setup = [&]() -> int {
        if (net_netstim(ctx, nstep)) return -1;
        if (capture && net_plan_tape(ctx, nstep, W)) return -1;
        ctx->log_cap = (int)std::min<long long>((long long)ncell * std::max(64, nstep / 20 + 1), 1LL << 26);
        HXC(ctx->spk_log.ensure(std::max(ctx->log_cap, 1)));
        if (ctx->ev_cap == 0) ctx->ev_cap = 16;
        HXC(ctx->ev_cnt.ensure(nbucket));
        return 0;
    };
    bool ok = setup() == 0;
    if (!ok && !multi) return -1;
    if (ctx->coupled && !ctx->N.gsync) W = 1;
    own_cap = ncell * ((W + 1) / 2) + 1;
    std::string local_err = ok ? std::string() : ctx->err;
    hx::DevProbe PV = hx_probe_view(ctx);
    const double half_dt = ctx->dt / 2;
    for (int attempt = 0; attempt < 6; attempt++) {
        ctx->win_cap = multi ? ctx->win_cap_cur : own_cap;
        HXC(ctx->win_send.ensure(ctx->win_cap));
        HXC(ctx->win_recv.ensure((size_t)ctx->win_cap * std::max(ctx->nranks, 1)));
        if (ok && ctx->ev_syn.ensure(nbucket * ctx->ev_cap) != cudaSuccess) {
            hx_fail(ctx, "event bucket allocation failed");
            if (!multi) return -1;
            ok = false;
            local_err = ctx->err;
        }
        auto init_attempt = [&]() -> int {
            HXC(cudaMemsetAsync(ctx->ev_cnt.p, 0, nbucket * 4, st));
            HXC(cudaMemsetAsync(ctx->dev_err.p, 0, 4, st));
            HXC(cudaMemsetAsync(ctx->win_max.p, 0, 4, st));
            HXC(cudaMemsetAsync(ctx->log_n.p, 0, 4, st));
            HXC(cudaMemsetAsync(ctx->cs_ps_flag.p, 0, (size_t)std::max(ncell, 1) * 4, st));
            if (ctx->N.gsync) HXC(cudaMemsetAsync(ctx->gs_err.p, 0, 4, st));
            double* v0 = ctx->coupled ? ctx->vbuf.p : ctx->sv.p;
            HXC(hx::launch_init(ctx->G, hx::DevState{v0, ctx->sm.p, ctx->sh.p, ctx->sn.p}, v_init, st));
            if (ctx->lib) HXC(hx::launch_lib_init(ctx->L, (int)nn, v_init, st));
            HXC(hx::launch_init_net(ctx->nsyn, ctx->sA.p, ctx->sB.p, ctx->ngr, ctx->prm[HX_P_GRADED_W].p,
                                    ctx->gr_vth.p, ctx->gr_delta.p, ctx->gr_g.p, ctx->gr_k.p, ctx->gr_erev.p,
                                    ctx->gr_s.p, v_init, st));
            if (attempt == 0) HXC(cudaEventRecord(ctx->ev[0], st));
            if (ctx->nsyn && ctx->ns_count)
                HXC(hx::launch_route(ctx->ns_spk.p, nullptr, ctx->ns_count, ctx->src_off.p, ctx->src_syn.p,
                                     ctx->nsrc, ctx->syn_delay.p, ctx->tstart.p, nstep, half_dt, 0, ctx->syn_pack.p,
                                     P.npack, ctx->ev_cnt.p, ctx->ev_syn.p, ctx->ev_cap, ctx->dev_err.p, st));
            return 0;
        };
        int launches = 0;
        // the window's compute: checkpoint, step kernel, spike log
        auto run_window = [&](int k0, int k1) -> int {
            double* vin = ctx->coupled ? ctx->vbuf.p + (size_t)(k0 & 1) * nn : ctx->sv.p;
            if (capture && !ctx->full_tape && k0 % ctx->seg == 0)
                if (net_ck(ctx, k0 / ctx->seg, true, vin)) return -1;
            HXC(cudaMemsetAsync(ctx->win_send.p, 0xFF, (size_t)ctx->win_cap * sizeof(int2), st));
            HXC(cudaMemsetAsync(ctx->win_n.p, 0, 4, st));
            hx::DevNet N = ctx->N;
            N.ev_cnt = ctx->ev_cnt.p;
            N.ev_syn = ctx->ev_syn.p;
            N.ev_cap = ctx->ev_cap;
            N.win_spk = ctx->win_send.p;
            N.win_cap = ctx->win_cap;
            N.detect = 1;
            N.vpeer = vin;
            N.vout = ctx->coupled ? ctx->vbuf.p + (size_t)((k0 + 1) & 1) * nn : nullptr;
            hx::DevTape T{nullptr, nullptr, nullptr, nullptr, 0};
            int write_tape = 0;
            if (capture && ctx->full_tape) {
                T = hx::DevTape{ctx->tv.p, ctx->tm.p, ctx->th.p, ctx->tn.p, 0};
                N.tA = ctx->tA.p;
                N.tB = ctx->tB.p;
                N.tS = ctx->tS.p;
                write_tape = 1;
            }
            if (N.gsync) {
                N.vout = ctx->vbuf.p + (size_t)(k1 & 1) * nn;  // stored by the last step
                HXC(cudaMemsetAsync(ctx->gs_bar.p, 0, 2 * sizeof(unsigned), st));
            }
            hx::DevState S{vin, ctx->sm.p, ctx->sh.p, ctx->sn.p};
            hx::DevLib Lv = ctx->L;
            Lv.tape = ctx->lib_tape.p;
            HXC(hx::launch_fwd(ctx->G, S, T, write_tape, PV, trace_dev, ctx->tmid.p, k0, k1, st, &N,
                               ctx->lib ? &Lv : nullptr));
            HXC(hx::launch_log_append(ctx->win_send.p, ctx->win_n.p, ctx->win_cap, ctx->spk_log.p, ctx->log_n.p,
                                      ctx->log_cap, ctx->dev_err.p, ctx->win_max.p, st));
            launches += 2;
            return 0;
        };
        auto route_window = [&](const int2* spk, const int* nspk, int nmax, int k1) -> int {
            HXC(hx::launch_route(spk, nspk, nmax, ctx->src_off.p, ctx->src_syn.p, ctx->nsrc, ctx->syn_delay.p,
                                 ctx->tstart.p, nstep, half_dt, k1, ctx->syn_pack.p, P.npack, ctx->ev_cnt.p,
                                 ctx->ev_syn.p, ctx->ev_cap, ctx->dev_err.p, st));
            launches++;
            return 0;
        };
        if (ok && init_attempt() != 0) {
            if (!multi) return -1;
            ok = false;
            local_err = ctx->err;
        }
        for (int k0 = 0; k0 < nstep; k0 += W) {
            const int k1 = std::min(nstep, k0 + W);
            if (ok && run_window(k0, k1) != 0) {
                if (!multi) return -1;
                ok = false;
                local_err = ctx->err;
            }
            if (multi) {
                if (!ok)  // stopped: keep the collective going with an empty window
                    cudaMemsetAsync(ctx->win_send.p, 0xFF, (size_t)ctx->win_cap * sizeof(int2), st);
                if (ctx->exchange(ctx->exchange_user, ctx->win_send.p, ctx->win_recv.p, ctx->win_cap, (void*)st) != 0)
                    return hx_fail(ctx, "spike exchange callback failed");
                if (ok && ctx->nsyn && route_window(ctx->win_recv.p, nullptr, ctx->win_cap * ctx->nranks, k1) != 0) {
                    ok = false;
                    local_err = ctx->err;
                }
            } else if (ctx->nsyn && k1 < nstep) {
                if (route_window(ctx->win_send.p, ctx->win_n.p, ctx->win_cap, k1) != 0) return -1;
            }
        }
        if (ok && ctx->coupled) {  // final voltages into the state vector
            HXC(cudaMemcpyAsync(ctx->sv.p, ctx->vbuf.p + (size_t)(nstep & 1) * nn, nn * 8, cudaMemcpyDeviceToDevice,
                                st));
        }
        int err = 0, need = 0, win_need = 0, bad_rank = -1;
        if (multi) {
            // every rank's (error bits, largest bucket count, largest window) after its last window
            if (ok && hx::launch_net_status(ctx->dev_err.p, ctx->ev_cnt.p, (int)nbucket, ctx->win_max.p, 0,
                                            ctx->st_send.p, st) != cudaSuccess) {
                ok = false;
                local_err = "status kernel launch failed";
            }
            if (!ok) {  // a stopped rank reports only that it stopped
                const int2 ab[2] = {make_int2(HX_XS_ABORT, 0), make_int2(0, 0)};
                cudaMemcpyAsync(ctx->st_send.p, ab, sizeof(ab), cudaMemcpyHostToDevice, st);
            }
            if (ctx->exchange(ctx->exchange_user, ctx->st_send.p, ctx->st_recv.p, 2, (void*)st) != 0)
                return hx_fail(ctx, "spike exchange callback failed (status)");
            std::vector<int2> all(2 * (size_t)ctx->nranks);
            HXC(cudaMemcpyAsync(all.data(), ctx->st_recv.p, all.size() * sizeof(int2), cudaMemcpyDeviceToHost, st));
            HXC(cudaEventRecord(ctx->ev[1], st));
            HXC(cudaStreamSynchronize(st));
            hx_exchange_merge_status(reinterpret_cast<const int*>(all.data()), ctx->nranks, &err, &need, &win_need,
                                     &bad_rank);
            if (err & HX_XS_ABORT)
                return hx_fail(ctx, local_err.empty()
                                        ? "rank " + std::to_string(bad_rank) + " failed in the multi-rank forward"
                                        : local_err);
        } else {
            HXC(cudaEventRecord(ctx->ev[1], st));
            HXC(cudaMemcpyAsync(&err, ctx->dev_err.p, 4, cudaMemcpyDeviceToHost, st));
            int gerr = 0;
            if (ctx->N.gsync) HXC(cudaMemcpyAsync(&gerr, ctx->gs_err.p, 4, cudaMemcpyDeviceToHost, st));
            HXC(cudaStreamSynchronize(st));
            if (gerr) return hx_fail(ctx, "a grid barrier of the coupled-network kernels timed out");
        }
        ctx->launches[0] = launches + (multi ? 1 : 0);
        if (err & HX_XS_LATE_EVENT)
            return hx_fail(ctx, "an event fell inside a simulated window (window longer than the delay)");
        if (err & HX_XS_WINDOW) {
            if (!multi) return hx_fail(ctx, "window spike buffer overflow");
            // the largest window over all ranks, so every rank grows alike
            ctx->win_cap_cur = std::max(ctx->win_cap_cur * 2, win_need + win_need / 4 + 8);
        }
        if (err & HX_XS_BUCKET) {
            if (!multi) {
                std::vector<int> cnt(nbucket);
                HXC(cudaMemcpy(cnt.data(), ctx->ev_cnt.p, cnt.size() * 4, cudaMemcpyDeviceToHost));
                need = *std::max_element(cnt.begin(), cnt.end());
            }
            // every rank takes the same (largest) need, so all rerun alike
            ctx->ev_cap = std::max(ctx->ev_cap * 2, need + need / 4 + 8);
        }
        if (err & (HX_XS_BUCKET | HX_XS_WINDOW))
            continue;  // the run depended on dropped events or spikes: run it again with room for all
        ctx->captured = capture;
        ctx->nstep = nstep;
        return 0;
    }
    return hx_fail(ctx, "event buckets or window buffers kept overflowing");
}

// ---------------------------------------------------------------- backward
int hx_net_backward(hx_ctx* ctx, const double* dLdv_dev) {
    cudaStream_t st = ctx->st;
    const size_t nn = ctx->P.nnode;
    const int nstep = ctx->nstep;
    const size_t nx = (size_t)ctx->nhg + ctx->ngj + ctx->ngr;
    for (DevBuf<double>* b : {&ctx->lv, &ctx->lm, &ctx->lh, &ctx->ln}) HXC(cudaMemsetAsync(b->p, 0, nn * 8, st));
    if (ctx->nsyn) {
        HXC(cudaMemsetAsync(ctx->lA.p, 0, (size_t)ctx->nsyn * 8, st));
        HXC(cudaMemsetAsync(ctx->lB.p, 0, (size_t)ctx->nsyn * 8, st));
    }
    if (ctx->ngr) HXC(cudaMemsetAsync(ctx->lS.p, 0, (size_t)ctx->ngr * 8, st));
    if (ctx->lib && ctx->lib_nst) HXC(cudaMemsetAsync(ctx->lib_lam.p, 0, (size_t)ctx->lib_nst * 8, st));
    hx::DevLib Lv = ctx->L;
    Lv.tape = ctx->lib_tape.p;
    const hx::DevLib* LP = ctx->lib ? &Lv : nullptr;
    if (ctx->coupled) HXC(cudaMemsetAsync(ctx->xbuf.p, 0, 2 * std::max<size_t>(nx, 1) * 8, st));
    const bool gsync = ctx->coupled && ctx->N.gsync;
    if (gsync) HXC(cudaMemsetAsync(ctx->gs_err.p, 0, 4, st));
    HXC(cudaMemsetAsync(ctx->grad.p, 0, ctx->grad_off[HX_P_COUNT] * 8, st));
    double* g = ctx->grad.p;
    hx::DevGrad GR{g + ctx->grad_off[HX_P_HH_GNABAR], g + ctx->grad_off[HX_P_HH_GKBAR], g + ctx->grad_off[HX_P_HH_GL],
                   g + ctx->grad_off[HX_P_HH_EL],     g + ctx->grad_off[HX_P_PAS_G],   g + ctx->grad_off[HX_P_PAS_E],
                   g + ctx->grad_off[HX_P_CM],        g + ctx->grad_off[HX_P_IC_AMP],  g + ctx->grad_off[HX_P_EXPSYN_W],
                   g + ctx->grad_off[HX_P_EXPSYN_E],  g + ctx->grad_off[HX_P_HALFGAP_G], g + ctx->grad_off[HX_P_GAPJ_G],
                   g + ctx->grad_off[HX_P_GAPJ_W],    g + ctx->grad_off[HX_P_GRADED_W]};
    GR.skip = ctx->grad_skip;
    hx::DevAdj A{ctx->lv.p, ctx->lm.p, ctx->lh.p, ctx->ln.p, ctx->lA.p, ctx->lB.p};
    hx::DevProbe PV = hx_probe_view(ctx);
    hx::DevNet N = ctx->N;
    N.ev_cnt = ctx->ev_cnt.p;
    N.ev_syn = ctx->ev_syn.p;
    N.ev_cap = ctx->ev_cap;
    N.detect = 0;
    N.tA = ctx->tA.p;
    N.tB = ctx->tB.p;
    N.tS = ctx->tS.p;
    double* xb = ctx->xbuf.p;
    const size_t xs = std::max<size_t>(nx, 1);
    auto set_x = [&](int k) {  // launch of step k reads parity (k+1), writes parity k
        double* in = xb + (size_t)((k + 1) & 1) * xs;
        double* out = xb + (size_t)(k & 1) * xs;
        N.x_hg_in = in;
        N.x_gj_in = in + ctx->nhg;
        N.x_gr_in = in + ctx->nhg + ctx->ngj;
        N.x_hg_out = out;
        N.x_gj_out = out + ctx->nhg;
        N.x_gr_out = out + ctx->nhg + ctx->ngj;
    };
    auto sweep = [&](int k_hi, int k_lo, const hx::DevTape& T) -> int {
        if (hx_kev_mark(ctx, st)) return -1;
        if (!ctx->coupled || gsync) {
            if (gsync) HXC(cudaMemsetAsync(ctx->gs_bar.p, 0, 2 * sizeof(unsigned), st));
            HXC(hx::launch_bwd(ctx->G, T, A, GR, PV, dLdv_dev, ctx->tmid.p, k_hi, k_lo, st, &N, LP));
        } else {
            for (int k = k_hi - 1; k >= k_lo; --k) {
                set_x(k);
                HXC(hx::launch_bwd(ctx->G, T, A, GR, PV, dLdv_dev, ctx->tmid.p, k + 1, k, st, &N, LP));
            }
        }
        if (hx_kev_mark(ctx, st)) return -1;
        return ctx->coupled && !gsync ? k_hi - k_lo : 1;
    };
    HXC(cudaEventRecord(ctx->ev[2], st));
    ctx->kev_n = 0;
    int launches = 0;
    if (ctx->full_tape) {
        hx::DevTape T{ctx->tv.p, ctx->tm.p, ctx->th.p, ctx->tn.p, 0};
        int r = sweep(nstep, 0, T);
        if (r < 0) return -1;
        launches += r;
    } else {
        for (int s = ctx->nseg - 1; s >= 0; s--) {
            const int k0 = s * ctx->seg, k1 = std::min(nstep, k0 + ctx->seg);
            hx::DevTape T{ctx->tv.p, ctx->tm.p, ctx->th.p, ctx->tn.p, k0};
            if (!ctx->coupled) {
                if (net_ck(ctx, s, false, ctx->sv.p)) return -1;
                hx::DevState S{ctx->sv.p, ctx->sm.p, ctx->sh.p, ctx->sn.p};
                HXC(hx::launch_fwd(ctx->G, S, T, 1, PV, nullptr, ctx->tmid.p, k0, k1, st, &N, LP));
                launches++;
            } else if (gsync) {  // the segment's recompute in one grid-synchronous launch
                double* vin = ctx->vbuf.p + (size_t)(k0 & 1) * nn;
                if (net_ck(ctx, s, false, vin)) return -1;
                hx::DevNet NF = N;
                NF.vpeer = vin;
                NF.vout = ctx->vbuf.p + (size_t)(k1 & 1) * nn;
                hx::DevState S{vin, ctx->sm.p, ctx->sh.p, ctx->sn.p};
                HXC(cudaMemsetAsync(ctx->gs_bar.p, 0, 2 * sizeof(unsigned), st));
                HXC(hx::launch_fwd(ctx->G, S, T, 1, PV, nullptr, ctx->tmid.p, k0, k1, st, &NF, LP));
                launches++;
            } else {
                if (net_ck(ctx, s, false, ctx->vbuf.p + (size_t)(k0 & 1) * nn)) return -1;
                for (int k = k0; k < k1; k++) {
                    hx::DevNet NF = N;
                    NF.vpeer = ctx->vbuf.p + (size_t)(k & 1) * nn;
                    NF.vout = ctx->vbuf.p + (size_t)((k + 1) & 1) * nn;
                    hx::DevState S{const_cast<double*>(NF.vpeer), ctx->sm.p, ctx->sh.p, ctx->sn.p};
                    HXC(hx::launch_fwd(ctx->G, S, T, 1, PV, nullptr, ctx->tmid.p, k, k + 1, st, &NF, LP));
                    launches++;
                }
            }
            int r = sweep(k1, k0, T);
            if (r < 0) return -1;
            launches += r;
        }
    }
    HXC(cudaEventRecord(ctx->ev[3], st));
    ctx->launches[1] = launches;
    if (gsync) {
        int gerr = 0;
        HXC(cudaMemcpyAsync(&gerr, ctx->gs_err.p, 4, cudaMemcpyDeviceToHost, st));
        HXC(cudaStreamSynchronize(st));
        if (gerr) return hx_fail(ctx, "a grid barrier of the coupled-network kernels timed out");
    }
    return 0;
}

// ---------------------------------------------------------------- C ABI
extern "C" {

int hx_get_spikes(hx_ctx* ctx, int cap, int* gid, double* t, int* n) {
    if (!ctx || !n || (cap > 0 && (!gid || !t))) return hx_fail(ctx, "bad argument");
    if (!ctx->net) return hx_fail(ctx, "the loaded group has no spike detection");
    HXC(cudaSetDevice(ctx->device));
    int total = 0;
    HXC(cudaMemcpyAsync(&total, ctx->log_n.p, 4, cudaMemcpyDeviceToHost, ctx->st));
    HXC(cudaStreamSynchronize(ctx->st));
    *n = total;
    const int k = std::min(std::min(total, ctx->log_cap), std::max(cap, 0));
    if (k <= 0) return 0;
    std::vector<int2> buf(k);
    HXC(cudaMemcpy(buf.data(), ctx->spk_log.p, (size_t)k * sizeof(int2), cudaMemcpyDeviceToHost));
    // step -> time: the start-of-step time accumulated in half steps
    int maxstep = 0;
    for (const int2& b : buf) maxstep = std::max(maxstep, b.y);
    std::vector<double> ts(maxstep + 1);
    double tt = 0.0;
    for (int s = 0; s <= maxstep; s++) {
        ts[s] = tt;
        tt += 0.5 * ctx->dt;
        tt += 0.5 * ctx->dt;
    }
    for (int i = 0; i < k; i++) {
        gid[i] = buf[i].x;
        t[i] = ts[buf[i].y];
    }
    return 0;
}

int hx_netstim_trains(const hx_group_desc* d, int nstep, int cap, int* id, int* step, int* n) {
    if (!d || nstep < 0 || !n || (cap > 0 && (!id || !step))) return -1;
    if (d->nnetstim > 0 && (!d->ns_interval || !d->ns_number || !d->ns_start || !d->ns_noise)) return -1;
    std::vector<double> ts(std::max(nstep, 1));
    double t = 0.0;
    for (int k = 0; k < nstep; k++) {
        ts[k] = t;
        t += 0.5 * d->dt;
        t += 0.5 * d->dt;
    }
    hx::NetStimTable tab;
    tab.n = std::max(d->nnetstim, 0);
    tab.interval = d->ns_interval;
    tab.number = d->ns_number;
    tab.start = d->ns_start;
    tab.noise = d->ns_noise;
    tab.rng_mode = d->netstim_rng;
    std::vector<int> ids, steps;
    hx::netstim_trains(tab, ts, d->dt, nstep, ids, steps);
    *n = (int)ids.size();
    for (int i = 0; i < std::min(*n, cap); i++) {
        id[i] = ids[i];
        step[i] = steps[i];
    }
    return 0;
}

int hx_set_exchange(hx_ctx* ctx, hx_exchange_fn exchange, void* user, int nranks, int cap_entries) {
    if (!ctx) return -1;
    if (nranks < 1 || cap_entries < 0) return hx_fail(ctx, "nranks must be >= 1, cap_entries >= 0");
    ctx->exchange = exchange;
    ctx->exchange_user = user;
    ctx->nranks = exchange ? nranks : 1;
    ctx->win_cap_user = exchange ? cap_entries : 0;
    ctx->win_cap_cur = exchange ? (cap_entries > 0 ? cap_entries : 1024) : 0;
    ctx->ev_cap = 0;
    return 0;
}

int hx_exchange_merge_status(const int* status, int nranks, int* flags, int* need, int* win_need, int* first_rank) {
    if (!status || nranks < 1 || !flags || !need || !win_need || !first_rank) return -1;
    int f = 0, nd = 0, wn = 0, hard = -1, soft = -1;
    for (int r = 0; r < nranks; r++) {
        const int* q = status + 4 * r;
        const int b = q[0];
        f |= b;
        nd = std::max(nd, q[1]);
        wn = std::max(wn, q[2]);
        if ((b & ~(HX_XS_BUCKET | HX_XS_WINDOW)) && hard < 0) hard = r;
        if ((b & (HX_XS_BUCKET | HX_XS_WINDOW)) && soft < 0) soft = r;
    }
    *flags = f;
    *need = nd;
    *win_need = wn;
    *first_rank = hard >= 0 ? hard : soft;
    return 0;
}

int hx_set_window(hx_ctx* ctx, int steps) {
    if (!ctx) return -1;
    if (steps < 0) return hx_fail(ctx, "window must be >= 0");
    ctx->window_user = steps;
    return 0;
}

int hx_get_window(hx_ctx* ctx, int* steps) {
    if (!ctx || !steps) return -1;
    if (!ctx->loaded) return hx_fail(ctx, "no group loaded");
    *steps = ctx->window_user > 0 ? ctx->window_user : ctx->window;
    if (ctx->coupled && !ctx->N.gsync) *steps = 1;
    return 0;
}

}  // extern "C"
