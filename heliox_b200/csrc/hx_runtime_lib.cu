// hx_runtime_lib.cu -- host side of the library mechanisms (hx_lib.cuh):
// the per-node entry tables in GPU order, the parameter kinds
// HX_P_CADYN_GAMMA .. HX_P_UNC2_G, and the device arrays of DevLib.
//
// The reference keeps one instance table per mechanism type
// (MechTemp::reg_node_indices / read_data_from_coredat,
// src/mech/mech_template.cuh:192-368) and reaches an instance's ion through
// the node (var_struct.cuh:376-470).  Here the instances of all library types
// on one node are one run of entries, in type order, so that the thread that
// owns the node walks them in the order the reference's type loop applies
// them.
#include <cmath>
#include <map>
#include <string>
#include <vector>

#include "hx_ctx.hpp"
#include "hx_lib.cuh"

namespace {

int fail(hx_ctx* c, const std::string& m) { return hx_fail(c, m); }

#define HXC(call)                                                                                    \
    do {                                                                                             \
        cudaError_t _e = (call);                                                                     \
        if (_e != cudaSuccess) return fail(ctx, std::string(#call) + ": " + cudaGetErrorString(_e)); \
    } while (0)

const char* kTypeName[HX_LIB_NTYPE] = {"na_ion", "k_ion", "ca_ion",  "CaDynamics_E2", "Ca_HVA",
                                       "Ca_LVAst", "Im",   "K_Pst",   "K_Tst",         "NaTg",
                                       "Nap_Et2", "SK_E2", "SKv3_1", "hd_la",         "km_la",
                                       "kca_la", "it2_la", "kdr_la", "sca_la",        "Ca",
                                       "shl1_lr", "kvs1_lr", "irk_lr", "egl36_lr",    "shk1_lr",
                                       "egl2_lr", "cca1_lr", "egl19_lr", "unc2_lr", "kcnl_lr", "nca_lr",
                                       "kqt3_lr", "cainternm_lr", "shl1", "kvs1", "irk", "egl36", "shk1",
                                       "egl2", "cca1", "egl19", "unc2"};

// worm-mech channels (src/mech/worm-mech/<name>.cu): the device runs them
// through their worm-lr sibling's gates with the fixed vector 1, -80 (the
// hard-coded reversal potential; 60 for the calcium ones), 0, then the kinetics constants of their
// setparames (kvs1: its GLOBALs), in the worm-lr GLOBAL order
const double kShl1K[18] = {11.2, 14.1, -33.1, 8.3, 13.8, -17.5, 12.9, -3.7, 6.5,
                           1.9, 539.2, -28.2, 4.9, 27.3, 8422.0, -37.7, 6.4, 118.9};  // shl1.cu setparames
const double kIrkK[8] = {-82.0, 13.0, 17.1, -17.8, 20.3, -43.4, 11.2, 3.8};            // irk.cu
const double kEgl36K[5] = {63.0, 28.5, 355.0, 63.0, 13.0};                             // egl36.cu
const double kShk1K[11] = {20.4, 7.7, -7.0, 5.8, 26.6, -33.7, 15.8, -33.7, 15.4, 2.0, 1400.0};  // shk1.cu
const double kEgl2K[6] = {-6.9, 14.9, 1845.8, -122.6, 13.8, 1517.74};                  // egl2.cu
const double kCca1K[12] = {-43.32, 7.6, -58.0, 7.0, 40.0, -62.5, -12.6, 0.7, 280.0, -60.7, 8.5, 19.8};  // cca1.cu
const double kEgl19K[25] = {5.6, 7.5, 24.9, 12.0, -20.5, 8.1, 1.43, 0.14, 5.96, 0.60, 2.9, 5.2, 6.0,
                            1.9, 1.4, 30.0, 2.3, 0.4, 44.6, -23.0, 5.0, 36.4, 28.7, 3.7, 43.1};  // egl19.cu
const double kUnc2K[15] = {-12.2, 4.0, -52.5, 5.6, 1.5, -8.2, 9.1, 15.4, 0.1, 83.8, 52.9, -3.5, 72.1, 23.9, -3.6};  // unc2.cu
bool worm_mech(int t) { return t >= HX_LIB_SHL1 && t <= HX_LIB_UNC2; }
// the calcium ones: erev 60 mV (gb ... (v - 60)), current into ica
bool worm_mech_ca(int t) { return t >= HX_LIB_CCA1 && t <= HX_LIB_UNC2; }

// columns of a type's hx_lib_table rows (trainable first, then fixed); hd_la's
// GLOBALs q10 and qtl enter the device's fixed parameters as one factor
int desc_cols(int t) {
    if (t == HX_LIB_HD_LA) return 11;
    if (worm_mech(t)) return t == HX_LIB_KVS1 ? 13 : 1;
    return hx::lib::ntrain(t) + hx::lib::nfix(t);
}

// ions a type needs on its node: bit 0 Na, 1 K, 2 Ca
int ions_needed(int t) {
    switch (t) {
        case HX_LIB_NATG:
        case HX_LIB_NAP_ET2:
            return 1;
        case HX_LIB_IM:
        case HX_LIB_K_PST:
        case HX_LIB_K_TST:
        case HX_LIB_SKV3_1:
        case HX_LIB_KM_LA:
        case HX_LIB_KDR_LA:
        case HX_LIB_SHL1_LR:
        case HX_LIB_KVS1_LR:
        case HX_LIB_IRK_LR:
        case HX_LIB_EGL36_LR:
        case HX_LIB_SHK1_LR:
        case HX_LIB_EGL2_LR:
        case HX_LIB_KQT3_LR:
        case HX_LIB_SHL1:
        case HX_LIB_KVS1:
        case HX_LIB_IRK:
        case HX_LIB_EGL36:
        case HX_LIB_SHK1:
        case HX_LIB_EGL2:
            return 2;
        case HX_LIB_SK_E2:
        case HX_LIB_KCA_LA:
        case HX_LIB_KCNL_LR:
            return 2 | 4;
        case HX_LIB_NCA_LR:
            return 1;
        case HX_LIB_IT2_LA:
        case HX_LIB_SCA_LA:
        case HX_LIB_CA:
        case HX_LIB_CCA1_LR:
        case HX_LIB_EGL19_LR:
        case HX_LIB_UNC2_LR:
        case HX_LIB_CCA1:
        case HX_LIB_EGL19:
        case HX_LIB_UNC2:
            return 4;
        case HX_LIB_CADYN:
        case HX_LIB_CAINTERNM_LR:
        case HX_LIB_CA_HVA:
        case HX_LIB_CA_LVAST:
            return 4;
    }
    return 0;
}

}  // namespace

// one past the last library kind (the kinds after it are network kinds again)
static constexpr int kLibKindEnd = HX_P_UNC2_G + 1;
static_assert(kLibKindEnd - HX_P_CADYN_GAMMA == hx::kLibKinds, "library kinds");

int hx_lib_type_of_kind(int kind) {
    if (kind >= HX_P_CADYN_GAMMA && kind <= HX_P_CADYN_MINCAI) return HX_LIB_CADYN;
    if (kind >= HX_P_CA_HVA_G && kind < kLibKindEnd) return kind - HX_P_CA_HVA_G + HX_LIB_CA_HVA;
    return -1;
}

int hx_lib_load(hx_ctx* ctx, const hx_group_desc* desc) {
    namespace L = hx::lib;
    ctx->lib = false;
    ctx->lib_nst = 0;
    ctx->L = hx::DevLib{};
    for (int t = 0; t < HX_LIB_NTYPE; t++) ctx->lib_n[t] = 0;
    const hx_lib_desc* D = desc->lib;
    bool any = false;
    if (D)
        for (int t = 0; t < HX_LIB_NTYPE; t++) {
            if (D->t[t].n < 0) return fail(ctx, std::string("negative count of library table ") + kTypeName[t]);
            if (D->t[t].n > 0 && (!D->t[t].node || !D->t[t].par))
                return fail(ctx, std::string("library table ") + kTypeName[t] + " needs node and par arrays");
            if (D->t[t].n >= (1 << 24)) return fail(ctx, std::string("too many instances of ") + kTypeName[t]);
            any = any || D->t[t].n > 0;
        }
    cudaStream_t st = ctx->st;
    if (!any) {
        for (int k = HX_P_CADYN_GAMMA; k < kLibKindEnd; k++) {
            ctx->kmap_h[k].assign(1, 0);
            HXC(ctx->kmap[k].upload(ctx->kmap_h[k], st));
            HXC(ctx->prm[k].ensure(1));
        }
        return 0;
    }
    const hx::Plan& P = ctx->P;
    const int nn = P.nnode;
    // reference node -> instance of each type
    std::vector<std::vector<int>> at(HX_LIB_NTYPE, std::vector<int>(nn, -1));
    for (int t = 0; t < HX_LIB_NTYPE; t++) {
        const hx_lib_table& T = D->t[t];
        for (int j = 0; j < T.n; j++) {
            const int r = T.node[j];
            if (r < 0 || r >= nn) return fail(ctx, std::string(kTypeName[t]) + ": node index out of range");
            if (j > 0 && r <= T.node[j - 1])
                return fail(ctx, std::string(kTypeName[t]) + ": nodes must be sorted, one instance per node");
            at[t][r] = j;
        }
        ctx->lib_n[t] = T.n;
    }
    for (int t = HX_LIB_CADYN; t < HX_LIB_NTYPE; t++) {
        const int need = ions_needed(t);
        for (int j = 0; j < D->t[t].n; j++) {
            const int r = D->t[t].node[j];
            if (((need & 1) && at[HX_LIB_NA_ION][r] < 0) || ((need & 2) && at[HX_LIB_K_ION][r] < 0) ||
                ((need & 4) && at[HX_LIB_CA_ION][r] < 0))
                return fail(ctx, std::string(kTypeName[t]) + " on node " + std::to_string(r) +
                                     " needs its ion (na_ion / k_ion / ca_ion) on that node");
        }
    }
    for (int j = 0; j < D->t[HX_LIB_CA_ION].n; j++)
        if (!(D->t[HX_LIB_CA_ION].par[4 * j] > 0.0)) return fail(ctx, "ca_ion: cai must be positive");
    for (int j = 0; j < D->t[HX_LIB_CAINTERNM_LR].n; j++)
        if (at[HX_LIB_CADYN][D->t[HX_LIB_CAINTERNM_LR].node[j]] >= 0)
            return fail(ctx, "CaDynamics_E2 and cainternm_lr on one node: one calcium dynamics per node");
    // entries in GPU node order, types ascending on a node
    std::vector<int> node_off(nn + 1, 0), ent, ent_st, ent_fix;
    std::vector<unsigned long long> mask(std::max(nn, 1), 0);
    std::vector<double> fix;
    std::vector<std::map<std::vector<double>, int>> fix_of(HX_LIB_NTYPE);
    std::vector<int> inst(HX_LIB_NTYPE, 0);
    std::vector<std::vector<double>> prm(hx::kLibKinds);
    for (int k = 0; k < hx::kLibKinds; k++) prm[k].assign(1, 0.0);
    for (int k = HX_P_CADYN_GAMMA; k < kLibKindEnd; k++)
        ctx->kmap_h[k].assign(std::max(ctx->lib_n[hx_lib_type_of_kind(k)], 1), 0);
    int nst = 0;
    for (int gi = 0; gi < nn; gi++) {
        const int r = P.gpu2ref[gi];
        for (int t = 0; t < HX_LIB_NTYPE; t++) {
            const int j = at[t][r];
            if (j < 0) continue;
            const int ntr = L::ntrain(t), nfx = L::nfix(t), q = inst[t]++;
            const double* par = D->t[t].par + (size_t)desc_cols(t) * j;
            ent.push_back(t << 24 | q);
            mask[gi] |= 1ull << t;
            ent_st.push_back(nst);
            nst += L::nstate(t);
            std::vector<double> fv;
            if (t == HX_LIB_HD_LA) {
                // vhalfl, tau, ehd, kl, vhalft, a0t, zetat, gmt, then qtl * qt * a0t with
                // qt = pow(q10, (celsius - 33) / 10) as hd_la.cu:94 computes it
                for (int c = 1; c <= 8; c++) fv.push_back(par[c]);
                const double qt = std::pow(par[9], ((desc->celsius - 33.0) / 10.0));
                fv.push_back(par[10] * qt * par[6]);
            } else if (worm_mech(t)) {
                fv = {1.0, worm_mech_ca(t) ? 60.0 : -80.0, 0.0};
                const double* k = t == HX_LIB_SHL1 ? kShl1K : t == HX_LIB_IRK ? kIrkK : t == HX_LIB_EGL36 ? kEgl36K
                                  : t == HX_LIB_SHK1 ? kShk1K : t == HX_LIB_EGL2 ? kEgl2K : t == HX_LIB_CCA1 ? kCca1K
                                  : t == HX_LIB_EGL19 ? kEgl19K : t == HX_LIB_UNC2 ? kUnc2K : par + 1;
                fv.insert(fv.end(), k, k + (nfx - 3));
            } else {
                for (int c = 0; c < nfx; c++) fv.push_back(par[ntr + c]);
            }
            // entries with equal fixed parameters (GLOBALs, shared ion constants)
            // share one copy, so that their reads stay in cache
            auto it = fix_of[t].find(fv);
            if (it == fix_of[t].end()) {
                it = fix_of[t].emplace(fv, (int)fix.size()).first;
                fix.insert(fix.end(), fv.begin(), fv.end());
            }
            ent_fix.push_back(it->second);
            const int k0 = L::kind0(t);
            for (int c = 0; c < ntr; c++) {
                std::vector<double>& pv = prm[k0 + c];
                if ((int)pv.size() < ctx->lib_n[t]) pv.resize(ctx->lib_n[t], 0.0);
                pv[q] = par[c];
                ctx->kmap_h[HX_P_CADYN_GAMMA + k0 + c][j] = q;
            }
        }
        node_off[gi + 1] = (int)ent.size();
    }
    ent_st.push_back(nst);
    if (fix.empty()) fix.push_back(0.0);
    if (ent.empty()) ent.push_back(0);
    // GLOBALs of a mechanism: one value over its instances
    const int glo_t[19] = {HX_LIB_SK_E2,    HX_LIB_HD_LA,    HX_LIB_KM_LA,   HX_LIB_KCA_LA,   HX_LIB_IT2_LA,
                           HX_LIB_SCA_LA,   HX_LIB_SHL1_LR,  HX_LIB_KVS1_LR, HX_LIB_IRK_LR,   HX_LIB_EGL36_LR,
                           HX_LIB_SHK1_LR,  HX_LIB_EGL2_LR,  HX_LIB_CCA1_LR, HX_LIB_EGL19_LR, HX_LIB_UNC2_LR,
                           HX_LIB_KCNL_LR,  HX_LIB_KQT3_LR,  HX_LIB_CAINTERNM_LR, HX_LIB_KVS1};
    const int glo_c0[19] = {1, 3, 1, 1, 1, 3, 4, 4, 4, 4, 4, 4, 4, 4, 4, 3, 4, 1, 1};
    for (int u = 0; u < 19; u++) {
        const hx_lib_table& T = D->t[glo_t[u]];
        const int nc = desc_cols(glo_t[u]);
        for (int j = 1; j < T.n; j++)
            for (int c = glo_c0[u]; c < nc; c++)
                if (T.par[(size_t)nc * j + c] != T.par[c])
                    return fail(ctx, std::string(kTypeName[glo_t[u]]) +
                                         ": a GLOBAL of the mechanism differs between instances");
    }
    HXC(ctx->lib_node_off.upload(node_off, st));
    HXC(ctx->lib_mask.upload(mask, st));
    HXC(ctx->lib_ent.upload(ent, st));
    HXC(ctx->lib_ent_st.upload(ent_st, st));
    HXC(ctx->lib_ent_fix.upload(ent_fix, st));
    HXC(ctx->lib_fix.upload(fix, st));
    for (int k = HX_P_CADYN_GAMMA; k < kLibKindEnd; k++) {
        HXC(ctx->kmap[k].upload(ctx->kmap_h[k], st));
        HXC(ctx->prm[k].upload(prm[k - HX_P_CADYN_GAMMA], st));
    }
    HXC(ctx->lib_st.ensure(std::max(nst, 1)));
    HXC(ctx->lib_lam.ensure(std::max(nst, 1)));
    HXC(ctx->lib_nica.ensure(std::max(nn, 1)));
    HXC(ctx->lib_nlica.ensure(std::max(nn, 1)));
    HXC(cudaMemsetAsync(ctx->lib_nica.p, 0, sizeof(double) * std::max(nn, 1), st));
    HXC(cudaMemsetAsync(ctx->lib_nlica.p, 0, sizeof(double) * std::max(nn, 1), st));
    ctx->lib = true;
    ctx->lib_nst = nst;
    hx::DevLib& V = ctx->L;
    V.nst = nst;
    V.node_off = ctx->lib_node_off.p;
    V.mask = ctx->lib_mask.p;
    V.ent = ctx->lib_ent.p;
    V.ent_st = ctx->lib_ent_st.p;
    V.ent_fix = ctx->lib_ent_fix.p;
    V.fix = ctx->lib_fix.p;
    for (int k = 0; k < hx::kLibKinds; k++) V.prm[k] = ctx->prm[HX_P_CADYN_GAMMA + k].p;
    V.st = ctx->lib_st.p;
    V.lam = ctx->lib_lam.p;
    V.nica = ctx->lib_nica.p;
    V.nlica = ctx->lib_nlica.p;
    V.dt = desc->dt;
    // eion.cuh:38-41 with the 2018 CODATA constants of units.h
    const double faraday = 1.602176634e-19 * 6.02214076e+23;
    const double gas = 1.380649e-23 * 6.02214076e+23;
    V.ktf = 1000. * gas * (desc->celsius + 273.15) / faraday;
    return 0;
}
