// hx_ctx.hpp -- the library context behind the C ABI (shared by the runtime
// translation units).  Device buffers are grow-only and reused across calls
// like the reference's LearnRuntime::ensure_buf
// (src/runtime_api/learn/LearnRuntime.cpp:877-895).
#pragma once

#include <cuda_runtime.h>

#include <string>
#include <vector>

#include "heliox_b200.h"
#include "hx_dev.hpp"
#include "hx_plan.hpp"

namespace hxrt {

template <typename T>
struct DevBuf {
    T* p = nullptr;
    size_t n = 0;
    ~DevBuf() { release(); }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
    }
    cudaError_t ensure(size_t count) {
        if (count <= n && p) return cudaSuccess;
        release();
        size_t c = count ? count : 1;
        cudaError_t e = cudaMalloc((void**)&p, c * sizeof(T));
        if (e == cudaSuccess) n = c;
        return e;
    }
    cudaError_t upload(const std::vector<T>& v, cudaStream_t st) {
        cudaError_t e = ensure(v.size());
        if (e != cudaSuccess || v.empty()) return e;
        return cudaMemcpyAsync(p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice, st);
    }
};

struct PinBuf {
    void* p = nullptr;
    size_t bytes = 0;
    ~PinBuf() {
        if (p) cudaFreeHost(p);
    }
    cudaError_t ensure(size_t b) {
        if (b <= bytes && p) return cudaSuccess;
        if (p) cudaFreeHost(p);
        p = nullptr;
        bytes = 0;
        cudaError_t e = cudaMallocHost(&p, b ? b : 16);
        if (e == cudaSuccess) bytes = b ? b : 16;
        return e;
    }
};

}  // namespace hxrt

using hxrt::DevBuf;
using hxrt::PinBuf;

// Adam over external-gradient slots (one per registered parameter instance).
struct AdamOpt {
    double beta1 = 0.9, beta2 = 0.999, eps = 1e-8, impedance = 1.0;
    long long step = 0;
    int n = 0;
    std::vector<int> kind_h, ref_h;
    DevBuf<int> kind, slot, flat;
    DevBuf<double> grad, m, v;
    DevBuf<float> f32;
    hx_allreduce_fn allreduce = nullptr;  // sum of the slot gradients over ranks before each step
    void* allreduce_user = nullptr;
};

struct hx_ctx {
    int device = 0;
    cudaStream_t own = nullptr, st = nullptr;
    std::string err;
    int pack_target = 0;
    size_t tape_budget = 0;
    long long split_spin_limit = hx::kSplitSpinLimitDefault;
    unsigned grad_skip = 0;  // DevGrad::skip of the next backward (hx_set_grad_kinds)
    bool loaded = false;
    hx::Plan P;
    double dt = 0.025, celsius = 6.3;
    // plan arrays
    DevBuf<int> pack_node_off, pack_slot_off, pack_br_off, pack_bch_off, pack_nch_off;
    DevBuf<int> cs_node0, cs_nnode, cs_warp0, cs_nwarp, cs_bar, cs_lvl_off, cs_nlev, level_br_off;
    DevBuf<int> br_head, br_end, br_parent, br_child_off, br_child, br_child_br;
    DevBuf<int> node_parent, node_child_off, node_child, node_flags, node_ic_off, node_ic;
    // reference instance -> device index, per parameter kind (host + device copies)
    std::vector<int> kmap_h[HX_P_COUNT];
    DevBuf<int> kmap[HX_P_COUNT];
    // parameters: node-indexed (density mechanisms, cm) or per IClamp instance
    DevBuf<double> a, b, area;
    DevBuf<double> prm[HX_P_COUNT];
    DevBuf<double> hh_ena, hh_ek, ic_del, ic_dur;
    hx::DevGroup G{};
    // state, tape, checkpoints, adjoint, gradients
    DevBuf<double> sv, sm, sh, sn;
    DevBuf<double> tv, tm, th, tn;
    DevBuf<double> ck;  // nseg x 4 nnode (v, m, h, n)
    DevBuf<double> lv, lm, lh, ln;
    DevBuf<double> grad;  // concatenated per kind
    size_t grad_off[HX_P_COUNT + 1] = {0};
    DevBuf<double> tmid;
    int tmid_steps = -1;
    DevBuf<int> pr_off, pr_local, pr_slot;
    std::vector<int> probe_key;
    int nprobe = 0;
    DevBuf<double> trace_dev, dLdv_dev, stage_dev;
    DevBuf<double> mse_partial;
    DevBuf<int> red_off, red_flat;
    DevBuf<float> red_scale, red_out;
    PinBuf pin;
    // capture bookkeeping
    bool captured = false;
    int nstep = 0;
    int seg = 0, nseg = 0;  // steps per segment (checkpoint interval) and count
    bool full_tape = true;
    std::vector<AdamOpt*> opts;
    DevBuf<double*> prm_ptrs;  // device copy of prm[kind].p
    cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};
    int launches[2] = {0, 0};
    // event pairs around every reverse-kernel launch of the last backward
    // (a checkpointed backward alternates recompute and reverse launches)
    std::vector<cudaEvent_t> kev;
    int kev_n = 0;

    // ---- network (hx_runtime_net.cu)
    bool net = false, coupled = false;
    // ngj: device gap instances (gapjunction_lr ngj_lr, then gapjunction_noptr ngnp)
    int nexp = 0, nexp2 = 0, nsyn = 0, nstim = 0, nhg = 0, ngj = 0, ngj_lr = 0, ngnp = 0, ngr = 0;
    int gid_base = 0, nsrc_cells = 0, nsrc = 0;
    int window = 0, window_user = 0;
    double dmin = 0.0;
    hx::DevNet N{};
    DevBuf<int> node_syn_off, pack_syn_off, syn_kind, src_off, src_syn, syn_node, syn_pack;
    DevBuf<double> syn_tau1, syn_tau2, syn_cA, syn_cB, syn_fA, syn_fB, syn_delay;
    DevBuf<double> sA, sB, tA, tB, lA, lB;
    DevBuf<int> cs_ps_node, cs_gid, cs_ps_flag;
    DevBuf<double> cs_ps_thr;
    DevBuf<int> node_hg_off, hg_src, node_gj_off, gj_pre, node_gr_off, gr_pre, node_in_off, node_in;
    DevBuf<double> gr_g, gr_k, gr_erev, gr_delta, gr_vth, gr_s, tS, lS;
    DevBuf<double> vbuf;  // 2 x nnode ping-pong voltages of coupled launches
    DevBuf<double> xbuf;  // 2 x (nhg + ngj + ngr) partner contributions of coupled reverse launches
    // grid-synchronous coupled launches: allowed (hx_set_grid_sync), and every
    // pack co-resident with cooperative launch support (checked at load)
    bool gsync_allowed = true, gsync_fit = false;
    DevBuf<unsigned> gs_bar;
    DevBuf<int> gs_err;
    DevBuf<double> tstart;
    DevBuf<int> ev_cnt, ev_syn, dev_err;
    int ev_cap = 0;
    DevBuf<int2> win_send, win_recv, spk_log, ns_spk;
    DevBuf<int2> st_send, st_recv;  // per-rank status pair after the last window
    DevBuf<int> win_n, log_n;
    int win_cap = 0, log_cap = 0, win_cap_user = 0;
    int win_cap_cur = 0;    // agreed window buffer size of a multi-rank exchange (grows on overflow)
    DevBuf<int> win_max;    // largest window spike count of the current forward
    // NetStim trains of the last forward length (host generator, routed each forward)
    std::vector<double> ns_interval, ns_number, ns_start, ns_noise;
    int ns_rng = 0, ns_steps = -1, ns_count = 0;
    // multi-GPU exchange
    hx_exchange_fn exchange = nullptr;
    void* exchange_user = nullptr;
    int nranks = 1;
    size_t ck_net_stride = 0;  // doubles per checkpoint beyond v, m, h, n

    // ---- library mechanisms (hx_lib.cuh; hx_runtime_lib.cu)
    bool lib = false;
    int lib_n[HX_LIB_NTYPE] = {0};  // instances per type
    int lib_nst = 0;                // states over all entries
    hx::DevLib L{};
    DevBuf<int> lib_node_off, lib_ent, lib_ent_st, lib_ent_fix;
    DevBuf<unsigned long long> lib_mask;
    DevBuf<double> lib_fix, lib_st, lib_lam, lib_nica, lib_nlica, lib_tape, lib_ck;

    // ---- a cell split across CTAs (hx_split.cu)
    bool split = false;
    hx::DevSplit X{};
    DevBuf<int> sub_root, sub_parent, split_err;
    DevBuf<double> xd, xrhs, xx, xv, xvp;
    DevBuf<unsigned> split_bar;
};

// The runtime's own error path (sets hx_last_error, returns -1).
int hx_fail(hx_ctx* c, const std::string& m);
// shared runtime helpers (hx_runtime.cu)
int hx_setup_probes(hx_ctx* ctx, int nprobe, const int* probe_nodes);
hx::DevProbe hx_probe_view(hx_ctx* c);
int hx_setup_time(hx_ctx* ctx, int nstep);
// records the next event of the reverse-kernel pairs on stream st (kev_n = 0 starts a backward)
int hx_kev_mark(hx_ctx* ctx, cudaStream_t st);
double* hx_kind_ptr(hx_ctx* c, int kind);
size_t hx_grad_base(const hx_ctx* c, int kind);
// library mechanisms (hx_runtime_lib.cu): entry tables, kinds 16.. maps and
// device arrays; the type of a library parameter kind
int hx_lib_load(hx_ctx* ctx, const hx_group_desc* desc);
int hx_lib_type_of_kind(int kind);
// network parts (hx_runtime_net.cu)
int hx_net_load(hx_ctx* ctx, const hx_group_desc* desc);
int hx_net_forward(hx_ctx* ctx, int nstep, double v_init, double* trace_dev, bool capture);
int hx_net_backward(hx_ctx* ctx, const double* dLdv_dev);

