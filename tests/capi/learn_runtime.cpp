// learn_runtime.cpp -- a C++ host of the C ABI in the shape of the reference's
// LearnRuntime (src/runtime_api/learn/LearnRuntime.h:21-293): a runtime object
// that loads a group once and answers simulate_and_adjoint_into calls (the
// exact-adjoint counterpart of simulate_and_replay_dw_dx_streaming_into,
// LearnRuntime.h:72-100): forward with capture, dL/d(output) widened to
// double, reverse sweep, column reduction of the per-instance gradients into
// dw_out_n.  0 / -1 with the reason printed, like every LearnRuntime entry.
//
//   learn_runtime <case.bin> <out.bin>
// case.bin (little endian): int32 ncell nnode nhh npas nic nstep nprobe nparam;
// float64 celsius dt v_init; int32 parent[nnode]; float64 a, b, area, cm
// [nnode each]; int32 hh_node[nhh]; float64 gnabar gkbar gl el ena ek [nhh
// each]; int32 pas_node[npas]; float64 g e [npas each]; int32 ic_node[nic];
// float64 del dur amp [nic each]; int32 probes[nprobe]; float32
// dLtdv[nstep * nprobe] (row t: step t + 1); int32 kind[nparam] index[nparam]
// dest[nparam]; float32 scale[nparam]; int32 N.
// out.bin: float64 trace[(nstep + 1) * nprobe]; float32 dw_out_n[N].
#include <cstdint>
#include <cstdio>
#include <span>
#include <string>
#include <vector>

#include "heliox_b200.h"

namespace {

struct Reader {
    FILE* f;
    bool ok = true;
    template <typename T>
    std::vector<T> take(size_t n) {
        std::vector<T> v(n);
        if (n && std::fread(v.data(), sizeof(T), n, f) != n) ok = false;
        return v;
    }
};

class AdjointLearnRuntime {
   public:
    ~AdjointLearnRuntime() {
        if (ctx_) hx_destroy(ctx_);
    }
    int load(int device, const hx_group_desc& desc) {
        if (hx_create(&ctx_, device) != 0) return fail("hx_create");
        if (hx_load_group(ctx_, &desc) != 0) return fail("hx_load_group");
        return 0;
    }
    // LearnRuntime::simulate_and_adjoint_into as INTEGRATION.md describes it
    int simulate_and_adjoint_into(const float* dLtdv_to, int T, int n_output, const int32_t* poutput,
                                  std::span<const int> kinds, std::span<const int> indices,
                                  std::span<const int32_t> dest, std::span<const float> scale, float* dw_out_n,
                                  int N, double v_init, double* trace_out) {
        std::vector<double> trace((size_t)(T + 1) * n_output);
        if (hx_forward_capture(ctx_, T, v_init, n_output, poutput, trace.data()) != 0) return fail("forward");
        std::vector<double> dLdv((size_t)(T + 1) * n_output, 0.0);  // row 0 (the initial state) carries no loss
        for (size_t i = 0; i < (size_t)T * n_output; i++) dLdv[n_output + i] = dLtdv_to[i];
        if (hx_backward(ctx_, dLdv.data(), nullptr) != 0) return fail("backward");
        if (hx_reduce_grads_f32(ctx_, (int)kinds.size(), kinds.data(), indices.data(), dest.data(), scale.data(),
                                dw_out_n, N) != 0)
            return fail("reduce");
        if (trace_out) std::copy(trace.begin(), trace.end(), trace_out);
        return 0;
    }

   private:
    int fail(const char* what) {
        std::printf("[AdjointLearnRuntime] %s failed: %s\n", what, hx_last_error(ctx_));
        return -1;
    }
    hx_ctx* ctx_ = nullptr;
};

}  // namespace

int main(int argc, char** argv) {
    if (argc != 3) {
        std::fprintf(stderr, "usage: %s case.bin out.bin\n", argv[0]);
        return 2;
    }
    if (hx_abi_version() != HX_ABI_VERSION) {
        std::fprintf(stderr, "library ABI %d, header %d\n", hx_abi_version(), HX_ABI_VERSION);
        return 2;
    }
    FILE* f = std::fopen(argv[1], "rb");
    if (!f) return 3;
    Reader r{f};
    const auto h = r.take<int32_t>(8);
    const int ncell = h[0], nnode = h[1], nhh = h[2], npas = h[3], nic = h[4], nstep = h[5], nprobe = h[6],
              nparam = h[7];
    const auto fl = r.take<double>(3);
    const auto parent = r.take<int32_t>(nnode);
    const auto a = r.take<double>(nnode), b = r.take<double>(nnode), area = r.take<double>(nnode),
               cm = r.take<double>(nnode);
    const auto hh_node = r.take<int32_t>(nhh);
    const auto gna = r.take<double>(nhh), gk = r.take<double>(nhh), gl = r.take<double>(nhh),
               el = r.take<double>(nhh), ena = r.take<double>(nhh), ek = r.take<double>(nhh);
    const auto pas_node = r.take<int32_t>(npas);
    const auto pg = r.take<double>(npas), pe = r.take<double>(npas);
    const auto ic_node = r.take<int32_t>(nic);
    const auto idel = r.take<double>(nic), idur = r.take<double>(nic), iamp = r.take<double>(nic);
    const auto probes = r.take<int32_t>(nprobe);
    const auto dLtdv = r.take<float>((size_t)nstep * nprobe);
    const auto kind = r.take<int32_t>(nparam), index = r.take<int32_t>(nparam), dest = r.take<int32_t>(nparam);
    const auto scale = r.take<float>(nparam);
    const auto Nv = r.take<int32_t>(1);
    std::fclose(f);
    if (!r.ok) {
        std::fprintf(stderr, "truncated case file\n");
        return 3;
    }
    hx_group_desc d{};
    d.ncell = ncell;
    d.nnode = nnode;
    d.parent = parent.data();
    d.a = a.data();
    d.b = b.data();
    d.area = area.data();
    d.cm = cm.data();
    d.celsius = fl[0];
    d.dt = fl[1];
    d.nhh = nhh;
    d.hh_node = hh_node.data();
    d.hh_gnabar = gna.data();
    d.hh_gkbar = gk.data();
    d.hh_gl = gl.data();
    d.hh_el = el.data();
    d.hh_ena = ena.data();
    d.hh_ek = ek.data();
    d.npas = npas;
    d.pas_node = pas_node.data();
    d.pas_g = pg.data();
    d.pas_e = pe.data();
    d.nic = nic;
    d.ic_node = ic_node.data();
    d.ic_del = idel.data();
    d.ic_dur = idur.data();
    d.ic_amp = iamp.data();
    AdjointLearnRuntime rt;
    if (rt.load(0, d) != 0) return 1;
    const int N = Nv[0];
    std::vector<float> dw(N, 0.0f);
    std::vector<double> trace((size_t)(nstep + 1) * nprobe);
    if (rt.simulate_and_adjoint_into(dLtdv.data(), nstep, nprobe, probes.data(), kind, index, dest, scale, dw.data(),
                                     N, fl[2], trace.data()) != 0)
        return 1;
    FILE* o = std::fopen(argv[2], "wb");
    if (!o) return 3;
    std::fwrite(trace.data(), sizeof(double), trace.size(), o);
    std::fwrite(dw.data(), sizeof(float), dw.size(), o);
    std::fclose(o);
    return 0;
}
