// hx_kernels.hpp -- host-callable launchers of the kernels in hx_kernels.cu.
#pragma once

#include <cuda_runtime.h>

#include "hx_dev.hpp"

namespace hx {

size_t fwd_smem_bytes(const DevGroup& G);
size_t bwd_smem_bytes(const DevGroup& G);
size_t split_fwd_smem_bytes(const DevGroup& G);
size_t split_bwd_smem_bytes(const DevGroup& G);
cudaError_t configure_kernels(size_t smem_fwd, size_t smem_bwd, size_t smem_fwd_net, size_t smem_bwd_net);
// the coupled-network instantiations (occupancy checks of grid-synchronous launches)
const void* fwd_cpl_kernel_ptr(bool lib);
const void* bwd_cpl_kernel_ptr(bool lib);
cudaError_t launch_init(const DevGroup& G, const DevState& S, double v_init, cudaStream_t st);
cudaError_t launch_lib_init(const DevLib& L, int nnode, double v_init, cudaStream_t st);
// N and L null: the plain kernels; N: the network instantiation; L: the
// library-mechanism instantiation (its tape rows are counted from T.k_base);
// both: library mechanisms in a network group
cudaError_t launch_fwd(const DevGroup& G, const DevState& S, const DevTape& T, int write_tape, const DevProbe& P,
                       double* trace, const double* tmid, int k0, int k1, cudaStream_t st, const DevNet* N = nullptr,
                       const DevLib* L = nullptr);
cudaError_t launch_bwd(const DevGroup& G, const DevTape& T, const DevAdj& A, const DevGrad& GR, const DevProbe& P,
                       const double* dLdv, const double* tmid, int k_hi, int k_lo, cudaStream_t st,
                       const DevNet* N = nullptr, const DevLib* L = nullptr);
// split cell (hx_split.cu): cooperative launches over all packs
cudaError_t configure_split(size_t smem_fwd, size_t smem_bwd);
const void* split_fwd_kernel_ptr();
const void* split_bwd_kernel_ptr();
cudaError_t launch_split_fwd(const DevGroup& G, const DevState& S, const DevTape& T, int write_tape, const DevProbe& P,
                             double* trace, const double* tmid, int k0, int k1, const DevSplit& X, cudaStream_t st);
cudaError_t launch_split_bwd(const DevGroup& G, const DevTape& T, const DevAdj& A, const DevGrad& GR, const DevProbe& P,
                             const double* dLdv, const double* tmid, int k_hi, int k_lo, const DevSplit& X,
                             cudaStream_t st);
cudaError_t launch_syn_prep(int n, const int* kind, const double* tau1, const double* tau2, double dt, double* cA,
                            double* cB, double* fA, double* fB, cudaStream_t st);
cudaError_t launch_init_net(int nsyn, double* sA, double* sB, int ngr, const double* gr_w, const double* gr_vth,
                            const double* gr_delta, double* gr_g, double* gr_k, double* gr_erev, double* gr_s,
                            double v_init, cudaStream_t st);
cudaError_t launch_route(const int2* spk, const int* nspk_dev, int nspk_max, const int* src_off, const int* src_syn,
                         int nsrc, const double* delay, const double* tstart, int nstep, double half_dt, int k_min,
                         const int* syn_pack, int npack, int* ev_cnt, int* ev_syn, int ev_cap, int* err,
                         cudaStream_t st);
cudaError_t launch_log_append(const int2* win, const int* win_n, int win_cap, int2* log, int* log_n, int log_cap,
                              int* err, int* win_max, cudaStream_t st);
cudaError_t launch_rcp_nz(const double* x, double* y, int n, cudaStream_t st);
cudaError_t launch_net_status(const int* err, const int* ev_cnt, int nstep, const int* win_max, int extra, int2* out,
                              cudaStream_t st);
cudaError_t launch_gather(const double* src, const int* idx, double* dst, int n, cudaStream_t st);
cudaError_t launch_scatter(const double* src, const int* idx, double* dst, int n, cudaStream_t st);
constexpr int kMsePartials = 256;
cudaError_t launch_mse(const double* trace, const double* target, double* dLdv, double* partial, double* loss,
                       int nrow, int ncol, cudaStream_t st);
cudaError_t launch_adam(double* const* wbase, const int* kind, const int* slot, double* grad, double* m, double* v,
                        int n, double lr, double impedance, double inv_record_steps, double beta1, double beta2,
                        double eps, double bc1, double bc2, cudaStream_t st);
cudaError_t launch_take_scaled(const double* src, const int* flat, double* dst, int n, double scale, cudaStream_t st);
cudaError_t launch_f32_to_f64(const float* a, double* b, int n, cudaStream_t st);
cudaError_t launch_reduce_cols(const double* grad, const int* col_off, const int* flat, const float* scale,
                               float* out, int ncol, cudaStream_t st);

}  // namespace hx
