// hx_kernels.hpp -- host-callable launchers of the kernels in hx_kernels.cu.
#pragma once

#include <cuda_runtime.h>

#include "hx_dev.hpp"

namespace hx {

size_t fwd_smem_bytes(const DevGroup& G);
size_t bwd_smem_bytes(const DevGroup& G);
cudaError_t configure_kernels(size_t smem_fwd, size_t smem_bwd);
cudaError_t launch_init(const DevGroup& G, const DevState& S, double v_init, cudaStream_t st);
cudaError_t launch_fwd(const DevGroup& G, const DevState& S, const DevTape& T, int write_tape, const DevProbe& P,
                       double* trace, const double* tmid, int k0, int k1, cudaStream_t st);
cudaError_t launch_bwd(const DevGroup& G, const DevTape& T, const DevAdj& A, const DevGrad& GR, const DevProbe& P,
                       const double* dLdv, const double* tmid, int k_hi, int k_lo, cudaStream_t st);
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
