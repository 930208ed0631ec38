// hx_noalloc.cu -- the allocation-free variant of the soma-trace MSE objective.
//
// Some hosts of this library cannot let it allocate device memory while they
// run: a training driver that pre-plans every device byte through its own fixed
// pool and forbids cudaMalloc/cudaFree by libraries, or a loop that must not
// hit the implicit device synchronisation cudaFree performs.  For them
// hx_mse_loss_grad_noalloc computes the same loss and gradient as
// hx_mse_loss_grad_dev without a context and without allocating: its scratch
// (one partial sum per 65,536-element chunk) lives in the file-scope array
// below, 4,096 doubles (32 KiB) per device, held by every GPU that loads the
// library until the process exits.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "heliox_b200.h"

namespace {

constexpr int kChunk = 1 << 16;        // elements reduced by one CTA
constexpr int kMaxPartials = 4096;     // capacity of the static scratch
constexpr int kMaxDevices = 64;

static __device__ __align__(256) double g_mse_scratch[kMaxPartials];

// The scratch array's device address per device (in host code the symbol's
// name is a host-side stand-in, not a device address).  Resolved again on
// every call made outside stream capture, so an address a cudaDeviceReset
// made stale is never used; a call during capture uses the address resolved
// by the device's last call outside capture.
double* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mu;

// One CTA per chunk: elementwise gradient, then the chunk's sum of squares into
// partial[blockIdx.x] (every slot the final kernel reads is written here, so no
// slot has to start at zero).
__global__ void mse_chunk_kernel(const double* __restrict__ tr, const double* __restrict__ tg,
                                 double* __restrict__ g, double* __restrict__ partial, long long n, long long ncol,
                                 double scale) {
    __shared__ double red[256];
    const long long b0 = (long long)blockIdx.x * kChunk;
    const long long b1 = (b0 + kChunk < n) ? b0 + kChunk : n;
    double acc = 0.0;
    for (long long i = b0 + threadIdx.x; i < b1; i += blockDim.x) {
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

// Sums the first np partials in a fixed order (deterministic).
__global__ void mse_chunk_final_kernel(const double* __restrict__ partial, int np, double* __restrict__ loss,
                                       double scale) {
    __shared__ double red[256];
    double acc = 0.0;
    for (int i = threadIdx.x; i < np; i += blockDim.x) acc += partial[i];
    red[threadIdx.x] = acc;
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
        if ((int)threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
        __syncthreads();
    }
    if (threadIdx.x == 0) *loss = red[0] * scale;
}

}  // namespace

extern "C" int hx_mse_loss_grad_noalloc(const double* trace_dev, const double* target_dev, int nrow, int ncol,
                                        double* dLdv_dev, double* loss_dev, void* stream) {
    if (!trace_dev || !target_dev || !dLdv_dev || !loss_dev || nrow < 1 || ncol < 0) return -1;
    const long long n = (long long)nrow * ncol;
    if (n > (long long)kMaxPartials * kChunk) {
        fprintf(stderr,
                "hx_mse_loss_grad_noalloc: %lld elements exceed the static scratch capacity of %lld "
                "(%d partial sums of %d elements)\n",
                n, (long long)kMaxPartials * kChunk, kMaxPartials, kChunk);
        return -2;
    }
    // an error left by earlier work is the caller's to read: report it
    // without clearing it and without doing any work
    if (cudaPeekAtLastError() != cudaSuccess) return -4;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -3;
    cudaStream_t st = (cudaStream_t)stream;
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cap) != cudaSuccess) return -3;
    double* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_scratch_mu);
        if (cap == cudaStreamCaptureStatusNone) {  // (re)resolve the scratch array's device address
            double* p = nullptr;
            if (cudaGetSymbolAddress((void**)&p, g_mse_scratch) != cudaSuccess || !p) return -3;
            g_scratch_ptr[dev] = p;
        }
        scratch = g_scratch_ptr[dev];
    }
    if (!scratch) return -3;  // first call on this device made during capture
    const int np = n > 0 ? (int)((n + kChunk - 1) / kChunk) : 1;
    const double scale = (nrow > 1 && ncol > 0) ? 1.0 / ((double)(nrow - 1) * ncol) : 0.0;
    mse_chunk_kernel<<<np, 256, 0, st>>>(trace_dev, target_dev, dLdv_dev, scratch, n, ncol, scale);
    if (cudaGetLastError() != cudaSuccess) return -3;
    mse_chunk_final_kernel<<<1, 256, 0, st>>>(scratch, np, loss_dev, scale);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
