// ref_nodev.cpp -- TEST INFRASTRUCTURE ONLY.
//
// Host-only definitions of the CUDA runtime calls the reference makes even in
// its CPU mode: pinned host buffers for every VecData (src/utils/cuda_utils.cu:
// 58-86), the spike counters PreSyn allocates on the device unconditionally
// (src/spike/presyn.cpp:29-30, used only by the GPU path), one stream and event
// per mechanism (src/mech/mechanism.cpp:27-28) and error polling
// (CUDA_CHECK_ERR).  Defined in the harness executable, they take
// precedence over the shared CUDA runtime's, so the reference's CPU integrator
// runs on a host without a GPU; its arithmetic does not depend on any of them.
#include <cuda_runtime_api.h>

#include <cstdlib>

extern "C" {

cudaError_t cudaHostAlloc(void** p, size_t size, unsigned int) {
    *p = std::calloc(size ? size : 1, 1);
    return *p ? cudaSuccess : cudaErrorMemoryAllocation;
}
cudaError_t cudaMallocHost(void** p, size_t size) { return cudaHostAlloc(p, size, 0); }
cudaError_t cudaFreeHost(void* p) {
    std::free(p);
    return cudaSuccess;
}
cudaError_t cudaMalloc(void** p, size_t size) { return cudaHostAlloc(p, size, 0); }
cudaError_t cudaFree(void* p) {
    std::free(p);
    return cudaSuccess;
}
cudaError_t cudaMemset(void* p, int v, size_t n) {
    unsigned char* c = static_cast<unsigned char*>(p);
    for (size_t i = 0; i < n; i++) c[i] = (unsigned char)v;
    return cudaSuccess;
}
cudaError_t cudaStreamCreateWithFlags(cudaStream_t* s, unsigned int) {
    static char token;
    *s = reinterpret_cast<cudaStream_t>(&token);
    return cudaSuccess;
}
cudaError_t cudaStreamCreate(cudaStream_t* s) {
    static char token;
    *s = reinterpret_cast<cudaStream_t>(&token);
    return cudaSuccess;
}
cudaError_t cudaStreamDestroy(cudaStream_t) { return cudaSuccess; }
cudaError_t cudaStreamSynchronize(cudaStream_t) { return cudaSuccess; }
cudaError_t cudaEventCreateWithFlags(cudaEvent_t* e, unsigned int) {
    static char token;
    *e = reinterpret_cast<cudaEvent_t>(&token);
    return cudaSuccess;
}
cudaError_t cudaEventDestroy(cudaEvent_t) { return cudaSuccess; }
cudaError_t cudaGetLastError(void) { return cudaSuccess; }
cudaError_t cudaDeviceSynchronize(void) { return cudaSuccess; }

}  // extern "C"
