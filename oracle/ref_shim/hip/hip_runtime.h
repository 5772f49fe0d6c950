// HIP -> CUDA shim: just enough of the HIP runtime API, spelled with CUDA, to compile the
// reference harness (bench/bench_main.cpp, common/backend.hpp) unmodified with nvcc.
// Test infrastructure only (oracle/).
#pragma once

#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>

using hipError_t = cudaError_t;
using hipStream_t = cudaStream_t;
using hipEvent_t = cudaEvent_t;
constexpr hipError_t hipSuccess = cudaSuccess;
constexpr unsigned hipStreamNonBlocking = cudaStreamNonBlocking;
constexpr cudaMemcpyKind hipMemcpyHostToDevice = cudaMemcpyHostToDevice;
constexpr cudaMemcpyKind hipMemcpyDeviceToHost = cudaMemcpyDeviceToHost;

// hipDeviceProp_t: the two fields the harness prints (name, gcnArchName).
struct hipDeviceProp_t {
    char name[256];
    char gcnArchName[256];
};

inline const char *hipGetErrorString(hipError_t e) { return cudaGetErrorString(e); }
inline hipError_t hipGetLastError() { return cudaGetLastError(); }
inline hipError_t hipGetDeviceProperties(hipDeviceProp_t *p, int dev) {
    cudaDeviceProp cp;
    const cudaError_t e = cudaGetDeviceProperties(&cp, dev);
    if (e != cudaSuccess)
        return e;
    std::snprintf(p->name, sizeof(p->name), "%s", cp.name);
    std::snprintf(p->gcnArchName, sizeof(p->gcnArchName), "sm_%d%d", cp.major, cp.minor);
    return cudaSuccess;
}
template <typename T> inline hipError_t hipMalloc(T **p, size_t n) { return cudaMalloc(reinterpret_cast<void **>(p), n); }
inline hipError_t hipFree(void *p) { return cudaFree(p); }
template <typename T> inline hipError_t hipHostMalloc(T **p, size_t n, unsigned = 0) {
    return cudaMallocHost(reinterpret_cast<void **>(p), n);
}
inline hipError_t hipHostFree(void *p) { return cudaFreeHost(p); }
inline hipError_t hipMemcpyAsync(void *d, const void *s, size_t n, cudaMemcpyKind k, hipStream_t st) {
    return cudaMemcpyAsync(d, s, n, k, st);
}
inline hipError_t hipMemsetAsync(void *d, int v, size_t n, hipStream_t st) { return cudaMemsetAsync(d, v, n, st); }
inline hipError_t hipStreamCreateWithFlags(hipStream_t *s, unsigned f) { return cudaStreamCreateWithFlags(s, f); }
inline hipError_t hipStreamDestroy(hipStream_t s) { return cudaStreamDestroy(s); }
inline hipError_t hipStreamSynchronize(hipStream_t s) { return cudaStreamSynchronize(s); }
inline hipError_t hipEventCreate(hipEvent_t *e) { return cudaEventCreate(e); }
inline hipError_t hipEventDestroy(hipEvent_t e) { return cudaEventDestroy(e); }
inline hipError_t hipEventRecord(hipEvent_t e, hipStream_t s) { return cudaEventRecord(e, s); }
inline hipError_t hipEventSynchronize(hipEvent_t e) { return cudaEventSynchronize(e); }
inline hipError_t hipEventElapsedTime(float *ms, hipEvent_t a, hipEvent_t b) { return cudaEventElapsedTime(ms, a, b); }
