// crx_checksum_noalloc: the full weight checksum (the reference's codec.checksum,
// src/crukx_sync/codec.py:61-68) for callers that must not allocate.  It uses no context and
// no cudaMalloc/cudaFree: its only scratch is the file-scope device array below, sized for
// kNoAllocSlots chunks of kNoAllocChunk elements.
//
//   * Set-up: the first call on each device (with that device current) looks up the array's
//     device address with cudaGetSymbolAddress, which loads this library's module on that
//     device.  Make one call before capturing a stream.
//   * Nothing has to start at zero: k_noalloc_partials writes every slot that k_noalloc_total
//     reads, and k_noalloc_total writes *out without reading it.
//   * One scratch array per device: calls that overlap on one device (two streams, or two host
//     threads without ordering between them) race on it.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "crukx_b200.h"

namespace {

using crx::splitmix_weight;
using crx::tmin;

constexpr int kNoAllocThreads = 256;
constexpr int64_t kNoAllocChunk = int64_t(1) << 16;      // elements per partial sum
constexpr int kNoAllocSlots = 16384;                       // 128 KiB of partial sums
constexpr int kMaxDevices = 64;
static_assert(int64_t(kNoAllocSlots) * kNoAllocChunk == CRX_CHECKSUM_NOALLOC_MAX, "limit in the header");

static __device__ __align__(256) unsigned long long g_partials[kNoAllocSlots];

std::mutex g_setup_mu;
unsigned long long* g_partials_addr[kMaxDevices];   // device address of g_partials, per device

// one block per chunk: Σ u16(p[i]) · w(i) over the chunk, mod 2^64, into partials[chunk]
__global__ void __launch_bounds__(kNoAllocThreads) k_noalloc_partials(const int16_t* __restrict__ p, int64_t n,
                                                                      unsigned long long* __restrict__ partials) {
    __shared__ uint64_t red[kNoAllocThreads / 32];
    const int64_t lo = int64_t(blockIdx.x) * kNoAllocChunk;
    const int64_t hi = tmin(n, lo + kNoAllocChunk);
    uint64_t s = 0;
#pragma unroll 8
    for (int64_t i = lo + threadIdx.x; i < hi; i += kNoAllocThreads)
        s += uint64_t(uint16_t(p[i])) * splitmix_weight(uint64_t(i));
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint64_t t = 0;
        for (int k = 0; k < kNoAllocThreads / 32; ++k) t += red[k];
        partials[blockIdx.x] = t;
    }
}

// one block: the sum of the first `chunks` partial sums into *out (0 when chunks == 0)
__global__ void __launch_bounds__(kNoAllocThreads) k_noalloc_total(const unsigned long long* __restrict__ partials,
                                                                   int chunks, unsigned long long* __restrict__ out) {
    __shared__ uint64_t red[kNoAllocThreads / 32];
    uint64_t s = 0;
    for (int k = threadIdx.x; k < chunks; k += kNoAllocThreads) s += partials[k];
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint64_t t = 0;
        for (int k = 0; k < kNoAllocThreads / 32; ++k) t += red[k];
        *out = t;
    }
}

int fail(char* err, size_t errlen, int status, const char* msg, cudaError_t e = cudaSuccess) {
    if (err && errlen) {
        if (e != cudaSuccess) std::snprintf(err, errlen, "crx_checksum_noalloc: %s: %s", msg, cudaGetErrorString(e));
        else std::snprintf(err, errlen, "crx_checksum_noalloc: %s", msg);
    }
    return status;
}

// true when p is memory a kernel on device `dev` can use as plain device memory: allocated on that
// device, or managed.  cudaPointerGetAttributes looks the pointer up and allocates nothing.
bool on_device(const void* p, int dev) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();   // an unknown pointer is an argument error, not a sticky one
        return false;
    }
    return a.type == cudaMemoryTypeManaged || (a.type == cudaMemoryTypeDevice && a.device == dev);
}

}  // namespace

extern "C" int crx_checksum_noalloc(const int16_t* data, int64_t n, void* stream, uint64_t* out, char* err,
                                    size_t errlen) {
    if (n < 0 || (n && !data) || !out) return fail(err, errlen, CRX_BAD_ARGUMENT, "null pointer or negative size");
    // a misaligned or host pointer would make the kernels fault (a sticky error for the whole
    // context), so both are rejected here, before anything is launched
    if (reinterpret_cast<uintptr_t>(out) & 7) return fail(err, errlen, CRX_BAD_ARGUMENT, "out is not 8-byte aligned");
    if (n && (reinterpret_cast<uintptr_t>(data) & 1))
        return fail(err, errlen, CRX_BAD_ARGUMENT, "data is not 2-byte aligned");
    if (n > CRX_CHECKSUM_NOALLOC_MAX) {
        char msg[160];
        std::snprintf(msg, sizeof msg, "%lld elements exceed the limit of %lld (a fixed %d KiB scratch); use crx_checksum",
                      static_cast<long long>(n), static_cast<long long>(CRX_CHECKSUM_NOALLOC_MAX),
                      int(sizeof(unsigned long long) * kNoAllocSlots / 1024));
        return fail(err, errlen, CRX_VALUE_ERROR, msg);
    }
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(err, errlen, CRX_CUDA_ERROR, "cudaGetDevice", e);
    if (dev < 0 || dev >= kMaxDevices) return fail(err, errlen, CRX_BAD_ARGUMENT, "device index out of range");
    if (!on_device(out, dev)) return fail(err, errlen, CRX_BAD_ARGUMENT, "out is not device memory of the current device");
    if (n && !on_device(data, dev))
        return fail(err, errlen, CRX_BAD_ARGUMENT, "data is not device memory of the current device");
    unsigned long long* partials;
    {
        std::lock_guard<std::mutex> g(g_setup_mu);
        if (!g_partials_addr[dev]) {   // set-up, once per device, with that device current
            void* addr = nullptr;
            e = cudaGetSymbolAddress(&addr, g_partials);
            if (e != cudaSuccess || !addr) return fail(err, errlen, CRX_CUDA_ERROR, "cudaGetSymbolAddress", e);
            g_partials_addr[dev] = static_cast<unsigned long long*>(addr);
        }
        partials = g_partials_addr[dev];
    }
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int chunks = int((n + kNoAllocChunk - 1) / kNoAllocChunk);
    if (chunks) k_noalloc_partials<<<unsigned(chunks), kNoAllocThreads, 0, st>>>(data, n, partials);
    k_noalloc_total<<<1, kNoAllocThreads, 0, st>>>(partials, chunks, reinterpret_cast<unsigned long long*>(out));
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail(err, errlen, CRX_CUDA_ERROR, "kernel launch", e);
    return CRX_OK;
}
