// Scans used by both directions: per-tensor column scans of [rows][256] histogram tables and a
// device-wide exclusive scan of u64 values (block bit lengths, block sums).
#include "common.cuh"
#include "context.h"

namespace crx {

namespace {

__device__ __forceinline__ int tensor_of_chunk(const int64_t* chunk_begin, int n_tensors, int64_t c) {
    int lo = 0, hi = n_tensors - 1;              // last t with chunk_begin[t] <= c
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (chunk_begin[mid] <= c) lo = mid; else hi = mid - 1;
    }
    return lo;
}

__global__ void __launch_bounds__(256) k_chunk_sums(const uint32_t* __restrict__ table, const int64_t* __restrict__ row_begin,
                                                    int n_tensors, const int64_t* __restrict__ chunk_begin,
                                                    uint32_t* __restrict__ chunk_sums) {
    const int64_t c = blockIdx.x;
    const int t = tensor_of_chunk(chunk_begin, n_tensors, c);
    const int64_t r0 = row_begin[t] + (c - chunk_begin[t]) * SCAN_CHUNK;
    const int64_t r1 = min(r0 + SCAN_CHUNK, row_begin[t + 1]);
    uint32_t s = 0;
    for (int64_t r = r0; r < r1; ++r) s += table[r * 256 + threadIdx.x];
    chunk_sums[c * 256 + threadIdx.x] = s;
}

__global__ void __launch_bounds__(256) k_chunk_scan(const int64_t* __restrict__ chunk_begin, uint32_t* __restrict__ chunk_sums,
                                                    uint64_t* __restrict__ totals) {
    const int t = blockIdx.x;
    uint64_t run = 0;
    for (int64_t c = chunk_begin[t]; c < chunk_begin[t + 1]; ++c) {
        const uint32_t v = chunk_sums[c * 256 + threadIdx.x];
        chunk_sums[c * 256 + threadIdx.x] = uint32_t(run);
        run += v;
    }
    totals[int64_t(t) * 256 + threadIdx.x] = run;
}

__global__ void __launch_bounds__(256) k_chunk_rescan(uint32_t* __restrict__ table, const int64_t* __restrict__ row_begin,
                                                      int n_tensors, const int64_t* __restrict__ chunk_begin,
                                                      const uint32_t* __restrict__ chunk_sums) {
    const int64_t c = blockIdx.x;
    const int t = tensor_of_chunk(chunk_begin, n_tensors, c);
    const int64_t r0 = row_begin[t] + (c - chunk_begin[t]) * SCAN_CHUNK;
    const int64_t r1 = min(r0 + SCAN_CHUNK, row_begin[t + 1]);
    uint32_t p = chunk_sums[c * 256 + threadIdx.x];
    for (int64_t r = r0; r < r1; ++r) {
        const uint32_t v = table[r * 256 + threadIdx.x];
        table[r * 256 + threadIdx.x] = p;
        p += v;
    }
}

constexpr int SCAN_T = 1024;
constexpr int SCAN_PER = 4;
constexpr int SCAN_TILE = SCAN_T * SCAN_PER;

__device__ __forceinline__ uint64_t block_exclusive_scan(uint64_t v, uint64_t* sh, uint64_t* total) {
    const int l = threadIdx.x & 31, w = threadIdx.x >> 5;
    uint64_t x = v;
    for (int o = 1; o < 32; o <<= 1) {
        const uint64_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (l >= o) x += y;
    }
    if (l == 31) sh[w] = x;
    __syncthreads();
    if (w == 0) {
        uint64_t s = sh[l];
        for (int o = 1; o < 32; o <<= 1) {
            const uint64_t y = __shfl_up_sync(0xffffffffu, s, o);
            if (l >= o) s += y;
        }
        sh[l] = s;
    }
    __syncthreads();
    const uint64_t before = (w ? sh[w - 1] : 0) + x - v;
    *total = sh[31];
    __syncthreads();
    return before;
}

__global__ void __launch_bounds__(SCAN_T) k_scan_reduce(const uint64_t* __restrict__ d, int64_t n, uint64_t* __restrict__ sums) {
    __shared__ uint64_t sh[32];
    const int64_t base = int64_t(blockIdx.x) * SCAN_TILE + threadIdx.x * SCAN_PER;
    uint64_t s = 0;
    for (int k = 0; k < SCAN_PER; ++k) if (base + k < n) s += d[base + k];
    uint64_t tot;
    block_exclusive_scan(s, sh, &tot);
    if (threadIdx.x == 0) sums[blockIdx.x] = tot;
}

__global__ void __launch_bounds__(SCAN_T) k_scan_top(uint64_t* __restrict__ sums, int64_t m, uint64_t* __restrict__ total) {
    __shared__ uint64_t sh[32];
    uint64_t carry = 0;
    for (int64_t b = 0; b < m; b += SCAN_T) {
        const int64_t i = b + threadIdx.x;
        const uint64_t v = i < m ? sums[i] : 0;
        uint64_t tot;
        const uint64_t ex = block_exclusive_scan(v, sh, &tot);
        if (i < m) sums[i] = carry + ex;
        carry += tot;
    }
    if (threadIdx.x == 0) *total = carry;
}

__global__ void __launch_bounds__(SCAN_T) k_scan_down(uint64_t* __restrict__ d, int64_t n, const uint64_t* __restrict__ sums) {
    __shared__ uint64_t sh[32];
    const int64_t base = int64_t(blockIdx.x) * SCAN_TILE + threadIdx.x * SCAN_PER;
    uint64_t v[SCAN_PER];
    uint64_t s = 0;
    for (int k = 0; k < SCAN_PER; ++k) { v[k] = base + k < n ? d[base + k] : 0; s += v[k]; }
    uint64_t tot;
    uint64_t p = block_exclusive_scan(s, sh, &tot) + sums[blockIdx.x];
    for (int k = 0; k < SCAN_PER; ++k) {
        if (base + k < n) d[base + k] = p;
        p += v[k];
    }
}

}  // namespace

void launch_column_scan(Ctx& C, uint32_t* table, int64_t n_rows, const int64_t* d_row_begin, int n_tensors,
                        const int64_t* d_chunk_begin, int64_t n_chunks, uint32_t* chunk_sums, uint64_t* totals,
                        cudaStream_t s) {
    (void)n_rows;
    if (n_chunks == 0) return;
    { KernelScope ks_(C, "k_chunk_sums", s);
    k_chunk_sums<<<unsigned(n_chunks), 256, 0, s>>>(table, d_row_begin, n_tensors, d_chunk_begin, chunk_sums);
    }
    { KernelScope ks_(C, "k_chunk_scan", s);
    k_chunk_scan<<<unsigned(n_tensors), 256, 0, s>>>(d_chunk_begin, chunk_sums, totals);
    }
    { KernelScope ks_(C, "k_chunk_rescan", s);
    k_chunk_rescan<<<unsigned(n_chunks), 256, 0, s>>>(table, d_row_begin, n_tensors, d_chunk_begin, chunk_sums);
    }
}

size_t exclusive_scan_tmp_elems(int64_t n) { return size_t((n + SCAN_TILE - 1) / SCAN_TILE) + 1; }

void launch_exclusive_scan_u64(Ctx& C, uint64_t* data, int64_t n, uint64_t* block_tmp, uint64_t* d_total, cudaStream_t s) {
    const int64_t m = (n + SCAN_TILE - 1) / SCAN_TILE;
    if (n == 0) {
        cudaMemsetAsync(d_total, 0, sizeof(uint64_t), s);
        return;
    }
    { KernelScope ks_(C, "k_scan_reduce", s);
    k_scan_reduce<<<unsigned(m), SCAN_T, 0, s>>>(data, n, block_tmp);
    }
    { KernelScope ks_(C, "k_scan_top", s);
    k_scan_top<<<1, SCAN_T, 0, s>>>(block_tmp, m, d_total);
    }
    { KernelScope ks_(C, "k_scan_down", s);
    k_scan_down<<<unsigned(m), SCAN_T, 0, s>>>(data, n, block_tmp);
    }
}

}  // namespace crx
