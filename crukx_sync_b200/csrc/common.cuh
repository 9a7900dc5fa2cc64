// Shared device code for the crukx-sync B200 kernels (sm_100a).
//
// Layout conventions used by every kernel:
//   * A weight tensor is a flat array of int16 bit patterns (bf16 bits).  Its old exponent is
//     (bits >> 7) & 0xFF (docs/FORMAT.md:21-24 of the reference).
//   * Tensors are cut into SUB_N-element sub-tiles; SUPER sub-tiles form a super-tile, which is
//     what one CTA walks.  Per-super-tile exponent histograms [n_super][256] (u32) are scanned
//     per tensor to give every super-tile the number of same-exponent elements before it, which
//     turns "stable rank by old exponent" (the reference's argsort, codec.py:124-147) into a
//     histogram + scan + in-CTA counting pass.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace crx {

struct Ctx;

constexpr int SUB_N = 8192;                  // elements per sub-tile (held in shared memory)
constexpr int SUPER = 32;                    // sub-tiles per super-tile
constexpr int64_t SUPER_N = int64_t(SUB_N) * SUPER;   // 2^18: ranks local to a super-tile fit 18 bits
constexpr int RANK_THREADS = 512;            // 16 warps; each warp owns SUB_N/16 = 512 elements
constexpr int RANK_WARPS = RANK_THREADS / 32;
constexpr int WARP_SPAN = SUB_N / RANK_WARPS;
constexpr int CHUNKS_PER_WARP = WARP_SPAN / 32;

// Error bits reduced into one status word on the device.
enum : uint32_t {
    ERR_DECODE = 1u << 0,       // a block did not decode exactly to its length
    ERR_RANGE = 1u << 1,        // a change lies outside its exponent group
    ERR_RECORD_OVERFLOW = 1u << 2,
    ERR_BLOCK_TOO_LONG = 1u << 3,
    ERR_INTERNAL = 1u << 4,
};

__host__ __device__ __forceinline__ uint64_t splitmix_weight(uint64_t i) {
    // w_i = splitmix64(i) | 1 with splitmix64 seeded by i + 1 (reference docs/FORMAT.md:61-64)
    uint64_t z = (i + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return (z ^ (z >> 31)) | 1ull;
}

template <class T>
__host__ __device__ __forceinline__ T tmin(T a, T b) { return a < b ? a : b; }
template <class T>
__host__ __device__ __forceinline__ T tmax(T a, T b) { return a < b ? b : a; }

__device__ __forceinline__ uint32_t lanemask_lt() {
    uint32_t m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

__device__ __forceinline__ uint32_t bswap32(uint32_t x) { return __byte_perm(x, 0, 0x0123); }

// Start moving [p, p + bytes) from HBM into L2 (one bulk prefetch, no data returned).  Only the
// 16-byte-aligned interior is requested, so the range never reaches past the caller's buffer.
__device__ __forceinline__ void prefetch_l2(const void* p, size_t bytes) {
    const uintptr_t lo = (reinterpret_cast<uintptr_t>(p) + 15) & ~uintptr_t(15);
    const uintptr_t hi = (reinterpret_cast<uintptr_t>(p) + bytes) & ~uintptr_t(15);
    if (hi > lo)
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(lo), "r"(uint32_t(hi - lo)) : "memory");
}

// Stable rank of this lane's key (0..255) among the same-key lanes of this chunk and of every
// earlier chunk this warp ranked with the same counters.  The lowest lane of each peer group adds
// the group's size to the warp's counter with one shared-memory atomic and broadcasts the old
// value; the next chunk's atomics are issued only after that value came back, so each counter
// sees its updates in chunk order.  Inactive lanes (act = false) get a key no other lane has.
__device__ __forceinline__ uint32_t warp_rank(uint32_t* cnt, uint32_t key, bool act, uint32_t lt, int lane) {
    const uint32_t peers = __match_any_sync(0xffffffffu, act ? key : 0x100u + uint32_t(lane));
    const int leader = __ffs(peers) - 1;
    uint32_t base = 0;
    if (act && lane == leader) base = atomicAdd(&cnt[key], uint32_t(__popc(peers)));
    base = __shfl_sync(0xffffffffu, base, leader);
    return base + __popc(peers & lt);
}

__device__ __forceinline__ int exp_of(uint32_t bits16) { return int((bits16 >> 7) & 0xFFu); }

// Sum of a u64 over the CTA into *dst with one atomic (all threads must call).
template <int NT>
__device__ __forceinline__ void block_add_u64(uint64_t v, unsigned long long* dst, uint64_t* red) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    if (w == 0) {
        v = l < NT / 32 ? red[l] : 0;
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (l == 0 && v) atomicAdd(dst, (unsigned long long)v);
    }
    __syncthreads();
}

// ------------------------------------------------------------------ per-tensor column scans
// Tables are [rows][256] u32, rows of one tensor contiguous: rows [row_begin[t], row_begin[t+1]).
// scan_* turns each column of each tensor into its exclusive prefix (in place) and writes the
// tensor's column totals to totals[t][256].  Three launches: chunk sums, chunk scan, rescan.

constexpr int SCAN_CHUNK = 32;  // rows per chunk

void launch_column_scan(Ctx& C, uint32_t* table, int64_t n_rows, const int64_t* d_row_begin /* n_t+1 */,
                        int n_tensors, const int64_t* d_chunk_begin /* n_t+1, chunks per tensor */,
                        int64_t n_chunks, uint32_t* chunk_sums /* n_chunks*256 */, uint64_t* totals /* n_t*256 */,
                        cudaStream_t s);

// Generic exclusive scan of n u64 values (in place), total to *d_total.
void launch_exclusive_scan_u64(Ctx& C, uint64_t* data, int64_t n, uint64_t* block_tmp, uint64_t* d_total, cudaStream_t s);
size_t exclusive_scan_tmp_elems(int64_t n);

}  // namespace crx
