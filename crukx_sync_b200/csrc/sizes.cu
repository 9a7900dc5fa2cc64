// Statistics behind the update-size comparison of the reference's bench/compare.py (its raw,
// sparserl and ctxfree columns, bench/compare.py:56-100 of crukx-sync), computed on the device in
// one pass over prev and cur.  Per changed element, in index order per tensor (the reference's
// torch.nonzero(a != b)):
//   * the new value's and the xor value's 16-bit patterns, counted in two 65536-bin histograms;
//   * the gap to the tensor's previous change (first change: its index), counted by bit length
//     (64 bins) with the sum of max(bit length - 1, 0) beside it;
//   * whether the position delta (gap + 1; first change: its index) needs more than 16 bits.
// The host turns the histograms into sizes with the reference's own formulas (order-0 entropies
// over the histograms in ascending value order).
//
//   k_size_tile   one CTA per tile of SZ_TILE elements of one tensor: each lane walks 32
//                 consecutive elements; a change's gap comes from the lane's previous change, or
//                 from the lanes and warps before it (max-scans of the last change index); the
//                 tile's first change is left to k_size_link, the tile records its first and last
//   k_size_link   one thread per tile: its first change against the last change of the nearest
//                 earlier tile of the same tensor that has one
#include <cstring>
#include <string>
#include <vector>

#include "capi_internal.h"
#include "common.cuh"

namespace crx {

namespace {

constexpr int SZ_THREADS = 256;
constexpr int SZ_TILE = SZ_THREADS * 32;   // 8192 elements per tile
constexpr int SZ_CLS = 64;                 // bit-length bins

// stats layout (u64 words): [0] changes, [1] escapes, [2] mantissa bits, [3, 3 + 64) bit-length
// histogram, then the new-value histogram (65536) and the xor histogram (65536)
constexpr int W_CHANGES = 0, W_ESC = 1, W_MANT = 2, W_CLS = 3, W_VAL = W_CLS + SZ_CLS, W_XOR = W_VAL + 65536;
constexpr int W_TOTAL = W_XOR + 65536;

struct SzTensor {
    const int16_t* prev;
    const int16_t* cur;
    int64_t numel;
    int64_t tile_begin;
};

__device__ __forceinline__ int tensor_of_tile(const SzTensor* T, int nT, int64_t s) {
    int lo = 0, hi = nT - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (T[mid].tile_begin <= s) lo = mid; else hi = mid - 1;
    }
    return lo;
}

__device__ __forceinline__ int bit_length(uint64_t g) { return g ? 64 - __clzll(static_cast<long long>(g)) : 0; }

__global__ void __launch_bounds__(SZ_THREADS) k_size_tile(const SzTensor* __restrict__ T, int nT,
                                                          unsigned long long* __restrict__ stats,
                                                          int64_t* __restrict__ tfirst, int64_t* __restrict__ tlast) {
    __shared__ unsigned long long cls[SZ_CLS];
    __shared__ int64_t wlast[SZ_THREADS / 32];
    __shared__ int64_t wfirst[SZ_THREADS / 32];
    __shared__ unsigned long long red[3];
    const int64_t s = blockIdx.x;
    const int t = tensor_of_tile(T, nT, s);
    const SzTensor tt = T[t];
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    if (tid < SZ_CLS) cls[tid] = 0;
    if (tid < 3) red[tid] = 0;
    const int64_t base = (s - tt.tile_begin) * SZ_TILE + int64_t(tid) * 32;   // this lane's 32 elements
    const int n = int(tmax<int64_t>(0, tmin<int64_t>(32, tt.numel - base)));
    const int16_t* pa = tt.prev + base;
    const int16_t* pb = tt.cur + base;
    uint32_t chg = 0;   // bit k: element base + k changed
    if (n == 32 && ((reinterpret_cast<uintptr_t>(pa) | reinterpret_cast<uintptr_t>(pb)) & 15) == 0) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint4 a = reinterpret_cast<const uint4*>(pa)[c], b = reinterpret_cast<const uint4*>(pb)[c];
            const uint32_t x[4] = {a.x ^ b.x, a.y ^ b.y, a.z ^ b.z, a.w ^ b.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                chg |= ((x[h] & 0xFFFFu) ? 1u : 0u) << (8 * c + 2 * h);
                chg |= ((x[h] >> 16) ? 1u : 0u) << (8 * c + 2 * h + 1);
            }
        }
    } else {
        for (int k = 0; k < n; ++k) chg |= (pa[k] != pb[k] ? 1u : 0u) << k;
    }
    // the last change of every earlier lane of the tile (max-scan), and whether the lane has any
    int64_t last = chg ? base + 31 - __clz(chg) : -1;
    int64_t incl = last;
    for (int o = 1; o < 32; o <<= 1) {
        const int64_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl = tmax(incl, y);
    }
    int64_t before = __shfl_up_sync(0xffffffffu, incl, 1);
    if (lane == 0) before = -1;
    const int64_t first = chg ? base + __ffs(chg) - 1 : -1;
    // first change of the warp: the lowest lane with one
    const uint32_t has = __ballot_sync(0xffffffffu, chg != 0);
    const int64_t wf = __shfl_sync(0xffffffffu, first, has ? __ffs(has) - 1 : 0);
    if (lane == 31) wlast[w] = incl;
    if (lane == 0) wfirst[w] = has ? wf : -1;
    __syncthreads();
    if (before < 0) {   // an earlier warp of the tile
        for (int ww = w - 1; ww >= 0 && before < 0; --ww) before = wlast[ww];
    }
    unsigned long long mant = 0, esc = 0, nch = 0;
    int64_t prev_i = before;
    for (uint32_t m = chg; m; m &= m - 1) {
        const int k = __ffs(m) - 1;
        const int64_t i = base + k;
        const uint32_t a = uint16_t(pa[k]), b = uint16_t(pb[k]);
        atomicAdd(&stats[W_VAL + b], 1ull);
        atomicAdd(&stats[W_XOR + (a ^ b)], 1ull);
        ++nch;
        if (prev_i >= 0) {   // the tile's first change (prev_i < 0) is linked by k_size_link
            const uint64_t gap = uint64_t(i - prev_i - 1);
            const int c = bit_length(gap);
            atomicAdd(&cls[c], 1ull);
            mant += uint64_t(c > 1 ? c - 1 : 0);
            esc += gap + 1 > 0xFFFFu ? 1u : 0u;
        }
        prev_i = i;
    }
    for (int o = 16; o; o >>= 1) {
        mant += __shfl_xor_sync(0xffffffffu, mant, o);
        esc += __shfl_xor_sync(0xffffffffu, esc, o);
        nch += __shfl_xor_sync(0xffffffffu, nch, o);
    }
    if (lane == 0) {
        atomicAdd(&red[0], nch);
        atomicAdd(&red[1], esc);
        atomicAdd(&red[2], mant);
    }
    __syncthreads();
    if (tid < SZ_CLS && cls[tid]) atomicAdd(&stats[W_CLS + tid], cls[tid]);
    if (tid < 3 && red[tid]) atomicAdd(&stats[tid], red[tid]);
    if (tid == 0) {
        int64_t f = -1, l = -1;
        for (int ww = 0; ww < SZ_THREADS / 32 && f < 0; ++ww) f = wfirst[ww];
        for (int ww = SZ_THREADS / 32 - 1; ww >= 0 && l < 0; --ww) l = wlast[ww];
        tfirst[s] = f;
        tlast[s] = l;
    }
}

__global__ void k_size_link(const SzTensor* __restrict__ T, int nT, int64_t n_tiles, unsigned long long* __restrict__ stats,
                            const int64_t* __restrict__ tfirst, const int64_t* __restrict__ tlast) {
    const int64_t s = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (s >= n_tiles || tfirst[s] < 0) return;
    const int t = tensor_of_tile(T, nT, s);
    int64_t pred = -1;
    for (int64_t q = s - 1; q >= T[t].tile_begin && pred < 0; --q) pred = tlast[q];
    const int64_t i = tfirst[s];
    // the reference: gaps = diff(i, prepend=-1) - 1 and d = diff(i, prepend=0), so the tensor's
    // first change has gap = d = its index, every later one d = gap + 1
    const uint64_t gap = pred < 0 ? uint64_t(i) : uint64_t(i - pred - 1);
    const uint64_t d = pred < 0 ? uint64_t(i) : gap + 1;
    const int c = bit_length(gap);
    atomicAdd(&stats[W_CLS + c], 1ull);
    if (c > 1) atomicAdd(&stats[W_MANT], uint64_t(c - 1));
    if (d > 0xFFFFu) atomicAdd(&stats[W_ESC], 1ull);
}

}  // namespace

int size_stats_words() { return W_TOTAL; }

Status size_stats_impl(Ctx& C, int nT, const int16_t* const* prev, const int16_t* const* cur, const int64_t* numel,
                       cudaStream_t st, uint64_t* out, std::string* err) {
    std::vector<SzTensor> T;
    int64_t tiles = 0;
    for (int t = 0; t < nT; ++t) {
        if (numel[t] < 0) { *err = "negative numel"; return kBadArgument; }
        if (numel[t] >= (int64_t(1) << 32)) { *err = "tensors of 2^32 or more elements are not supported"; return kValueError; }
        if (numel[t] == 0) continue;
        T.push_back(SzTensor{prev[t], cur[t], numel[t], tiles});
        tiles += (numel[t] + SZ_TILE - 1) / SZ_TILE;
    }
    std::memset(out, 0, sizeof(uint64_t) * W_TOTAL);
    if (T.empty()) return kOk;
    const int nt = int(T.size());
    CRX_CUDA(ensure_dev(C.b[S_SZ_STATS], sizeof(uint64_t) * W_TOTAL, st));
    CRX_CUDA(ensure_dev(C.b[S_SZ_TILES], sizeof(SzTensor) * size_t(nt) + 16 * size_t(tiles), st));
    auto* stats = static_cast<unsigned long long*>(C.b[S_SZ_STATS].p);
    auto* dT = static_cast<SzTensor*>(C.b[S_SZ_TILES].p);
    auto* tfirst = reinterpret_cast<int64_t*>(dT + nt);
    auto* tlast = tfirst + tiles;
    CRX_CUDA(ensure_host(C, std::max(sizeof(SzTensor) * size_t(nt), sizeof(uint64_t) * W_TOTAL), st));
    std::memcpy(C.host, T.data(), sizeof(SzTensor) * size_t(nt));
    CRX_CUDA(cudaMemcpyAsync(dT, C.host, sizeof(SzTensor) * size_t(nt), cudaMemcpyHostToDevice, st));
    CRX_CUDA(cudaMemsetAsync(stats, 0, sizeof(uint64_t) * W_TOTAL, st));
    { KernelScope ks_(C, "k_size_tile", st);
    k_size_tile<<<unsigned(tiles), SZ_THREADS, 0, st>>>(dT, nt, stats, tfirst, tlast);
    }
    CRX_CUDA(cudaGetLastError());
    { KernelScope ks_(C, "k_size_link", st);
    k_size_link<<<unsigned((tiles + 255) / 256), 256, 0, st>>>(dT, nt, tiles, stats, tfirst, tlast);
    }
    CRX_CUDA(cudaGetLastError());
    CRX_CUDA(cudaMemcpyAsync(C.host, stats, sizeof(uint64_t) * W_TOTAL, cudaMemcpyDeviceToHost, st));
    CRX_CUDA(cudaStreamSynchronize(st));
    std::memcpy(out, C.host, sizeof(uint64_t) * W_TOTAL);
    return kOk;
}

}  // namespace crx
