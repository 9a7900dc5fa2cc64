// Encoder: bf16 prev/cur -> crukx-sync update bytes (wire format version 2), byte-identical to
// the reference's encode_update (src/crukx_sync/codec.py:278-420, wire.py:64-89).
//
// Pipeline (one CUDA stream, four small host round trips: the record count, the group table,
// the statistics and the block lengths; a device result is then returned without waiting):
//   k_enc_rank     one pass over prev+cur.  Per super-tile: old-exponent histogram and changed
//                  count per exponent; every changed element becomes a record holding its rank
//                  among same-exponent elements and among same-exponent changes, both local to
//                  the super-tile.  Checksum delta (and the full checksum when no cache) fused.
//                  Replaces the reference's stable argsort ranking (codec.py:124-194).
//   column scans   per tensor and exponent, exclusive prefix over super-tiles (scan.cu).
//   k_groups       (tensor, exponent) groups in the reference's order, change offsets.
//   k_place        records -> group order: local index and old|new bits per change.
//   k_r0 / k_stats Golomb-Rice candidate costs per group (codec.py:268-275) and the
//                  (exponent, zigzag residual) symbol histogram (codec.py:355-367).
//   host           Rice choice, length-limited Huffman per exponent (codec.py:71-111, 369-392).
//   k_pack_slots   one warp per 256-change block assembles its bits MSB-first (codec.py:218-257)
//                  from bit 0 of the block's slot and records its length (codec.py:411-416);
//                  an exclusive scan of the lengths gives every block's offset.
//   k_compact      every block's slot shifted into place in the payload.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "capi_internal.h"
#include "common.cuh"

namespace crx {

namespace {

constexpr uint32_t FULL = 0xffffffffu;
constexpr int DENSE_SYM = 64;          // residual symbols below this are counted per CTA in smem
constexpr int STATS_PER_CTA = 8192;    // changes per k_stats CTA
constexpr int STATS_LOCAL_GROUPS = 64; // groups a k_stats CTA accumulates in smem

struct EncTensor {
    const int16_t* prev;
    const int16_t* cur;
    int64_t numel;
    int64_t super_begin;
    int32_t want_full;
    int32_t pad;
};

__device__ __forceinline__ int tensor_of_super(const EncTensor* T, int nT, int64_t s) {
    int lo = 0, hi = nT - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (T[mid].super_begin <= s) lo = mid; else hi = mid - 1;
    }
    return lo;
}

__device__ __forceinline__ int64_t group_of(const uint64_t* __restrict__ start, int64_t ng, uint64_t j) {
    int64_t lo = 0, hi = ng - 1;             // last g with start[g] <= j
    while (lo < hi) {
        const int64_t mid = (lo + hi + 1) >> 1;
        if (start[mid] <= j) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// ------------------------------------------------------------------ k_enc_rank
//
// Stable rank by old exponent without a sort: every lane takes a run of 32 elements and marks, per
// exponent of a 16-exponent window ending at the sub-tile's largest old exponent, which of its
// elements carry it (one 32-bit mask per window row).  An element's rank among the equal exponents
// is then the running total of earlier sub-tiles + earlier warps + earlier lanes (prefixes of the
// masks' population counts) + the set bits of its own mask below it; the rank among the changed
// ones likewise with the run's changed-bit mask.  Elements below the window (zeros, tiny weights)
// are ranked by warp matching, in index order.

constexpr int ER_THREADS = 256;
constexpr int ER_WARPS = ER_THREADS / 32;
constexpr int ER_MINB = 6;                   // CTAs per SM (40 registers a thread, 37 KB of shared memory)
constexpr int ER_SPAN = 1024;                // elements per warp
constexpr int ER_SUB = ER_SPAN * ER_WARPS;   // elements per sub-tile
constexpr int ER_RUN = ER_SPAN / 32;         // 32 per lane
constexpr int WIN = 16;                      // window rows
constexpr int WLIST = 256;                   // in-window changes of a span listed for the CTA's record writes
static_assert(SUPER_N % ER_SUB == 0 && ER_SUB <= 0xFFFF, "whole sub-tiles per super-tile; 16-bit packed counts");

struct RankSmem {
    // old exponent bytes; run r (32 elements) in words 9r..9r+7.  Once a warp has marked its runs it
    // reuses their words for its lane prefixes (pre_of): exclusive prefixes of the rows' counts at
    // even lanes, all | changed << 16 (first every lane's counts as a halfword, in the same 64 bytes
    // a row).  Exponents needed later are taken from the elements' bits instead.
    uint32_t texp[ER_SUB / 32 * 9];
    uint32_t chm[ER_SUB / 32];            // changed bit of every element, one word per run
    uint32_t msk[ER_WARPS][WIN + 1][32];  // per lane and window row: its run's elements of that exponent (row WIN: below)
    uint32_t wwin[ER_WARPS][WIN];         // per-warp row totals, then warp bases (all | changed << 16)
    uint32_t ocnt[256];                   // below-window counts per exponent, all | changed << 16
    uint32_t runA[256], runC[256];        // super-tile running totals
    uint32_t tot[256];                    // this sub-tile's totals, all | changed << 16
    uint16_t cstart[256];                 // exclusive scan of the changed totals: records sorted by exponent
    uint16_t wl[ER_WARPS][WLIST];         // a warp's in-window changes (sub-tile indices)
    uint32_t wcnt[ER_WARPS];              // listed changes per warp, then (lbase) their exclusive prefix
    uint32_t lbase[ER_WARPS + 1];
    uint32_t oowm[ER_WARPS];              // per warp: its runs holding below-window elements
    unsigned long long rec_base;
    int emax[2];                          // largest old exponent, alternating between sub-tiles
    uint64_t red[ER_WARPS];
};

// warp w's lane prefixes: [WIN][16] words in the exponent words of its own 32 runs
__device__ __forceinline__ uint32_t (*pre_of(RankSmem& S, int w))[16] {
    return reinterpret_cast<uint32_t(*)[16]>(&S.texp[w * 32 * 9]);
}
static_assert(offsetof(RankSmem, texp) % 16 == 0 && (32 * 9 * 4) % 16 == 0, "16-byte prefix pieces");
static_assert(32 * 9 >= WIN * 16, "a warp's lane prefixes fit in its runs' exponent words");

__device__ __forceinline__ void put_record(uint64_t* rec_key, uint32_t* rec_val, uint64_t rec_cap, uint64_t j, int64_t s,
                                           uint32_t rankA, uint32_t rankC, uint32_t x) {
    if (j < rec_cap) {
        rec_key[j] = (uint64_t(s) << 36) | (uint64_t(rankA) << 18) | uint64_t(rankC);
        rec_val[j] = x;
    }
}

// (new - old) * w(position), the change's term of the checksum delta (codec.py:325)
__device__ __forceinline__ uint64_t change_delta(uint32_t x, int64_t pos) {
    return (uint64_t(x >> 16) - uint64_t(x & 0xFFFFu)) * splitmix_weight(uint64_t(pos));
}

// warp_rank with counters packed as A | C << 16: adds to the half selected by `shift`
__device__ __forceinline__ uint32_t warp_rank_packed(uint32_t* cnt, uint32_t key, bool act, int shift, uint32_t lt, int lane) {
    const uint32_t peers = __match_any_sync(0xffffffffu, act ? key : 0x100u + uint32_t(lane));
    const int leader = __ffs(peers) - 1;
    uint32_t base = 0;
    if (act && lane == leader) base = atomicAdd(&cnt[key], uint32_t(__popc(peers)) << shift);
    base = __shfl_sync(0xffffffffu, base, leader);
    return ((base >> shift) & 0xFFFFu) + __popc(peers & lt);
}

__device__ __forceinline__ bool changed_bits(uint32_t x) { return ((x ^ (x >> 16)) & 0xFFFFu) != 0; }

// warp 0: cstart[e] = number of this sub-tile's changed elements with a smaller exponent, so each
// sub-tile's records land sorted by (exponent, rank) and k_place writes runs of consecutive changes
__device__ __forceinline__ void scan_change_starts(const uint32_t* tot, uint16_t* cstart, int lane) {
    uint32_t v[8], sum = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) { v[k] = tot[lane * 8 + k] >> 16; sum += v[k]; }
    uint32_t incl = sum;
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    uint32_t run = incl - sum;
#pragma unroll
    for (int k = 0; k < 8; ++k) { cstart[lane * 8 + k] = run; run += v[k]; }
}

__global__ void __launch_bounds__(ER_THREADS, ER_MINB)
k_enc_rank(const EncTensor* __restrict__ T, int nT, uint64_t* __restrict__ rec_key, uint32_t* __restrict__ rec_val,
           uint64_t rec_cap, unsigned long long* __restrict__ counters, uint32_t* __restrict__ HS,
           uint32_t* __restrict__ CS, unsigned long long* __restrict__ chk_delta, unsigned long long* __restrict__ chk_full) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    RankSmem& S = *reinterpret_cast<RankSmem*>(smem_raw);
    const int64_t s = blockIdx.x;
    const int t = tensor_of_super(T, nT, s);
    const EncTensor tt = T[t];
    const int64_t e_begin = (s - tt.super_begin) * SUPER_N;
    const int64_t e_end = tmin(tt.numel, e_begin + SUPER_N);
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const uint32_t lt = lanemask_lt();
    const int span0 = w * ER_SPAN;
    uint64_t full = 0, delta = 0;   // checksum of cur (no cache) / checksum delta of the changes

    for (int e = tid; e < 256; e += ER_THREADS) {
        S.runA[e] = 0;
        S.runC[e] = 0;
    }
    if (tid == 0) { S.emax[0] = 0; S.emax[1] = 0; }
    __syncthreads();

    int it = 0;
    for (int64_t base = e_begin; base < e_end; base += ER_SUB, ++it) {
        const int n = int(tmin<int64_t>(ER_SUB, e_end - base));
        const int16_t* pp = tt.prev + base;
        const int16_t* cp = tt.cur + base;
        // the (prev, cur) bits of sub-tile element i; only changed elements are read back
        auto bits_of = [&](int i) { return uint32_t(uint16_t(pp[i])) | (uint32_t(uint16_t(cp[i])) << 16); };
        if (base + ER_SUB < e_end && (tid & 31) == 0 && w < 2) {   // the next sub-tile streams into L2 meanwhile
            const size_t nb = size_t(tmin<int64_t>(ER_SUB, e_end - base - ER_SUB)) * 2;
            prefetch_l2((w ? cp : pp) + ER_SUB, nb);
        }
        // ---- stage old exponents (bytes) and changed bits; largest old exponent
        uint32_t mx = 0;
        if (n == ER_SUB && ((reinterpret_cast<uintptr_t>(pp) | reinterpret_cast<uintptr_t>(cp)) & 15) == 0) {
            const uint4* pv = reinterpret_cast<const uint4*>(pp);
            const uint4* cv = reinterpret_cast<const uint4*>(cp);
#pragma unroll
            for (int k = 0; k < ER_SUB / 8 / ER_THREADS; ++k) {
                const int v = tid + k * ER_THREADS;     // elements 8v .. 8v+7: run v/4, quarter v%4
                const uint4 a = pv[v];
                const uint4 b = cv[v];
                const uint32_t x0 = (a.x >> 7) & 0x00FF00FFu, x1 = (a.y >> 7) & 0x00FF00FFu;
                const uint32_t x2 = (a.z >> 7) & 0x00FF00FFu, x3 = (a.w >> 7) & 0x00FF00FFu;
                const int r = v >> 2, q = v & 3;
                S.texp[r * 9 + 2 * q] = __byte_perm(x0, x1, 0x6420);
                S.texp[r * 9 + 2 * q + 1] = __byte_perm(x2, x3, 0x6420);
                mx = __vimax3_u16x2(mx, __vimax3_u16x2(x0, x1, x2), x3);   // exponents in 16-bit halves
                // changed bits of the 8 elements (low half of a word first), then the run's 32.
                // nzh: bit 15 / bit 31 set where the low / high 16-bit half is nonzero (the masked
                // halves plus 0x7FFF carry into bit 15 exactly when nonzero, never into bit 16)
                auto nzh = [](uint32_t x) { return (((x & 0x7FFF7FFFu) + 0x7FFF7FFFu) | x) & 0x80008000u; };
                const uint32_t c0 = nzh(a.x ^ b.x), c1 = nzh(a.y ^ b.y), c2 = nzh(a.z ^ b.z), c3 = nzh(a.w ^ b.w);
                // word h's two bits (15, 31) to bits 2h and 16 + 2h, then the high ones down to 2h + 1
                const uint32_t cx = (c0 >> 15) | (c1 >> 13) | (c2 >> 11) | (c3 >> 9);
                uint32_t cb = (cx | (cx >> 15)) & 0xFFu;
                cb <<= 8 * q;
                cb |= __shfl_xor_sync(FULL, cb, 1);
                cb |= __shfl_xor_sync(FULL, cb, 2);
                if (q == 0) S.chm[r] = cb;
                if (tt.want_full) {
                    const uint32_t cw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
                    for (int h = 0; h < 4; ++h) {
                        full += uint64_t(cw[h] & 0xFFFFu) * splitmix_weight(uint64_t(base + 8 * v + 2 * h));
                        full += uint64_t(cw[h] >> 16) * splitmix_weight(uint64_t(base + 8 * v + 2 * h + 1));
                    }
                }
            }
            mx = tmax(mx & 0xFFFFu, mx >> 16);
        } else {
            uint8_t* tb = reinterpret_cast<uint8_t*>(S.texp);
            for (int k = tid; k < ER_SUB / 32; k += ER_THREADS) S.chm[k] = 0;
            __syncthreads();
            for (int i = tid; i < n; i += ER_THREADS) {
                const uint32_t x = bits_of(i);
                const uint32_t e = (x >> 7) & 0xFFu;
                tb[(i >> 5) * 36 + (i & 31)] = uint8_t(e);
                if (changed_bits(x)) atomicOr(&S.chm[i >> 5], 1u << (i & 31));
                mx = tmax(mx, e);
                if (tt.want_full) full += uint64_t(x >> 16) * splitmix_weight(uint64_t(base + i));
            }
        }
        mx = __reduce_max_sync(FULL, mx);
        if (lane == 0) atomicMax(&S.emax[it & 1], int(mx));
        {   // this warp's masks to zero
            static_assert(sizeof(S.msk[0]) % 16 == 0 && offsetof(RankSmem, msk) % 16 == 0, "uint4 zeroing");
            uint4* m4 = reinterpret_cast<uint4*>(&S.msk[w][0][0]);
#pragma unroll
            for (int k = lane; k < int(sizeof(S.msk[0]) / 16); k += 32) m4[k] = make_uint4(0, 0, 0, 0);
        }
        __syncthreads();
        if (tid == 0) S.emax[(it + 1) & 1] = 0;   // the next sub-tile's (its atomics come after later barriers)
        const uint32_t ebase = uint32_t(tmax(S.emax[it & 1] - (WIN - 1), 0));
        auto row_of = [&](uint32_t e) { return tmin(e - ebase, uint32_t(WIN)); };   // below: wraps to WIN
        auto exp_at = [&](int i) { return (uint32_t(uint16_t(pp[i])) >> 7) & 0xFFu; };   // (from L1/L2: just staged)
        const int span_n = tmax(0, tmin(ER_SPAN, n - span0));
        const int vn = tmax(0, tmin(ER_RUN, span_n - lane * ER_RUN));
        // ---- lane walk: for every window row, which elements of the lane's run carry it
        {
            const uint32_t* ew = &S.texp[(w * 32 + lane) * 9];
            uint32_t* mine = &S.msk[w][0][lane];
            if (vn == ER_RUN) {
                // two exponent bytes per word at once: per 16-bit half, (e - ebase) mod 2^16 then
                // the minimum with 16 (below the window wraps to 65280 and up) -- row_of for both
                const uint32_t nb = ((0x10000u - ebase) & 0xFFFFu) * 0x00010001u;
#pragma unroll
                for (int g = 0; g < ER_RUN / 4; ++g) {
                    const uint32_t eb = ew[g];
                    const uint32_t r02 = __viaddmin_u16x2(eb & 0x00FF00FFu, nb, 0x00100010u);
                    const uint32_t r13 = __viaddmin_u16x2(__byte_perm(eb, 0u, 0x4341), nb, 0x00100010u);
                    atomicOr(mine + (r02 & 0xFFFFu) * 32, 1u << (4 * g));
                    atomicOr(mine + (r13 & 0xFFFFu) * 32, 2u << (4 * g));
                    atomicOr(mine + (r02 >> 16) * 32, 4u << (4 * g));
                    atomicOr(mine + (r13 >> 16) * 32, 8u << (4 * g));
                }
            } else {
                for (int k = 0; k < vn; ++k) mine[row_of((ew[k >> 2] >> (8 * (k & 3))) & 0xFFu) * 32] |= 1u << k;
            }
        }
        __syncwarp();
        const uint32_t outm = S.msk[w][WIN][lane];              // the run's elements below the window
        const uint32_t oowm = __ballot_sync(FULL, outm != 0);
        if (lane == 0) S.oowm[w] = oowm;
        const uint32_t cm = S.chm[w * 32 + lane];
        // this span's in-window changes, listed in index order for the CTA's record writes (a lane
        // keeps what does not fit)
        const uint32_t mine = cm & ~outm;
        uint32_t lpos = __popc(mine);
        {
            uint32_t incl = lpos;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(FULL, incl, o);
                if (lane >= o) incl += y;
            }
            lpos = incl - lpos;
            uint32_t at = lpos;
            for (uint32_t b = mine; b && at < uint32_t(WLIST); b &= b - 1, ++at)
                S.wl[w][at] = uint16_t(span0 + lane * 32 + (__ffs(b) - 1));
            if (lane == 31) S.wcnt[w] = tmin(incl, uint32_t(WLIST));
        }
        // ---- lane prefixes per window row of (all, changed) counts.  Every lane writes its run's two
        //      counts of each row as a halfword (all | changed << 8), into the row's prefix slots;
        //      then lane 2d + h turns the 32 bytes of row d's lanes 16h..16h+15 in place into the
        //      exclusive prefixes of its even lanes (all | changed << 16): a word holds two lanes.
        {
            uint32_t (*const pw)[16] = pre_of(S, w);
            uint16_t* const ch = reinterpret_cast<uint16_t*>(&pw[0][0]);
#pragma unroll
            for (int d = 0; d < WIN; ++d) {
                const uint32_t m = S.msk[w][d][lane];
                ch[d * 32 + lane] = uint16_t(uint32_t(__popc(m)) | (uint32_t(__popc(m & cm)) << 8));
            }
            __syncwarp();
            const int d = lane >> 1, h = lane & 1;
            uint4* const q = reinterpret_cast<uint4*>(&pw[d][8 * h]);   // this lane's 32 bytes, in and out
            const uint4 c0 = q[0], c1 = q[1];
            const uint32_t wd[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
            uint32_t run = 0, out[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {   // bytes (a0, c0, a1, c1): add a0 + a1 | (c0 + c1) << 16
                out[k] = run;
                run += __byte_perm(wd[k], 0u, 0x4140) + __byte_perm(wd[k], 0u, 0x4342);
            }
            const uint32_t lo = __shfl_xor_sync(FULL, run, 1);   // at odd lanes: the first 16 lanes' totals
            if (h) {
#pragma unroll
                for (int k = 0; k < 8; ++k) out[k] += lo;
                S.wwin[w][d] = run + lo;
            }
            q[0] = make_uint4(out[0], out[1], out[2], out[3]);
            q[1] = make_uint4(out[4], out[5], out[6], out[7]);
        }
        const bool any_out = __syncthreads_or(oowm != 0);
        // elements below the window, whole sub-tile in index order, by one warp (they are rare):
        // ranks (all, changed) by warp matching; the second pass writes the changes' records
        auto rank_outside = [&](bool write) {
            for (int k = lane; k < 256; k += 32) S.ocnt[k] = 0;
            __syncwarp();
            const uint64_t rb = S.rec_base;
            for (int ww = 0; ww < ER_WARPS; ++ww) {
                const int sn = tmax(0, tmin(ER_SPAN, n - ww * ER_SPAN));
                for (uint32_t m = S.oowm[ww]; m; m &= m - 1) {
                    const int run = __ffs(m) - 1;
                    const int ii = run * ER_RUN + lane;
                    const int i = ww * ER_SPAN + ii;
                    const bool outside = ii < sn && row_of(exp_at(i)) == uint32_t(WIN);
                    const uint32_t e = outside ? exp_at(i) : 0u;
                    const bool ch = outside && ((S.chm[i >> 5] >> (i & 31)) & 1u);
                    const uint32_t rA = warp_rank_packed(S.ocnt, e, outside, 0, lt, lane);
                    const uint32_t rC = warp_rank_packed(S.ocnt, e, ch, 16, lt, lane);
                    if (write && ch) {
                        const uint32_t x = bits_of(i);
                        put_record(rec_key, rec_val, rec_cap, rb + S.cstart[e] + rC, s, S.runA[e] + rA, S.runC[e] + rC, x);
                        delta += change_delta(x, base + i);
                    }
                }
            }
        };
        if (any_out) {   // first pass: the counts
            if (w == 0) rank_outside(false);
            __syncthreads();
        }
        for (int e = tid; e < 256; e += ER_THREADS) {   // warp bases of the window rows and the sub-tile's totals (all | changed << 16)
            uint32_t o = any_out ? S.ocnt[e] : 0u;
            const uint32_t d = uint32_t(e) - ebase;
            if (d < uint32_t(WIN)) {
                uint32_t a = 0;
                for (int ww = 0; ww < ER_WARPS; ++ww) {
                    const uint32_t v = S.wwin[ww][d];
                    S.wwin[ww][d] = a;
                    a += v;
                }
                o += a;
            }
            S.tot[e] = o;
        }
        if (tid == 0) {
            uint32_t r = 0;
            for (int ww = 0; ww < ER_WARPS; ++ww) { S.lbase[ww] = r; r += S.wcnt[ww]; }
            S.lbase[ER_WARPS] = r;
        }
        __syncthreads();
        if (w == 0) {   // record slots: the sub-tile's changes sorted by exponent, one atomic
            scan_change_starts(S.tot, S.cstart, lane);
            __syncwarp();
            if (lane == 31) {
                const uint32_t r = S.cstart[255] + (S.tot[255] >> 16);
                S.rec_base = r ? atomicAdd(&counters[0], (unsigned long long)r) : 0ull;
            }
        }
        __syncthreads();
        if (any_out && w == 0) rank_outside(true);
        // ---- records of the in-window changes: the listed ones by all threads, two at a time (their
        //      bits load together); a lane then writes those of its run that did not fit the list
        {
            const uint64_t rb = S.rec_base;
            auto record = [&](int i, uint32_t x) {   // i: index in the sub-tile
                const int ww = i >> 10, l = (i >> 5) & 31, k = i & 31;
                const uint32_t e = (x >> 7) & 0xFFu;   // the old exponent
                const uint32_t d = e - ebase;
                const uint32_t below = (1u << k) - 1u;
                const uint32_t m = S.msk[ww][d][l];
                const uint32_t c = S.chm[i >> 5];
                uint32_t pr = pre_of(S, ww)[d][l >> 1];   // even lanes' prefixes: an odd lane adds its neighbour's counts
                if (l & 1) {
                    const uint32_t mp = S.msk[ww][d][l - 1];
                    pr += uint32_t(__popc(mp)) | (uint32_t(__popc(mp & S.chm[(i >> 5) - 1])) << 16);
                }
                const uint32_t wb = S.wwin[ww][d];
                const uint32_t rA = (wb & 0xFFFFu) + (pr & 0xFFFFu) + uint32_t(__popc(m & below));
                const uint32_t rC = (wb >> 16) + (pr >> 16) + uint32_t(__popc(m & c & below));
                put_record(rec_key, rec_val, rec_cap, rb + S.cstart[e] + rC, s, S.runA[e] + rA, S.runC[e] + rC, x);
                delta += change_delta(x, base + i);
            };
            auto entry = [&](uint32_t g) {
                int ww = 0;
#pragma unroll
                for (int q = 1; q < ER_WARPS; ++q) ww += S.lbase[q] <= g;
                return int(S.wl[ww][g - S.lbase[ww]]);
            };
            const uint32_t nl = S.lbase[ER_WARPS];
            for (uint32_t g = tid; g < nl; g += 2 * ER_THREADS) {
                const uint32_t g2 = g + ER_THREADS;
                const int i0 = entry(g), i1 = g2 < nl ? entry(g2) : -1;
                const uint32_t x0 = bits_of(i0), x1 = i1 >= 0 ? bits_of(i1) : 0u;
                record(i0, x0);
                if (i1 >= 0) record(i1, x1);
            }
            if (lpos + __popc(mine) > uint32_t(WLIST)) {
                uint32_t at = lpos;
                for (uint32_t b = mine; b; b &= b - 1, ++at) {
                    if (at < uint32_t(WLIST)) continue;
                    const int i = span0 + lane * 32 + (__ffs(b) - 1);
                    record(i, bits_of(i));
                }
            }
        }
        __syncthreads();
        for (int e = tid; e < 256; e += ER_THREADS) {
            S.runA[e] += S.tot[e] & 0xFFFFu;
            S.runC[e] += S.tot[e] >> 16;
        }
    }
    for (int e = tid; e < 256; e += ER_THREADS) {
        HS[s * 256 + e] = S.runA[e];
        CS[s * 256 + e] = S.runC[e];
    }
    block_add_u64<ER_THREADS>(delta, &chk_delta[t], S.red);
    if (tt.want_full) block_add_u64<ER_THREADS>(full, &chk_full[t], S.red);
}

// ------------------------------------------------------------------ groups in reference order

__device__ __forceinline__ uint32_t block_scan_u32(uint32_t v, uint32_t* sh, uint32_t* total) {
    const int l = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    uint32_t x = v;
    for (int o = 1; o < 32; o <<= 1) { const uint32_t y = __shfl_up_sync(FULL, x, o); if (l >= o) x += y; }
    if (l == 31) sh[w] = x;
    __syncthreads();
    if (w == 0) {
        uint32_t q = l < nw ? sh[l] : 0;
        for (int o = 1; o < 32; o <<= 1) { const uint32_t y = __shfl_up_sync(FULL, q, o); if (l >= o) q += y; }
        sh[l] = q;
    }
    __syncthreads();
    const uint32_t ex = (w ? sh[w - 1] : 0) + x - v;
    *total = sh[nw - 1];
    __syncthreads();
    return ex;
}

__device__ __forceinline__ uint64_t block_scan_u64(uint64_t v, uint64_t* sh, uint64_t* total) {
    const int l = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    uint64_t x = v;
    for (int o = 1; o < 32; o <<= 1) { const uint64_t y = __shfl_up_sync(FULL, x, o); if (l >= o) x += y; }
    if (l == 31) sh[w] = x;
    __syncthreads();
    if (w == 0) {
        uint64_t q = l < nw ? sh[l] : 0;
        for (int o = 1; o < 32; o <<= 1) { const uint64_t y = __shfl_up_sync(FULL, q, o); if (l >= o) q += y; }
        sh[l] = q;
    }
    __syncthreads();
    const uint64_t ex = (w ? sh[w - 1] : 0) + x - v;
    *total = sh[nw - 1];
    __syncthreads();
    return ex;
}

// Groups are the (tensor, exponent) cells with changes, tensors in caller order, exponents
// ascending (codec.py:146, :317-323): one CTA scans the cells.
__global__ void __launch_bounds__(1024) k_groups(const uint64_t* __restrict__ GC, int64_t n_cells, uint64_t* __restrict__ gcell,
                                                 int32_t* __restrict__ g_tensor, int32_t* __restrict__ g_exp,
                                                 uint64_t* __restrict__ g_start, uint64_t* __restrict__ g_count,
                                                 unsigned long long* __restrict__ counters) {
    __shared__ uint32_t sh32[32];
    __shared__ uint64_t sh64[32];
    uint32_t gbase = 0;
    uint64_t cbase = 0;
    for (int64_t b = 0; b < n_cells; b += 1024) {
        const int64_t cell = b + threadIdx.x;
        const uint64_t cnt = cell < n_cells ? GC[cell] : 0;
        const uint32_t f = cnt ? 1u : 0u;
        uint32_t nf;
        uint64_t nc;
        const uint32_t exf = block_scan_u32(f, sh32, &nf);
        const uint64_t exc = block_scan_u64(cnt, sh64, &nc);
        if (cell < n_cells) {
            if (f) {
                const uint32_t g = gbase + exf;
                gcell[cell] = cbase + exc;
                g_tensor[g] = int32_t(cell >> 8);
                g_exp[g] = int32_t(cell & 255);
                g_start[g] = cbase + exc;
                g_count[g] = cnt;
            } else {
                gcell[cell] = ~0ull;
            }
        }
        gbase += nf;
        cbase += nc;
    }
    if (threadIdx.x == 0) {
        g_start[gbase] = cbase;           // sentinel: start of the (absent) next group
        counters[2] = gbase;
        counters[3] = cbase;
    }
}

// records -> changes in group order.  Each sub-tile's records are sorted by (exponent, rank), so
// consecutive lanes mostly write consecutive destinations.
__global__ void __launch_bounds__(256) k_place(const uint64_t* __restrict__ rec_key, const uint32_t* __restrict__ rec_val,
                                               uint64_t n_rec, const uint32_t* __restrict__ HSP,
                                               const uint32_t* __restrict__ CSP, const uint64_t* __restrict__ gcell,
                                               const int32_t* __restrict__ super_t, uint32_t* __restrict__ local,
                                               uint32_t* __restrict__ vals, uint64_t total,
                                               unsigned long long* __restrict__ counters) {
    const uint64_t j = uint64_t(blockIdx.x) * 256 + threadIdx.x;
    if (j >= n_rec) return;
    const uint64_t key = rec_key[j];
    const uint32_t x = rec_val[j];
    const int64_t s = int64_t(key >> 36);
    const int e = exp_of(x & 0xFFFFu);
    const int t = super_t[s];
    const uint32_t csp = CSP[s * 256 + e], hsp = HSP[s * 256 + e];
    const uint64_t gs = gcell[int64_t(t) * 256 + e];
    const uint64_t dest = gs == ~0ull ? total : gs + csp + (uint32_t(key) & 0x3FFFFu);
    if (dest < total) {
        local[dest] = hsp + (uint32_t(key >> 18) & 0x3FFFFu);
        vals[dest] = x;
    } else {
        atomicOr(&counters[1], (unsigned long long)ERR_INTERNAL);
    }
}

// floor(log2(max(mean gap, 1))) clamped to [0, 30], by exact integer comparison: the mean is
// sum/count with sum < 2^33, so double rounding can never cross a power of two (codec.py:271-272)
__global__ void k_r0(const uint64_t* __restrict__ g_start, const uint64_t* __restrict__ g_count, int64_t ng,
                     const uint32_t* __restrict__ local, uint32_t* __restrict__ g_cand) {
    const int64_t g = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (g >= ng) return;
    const uint64_t cnt = g_count[g];
    const uint64_t last = local[g_start[g] + cnt - 1];
    const uint64_t sum = last - (cnt - 1);        // gaps telescope: sum = last local - (count - 1)
    int r0 = 0;
    while (r0 < 30 && (cnt << (r0 + 1)) <= sum) ++r0;
    const int c0 = max(r0 - 1, 0), c1 = r0, c2 = min(r0 + 1, 30);
    g_cand[g] = uint32_t(c0) | (uint32_t(c1) << 8) | (uint32_t(c2) << 16);
}

__device__ __forceinline__ uint32_t zigzag_of(uint32_t x) {
    const int32_t res = int32_t(int16_t(x >> 16)) - int32_t(int16_t(x & 0xFFFFu));
    return uint32_t((res << 1) ^ (res >> 31));
}

struct StatsSmem {
    uint32_t hist[STATS_LOCAL_GROUPS][DENSE_SYM];
    unsigned long long cost[STATS_LOCAL_GROUPS][3];
    int32_t gexp[STATS_LOCAL_GROUPS];
    int64_t g0;
};

// Rice candidate costs sum((gap >> c) + 1 + c) per group (codec.py:274) and (exponent, zigzag)
// symbol counts (codec.py:355-367).  Lanes take consecutive changes; each lane keeps its sums and
// a packed count of the symbols 0..7 in registers while its group stays the same, so atomics are
// needed only at group boundaries and for larger symbols.
__global__ void __launch_bounds__(256, 5) k_stats(const uint64_t* __restrict__ g_start, const int32_t* __restrict__ g_exp,
                                               const uint32_t* __restrict__ g_cand, int64_t ng, uint64_t total,
                                               const uint32_t* __restrict__ local, const uint32_t* __restrict__ vals,
                                               unsigned long long* __restrict__ costs, unsigned long long* __restrict__ dense_hist,
                                               uint32_t* __restrict__ rare_hist, uint32_t* __restrict__ rare_flag) {
    __shared__ StatsSmem S;
    const uint64_t j0 = uint64_t(blockIdx.x) * STATS_PER_CTA;
    const uint64_t j1 = tmin<uint64_t>(j0 + STATS_PER_CTA, total);
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) S.g0 = group_of(g_start, ng, j0);
    for (int k = threadIdx.x; k < STATS_LOCAL_GROUPS * DENSE_SYM; k += blockDim.x) (&S.hist[0][0])[k] = 0;
    for (int k = threadIdx.x; k < STATS_LOCAL_GROUPS * 3; k += blockDim.x) (&S.cost[0][0])[k] = 0;
    __syncthreads();
    const int64_t g0 = S.g0;
    if (threadIdx.x < STATS_LOCAL_GROUPS && g0 + threadIdx.x < ng) S.gexp[threadIdx.x] = g_exp[g0 + threadIdx.x];
    __syncthreads();

    int64_t g = -1;                    // this lane's current group and its register accumulators
    uint64_t ge = 0, gs = 0, acc0 = 0, acc1 = 0, acc2 = 0;
    uint32_t small_lo = 0, small_hi = 0;   // counts of the symbols 0..3 and 4..7, a byte each
    uint32_t cand = 0;
    int e = 0;
    auto flush = [&]() {
        if (g < 0) return;
        const int64_t lg = g - g0;
        if (lg < STATS_LOCAL_GROUPS) {
            if (acc0) atomicAdd(&S.cost[lg][0], (unsigned long long)acc0);
            if (acc1) atomicAdd(&S.cost[lg][1], (unsigned long long)acc1);
            if (acc2) atomicAdd(&S.cost[lg][2], (unsigned long long)acc2);
            for (int z = 0; z < 8; ++z) {
                const uint32_t c = ((z < 4 ? small_lo : small_hi) >> (8 * (z & 3))) & 0xFFu;
                if (c) atomicAdd(&S.hist[lg][z], c);
            }
        } else {
            if (acc0) atomicAdd(&costs[3 * g + 0], (unsigned long long)acc0);
            if (acc1) atomicAdd(&costs[3 * g + 1], (unsigned long long)acc1);
            if (acc2) atomicAdd(&costs[3 * g + 2], (unsigned long long)acc2);
            for (int z = 0; z < 8; ++z) {
                const uint64_t c = ((z < 4 ? small_lo : small_hi) >> (8 * (z & 3))) & 0xFFu;
                if (c) atomicAdd(&dense_hist[e * DENSE_SYM + z], (unsigned long long)c);
            }
        }
        acc0 = acc1 = acc2 = 0;
        small_lo = small_hi = 0;
    };
    // each warp takes a contiguous quarter of the CTA's changes, four chunks of 32 loaded at once
    const uint64_t wb = j0 + uint64_t(threadIdx.x >> 5) * (STATS_PER_CTA / 8);
    const uint64_t we = tmin<uint64_t>(wb + STATS_PER_CTA / 8, j1);
    for (uint64_t jb = wb; jb < we; jb += 128) {
        uint32_t locs[4], vs[4], pl[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const uint64_t j = jb + 32 * u + lane;
            const bool v = j < we;
            locs[u] = v ? local[j] : 0u;
            vs[u] = v ? vals[j] : 0u;
            pl[u] = (lane == 0 && v && j > 0) ? local[j - 1] : 0u;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const uint64_t j = jb + 32 * u + lane;
            const bool valid = j < we;
            const uint32_t loc = locs[u];
            const uint32_t prevw = __shfl_up_sync(FULL, loc, 1);
            if (valid) {
                if (j >= ge) {
                    flush();
                    g = g < 0 ? group_of(g_start, ng, j) : g + 1;
                    while (g_start[g + 1] <= j) ++g;
                    gs = g_start[g];
                    ge = g_start[g + 1];
                    cand = g_cand[g];
                    e = g_exp[g];
                }
                const uint32_t prev = lane ? prevw : (j > gs ? pl[u] : 0u);
                const uint32_t gap = j == gs ? loc : loc - prev - 1;   // locals ascend within a group
                const uint32_t c0 = cand & 255, c1 = (cand >> 8) & 255, c2 = (cand >> 16) & 255;
                acc0 += uint64_t(gap >> c0) + (1 + c0);
                acc1 += uint64_t(gap >> c1) + (1 + c1);
                acc2 += uint64_t(gap >> c2) + (1 + c2);
                const uint32_t z = zigzag_of(vs[u]);
                if (z < 8) {
                    const uint32_t one = 1u << (8 * (z & 3));
                    if (z < 4) small_lo += one; else small_hi += one;
                } else if (z < DENSE_SYM) {
                    const int64_t lg = g - g0;
                    if (lg < STATS_LOCAL_GROUPS) atomicAdd(&S.hist[lg][z], 1u);
                    else atomicAdd(&dense_hist[e * DENSE_SYM + z], 1ull);
                } else {
                    atomicAdd(&rare_hist[int64_t(e) * kSymSpace + z], 1u);
                    if (!rare_flag[e]) rare_flag[e] = 1;
                }
            }
        }
    }
    flush();
    __syncthreads();
    for (int k = threadIdx.x; k < STATS_LOCAL_GROUPS * DENSE_SYM; k += blockDim.x) {
        const int lg = k / DENSE_SYM;
        const uint32_t v = (&S.hist[0][0])[k];
        if (v && g0 + lg < ng) atomicAdd(&dense_hist[S.gexp[lg] * DENSE_SYM + (k % DENSE_SYM)], (unsigned long long)v);
    }
    for (int k = threadIdx.x; k < STATS_LOCAL_GROUPS * 3; k += blockDim.x) {
        const int lg = k / 3;
        const unsigned long long v = (&S.cost[0][0])[k];
        if (v && g0 + lg < ng) atomicAdd(&costs[3 * (g0 + lg) + (k % 3)], v);
    }
}

// Rare symbols of one exponent, ascending, as (symbol << 32 | count); the histogram row is
// zeroed again so the buffer stays clean between calls.
__global__ void __launch_bounds__(1024) k_rare_compact(uint32_t* __restrict__ rare_hist, uint32_t* __restrict__ rare_flag,
                                                       uint64_t* __restrict__ out, uint64_t out_cap,
                                                       unsigned long long* __restrict__ rare_total,
                                                       uint64_t* __restrict__ rare_base, uint32_t* __restrict__ rare_cnt) {
    constexpr uint32_t SLICE = (kSymSpace + 32 * 32 - 1) / (32 * 32) * 32;   // each of the 32 warps takes one slice, in order
    __shared__ uint32_t wbase[32];
    __shared__ uint64_t base_sh;
    const int e = blockIdx.x;
    const int w = int(threadIdx.x >> 5), lane = int(threadIdx.x & 31);
    if (!rare_flag[e]) { if (threadIdx.x == 0) rare_cnt[e] = 0; return; }
    uint32_t* row = rare_hist + int64_t(e) * kSymSpace;
    const uint32_t s0 = uint32_t(w) * SLICE;
    uint32_t nz = 0;
    for (uint32_t i = s0 + lane; i < s0 + SLICE && i < kSymSpace; i += 32) nz += row[i] != 0;
    nz = __reduce_add_sync(FULL, nz);
    if (lane == 0) wbase[w] = nz;
    __syncthreads();
    if (w == 0) {   // warp bases, the exponent's total and its place in the list
        const uint32_t v = wbase[lane];
        uint32_t incl = v;
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(FULL, incl, o);
            if (lane >= o) incl += y;
        }
        wbase[lane] = incl - v;
        if (lane == 31) {
            base_sh = atomicAdd(rare_total, (unsigned long long)incl);
            rare_base[e] = base_sh;
            rare_cnt[e] = incl;
            rare_flag[e] = 0;
        }
    }
    __syncthreads();
    uint64_t pos = base_sh + wbase[w];
    const uint32_t lt = lanemask_lt();
    for (uint32_t b = s0; b < s0 + SLICE; b += 32) {
        const uint32_t i = b + uint32_t(lane);
        const uint32_t v = i < kSymSpace ? row[i] : 0u;
        const uint32_t m = __ballot_sync(FULL, v != 0);
        if (v) {
            const uint64_t at = pos + uint64_t(__popc(m & lt));
            if (at < out_cap) out[at] = (uint64_t(i) << 32) | v;
            row[i] = 0;
        }
        pos += uint64_t(__popc(m));
    }
}

__global__ void k_scatter_codes(const uint64_t* __restrict__ list, int64_t n, uint32_t* __restrict__ big_code) {
    const int64_t k = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (k >= n) return;
    const uint64_t v = list[k];   // (exp << 17 | sym) << 32 | (code | len << 24)
    const uint32_t key = uint32_t(v >> 32);
    big_code[int64_t(key >> 17) * kSymSpace + (key & 0x1FFFFu)] = uint32_t(v);
}

__device__ __forceinline__ uint32_t code_of(const uint32_t* __restrict__ dense_code, const uint32_t* __restrict__ big_code,
                                            int e, uint32_t z) {
    return z < DENSE_SYM ? dense_code[e * DENSE_SYM + z] : big_code[int64_t(e) * kSymSpace + z];
}

__device__ __forceinline__ void or_word(uint32_t* words, uint64_t w, uint32_t v) {
    if (v) atomicOr(&words[w], bswap32(v));
}

// write `len` (<= 64) low bits of v at bit position pos (MSB-first stream)
__device__ __forceinline__ void put_bits(uint32_t* words, uint64_t pos, uint64_t v, int len) {
    if (len == 0) return;
    const int o = int(pos & 31);
    const uint64_t w0 = pos >> 5;
    const unsigned __int128 win = (unsigned __int128)v << (96 - o - len);
    or_word(words, w0, uint32_t(win >> 64));
    if (o + len > 32) or_word(words, w0 + 1, uint32_t(win >> 32));
    if (o + len > 64) or_word(words, w0 + 2, uint32_t(win));
}

// q one-bits starting at pos: partial edge words by atomicOr, whole words by plain stores
__device__ void put_ones(uint32_t* words, uint64_t pos, uint64_t q) {
    const uint64_t end = pos + q;
    while (pos < end && (pos & 31)) {
        const int o = int(pos & 31);
        const int k = int(tmin<uint64_t>(32 - o, end - pos));
        const uint32_t m = (k == 32 ? FULL : ((1u << k) - 1u)) << (32 - o - k);
        or_word(words, pos >> 5, m);
        pos += k;
    }
    while (end - pos >= 32) { words[pos >> 5] = FULL; pos += 32; }
    if (pos < end) {
        const int k = int(end - pos);
        or_word(words, pos >> 5, ((1u << k) - 1u) << (32 - k));
    }
}

// `len` (<= 64) low bits of v at bit `rel` of a warp's shared-memory words (MSB-first stream)
__device__ __forceinline__ void stage_bits(uint32_t* sw, uint32_t rel, uint64_t v, int len) {
    if (len == 0) return;
    const int o = int(rel & 31);
    uint32_t* w = sw + (rel >> 5);
    if (o + len <= 64) {
        const uint64_t x = v << (64 - o - len);
        if (uint32_t(x >> 32)) atomicOr(w, uint32_t(x >> 32));
        if (o + len > 32 && uint32_t(x)) atomicOr(w + 1, uint32_t(x));
    } else {   // 65..95 bits of window: three words
        const int sh = 96 - o - len;   // 1..31
        if (uint32_t(v >> (64 - sh))) atomicOr(w, uint32_t(v >> (64 - sh)));
        if (uint32_t((v << sh) >> 32)) atomicOr(w + 1, uint32_t((v << sh) >> 32));
        if (uint32_t(v << sh)) atomicOr(w + 2, uint32_t(v << sh));
    }
}

constexpr int SLOT_WORDS = 128;   // a block of up to 4 Kbit is assembled in shared memory and kept in its slot

// One warp per 256-change block: Rice gap then canonical Huffman code per change, MSB first
// (codec.py:218-257).  The block's bit count goes to the block table (bb32, and bb64 for the offset
// scan; codec.py:411-416).  A block that fits its slot is assembled in shared memory from bit 0 and stored there
// whole; k_compact later moves it to its place in the payload.  Longer blocks (rare) are encoded
// again by k_compact straight into the payload.
__global__ void __launch_bounds__(256, 5) k_pack_slots(const uint64_t* __restrict__ g_start, const int32_t* __restrict__ g_exp,
                                                    const uint8_t* __restrict__ g_rice, const uint64_t* __restrict__ g_block,
                                                    int64_t ng, int64_t n_blocks, const uint32_t* __restrict__ local,
                                                    const uint32_t* __restrict__ vals, const uint32_t* __restrict__ dense_code,
                                                    const uint32_t* __restrict__ big_code, uint32_t* __restrict__ slots,
                                                    uint64_t* __restrict__ bb64, uint32_t* __restrict__ bb32,
                                                    unsigned long long* __restrict__ counters) {
    __shared__ uint32_t stage[256 / 32][SLOT_WORDS];
    const int64_t b = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (b >= n_blocks) return;
    const int64_t g = group_of(g_block, ng, uint64_t(b));
    const uint64_t gs = g_start[g], ge = g_start[g + 1];
    const uint64_t j0 = gs + uint64_t(b - int64_t(g_block[g])) * kBlock;
    const uint64_t j1 = tmin<uint64_t>(j0 + kBlock, ge);
    const int r = g_rice[g];
    const int e = g_exp[g];
    uint32_t* sw = stage[threadIdx.x >> 5];
    for (int k = lane; k < SLOT_WORDS; k += 32) sw[k] = 0;
    __syncwarp();
    static_assert(kBlock == 256, "eight chunks of 32 per block");
    uint32_t locs[8], vs[8];   // the block's loads issued together; previous indices by shuffle
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        const uint64_t j = j0 + 32 * u + lane;
        locs[u] = j < j1 ? local[j] : 0u;
        vs[u] = j < j1 ? vals[j] : 0u;
    }
    uint32_t carry = lane == 0 && j0 > gs ? local[j0 - 1] : 0u;
    uint64_t rel = 0;     // the block's bits so far (warp-uniform)
    bool fits = true;     // every chunk so far was staged (warp-uniform)
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        const uint64_t j = j0 + 32 * u + lane;
        const uint32_t up = __shfl_up_sync(FULL, locs[u], 1);
        const uint32_t prev = lane ? up : carry;
        carry = __shfl_sync(FULL, locs[u], 31);
        uint32_t cl = 0;
        uint64_t gap = 0, L = 0;
        if (j < j1) {
            gap = j == gs ? locs[u] : uint64_t(locs[u]) - prev - 1;
            cl = code_of(dense_code, big_code, e, zigzag_of(vs[u]));
            L = (gap >> r) + 1 + uint64_t(r) + (cl >> 24);
        }
        uint64_t incl;
        if (__all_sync(FULL, L < (1u << 26))) {   // the usual case: 32-bit sums
            uint32_t in32 = uint32_t(L);
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(FULL, in32, o);
                if (lane >= o) in32 += y;
            }
            incl = in32;
        } else {
            incl = L;
            for (int o = 1; o < 32; o <<= 1) {
                const uint64_t y = __shfl_up_sync(FULL, incl, o);
                if (lane >= o) incl += y;
            }
        }
        const uint64_t ctot = __shfl_sync(FULL, incl, 31);
        fits = fits && rel + ctot <= uint64_t(SLOT_WORDS) * 32;
        if (fits && j < j1) {
            uint32_t at = uint32_t(rel + incl - L);
            uint32_t q = uint32_t(gap >> r);
            const int hl = int(cl >> 24);
            const uint64_t rem = r ? (gap & ((1ull << r) - 1)) : 0;
            const int tail_len = 1 + r + hl;                          // the 0, r remainder bits, code
            const uint64_t tail = (rem << hl) | (cl & 0xFFFFFFu);     // leading 0 is implicit
            while (q + uint32_t(tail_len) > 64u) {   // long unary runs: ones 32 at a time
                const uint32_t c = tmin(q, 32u);
                stage_bits(sw, at, (1ull << c) - 1, int(c));
                q -= c;
                at += c;
            }
            stage_bits(sw, at, q ? ((((1ull << q) - 1) << tail_len) | tail) : tail, int(q) + tail_len);
        }
        rel += ctot;
    }
    if (lane == 0) {
        bb64[b] = rel;
        bb32[b] = uint32_t(rel);
        if (rel >> 32) atomicOr(&counters[1], (unsigned long long)ERR_BLOCK_TOO_LONG);
    }
    if (fits) {
        __syncwarp();
        uint32_t* dst = slots + b * SLOT_WORDS;
        const uint32_t nw = uint32_t((rel + 31) >> 5);
        for (uint32_t k = lane; k < nw; k += 32) dst[k] = sw[k];
    }
}

// One warp per block: its slot's words shifted to the block's bit offset in the payload (the two
// edge words, which it may share with its neighbours, by atomic OR into the zeroed payload; the
// others by plain stores).  A block longer than a slot is encoded here again, straight into the
// payload.  block_off: exclusive scan of the blocks' bits; bit0: where this part starts inside its
// first byte (a rank's part of a global update).
__global__ void __launch_bounds__(256) k_compact(const uint64_t* __restrict__ g_start, const int32_t* __restrict__ g_exp,
                                                 const uint8_t* __restrict__ g_rice, const uint64_t* __restrict__ g_block,
                                                 int64_t ng, int64_t n_blocks, const uint32_t* __restrict__ local,
                                                 const uint32_t* __restrict__ vals, const uint32_t* __restrict__ dense_code,
                                                 const uint32_t* __restrict__ big_code, const uint32_t* __restrict__ slots,
                                                 const uint64_t* __restrict__ block_off, const uint32_t* __restrict__ block_bits,
                                                 uint32_t* __restrict__ words, uint32_t bit0) {
    const int64_t b = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (b >= n_blocks) return;
    uint64_t pos = block_off[b] + bit0;
    const uint32_t bits = block_bits[b];
    if (bits <= uint32_t(SLOT_WORDS) * 32) {
        const uint32_t* src = slots + b * SLOT_WORDS;
        const uint32_t o = uint32_t(pos & 31);
        const uint64_t w0 = pos >> 5;
        const uint32_t nin = (bits + 31) >> 5, nout = (o + bits + 31) >> 5;
        for (uint32_t k = lane; k < nout; k += 32) {
            const uint32_t hi = k < nin ? src[k] : 0u;
            const uint32_t lo = k >= 1 && k - 1 < nin ? src[k - 1] : 0u;
            const uint32_t v = o ? (hi >> o) | (lo << (32 - o)) : hi;
            if (k == 0 || k + 1 == nout) or_word(words, w0 + k, v);
            else words[w0 + k] = bswap32(v);
        }
        return;
    }
    const int64_t g = group_of(g_block, ng, uint64_t(b));
    const uint64_t gs = g_start[g], ge = g_start[g + 1];
    const uint64_t j0 = gs + uint64_t(b - int64_t(g_block[g])) * kBlock;
    const uint64_t j1 = tmin<uint64_t>(j0 + kBlock, ge);
    const int r = g_rice[g];
    const int e = g_exp[g];
    for (uint64_t jb = j0; jb < j1; jb += 32) {
        const uint64_t j = jb + lane;
        uint64_t L = 0, gap = 0;
        uint32_t cl = 0;
        if (j < j1) {
            const uint32_t loc = local[j];
            gap = j == gs ? loc : uint64_t(loc) - local[j - 1] - 1;
            cl = code_of(dense_code, big_code, e, zigzag_of(vals[j]));
            L = (gap >> r) + 1 + r + (cl >> 24);
        }
        uint64_t incl = L;
        for (int o = 1; o < 32; o <<= 1) {
            const uint64_t y = __shfl_up_sync(FULL, incl, o);
            if (lane >= o) incl += y;
        }
        const uint64_t at = pos + incl - L;
        if (j < j1) {
            const uint64_t q = gap >> r;
            const int hl = int(cl >> 24);
            const uint64_t code = cl & 0xFFFFFFu;
            const uint64_t rem = r ? (gap & ((1ull << r) - 1)) : 0;
            const int tail_len = 1 + r + hl;                          // the 0, r remainder bits, code
            const uint64_t tail = (rem << hl) | code;                 // leading 0 is implicit
            if (q + tail_len <= 64) {
                const uint64_t v = q ? ((((1ull << q) - 1) << tail_len) | tail) : tail;
                put_bits(words, at, v, int(q) + tail_len);
            } else {
                put_ones(words, at, q);
                put_bits(words, at + q, tail, tail_len);
            }
        }
        pos += __shfl_sync(FULL, incl, 31);
    }
}

}  // namespace

// ------------------------------------------------------------------ host driver

namespace {

template <class T>
T* dev(Ctx& c, Slot s) { return reinterpret_cast<T*>(c.b[s].p); }

struct HostTables {
    // per exponent: ascending symbols, their counts, lengths and codes
    std::vector<uint32_t> sym[256];
    std::vector<uint64_t> cnt[256];
    std::vector<uint8_t> len[256];
    std::vector<uint32_t> code[256];
};

// Huffman tables from the symbol histogram: dense counts [256][DENSE_SYM] and the larger symbols
// as (exponent << 17 | symbol, count) pairs sorted by key (codec.py:369-392).
void build_tables(const std::vector<uint64_t>& dense, const std::vector<std::pair<uint64_t, uint64_t>>& rare,
                  HostTables* tabs) {
    size_t r = 0;
    for (int e = 0; e < 256; ++e) {
        for (int z = 0; z < DENSE_SYM; ++z) {
            const uint64_t c = dense[size_t(e) * DENSE_SYM + size_t(z)];
            if (c) { tabs->sym[e].push_back(uint32_t(z)); tabs->cnt[e].push_back(c); }
        }
        for (; r < rare.size() && (rare[r].first >> 17) == uint64_t(e); ++r) {
            tabs->sym[e].push_back(uint32_t(rare[r].first & 0x1FFFFu));
            tabs->cnt[e].push_back(rare[r].second);
        }
    }
    // the exponents' tables are independent: built on the host pool, the largest first
    std::vector<int> todo;
    for (int e = 0; e < 256; ++e)
        if (!tabs->sym[e].empty()) todo.push_back(e);
    std::sort(todo.begin(), todo.end(), [&](int a, int b) { return tabs->sym[a].size() > tabs->sym[b].size(); });
    size_t total = 0;
    for (int e : todo) total += tabs->sym[e].size();
    auto one = [&](size_t k) {
        const int e = todo[k];
        const size_t ns = tabs->sym[e].size();
        tabs->len[e].resize(ns);
        tabs->code[e].resize(ns);
        huffman_lengths(tabs->cnt[e].data(), int64_t(ns), tabs->len[e].data());
        canonical_codes(tabs->len[e].data(), int64_t(ns), tabs->code[e].data());
    };
    if (total < 8192) {   // small alphabets: waking the pool costs more than the work
        for (size_t k = 0; k < todo.size(); ++k) one(k);
    } else {
        parallel_for(todo.size(), one);
    }
}

// Global mode: the histogram summed over ranks (dense part by sum, rare pairs gathered and merged)
Status exchange_histogram(const GlobalExchange& gx, std::vector<uint64_t>* dense,
                          std::vector<std::pair<uint64_t, uint64_t>>* rare, std::string* err) {
    if (gx.sum_u64(gx.user, dense->data(), int64_t(dense->size()))) { *err = "histogram sum failed"; return kCudaError; }
    std::vector<uint64_t> mine;
    for (const auto& p : *rare) { mine.push_back(p.first); mine.push_back(p.second); }
    const uint8_t* all = nullptr;
    int64_t all_len = 0;
    if (gx.allgather_bytes(gx.user, reinterpret_cast<const uint8_t*>(mine.data()), int64_t(8 * mine.size()), &all, &all_len) ||
        all_len % 16 || (all_len && !all)) {
        *err = "rare-symbol gather failed";
        return kCudaError;
    }
    std::vector<std::pair<uint64_t, uint64_t>> merged(size_t(all_len / 16));
    for (size_t k = 0; k < merged.size(); ++k) {
        std::memcpy(&merged[k].first, all + 16 * k, 8);
        std::memcpy(&merged[k].second, all + 16 * k + 8, 8);
    }
    std::sort(merged.begin(), merged.end());
    rare->clear();
    for (const auto& p : merged) {
        if (!rare->empty() && rare->back().first == p.first) rare->back().second += p.second;
        else rare->push_back(p);
    }
    return kOk;
}

// Global mode: every rank's value gathered by a sum over a one-hot vector
Status exchange_per_rank(const GlobalExchange& gx, uint64_t mine, std::vector<uint64_t>* all, std::string* err) {
    all->assign(size_t(gx.world), 0);
    (*all)[size_t(gx.rank)] = mine;
    if (gx.sum_u64(gx.user, all->data(), int64_t(gx.world))) { *err = "per-rank exchange failed"; return kCudaError; }
    return kOk;
}

// magic, version and tables of an update (wire.py:64-78); the tensor count follows
void put_prefix(std::vector<uint8_t>& ob, const HostTables& tabs) {
    const uint8_t magic[5] = {'C', 'R', 'X', 'S', 2};
    ob.insert(ob.end(), magic, magic + 5);
    int n_tables = 0;
    for (int e = 0; e < 256; ++e) n_tables += !tabs.sym[e].empty();
    put_varint(ob, uint64_t(n_tables));
    for (int e = 0; e < 256; ++e) {
        if (tabs.sym[e].empty()) continue;
        ob.push_back(uint8_t(e));
        put_varint(ob, tabs.sym[e].size());
        for (size_t k = 0; k < tabs.sym[e].size(); ++k) {
            put_varint(ob, tabs.sym[e][k]);
            ob.push_back(tabs.len[e][k]);
        }
    }
}

// Global mode for a rank without changes: the same collectives with empty contributions
Status global_empty_part(const GlobalExchange& gx, Encoded* out, std::string* err) {
    std::vector<uint64_t> dense(size_t(256) * DENSE_SYM, 0);
    std::vector<std::pair<uint64_t, uint64_t>> rare;
    Status s = exchange_histogram(gx, &dense, &rare, err);
    if (s != kOk) return s;
    std::vector<uint64_t> np, bits;
    if ((s = exchange_per_rank(gx, 0, &np, err)) != kOk) return s;
    HostTables tabs;
    build_tables(dense, rare, &tabs);
    out->head.clear();
    put_prefix(out->head, tabs);
    uint64_t n_tensors = 0;
    for (uint64_t v : np) n_tensors += v;
    put_varint(out->head, n_tensors);
    if ((s = exchange_per_rank(gx, 0, &bits, err)) != kOk) return s;
    uint64_t before = 0, total = 0;
    for (int r = 0; r < gx.world; ++r) { if (r < gx.rank) before += bits[size_t(r)]; total += bits[size_t(r)]; }
    out->part = true;
    out->bit_offset = before;
    out->total_bits = total;
    out->len_varint.clear();
    put_varint(out->len_varint, (total + 7) / 8);
    return kOk;
}

}  // namespace

Status encode_impl(Ctx& C, int nT, const int16_t* const* prev, const int16_t* const* cur, const int64_t* numel,
                   const uint8_t* const* names, const int64_t* name_len, const uint64_t* cache_chk,
                   const uint8_t* has_cache, cudaStream_t st, Encoded* out, std::string* err, bool device_result,
                   const GlobalExchange* gx) {
    if (C.live) {           // an earlier result still reads the output buffers: give it its own copy
        const cudaError_t de = C.live->detach();
        C.live = nullptr;
        if (de != cudaSuccess) { *err = std::string("detaching the previous update: ") + cudaGetErrorString(de); return kCudaError; }
    }
    // copies of an earlier device result may still read the block table and payload workspace
    if (C.wd_busy) CRX_CUDA(cudaStreamWaitEvent(st, C.wd_ev, 0));
    out->ctx = &C;
    out->head.clear();
    out->len_varint.assign(1, 0);
    out->checksums.assign(size_t(nT), 0);
    out->present.assign(size_t(nT), 0);
    trace_phase(C, "encode: start");
    // ---- tensor descriptors
    std::vector<EncTensor> T;
    std::vector<int> tmap;  // index into caller arrays
    int64_t n_super = 0;
    for (int t = 0; t < nT; ++t) {
        if (numel[t] < 0) { *err = "negative numel"; return kBadArgument; }
        if (numel[t] >= (int64_t(1) << 32)) { *err = "tensors of 2^32 or more elements are not supported"; return kValueError; }
        if (numel[t] == 0) continue;
        EncTensor d{};
        d.prev = prev[t];
        d.cur = cur[t];
        d.numel = numel[t];
        d.super_begin = n_super;
        d.want_full = has_cache && has_cache[t] ? 0 : 1;
        n_super += (numel[t] + SUPER_N - 1) / SUPER_N;
        T.push_back(d);
        tmap.push_back(t);
    }
    const int nt = int(T.size());
    auto empty_update = [&]() {   // "CRXS" 2, no tables, no tensors, payload_len 0
        static const uint8_t kEmpty[7] = {'C', 'R', 'X', 'S', 2, 0, 0};
        out->head.assign(kEmpty, kEmpty + 7);
        return kOk;
    };
    if (nt == 0) return gx ? global_empty_part(*gx, out, err) : empty_update();
    if (n_super >= (int64_t(1) << 28)) { *err = "update too large for one call"; return kValueError; }

    // ---- buffers
    const size_t cells = size_t(nt) * 256;
    std::vector<int64_t> row_begin(static_cast<size_t>(nt) + 1), chunk_begin(static_cast<size_t>(nt) + 1);
    for (int t = 0; t < nt; ++t) {
        row_begin[size_t(t)] = T[size_t(t)].super_begin;
        const int64_t rows = (T[size_t(t)].numel + SUPER_N - 1) / SUPER_N;
        chunk_begin[size_t(t) + 1] = chunk_begin[size_t(t)] + (rows + SCAN_CHUNK - 1) / SCAN_CHUNK;
    }
    row_begin[size_t(nt)] = n_super;
    const int64_t n_chunks = chunk_begin[size_t(nt)];
    CRX_CUDA(ensure_dev(C.b[S_TENS], sizeof(EncTensor) * size_t(nt), st));
    CRX_CUDA(ensure_dev(C.b[S_HS], sizeof(uint32_t) * 256 * size_t(n_super), st));
    CRX_CUDA(ensure_dev(C.b[S_CS], sizeof(uint32_t) * 256 * size_t(n_super), st));
    CRX_CUDA(ensure_dev(C.b[S_CHUNK_ROWS], sizeof(int64_t) * 2 * (size_t(nt) + 1), st));
    CRX_CUDA(ensure_dev(C.b[S_CHUNK_SUMS], sizeof(uint32_t) * 256 * size_t(n_chunks), st));
    CRX_CUDA(ensure_dev(C.b[S_TOTALS_A], sizeof(uint64_t) * cells, st));
    CRX_CUDA(ensure_dev(C.b[S_TOTALS_C], sizeof(uint64_t) * cells, st));
    CRX_CUDA(ensure_dev(C.b[S_COUNTERS], sizeof(uint64_t) * 16, st));
    CRX_CUDA(ensure_dev(C.b[S_CHK], sizeof(uint64_t) * 2 * size_t(nt), st));
    CRX_CUDA(ensure_dev(C.b[S_GIDX], sizeof(uint64_t) * cells, st));
    CRX_CUDA(ensure_dev(C.b[S_SUPER_T], sizeof(int32_t) * size_t(n_super), st));
    // groups: tensor, exp (i32), start (cells+1), count, cand (u32), costs (3 u64), rice (u8), block start
    CRX_CUDA(ensure_dev(C.b[S_GROUPS], (4 + 4 + 8 + 8 + 4 + 24 + 1 + 8) * (cells + 1) + 64, st));
    int64_t total_el = 0;
    for (auto& d : T) total_el += d.numel;
    uint64_t rec_cap = C.b[S_REC_KEY].cap / sizeof(uint64_t);
    const uint64_t want_cap = std::max<uint64_t>(uint64_t(total_el / 16) + 4096, rec_cap);
    CRX_CUDA(ensure_dev(C.b[S_REC_KEY], sizeof(uint64_t) * want_cap, st));
    CRX_CUDA(ensure_dev(C.b[S_REC_VAL], sizeof(uint32_t) * want_cap, st));
    rec_cap = want_cap;

    const size_t meta_bytes = sizeof(EncTensor) * size_t(nt) + sizeof(int64_t) * 2 * (size_t(nt) + 1) +
                              sizeof(int32_t) * size_t(n_super);
    CRX_CUDA(ensure_host(C, std::max<size_t>(meta_bytes, 1 << 20), st));
    {
        uint8_t* h = static_cast<uint8_t*>(C.host);
        std::memcpy(h, T.data(), sizeof(EncTensor) * size_t(nt));
        CRX_CUDA(cudaMemcpyAsync(C.b[S_TENS].p, h, sizeof(EncTensor) * size_t(nt), cudaMemcpyHostToDevice, st));
        int64_t* rb = reinterpret_cast<int64_t*>(h + sizeof(EncTensor) * size_t(nt));
        std::memcpy(rb, row_begin.data(), sizeof(int64_t) * (size_t(nt) + 1));
        std::memcpy(rb + nt + 1, chunk_begin.data(), sizeof(int64_t) * (size_t(nt) + 1));
        CRX_CUDA(cudaMemcpyAsync(C.b[S_CHUNK_ROWS].p, rb, sizeof(int64_t) * 2 * (size_t(nt) + 1), cudaMemcpyHostToDevice, st));
        int32_t* stt = reinterpret_cast<int32_t*>(rb + 2 * (nt + 1));
        for (int t = 0; t < nt; ++t)
            for (int64_t s = row_begin[size_t(t)]; s < row_begin[size_t(t) + 1]; ++s) stt[s] = t;
        CRX_CUDA(cudaMemcpyAsync(C.b[S_SUPER_T].p, stt, sizeof(int32_t) * size_t(n_super), cudaMemcpyHostToDevice, st));
    }
    const int64_t* d_row_begin = dev<int64_t>(C, S_CHUNK_ROWS);
    const int64_t* d_chunk_begin = d_row_begin + nt + 1;
    auto* counters = dev<unsigned long long>(C, S_COUNTERS);
    auto* chk_delta = dev<unsigned long long>(C, S_CHK);
    auto* chk_full = chk_delta + nt;
    const size_t rank_smem = sizeof(RankSmem);
    CRX_CUDA(cudaFuncSetAttribute(k_enc_rank, cudaFuncAttributeMaxDynamicSharedMemorySize, int(rank_smem)));

    uint64_t* hostc = C.small;
    for (int attempt = 0; attempt < 2; ++attempt) {
        CRX_CUDA(cudaMemsetAsync(counters, 0, sizeof(uint64_t) * 16, st));
        CRX_CUDA(cudaMemsetAsync(chk_delta, 0, sizeof(uint64_t) * 2 * size_t(nt), st));
        { KernelScope ks_(C, "k_enc_rank", st);
        k_enc_rank<<<unsigned(n_super), ER_THREADS, rank_smem, st>>>(
            dev<EncTensor>(C, S_TENS), nt, dev<uint64_t>(C, S_REC_KEY), dev<uint32_t>(C, S_REC_VAL), rec_cap, counters,
            dev<uint32_t>(C, S_HS), dev<uint32_t>(C, S_CS), chk_delta, chk_full);
        }
        CRX_CUDA(cudaGetLastError());
        CRX_CUDA(cudaMemcpyAsync(hostc, counters, sizeof(uint64_t) * 2, cudaMemcpyDeviceToHost, st));
        CRX_CUDA(cudaStreamSynchronize(st));
        if (hostc[0] <= rec_cap) break;
        const uint64_t need = hostc[0] + 4096;
        CRX_CUDA(ensure_dev(C.b[S_REC_KEY], sizeof(uint64_t) * need, st));
        CRX_CUDA(ensure_dev(C.b[S_REC_VAL], sizeof(uint32_t) * need, st));
        rec_cap = need;
    }
    const uint64_t n_rec = hostc[0];
    trace_phase(C, "encode: ranked (sync 1)");
    if (n_rec == 0) return gx ? global_empty_part(*gx, out, err) : empty_update();

    // ---- per tensor column scans and the group table
    launch_column_scan(C, dev<uint32_t>(C, S_HS), n_super, d_row_begin, nt, d_chunk_begin, n_chunks,
                       dev<uint32_t>(C, S_CHUNK_SUMS), dev<uint64_t>(C, S_TOTALS_A), st);
    launch_column_scan(C, dev<uint32_t>(C, S_CS), n_super, d_row_begin, nt, d_chunk_begin, n_chunks,
                       dev<uint32_t>(C, S_CHUNK_SUMS), dev<uint64_t>(C, S_TOTALS_C), st);
    uint8_t* gb = dev<uint8_t>(C, S_GROUPS);
    const size_t gcap = cells + 1;
    auto* g_start = reinterpret_cast<uint64_t*>(gb);
    auto* g_count = reinterpret_cast<uint64_t*>(gb + 8 * gcap);
    auto* costs = reinterpret_cast<unsigned long long*>(gb + 16 * gcap);
    auto* g_block = reinterpret_cast<uint64_t*>(gb + 40 * gcap);
    auto* g_tensor = reinterpret_cast<int32_t*>(gb + 48 * gcap);
    auto* g_exp = reinterpret_cast<int32_t*>(gb + 52 * gcap);
    auto* g_cand = reinterpret_cast<uint32_t*>(gb + 56 * gcap);
    auto* g_rice = reinterpret_cast<uint8_t*>(gb + 60 * gcap);
    { KernelScope ks_(C, "k_groups", st);
    k_groups<<<1, 1024, 0, st>>>(dev<uint64_t>(C, S_TOTALS_C), int64_t(cells), dev<uint64_t>(C, S_GIDX), g_tensor, g_exp,
                                g_start, g_count, counters);
    }
    CRX_CUDA(cudaGetLastError());
    CRX_CUDA(cudaMemcpyAsync(hostc, counters, sizeof(uint64_t) * 4, cudaMemcpyDeviceToHost, st));
    CRX_CUDA(cudaStreamSynchronize(st));
    const int64_t ng = int64_t(hostc[2]);
    trace_phase(C, "encode: groups (sync 2)");
    const uint64_t total = hostc[3];
    if (total != n_rec || (hostc[1] & ERR_INTERNAL)) { *err = "internal: change count mismatch"; return kCudaError; }

    CRX_CUDA(ensure_dev(C.b[S_LOCAL], sizeof(uint32_t) * total, st));
    CRX_CUDA(ensure_dev(C.b[S_VALS], sizeof(uint32_t) * total, st));
    auto* local = dev<uint32_t>(C, S_LOCAL);
    auto* vals = dev<uint32_t>(C, S_VALS);
    { KernelScope ks_(C, "k_place", st);
    k_place<<<unsigned((n_rec + 255) / 256), 256, 0, st>>>(dev<uint64_t>(C, S_REC_KEY), dev<uint32_t>(C, S_REC_VAL), n_rec,
                                                           dev<uint32_t>(C, S_HS), dev<uint32_t>(C, S_CS), dev<uint64_t>(C, S_GIDX),
                                                           dev<int32_t>(C, S_SUPER_T), local, vals, total, counters);
    }
    CRX_CUDA(cudaGetLastError());
    { KernelScope ks_(C, "k_r0", st);
    k_r0<<<unsigned((ng + 255) / 256), 256, 0, st>>>(g_start, g_count, ng, local, g_cand);
    }
    CRX_CUDA(cudaGetLastError());

    // ---- symbol histogram + Rice costs
    CRX_CUDA(ensure_dev(C.b[S_DENSE_HIST], sizeof(uint64_t) * 256 * DENSE_SYM, st));
    CRX_CUDA(ensure_dev(C.b[S_RARE_FLAG], sizeof(uint32_t) * 256 * 2 + sizeof(uint64_t) * 256, st));
    if (C.b[S_RARE_HIST].cap < sizeof(uint32_t) * 256 * size_t(kSymSpace)) {
        CRX_CUDA(ensure_dev(C.b[S_RARE_HIST], sizeof(uint32_t) * 256 * size_t(kSymSpace), st));
        CRX_CUDA(cudaMemsetAsync(C.b[S_RARE_HIST].p, 0, C.b[S_RARE_HIST].cap, st));
        CRX_CUDA(cudaMemsetAsync(C.b[S_RARE_FLAG].p, 0, sizeof(uint32_t) * 256, st));
    }
    auto* rare_flag = dev<uint32_t>(C, S_RARE_FLAG);
    auto* rare_cnt = rare_flag + 256;
    auto* rare_base = reinterpret_cast<uint64_t*>(rare_flag + 512);
    CRX_CUDA(cudaMemsetAsync(C.b[S_DENSE_HIST].p, 0, sizeof(uint64_t) * 256 * DENSE_SYM, st));
    CRX_CUDA(cudaMemsetAsync(costs, 0, sizeof(uint64_t) * 3 * size_t(ng), st));
    { KernelScope ks_(C, "k_stats", st);
    k_stats<<<unsigned((total + STATS_PER_CTA - 1) / STATS_PER_CTA), 256, 0, st>>>(
        g_start, g_exp, g_cand, ng, total, local, vals, costs, dev<unsigned long long>(C, S_DENSE_HIST),
        dev<uint32_t>(C, S_RARE_HIST), rare_flag);
    }
    CRX_CUDA(cudaGetLastError());
    const uint64_t rare_cap = std::min<uint64_t>(total, uint64_t(256) * kSymSpace);
    CRX_CUDA(ensure_dev(C.b[S_RARE_OUT], sizeof(uint64_t) * rare_cap, st));
    { KernelScope ks_(C, "k_rare_compact", st);
    k_rare_compact<<<256, 1024, 0, st>>>(dev<uint32_t>(C, S_RARE_HIST), rare_flag, dev<uint64_t>(C, S_RARE_OUT), rare_cap,
                                         counters + 4, rare_base, rare_cnt);
    }
    CRX_CUDA(cudaGetLastError());

    // ---- download what the host needs for headers and Huffman tables
    const size_t off_gt = 0, off_ge = off_gt + 4 * size_t(ng), off_gc = off_ge + 4 * size_t(ng);
    const size_t off_cost = off_gc + 8 * size_t(ng), off_dense = off_cost + 24 * size_t(ng);
    const size_t off_rc = off_dense + 8 * 256 * DENSE_SYM, off_rb = off_rc + 4 * 256, off_chk = off_rb + 8 * 256;
    const size_t off_ctr = off_chk + 16 * size_t(nt), off_cand = off_ctr + 8 * 16;
    // the first rare-symbol pairs come down in the same round trip (most updates have few)
    const size_t off_rare = (off_cand + 4 * size_t(ng) + 7) & ~size_t(7);
    const uint64_t rare_eager = std::min<uint64_t>(rare_cap, 65536);
    const size_t down1 = off_rare + 8 * size_t(rare_eager);
    CRX_CUDA(ensure_host(C, down1, st));
    uint8_t* h = static_cast<uint8_t*>(C.host);
    CRX_CUDA(cudaMemcpyAsync(h + off_gt, g_tensor, 4 * size_t(ng), cudaMemcpyDeviceToHost, st));
    CRX_CUDA(cudaMemcpyAsync(h + off_ge, g_exp, 4 * size_t(ng), cudaMemcpyDeviceToHost, st));
    CRX_CUDA(cudaMemcpyAsync(h + off_gc, g_count, 8 * size_t(ng), cudaMemcpyDeviceToHost, st));
    CRX_CUDA(cudaMemcpyAsync(h + off_cost, costs, 24 * size_t(ng), cudaMemcpyDeviceToHost, st));
    CRX_CUDA(cudaMemcpyAsync(h + off_dense, C.b[S_DENSE_HIST].p, 8 * 256 * DENSE_SYM, cudaMemcpyDeviceToHost, st));
    CRX_CUDA(cudaMemcpyAsync(h + off_rc, rare_cnt, 4 * 256, cudaMemcpyDeviceToHost, st));
    CRX_CUDA(cudaMemcpyAsync(h + off_rb, rare_base, 8 * 256, cudaMemcpyDeviceToHost, st));
    CRX_CUDA(cudaMemcpyAsync(h + off_chk, chk_delta, 16 * size_t(nt), cudaMemcpyDeviceToHost, st));
    CRX_CUDA(cudaMemcpyAsync(h + off_ctr, counters, 8 * 16, cudaMemcpyDeviceToHost, st));
    CRX_CUDA(cudaMemcpyAsync(h + off_cand, g_cand, 4 * size_t(ng), cudaMemcpyDeviceToHost, st));
    if (rare_eager)
        CRX_CUDA(cudaMemcpyAsync(h + off_rare, C.b[S_RARE_OUT].p, 8 * size_t(rare_eager), cudaMemcpyDeviceToHost, st));
    CRX_CUDA(cudaStreamSynchronize(st));
    std::vector<uint32_t> hcand(static_cast<size_t>(ng));
    std::memcpy(hcand.data(), h + off_cand, 4 * size_t(ng));
    trace_phase(C, "encode: stats down (sync 3)");
    std::vector<int32_t> hg_tensor(static_cast<size_t>(ng)), hg_exp(static_cast<size_t>(ng));
    std::vector<uint64_t> hg_count(static_cast<size_t>(ng)), hcost(3 * static_cast<size_t>(ng)), hdense(256 * DENSE_SYM), hrb(256), hchk(2 * static_cast<size_t>(nt));
    std::vector<uint32_t> hrc(256);
    std::memcpy(hg_tensor.data(), h + off_gt, 4 * size_t(ng));
    std::memcpy(hg_exp.data(), h + off_ge, 4 * size_t(ng));
    std::memcpy(hg_count.data(), h + off_gc, 8 * size_t(ng));
    std::memcpy(hcost.data(), h + off_cost, 24 * size_t(ng));
    std::memcpy(hdense.data(), h + off_dense, 8 * 256 * DENSE_SYM);
    std::memcpy(hrc.data(), h + off_rc, 4 * 256);
    std::memcpy(hrb.data(), h + off_rb, 8 * 256);
    std::memcpy(hchk.data(), h + off_chk, 16 * size_t(nt));
    uint64_t hctr[16];
    std::memcpy(hctr, h + off_ctr, 8 * 16);
    if (hctr[1] & ERR_INTERNAL) { *err = "internal: a change has no group"; return kCudaError; }
    const uint64_t rare_total = hctr[4];
    if (rare_total > rare_cap) { *err = "internal: rare symbol overflow"; return kCudaError; }
    std::vector<uint64_t> hrare(rare_total);
    if (rare_total && rare_total <= rare_eager) {
        std::memcpy(hrare.data(), h + off_rare, 8 * rare_total);
    } else if (rare_total) {
        CRX_CUDA(ensure_host(C, 8 * rare_total, st));
        CRX_CUDA(cudaMemcpyAsync(C.host, C.b[S_RARE_OUT].p, 8 * rare_total, cudaMemcpyDeviceToHost, st));
        CRX_CUDA(cudaStreamSynchronize(st));
        std::memcpy(hrare.data(), C.host, 8 * rare_total);
    }
    trace_phase(C, "encode: rare symbols down");

    // ---- Rice per group: first cheapest of the three candidates (codec.py:273-275)
    std::vector<uint8_t> rice(static_cast<size_t>(ng));
    std::vector<uint64_t> gblock(static_cast<size_t>(ng) + 1, 0);
    for (int64_t g = 0; g < ng; ++g) {
        const uint64_t* cst = &hcost[3 * size_t(g)];
        int best = 0;
        for (int k = 1; k < 3; ++k) if (cst[k] < cst[best]) best = k;
        rice[size_t(g)] = uint8_t((hcand[size_t(g)] >> (8 * best)) & 255);
        gblock[size_t(g) + 1] = gblock[size_t(g)] + (hg_count[size_t(g)] + kBlock - 1) / kBlock;
    }
    const int64_t n_blocks = int64_t(gblock[size_t(ng)]);

    // ---- one Huffman table per exponent over the whole update (codec.py:369-392); a global
    //      update sums the histogram over its ranks first
    std::vector<std::pair<uint64_t, uint64_t>> rare_pairs;
    rare_pairs.reserve(rare_total);
    for (int e = 0; e < 256; ++e)
        for (uint32_t k = 0; k < hrc[size_t(e)]; ++k) {
            const uint64_t v = hrare[size_t(hrb[size_t(e)] + k)];
            rare_pairs.emplace_back((uint64_t(e) << 17) | (v >> 32), v & 0xFFFFFFFFull);
        }
    std::vector<uint64_t> np_all;
    int n_present_local = 0;
    {
        std::vector<uint8_t> has(static_cast<size_t>(nt), 0);
        for (int64_t g = 0; g < ng; ++g) has[size_t(hg_tensor[size_t(g)])] = 1;
        for (uint8_t x : has) n_present_local += x;
    }
    if (gx) {
        Status xs = exchange_histogram(*gx, &hdense, &rare_pairs, err);
        if (xs == kOk) xs = exchange_per_rank(*gx, uint64_t(n_present_local), &np_all, err);
        if (xs != kOk) return xs;
    }
    trace_phase(C, "encode: rice, rare pairs");
    HostTables tabs;
    build_tables(hdense, rare_pairs, &tabs);
    if (C.trace) {
        size_t nsym = 0, ntab = 0, biggest = 0;
        for (int e = 0; e < 256; ++e)
            if (!tabs.sym[e].empty()) { ++ntab; nsym += tabs.sym[e].size(); biggest = std::max(biggest, tabs.sym[e].size()); }
        std::fprintf(stderr, "[crx-host] tables: %zu, symbols %zu (largest %zu), rare pairs %zu, groups %lld\n", ntab, nsym,
                     biggest, rare_pairs.size(), static_cast<long long>(ng));
    }

    trace_phase(C, "encode: huffman (host)");
    // ---- upload rice, block starts, code tables
    std::vector<uint32_t> dense_code(256 * DENSE_SYM, 0);
    std::vector<uint64_t> rare_codes;
    rare_codes.reserve(rare_pairs.size());
    for (int e = 0; e < 256; ++e) {
        for (size_t k = 0; k < tabs.sym[e].size(); ++k) {
            const uint32_t z = tabs.sym[e][k];
            const uint32_t cl = tabs.code[e][k] | (uint32_t(tabs.len[e][k]) << 24);
            if (z < DENSE_SYM) dense_code[size_t(e) * DENSE_SYM + z] = cl;
            else rare_codes.push_back((uint64_t((uint32_t(e) << 17) | z) << 32) | cl);
        }
    }
    CRX_CUDA(ensure_dev(C.b[S_DENSE_CODE], sizeof(uint32_t) * 256 * DENSE_SYM, st));
    if (!rare_codes.empty()) {
        if (C.b[S_BIG_CODE].cap < sizeof(uint32_t) * 256 * size_t(kSymSpace))
            CRX_CUDA(ensure_dev(C.b[S_BIG_CODE], sizeof(uint32_t) * 256 * size_t(kSymSpace), st));
        CRX_CUDA(ensure_dev(C.b[S_RARE_CODES], sizeof(uint64_t) * rare_codes.size(), st));
    }
    const size_t up_bytes = ng + 8 * (size_t(ng) + 1) + 4 * 256 * DENSE_SYM + 8 * rare_codes.size() + 64;
    CRX_CUDA(ensure_host(C, up_bytes, st));
    h = static_cast<uint8_t*>(C.host);
    size_t o = 0;
    std::memcpy(h + o, gblock.data(), 8 * (size_t(ng) + 1));
    CRX_CUDA(cudaMemcpyAsync(g_block, h + o, 8 * (size_t(ng) + 1), cudaMemcpyHostToDevice, st));
    o += 8 * (size_t(ng) + 1);
    std::memcpy(h + o, dense_code.data(), 4 * 256 * DENSE_SYM);
    CRX_CUDA(cudaMemcpyAsync(C.b[S_DENSE_CODE].p, h + o, 4 * 256 * DENSE_SYM, cudaMemcpyHostToDevice, st));
    o += 4 * 256 * DENSE_SYM;
    if (!rare_codes.empty()) {
        std::memcpy(h + o, rare_codes.data(), 8 * rare_codes.size());
        CRX_CUDA(cudaMemcpyAsync(C.b[S_RARE_CODES].p, h + o, 8 * rare_codes.size(), cudaMemcpyHostToDevice, st));
        o += 8 * rare_codes.size();
        { KernelScope ks_(C, "k_scatter_codes", st);
        k_scatter_codes<<<unsigned((rare_codes.size() + 255) / 256), 256, 0, st>>>(
            dev<uint64_t>(C, S_RARE_CODES), int64_t(rare_codes.size()), dev<uint32_t>(C, S_BIG_CODE));
        }
        CRX_CUDA(cudaGetLastError());
    }
    std::memcpy(h + o, rice.data(), size_t(ng));
    CRX_CUDA(cudaMemcpyAsync(g_rice, h + o, size_t(ng), cudaMemcpyHostToDevice, st));
    o += size_t(ng);
    trace_phase(C, "encode: code tables up");

    // ---- block lengths, offsets, payload
    CRX_CUDA(ensure_dev(C.b[S_BLOCK_BITS], sizeof(uint64_t) * size_t(n_blocks), st));
    CRX_CUDA(ensure_dev(C.b[S_BB32], sizeof(uint32_t) * size_t(n_blocks), st));
    CRX_CUDA(ensure_dev(C.b[S_SCAN_TMP], sizeof(uint64_t) * (exclusive_scan_tmp_elems(n_blocks) + 2), st));
    const uint32_t* big_code = rare_codes.empty() ? dev<uint32_t>(C, S_DENSE_CODE) : dev<uint32_t>(C, S_BIG_CODE);
    const unsigned warps_grid = unsigned((n_blocks * 32 + 255) / 256);
    CRX_CUDA(ensure_dev(C.b[S_PACK_SLOTS], sizeof(uint32_t) * SLOT_WORDS * size_t(n_blocks), st));
    { KernelScope ks_(C, "k_pack_slots", st);
    k_pack_slots<<<warps_grid, 256, 0, st>>>(g_start, g_exp, g_rice, g_block, ng, n_blocks, local, vals,
                                             dev<uint32_t>(C, S_DENSE_CODE), big_code, dev<uint32_t>(C, S_PACK_SLOTS),
                                             dev<uint64_t>(C, S_BLOCK_BITS), dev<uint32_t>(C, S_BB32), counters);
    }
    CRX_CUDA(cudaGetLastError());
    uint64_t* scan_tmp = dev<uint64_t>(C, S_SCAN_TMP);
    uint64_t* d_total_bits = scan_tmp + exclusive_scan_tmp_elems(n_blocks);
    launch_exclusive_scan_u64(C, dev<uint64_t>(C, S_BLOCK_BITS), n_blocks, scan_tmp, d_total_bits, st);
    CRX_CUDA(cudaMemcpyAsync(hostc, d_total_bits, 8, cudaMemcpyDeviceToHost, st));
    CRX_CUDA(cudaMemcpyAsync(hostc + 1, counters + 1, 8, cudaMemcpyDeviceToHost, st));
    // ---- header (wire.py:64-89), built while the GPU packs; a device result also gets its parse
    //      up to the block table now (the rest, the payload length, after the lengths are known)
    out->head.clear();
    out->head.reserve(4096);
    put_prefix(out->head, tabs);
    // tensors present = those with groups, in caller order; a part of a global update keeps its
    // tensor headers apart and counts the whole update's tensors
    std::vector<uint8_t>& ob = gx ? out->part_tensors : out->head;
    std::vector<int64_t> t_first(static_cast<size_t>(nt), -1), t_ng(static_cast<size_t>(nt), 0);
    for (int64_t g = 0; g < ng; ++g) {
        const int t = hg_tensor[size_t(g)];
        if (t_first[size_t(t)] < 0) t_first[size_t(t)] = g;
        t_ng[size_t(t)]++;
    }
    uint64_t n_present = uint64_t(n_present_local);
    if (gx) {
        n_present = 0;
        for (uint64_t v : np_all) n_present += v;
    }
    put_varint(out->head, n_present);
    for (int t = 0; t < nt; ++t) {
        if (!t_ng[size_t(t)]) continue;
        const int ct = tmap[size_t(t)];
        const uint64_t chk = T[size_t(t)].want_full ? hchk[size_t(nt + t)] : cache_chk[ct] + hchk[size_t(t)];
        out->checksums[size_t(ct)] = chk;
        out->present[size_t(ct)] = 1;
        put_varint(ob, uint64_t(name_len[ct]));
        ob.insert(ob.end(), names[ct], names[ct] + name_len[ct]);
        put_varint(ob, uint64_t(numel[ct]));
        for (int k = 0; k < 8; ++k) ob.push_back(uint8_t(chk >> (8 * k)));
        put_varint(ob, uint64_t(t_ng[size_t(t)]));
        for (int64_t g = t_first[size_t(t)]; g < t_first[size_t(t)] + t_ng[size_t(t)]; ++g) {
            ob.push_back(uint8_t(hg_exp[size_t(g)]));
            put_varint(ob, hg_count[size_t(g)]);
            ob.push_back(rice[size_t(g)]);
        }
    }
    if (device_result && !gx) {
        out->pre = std::make_unique<Update>();
        int64_t nd = 0;
        std::string pmsg;
        // the update's length is not known yet: any bound past the block table serves here
        const int64_t t1 = int64_t(out->head.size()) + 4 * n_blocks;
        const Status ps = parse_head_device_table(out->head.data(), int64_t(out->head.size()), t1 + (int64_t(1) << 60), 0,
                                                  out->pre.get(), &nd, &pmsg);
        if (ps != kNeedMore || out->pre->block_table_offset != int64_t(out->head.size()) || out->pre->n_blocks != n_blocks)
            out->pre.reset();   // (not expected) the parse is then done in full when asked for
    }
    CRX_CUDA(cudaStreamSynchronize(st));
    const uint64_t total_bits = hostc[0];
    trace_phase(C, "encode: block bits (sync 4)");
    if (hostc[1] & ERR_BLOCK_TOO_LONG) {
        *err = "a block exceeds 2^32 bits; the update cannot be represented";
        return kValueError;
    }
    uint64_t bit_before = 0, bits_all = total_bits;   // global mode: this part's offset, the update's bits
    if (gx) {
        std::vector<uint64_t> bits;
        const Status xs = exchange_per_rank(*gx, total_bits, &bits, err);
        if (xs != kOk) return xs;
        bits_all = 0;
        for (int r = 0; r < gx->world; ++r) { if (r < gx->rank) bit_before += bits[size_t(r)]; bits_all += bits[size_t(r)]; }
    }
    const uint32_t bit0 = uint32_t(bit_before & 7);
    const uint64_t payload_len = (bit0 + total_bits + 7) / 8;
    const size_t n_words = size_t((bit0 + total_bits + 31) / 32) + 4;
    CRX_CUDA(ensure_dev(C.b[S_PAYLOAD], 4 * n_words, st));
    CRX_CUDA(cudaMemsetAsync(C.b[S_PAYLOAD].p, 0, 4 * n_words, st));
    { KernelScope ks_(C, "k_compact", st);
    k_compact<<<warps_grid, 256, 0, st>>>(g_start, g_exp, g_rice, g_block, ng, n_blocks, local, vals,
                                          dev<uint32_t>(C, S_DENSE_CODE), big_code, dev<uint32_t>(C, S_PACK_SLOTS),
                                          dev<uint64_t>(C, S_BLOCK_BITS), dev<uint32_t>(C, S_BB32),
                                          dev<uint32_t>(C, S_PAYLOAD), bit0);
    }
    CRX_CUDA(cudaGetLastError());
    // block table and payload go to pinned memory in one pass each (below), or stay on the device
    out->len_varint.clear();
    put_varint(out->len_varint, gx ? (bits_all + 7) / 8 : payload_len);
    if (gx) {
        out->part = true;
        out->bit_offset = bit_before;
        out->total_bits = bits_all;
    }
    out->n_blocks = n_blocks;
    out->payload_len = payload_len;
    out->changes = total;
    if (!gx) out->total_bits = total_bits;
    if (device_result) {   // block table and payload stay on the device; only the error flags come back
        CRX_CUDA(chunk_events(C, 1));
        CRX_CUDA(cudaMemcpyAsync(C.small + kEncStatusWord, counters + 1, 8, cudaMemcpyDeviceToHost, st));
        CRX_CUDA(cudaEventRecord(C.copy_ev[0], st));
        out->stream = st;
        out->device = true;
        out->dtable = static_cast<const uint8_t*>(C.b[S_BB32].p);
        out->dpay = static_cast<const uint8_t*>(C.b[S_PAYLOAD].p);
        C.live = out;
        return kOk;
    }
    // block table, error flags and payload go to pinned memory behind k_compact; nothing waits for
    // them here: the serializer pre-faults its destination meanwhile (Encoded::write)
    const size_t bt = 4 * size_t(n_blocks);
    CRX_CUDA(ensure_pinned(C.out_host, bt + payload_len + 16, st));
    uint8_t* oh = static_cast<uint8_t*>(C.out_host.p);
    CRX_CUDA(chunk_events(C, 1 + size_t((payload_len + kCopyChunk - 1) / kCopyChunk)));
    CRX_CUDA(cudaMemcpyAsync(oh, C.b[S_BB32].p, bt, cudaMemcpyDeviceToHost, st));
    CRX_CUDA(cudaMemcpyAsync(C.small + kEncStatusWord, counters + 1, 8, cudaMemcpyDeviceToHost, st));
    CRX_CUDA(cudaEventRecord(C.copy_ev[0], st));
    const uint8_t* dpay = static_cast<const uint8_t*>(C.b[S_PAYLOAD].p);
    for (uint64_t off = 0, k = 0; off < payload_len; off += kCopyChunk, ++k) {
        const size_t len = size_t(std::min<uint64_t>(kCopyChunk, payload_len - off));
        CRX_CUDA(cudaMemcpyAsync(oh + bt + off, dpay + off, len, cudaMemcpyDeviceToHost, st));
        CRX_CUDA(cudaEventRecord(C.copy_ev[1 + k], st));
    }
    trace_phase(C, "encode: copies queued");
    out->stream = st;
    out->table = oh;
    out->pending = true;
    C.live = out;
    out->changes = total;
    return kOk;
}

}  // namespace crx
