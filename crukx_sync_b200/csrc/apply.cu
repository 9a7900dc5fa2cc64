// Apply: verify a parsed crukx-sync update against the receiver's bf16 weights and commit it in
// place, all or nothing (reference src/crukx_sync/codec.py:578-717).
//
//   k_app_hist     old-exponent histogram per super-tile (+ full checksum when the receiver has no
//                  trusted cached checksum, codec.py:702-705); column scans give every
//                  super-tile its per-exponent offset and every group its exact size.
//   k_decode       one thread per 256-change block: Golomb-Rice gap + canonical Huffman residual,
//                  with the reference's validation (codec.py:504-575, _triton.py:34-88): overrun,
//                  q > q_max, no code, block not consumed exactly.  Unary runs longer than one
//                  64-bit window are followed inside the block's own bits only.  It writes the
//                  running sum of gap + 1 inside the block and the block's group.
//   k_locals       group-local index = the block's base (the group's earlier blocks' sums) + the
//                  in-block running sum (codec.py:640-642), range checks (codec.py:696-697).
//   k_map          per super-tile: per-lane masks of the old exponents over a 16-exponent window,
//                  then every change is placed by (exponent, local rank) -> position through
//                  selection on the masks' counts (codec.py:654-694) and written in place (device
//                  weights; its old value kept in the commit list) or staged (host weights), the
//                  checksum delta accumulated (codec.py:698-700).
//   host verdict   one synchronisation: decode/range flags and per-tensor checksums; a failed one
//                  has k_commit write the old values back, so nothing is left written.
//   k_commit       scatter of the list's values at its positions (codec.py:713-714): the undo
//                  above, or the new values into the device copies of host weights.
#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "capi_internal.h"
#include "common.cuh"

namespace crx {

namespace {

constexpr uint32_t FULL = 0xffffffffu;
constexpr int LUT_BITS = 10;

struct AppTensor {
    int16_t* w;
    int64_t numel;
    int64_t super_begin;
    int32_t want_full;
    int32_t g_begin;
    int32_t g_end;
    int32_t pad;
    const uint32_t* hcache;   // the tensor's cached histogram rows (null: compute them)
};

struct AppGroup {
    uint64_t start;      // first change of the group (update-wide index)
    uint64_t count;
    int32_t tensor;
    int32_t exp;
    int32_t rice;
    int32_t table;
};

struct DecTable {
    uint32_t first[kMaxCodeLen + 1];
    uint32_t base[kMaxCodeLen + 1];
    uint32_t limit[kMaxCodeLen + 1];
    uint32_t sym_off;
    uint32_t nsym;
    uint32_t lut[1 << LUT_BITS];   // len << 24 | symbol for codes of <= LUT_BITS bits, else 0
};

__device__ __forceinline__ int tensor_of_super(const AppTensor* T, int nT, int64_t s) {
    int lo = 0, hi = nT - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (T[mid].super_begin <= s) lo = mid; else hi = mid - 1;
    }
    return lo;
}

__device__ __forceinline__ int64_t last_le(const uint64_t* __restrict__ a, int64_t n, uint64_t v) {
    int64_t lo = 0, hi = n - 1;
    while (lo < hi) {
        const int64_t mid = (lo + hi + 1) >> 1;
        if (a[mid] <= v) lo = mid; else hi = mid - 1;
    }
    return lo;
}

__device__ __forceinline__ uint64_t bswap64(uint64_t x) {
    const uint32_t lo = uint32_t(x), hi = uint32_t(x >> 32);
    return (uint64_t(bswap32(lo)) << 32) | bswap32(hi);
}

// 64 payload bits starting at bit `pos`, MSB first.  The buffer carries >= 16 zero bytes past the
// payload, so every read the decoder makes (pos <= block end) stays inside it.
__device__ __forceinline__ uint64_t read64(const uint64_t* __restrict__ W, uint64_t pos) {
    const uint64_t w = pos >> 6;
    const int s = int(pos & 63);
    const uint64_t hi = bswap64(__ldg(W + w));
    if (!s) return hi;
    const uint64_t lo = bswap64(__ldg(W + w + 1));
    return (hi << s) | (lo >> (64 - s));
}

// ------------------------------------------------------------------ histogram of old exponents

constexpr int HIST_THREADS = 512;

__global__ void __launch_bounds__(HIST_THREADS) k_app_hist(const AppTensor* __restrict__ T, int nT, uint32_t* __restrict__ HS,
                                                           unsigned long long* __restrict__ chk_full) {
    __shared__ uint32_t hist[HIST_THREADS / 32][256];
    __shared__ uint64_t red[HIST_THREADS / 32];
    const int64_t s = blockIdx.x;
    const int t = tensor_of_super(T, nT, s);
    const AppTensor tt = T[t];
    if (tt.hcache) {   // histogram cached by the previous apply: no pass over the weights
        for (int k = threadIdx.x; k < 256; k += HIST_THREADS) HS[s * 256 + k] = tt.hcache[(s - tt.super_begin) * 256 + k];
        return;
    }
    const int64_t e0 = (s - tt.super_begin) * SUPER_N;
    const int64_t e1 = min(tt.numel, e0 + SUPER_N);
    const int w = threadIdx.x >> 5;
    for (int k = threadIdx.x; k < (HIST_THREADS / 32) * 256; k += HIST_THREADS) (&hist[0][0])[k] = 0;
    __syncthreads();
    uint64_t full = 0;
    const int16_t* p = tt.w + e0;
    const int64_t n = e1 - e0;
    if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
        const uint4* v = reinterpret_cast<const uint4*>(p);
        const int64_t nv = n / 8;
        for (int64_t k = threadIdx.x; k < nv; k += HIST_THREADS) {
            const uint4 q = __ldcs(v + k);
            const uint32_t ws[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                atomicAdd(&hist[w][(ws[h] >> 7) & 0xFF], 1u);
                atomicAdd(&hist[w][(ws[h] >> 23) & 0xFF], 1u);
            }
            if (tt.want_full) {
                const uint64_t i0 = uint64_t(e0 + 8 * k);
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    full += uint64_t(ws[h] & 0xFFFF) * splitmix_weight(i0 + 2 * h);
                    full += uint64_t(ws[h] >> 16) * splitmix_weight(i0 + 2 * h + 1);
                }
            }
        }
        for (int64_t i = nv * 8 + threadIdx.x; i < n; i += HIST_THREADS) {
            const uint32_t x = uint16_t(p[i]);
            atomicAdd(&hist[w][(x >> 7) & 0xFF], 1u);
            if (tt.want_full) full += uint64_t(x) * splitmix_weight(uint64_t(e0 + i));
        }
    } else {
        for (int64_t i = threadIdx.x; i < n; i += HIST_THREADS) {
            const uint32_t x = uint16_t(p[i]);
            atomicAdd(&hist[w][(x >> 7) & 0xFF], 1u);
            if (tt.want_full) full += uint64_t(x) * splitmix_weight(uint64_t(e0 + i));
        }
    }
    __syncthreads();
    if (threadIdx.x < 256) {
        uint32_t a = 0;
        for (int ww = 0; ww < HIST_THREADS / 32; ++ww) a += hist[ww][threadIdx.x];
        HS[s * 256 + threadIdx.x] = a;
    }
    if (tt.want_full) block_add_u64<HIST_THREADS>(full, &chk_full[t], red);
}

// ------------------------------------------------------------------ block decoder
//
// One thread per 256-change block.  Each thread reads its block through a private 64-bit bit
// buffer (bits [pos, pos + avail) MSB-aligned, zeros below), refilled 32 big-endian bits at a time
// from 16-byte payload loads made ahead of use; no shared memory, so occupancy is set by
// registers.  Steps whose unary run, remainder and longest code do not fit in the buffer (long
// unary runs, large Rice parameters) take the generic reader at absolute positions.

constexpr int DEC_THREADS = 256;

// canonical code at the top of `peek` (17 bits): its length and symbol; false if none.  Codes of
// up to LUT_BITS bits (nearly all) take one table load; longer ones search the lengths.
__device__ __forceinline__ bool find_code(const DecTable* __restrict__ tab, const uint32_t* __restrict__ SY,
                                          uint32_t nsym1, uint32_t peek, int& L, uint32_t& sym) {
    const uint32_t lv = tab->lut[peek >> (kMaxCodeLen - LUT_BITS)];
    if (lv) {
        L = int(lv >> 24);
        sym = lv & 0xFFFFFFu;
        return true;
    }
    L = LUT_BITS + 1;   // no code of <= LUT_BITS bits starts with these bits
    while (L <= kMaxCodeLen && peek >= tab->limit[L]) ++L;
    if (L > kMaxCodeLen) return false;
    sym = SY[tmin(tab->base[L] + (peek >> (kMaxCodeLen - L)) - tab->first[L], nsym1)];
    return true;
}

// The generic step of k_decode: a unary run that does not fit the bit buffer (more than ~30 ones,
// or a large Rice parameter) is followed window by window at absolute positions, never past the
// block's end or past q_max, so hostile updates cost at most their own bits.  ok = false on a
// decode error; otherwise pos is past the change.  (Inlined: a call costs the main loop registers.)
struct GenericStep {
    uint64_t pos, gap;
    uint32_t sym;
    bool ok;
};

__device__ __forceinline__ GenericStep decode_generic(const uint64_t* __restrict__ W, uint64_t p, uint64_t end, uint64_t qmax,
                                                      int rice, const DecTable* __restrict__ tab,
                                                      const uint32_t* __restrict__ SY, uint32_t nsym1) {
    GenericStep r{p, 0, 0, false};
    uint64_t y = ~read64(W, p);
    uint64_t qq;
    if (y) {
        qq = uint64_t(__clzll(y));
    } else {
        qq = 64;
        while (qq <= qmax && p + qq < end) {
            y = ~read64(W, p + qq);
            if (y) { qq += uint64_t(__clzll(y)); break; }
            qq += 64;
        }
    }
    if (qq > qmax || p + qq >= end) return r;
    const uint64_t c = p + qq + 1;
    const uint64_t x = read64(W, c);
    const uint64_t rem = rice ? (x >> (64 - rice)) : 0;
    int L;
    if (!find_code(tab, SY, nsym1, uint32_t((x << rice) >> (64 - kMaxCodeLen)), L, r.sym)) return r;
    r.gap = (qq << rice) | rem;
    r.pos = c + uint64_t(rice) + uint64_t(L);
    r.ok = true;
    return r;
}

__device__ __forceinline__ uint32_t clamp32(uint64_t v) { return v > 0xFFFFFFFFull ? 0xFFFFFFFFu : uint32_t(v); }

// One thread per 256-change block.  Outputs go through shared memory: every DEC_CH changes a lane's
// values wait in its row, then the warp stores them with consecutive lanes on consecutive indices
// (16 lanes per block row), so a store instruction writes two runs of 64 bytes instead of 32
// scattered words.
constexpr int DEC_CH = 16;

__global__ void __launch_bounds__(DEC_THREADS) k_decode(const uint64_t* __restrict__ W, uint64_t n32,
                                                        const uint32_t* __restrict__ bb, const uint64_t* __restrict__ boff,
                                                        int64_t n_blocks, const AppGroup* __restrict__ G,
                                                        const uint64_t* __restrict__ gblock, int64_t ng,
                                                        const DecTable* __restrict__ TB, const uint32_t* __restrict__ SYMS,
                                                        const uint64_t* __restrict__ GS, uint32_t* __restrict__ inblk,
                                                        uint32_t* __restrict__ zz, uint64_t* __restrict__ bsum,
                                                        int32_t* __restrict__ bgroup, unsigned long long* __restrict__ counters) {
    __shared__ uint32_t sg[DEC_THREADS / 32][32 * (DEC_CH + 1)];   // per warp: each lane's staged gaps (rows padded)
    __shared__ uint32_t sz[DEC_THREADS / 32][32 * (DEC_CH + 1)];   // and residual symbols
    const int lane = threadIdx.x & 31, wq = threadIdx.x >> 5;
    const int64_t b = int64_t(blockIdx.x) * DEC_THREADS + threadIdx.x;
    const bool live = b < n_blocks;   // lanes past the last block only take part in the warp's stores
    const int64_t g = live ? last_le(gblock, ng, uint64_t(b)) : 0;
    if (live) bgroup[b] = int32_t(g);
    const AppGroup grp = live ? G[g] : AppGroup{};
    const uint64_t kb = live ? uint64_t(b) - gblock[g] : 0;
    const int cnt = live ? int(tmin<uint64_t>(kBlock, grp.count - kb * kBlock)) : 0;
    const uint64_t ebase = grp.start + kb * kBlock;
    const uint64_t pos0 = live ? boff[b] : 0;
    const uint64_t qmax = live ? GS[int64_t(grp.tensor) * 256 + grp.exp] >> grp.rice : 0;
    const uint32_t qmax32 = uint32_t(tmin<uint64_t>(qmax, 0xFFFFFFFFull));   // the fast path's q is below 64
    const int rice = grp.rice;
    const DecTable* tab = TB + (live ? grp.table : 0);
    const uint32_t* SY = SYMS + (live ? tab->sym_off : 0);
    const uint32_t nsym1 = live ? tab->nsym - 1 : 0;
    const uint32_t* W32 = reinterpret_cast<const uint32_t*>(W);
    const uint64_t last32 = n32 - 1;
    // bits [pos0 + rel, pos0 + rel + avail) of the payload sit MSB-aligned in buf (zeros below);
    // the next word to enter it is `nextw`, loaded one refill ahead; blen = the block's bits
    const uint64_t blen = live ? bb[b] : 0;
    uint64_t rel = 0;
    uint64_t wi = 0, buf = 0;
    uint32_t nextw = 0;
    int avail = 0;
    auto word = [&](uint64_t i) { return bswap32(__ldg(W32 + tmin(i, last32))); };
    auto fill = [&]() {   // buffer := 64 - (pos & 31) bits from pos
        const uint64_t p = pos0 + rel;
        wi = p >> 5;
        buf = ((uint64_t(word(wi)) << 32) | word(wi + 1)) << (p & 31);
        avail = 64 - int(p & 31);
        nextw = word(wi + 2);
        wi += 3;
    };
    if (live) fill();
    // one change: Rice gap and canonical-code symbol, with the reference's validation; false on error
    auto one = [&](uint64_t& gap, uint32_t& sym) -> bool {
        if (rel >= blen) return false;
        const int q = __clzll(~buf);   // ones ahead; bits past `avail` are zeros, so q < avail when it fits
        if (q + 1 + rice + kMaxCodeLen <= avail) {
            if (uint32_t(q) > qmax32 || rel + uint64_t(q) >= blen) return false;
            uint64_t t = buf << (q + 1);
            const uint64_t rem = rice ? (t >> (64 - rice)) : 0;
            t <<= rice;
            int L;
            if (!find_code(tab, SY, nsym1, uint32_t(t >> (64 - kMaxCodeLen)), L, sym)) return false;
            gap = (uint64_t(q) << rice) | rem;
            const int used = q + 1 + rice + L;
            buf = t << L;
            avail -= used;
            rel += uint64_t(used);
            if (avail <= 32) {   // used <= avail before, so one word brings it above 32 again
                buf |= uint64_t(nextw) << (32 - avail);
                avail += 32;
                nextw = word(wi++);
            }
            return true;
        }
        const GenericStep r = decode_generic(W, pos0 + rel, pos0 + blen, qmax, rice, tab, SY, nsym1);
        if (!r.ok) return false;
        rel = r.pos - pos0;
        gap = r.gap;
        sym = r.sym;
        fill();
        return true;
    };
    uint64_t sum = 0;
    bool ok = live;
    uint32_t* mg = &sg[wq][lane * (DEC_CH + 1)];
    uint32_t* mz = &sz[wq][lane * (DEC_CH + 1)];
    for (int c0 = 0; __any_sync(FULL, ok && c0 < cnt); c0 += DEC_CH) {
        const int n = ok ? tmax(0, tmin(DEC_CH, cnt - c0)) : 0;
        int got = 0;
        for (; got < n; ++got) {
            uint64_t gp;
            uint32_t sy;
            ok = one(gp, sy);
            if (!ok) break;
            sum += gp + 1;
            mg[got] = clamp32(sum - 1);   // in-block local index: gap 0 is the first change's
            mz[got] = sy;
        }
        __syncwarp();
        // lanes 0-15 store lane 2i's staged values, lanes 16-31 lane 2i+1's
        const int k2 = lane & 15;
#pragma unroll 4
        for (int i = 0; i < 16; ++i) {
            const int t = 2 * i + (lane >> 4);
            const int gt = __shfl_sync(FULL, got, t);
            const uint64_t dst = __shfl_sync(FULL, ebase, t) + uint64_t(c0 + k2);
            if (k2 < gt) {
                inblk[dst] = sg[wq][t * (DEC_CH + 1) + k2];
                zz[dst] = sz[wq][t * (DEC_CH + 1) + k2];
            }
        }
        __syncwarp();
    }
    if (!live) return;
    ok = ok && rel == blen;
    bsum[b] = ok ? sum : 0;
    if (!ok) atomicOr(&counters[1], (unsigned long long)ERR_DECODE);
}

// group-local index of every change: its block's base (the sums of gap + 1 over the group's earlier
// blocks, from the scan of the blocks' sums) plus the running sum inside the block that k_decode
// wrote.  An index at or past the group's size is a range error; since indices grow by at least
// one per change, that also covers every gap at or past the size (codec.py:696-697).  A warp per
// block, in place.
__global__ void __launch_bounds__(256) k_locals(const uint64_t* __restrict__ bscan, int64_t n_blocks,
                                                const AppGroup* __restrict__ G, const uint64_t* __restrict__ gblock,
                                                const int32_t* __restrict__ bgroup, const uint64_t* __restrict__ GS,
                                                uint32_t* __restrict__ local, unsigned long long* __restrict__ counters) {
    const int64_t b = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (b >= n_blocks) return;
    const int32_t g = bgroup[b];
    const AppGroup grp = G[g];
    const uint64_t gb = gblock[g];
    const uint64_t k = uint64_t(b) - gb;
    const uint32_t cnt = uint32_t(tmin<uint64_t>(kBlock, grp.count - k * kBlock));
    uint32_t* const v = local + grp.start + k * kBlock;
    const uint64_t size = GS[int64_t(grp.tensor) * 256 + grp.exp];
    const uint64_t base = bscan[b] - bscan[gb];
    bool bad = false;
    static_assert(kBlock == 256, "eight chunks of 32 per block");
    uint32_t in[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) in[u] = uint32_t(32 * u + lane) < cnt ? v[32 * u + lane] : 0u;   // loads together
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        if (uint32_t(32 * u + lane) < cnt) {
            const uint64_t loc = base + in[u];
            bad |= loc >= size;
            v[32 * u + lane] = loc > 0xFFFFFFFFull ? 0xFFFFFFFFu : uint32_t(loc);
        }
    }
    if (__any_sync(FULL, bad) && lane == 0) atomicOr(&counters[1], (unsigned long long)ERR_RANGE);
}

// ------------------------------------------------------------------ (exponent, rank) -> position
//
// Every super-tile picks the 16 consecutive old exponents that hold most of its elements (its
// histogram is known from the column scans).  Per sub-tile every lane marks, for its own run of 32
// elements, which elements carry each window exponent (one 32-bit mask per window row; one more
// row for the elements outside the window).  A change with exponent e and rank r among the
// sub-tile's elements of exponent e is then found by selection: the warp whose exclusive base is
// the last <= r, the lane likewise, and the r-th set bit of that lane's mask.  Elements outside the
// window (zeros, tiny or huge weights) are few: their positions are listed in (exponent, index)
// order by warp matching, into the super-tile's slot of a global scratch list.  Changes are
// written (and listed) in position order per warp span, which keeps the scattered 2-byte writes of
// one region together in L2.

constexpr int MP_THREADS = 256;
constexpr int MP_WARPS = MP_THREADS / 32;
constexpr int MP_SUB = 8192;
constexpr int MP_SPAN = MP_SUB / MP_WARPS;   // 1024
constexpr int MP_RUN = MP_SPAN / 32;         // 32
constexpr int MWIN = 16;
constexpr int MP_PRE = 3;                    // groups per warp whose first changes are loaded ahead
static_assert(MP_SUB * 32 == SUPER_N, "32 sub-tiles per super-tile");

struct MapSmem {
    uint32_t msk[MP_WARPS][MWIN + 1][32];  // per lane and window row: its run's elements of that exponent (row MWIN: outside)
    uint8_t nz8[MP_SUB];                   // zigzag residual of every changed position; 255: in the escape list.
                                           // Before the placement its first KB holds the outside-window counts.
    uint16_t pre[MP_WARPS][MWIN][16];      // exclusive prefixes over the lanes of the masks' counts, at even lanes
                                           // (first the lanes' counts as bytes, in the same 32 bytes a row)
    uint32_t mark[MP_SUB / 32];            // changed positions
    uint32_t wwin[MP_WARPS][MWIN];         // per-warp window totals, then warp bases
    uint16_t tot[256], estart[256];
    uint32_t pcur[256];
    uint32_t cursor[256], gend[256];      // per group: next change and end, relative to the tensor's first change
    uint32_t nextloc[256];                 // group-local index of each group's next change (~0: none)
    int32_t hdelta[256];                   // this super-tile's histogram, then plus its exponent moves
    uint8_t gexp[256];
    uint32_t oowm[MP_WARPS];               // per warp: its runs that hold outside-window elements
    unsigned long long wkey[MP_WARPS];
    uint32_t ebase;
    uint64_t red[MP_WARPS];
};

static_assert(offsetof(MapSmem, pre) % 16 == 0, "16-byte prefix pieces");

// For every byte value: the positions of its set bits, lowest first, four bits each.
struct NthBitTable {
    uint32_t v[256];
};
constexpr NthBitTable make_nth_bit_table() {
    NthBitTable t{};
    for (int m = 0; m < 256; ++m) {
        uint32_t e = 0;
        int k = 0;
        for (int b = 0; b < 8; ++b)
            if ((m >> b) & 1) e |= uint32_t(b) << (4 * k++);
        t.v[m] = e;
    }
    return t;
}
__device__ const NthBitTable kNthBit = make_nth_bit_table();

// position of the r-th (0-based) set bit of m; m has more than r set bits: the half, then the byte
// by population counts, then the byte's table entry
__device__ __forceinline__ uint32_t nth_set_bit(uint32_t m, uint32_t r) {
    uint32_t pos = 0;
    const uint32_t c16 = __popc(m & 0xFFFFu);
    if (r >= c16) { r -= c16; m >>= 16; pos = 16; }
    const uint32_t c8 = __popc(m & 0xFFu);
    if (r >= c8) { r -= c8; m >>= 8; pos += 8; }
    return pos + ((__ldg(&kNthBit.v[m & 0xFFu]) >> (4 * r)) & 0xFu);
}

__global__ void __launch_bounds__(MP_THREADS, 6)
k_map(const AppTensor* __restrict__ T, int nT, const AppGroup* __restrict__ G, const uint32_t* __restrict__ PS,
      const uint32_t* __restrict__ local, const uint32_t* __restrict__ zz, uint32_t* __restrict__ marks,
      unsigned long long* __restrict__ spanbase, uint16_t* __restrict__ cval, uint64_t stage_cap,
      unsigned long long* __restrict__ chk_delta,
      unsigned long long* __restrict__ staged, const uint64_t* __restrict__ GS, uint32_t* __restrict__ HNEW,
      uint16_t* __restrict__ order_scratch, uint16_t* __restrict__ esc_scratch, int inplace) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    MapSmem& S = *reinterpret_cast<MapSmem*>(smem_raw);
    const int64_t s = blockIdx.x;
    const int t = tensor_of_super(T, nT, s);
    const AppTensor tt = T[t];
    const int64_t e_begin = (s - tt.super_begin) * SUPER_N;
    const int64_t e_end = tmin(tt.numel, e_begin + SUPER_N);
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const uint32_t lt = lanemask_lt();
    const int ngt = tt.g_end - tt.g_begin;
    const int span0 = w * MP_SPAN;
    uint16_t* const order = order_scratch + s * MP_SUB;   // outside-window positions in (exponent, index) order
    uint16_t* const esc = esc_scratch + s * MP_SUB;       // residuals whose zigzag is 255 or more, by position
    uint32_t* const ocnt = reinterpret_cast<uint32_t*>(S.nz8);   // outside-window counts per exponent (before placement)
    const uint64_t tg0 = ngt ? G[tt.g_begin].start : 0;   // the tensor's first change: group cursors are relative to it
    const uint32_t* const lrel = local + tg0;               // indexed by those 32-bit cursors (a tensor has < 2^32 changes)
    const uint32_t* const zrel = zz + tg0;
    S.pcur[tid] = PS[s * 256 + tid];
    {   // this super-tile's histogram: the next row's prefix (or the tensor's total) minus this one's
        const bool last = e_end >= tt.numel;
        const uint32_t nxt = last ? uint32_t(GS[int64_t(t) * 256 + tid]) : PS[(s + 1) * 256 + tid];
        S.hdelta[tid] = int32_t(nxt - S.pcur[tid]);
    }
    __syncthreads();
    {   // the window: 16 consecutive exponents holding the most elements (ties: the lowest start)
        uint64_t key = 0;
        if (tid <= 256 - MWIN) {
            uint32_t sum = 0;
#pragma unroll
            for (int k = 0; k < MWIN; ++k) sum += uint32_t(S.hdelta[tid + k]);
            key = (uint64_t(sum) << 8) | uint64_t(255 - tid);
        }
        for (int o = 16; o; o >>= 1) key = tmax(key, (uint64_t)__shfl_xor_sync(FULL, key, o));
        if (lane == 0) S.wkey[w] = key;
    }
    if (tid < ngt) {
        const AppGroup grp = G[tt.g_begin + tid];
        const uint32_t p0 = S.pcur[grp.exp];
        uint64_t lo = grp.start, hi = grp.start + grp.count;      // first change with local >= p0
        while (lo < hi) {
            const uint64_t mid = (lo + hi) >> 1;
            if (local[mid] < p0) lo = mid + 1; else hi = mid;
        }
        S.cursor[tid] = uint32_t(lo - tg0);
        S.gend[tid] = uint32_t(grp.start + grp.count - tg0);
        S.gexp[tid] = uint8_t(grp.exp);
        S.nextloc[tid] = lo < grp.start + grp.count ? local[lo] : 0xFFFFFFFFu;
    }
    __syncthreads();
    if (tid == 0) {
        unsigned long long k = 0;
        for (int ww = 0; ww < MP_WARPS; ++ww) k = tmax(k, S.wkey[ww]);
        S.ebase = 255u - uint32_t(k & 0xFFu);
    }
    __syncthreads();
    const uint32_t ebase = S.ebase;
    auto row_of = [&](uint32_t e) { return tmin(e - ebase, uint32_t(MWIN)); };   // outside: wraps to MWIN
    uint64_t delta = 0;
    for (int64_t base = e_begin; base < e_end; base += MP_SUB) {
        const int n = int(tmin<int64_t>(MP_SUB, e_end - base));
        const int16_t* p = tt.w + base;
        if (tid == 0 && base + MP_SUB < e_end)     // the next sub-tile streams into L2 meanwhile
            prefetch_l2(p + MP_SUB, size_t(tmin<int64_t>(MP_SUB, e_end - base - MP_SUB)) * 2);
        const int span_n = tmax(0, tmin(MP_SPAN, n - span0));
        const int r0 = lane * MP_RUN;
        const int vn = tmax(0, tmin(MP_RUN, span_n - r0));
        // the first 32 changes of this warp's groups (group k belongs to warp k % MP_WARPS), loaded
        // now so that they arrive while the sub-tile is marked and scanned
        uint32_t pl[MP_PRE], pz[MP_PRE];
#pragma unroll
        for (int j = 0; j < MP_PRE; ++j) {
            const int k = w + MP_WARPS * j;
            pl[j] = 0xFFFFFFFFu;
            pz[j] = 0;
            if (k < ngt) {
                const uint32_t c = S.cursor[k];
                if (uint32_t(lane) < S.gend[k] - c) {   // issued here (volatile), consumed after the marking and scans
                    asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(pl[j]) : "l"(lrel + c + lane));
                    asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(pz[j]) : "l"(zrel + c + lane));
                }
            }
        }
        // ---- this warp's masks to zero, then each lane marks its run
        {
            uint4* m4 = reinterpret_cast<uint4*>(&S.msk[w][0][0]);
            static_assert(sizeof(S.msk[0]) % 16 == 0 && offsetof(MapSmem, msk) % 16 == 0, "uint4 zeroing");
#pragma unroll
            for (int k = lane; k < int(sizeof(S.msk[0]) / 16); k += 32) m4[k] = make_uint4(0, 0, 0, 0);
        }
        __syncwarp();
        {
            uint32_t* mine = &S.msk[w][0][lane];
            const int16_t* run = p + span0 + r0;
            if (vn == MP_RUN && (reinterpret_cast<uintptr_t>(run) & 15) == 0) {
                const uint4* rv = reinterpret_cast<const uint4*>(run);
                uint4 q[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) q[c] = rv[c];
                // both elements of a word at once: per 16-bit half, (e - ebase) mod 2^16 then the
                // minimum with 16 (below the window wraps to 65280 and up) -- row_of for both
                const uint32_t nb = ((0x10000u - ebase) & 0xFFFFu) * 0x00010001u;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const uint32_t wd[4] = {q[c].x, q[c].y, q[c].z, q[c].w};
#pragma unroll
                    for (int h = 0; h < 4; ++h) {
                        const int k = c * 8 + h * 2;
                        const uint32_t r2 = __viaddmin_u16x2((wd[h] >> 7) & 0x00FF00FFu, nb, 0x00100010u);
                        atomicOr(mine + (r2 & 0xFFFFu) * 32, 1u << k);
                        atomicOr(mine + (r2 >> 16) * 32, 2u << k);
                    }
                }
            } else {
                for (int k = 0; k < vn; ++k) mine[row_of((uint32_t(uint16_t(run[k])) >> 7) & 0xFFu) * 32] |= 1u << k;
            }
        }
        S.mark[(span0 >> 5) + lane] = 0;   // this warp's span (its staging below read the last ones)
        __syncwarp();
        const uint32_t oowm = __ballot_sync(FULL, S.msk[w][MWIN][lane] != 0);   // runs with outside elements
        if (lane == 0) S.oowm[w] = oowm;
        // ---- lane prefixes of the window rows.  Every lane writes its run's count of each row as a
        //      byte, into the row's prefix slots; then lane 2d + h turns the 16 bytes of row d's
        //      lanes 16h..16h+15 in place into the exclusive prefixes of its even lanes (16 bits
        //      each: per 4 lanes one byte-dot-product to the middle lane and one over all four)
        {
            uint8_t* const cb = reinterpret_cast<uint8_t*>(&S.pre[w][0][0]);
#pragma unroll
            for (int d = 0; d < MWIN; ++d) cb[d * 32 + lane] = uint8_t(__popc(S.msk[w][d][lane]));
            __syncwarp();
            const int d = lane >> 1, h = lane & 1;
            uint4* const q = reinterpret_cast<uint4*>(cb + d * 32 + h * 16);   // this lane's 16 bytes, in and out
            const uint4 c = *q;
            const uint32_t wd[4] = {c.x, c.y, c.z, c.w};
            uint32_t run = 0, out[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                out[k] = run | (__dp4a(wd[k], 0x0101u, run) << 16);   // lanes 4k and 4k + 2
                run = __dp4a(wd[k], 0x01010101u, run);
            }
            const uint32_t lo = __shfl_xor_sync(FULL, run, 1);   // at odd lanes: the first 16 lanes' total
            if (h) {
#pragma unroll
                for (int k = 0; k < 4; ++k) out[k] += lo * 0x00010001u;
                S.wwin[w][d] = run + lo;
            }
            *q = make_uint4(out[0], out[1], out[2], out[3]);
        }
        const bool any_out = __syncthreads_or(oowm != 0);
        auto exp_at = [&](int i) { return (uint32_t(uint16_t(p[i])) >> 7) & 0xFFu; };
        // outside-window elements of the whole sub-tile in index order, by one warp (they are rare):
        // slots from warp matching over the counters
        auto rank_outside = [&](bool list) {
            for (int k = lane; k < 256; k += 32) ocnt[k] = 0;
            __syncwarp();
            for (int ww = 0; ww < MP_WARPS; ++ww) {
                const int sn = tmax(0, tmin(MP_SPAN, n - ww * MP_SPAN));
                for (uint32_t m = S.oowm[ww]; m; m &= m - 1) {
                    const int ii = (__ffs(m) - 1) * MP_RUN + lane;
                    const uint32_t e = ii < sn ? exp_at(ww * MP_SPAN + ii) : 0u;
                    const bool outside = ii < sn && row_of(e) == uint32_t(MWIN);
                    const uint32_t r = warp_rank(ocnt, e, outside, lt, lane);
                    if (list && outside) order[S.estart[e] + r] = uint16_t(ww * MP_SPAN + ii);
                }
            }
        };
        if (any_out) {   // first pass: the counts
            if (w == 0) rank_outside(false);
            __syncthreads();
        }
        {   // warp bases of the window rows and the sub-tile's totals
            const int e = tid;
            uint32_t o = any_out ? ocnt[e] : 0u;
            const uint32_t d = uint32_t(e) - ebase;
            if (d < uint32_t(MWIN)) {
                uint32_t a = 0;
                for (int ww = 0; ww < MP_WARPS; ++ww) {
                    const uint32_t v = S.wwin[ww][d];
                    S.wwin[ww][d] = a;
                    a += v;
                }
                o += a;
            }
            S.tot[e] = uint16_t(o);
        }
        __syncthreads();
        if (any_out) {   // second pass: bucket starts, then every outside element's slot
            if (w == 0) {
                uint32_t v[8], sum = 0;
#pragma unroll
                for (int k = 0; k < 8; ++k) { v[k] = S.tot[lane * 8 + k]; sum += v[k]; }
                uint32_t incl = sum;
                for (int o = 1; o < 32; o <<= 1) {
                    const uint32_t y = __shfl_up_sync(FULL, incl, o);
                    if (lane >= o) incl += y;
                }
                uint32_t run = incl - sum;
#pragma unroll
                for (int k = 0; k < 8; ++k) { S.estart[lane * 8 + k] = uint16_t(run); run += v[k]; }
                __syncwarp();
                rank_outside(true);
            }
            __syncthreads();
        }
        // ---- place this sub-tile's changes: group k is placed by warp k % MP_WARPS, which knows its
        //      groups' first changes already; groups whose next change lies beyond this sub-tile are
        //      skipped from shared memory.  A change leaves its residual and its mark; the old value
        //      is read when the span is staged.  The next chunk of a group is loaded while this one is
        //      placed.
        auto place_group = [&](int k, uint32_t lc, uint32_t z) {
            const uint32_t e = S.gexp[k];
            const uint32_t lo = S.pcur[e], tot = S.tot[e];
            if (S.nextloc[k] - lo >= tot) return;
            const uint32_t d = row_of(e);
            const uint32_t ge = S.gend[k];
            uint32_t cur = S.cursor[k];   // <= ge, so ge - cur does not wrap
            uint32_t next;
            for (;;) {
                uint32_t lcn = 0xFFFFFFFFu, zn = 0;
                if (32u + uint32_t(lane) < ge - cur) { lcn = lrel[cur + 32u + lane]; zn = zrel[cur + 32u + lane]; }
                const bool valid = lc != 0xFFFFFFFFu && lc >= lo && lc - lo < tot;
                if (valid) {
                    uint32_t r = lc - lo;
                    int i;
                    if (d < uint32_t(MWIN)) {
                        int ww = 0;                  // last warp whose base is <= r
#pragma unroll
                        for (int st = MP_WARPS / 2; st; st >>= 1) ww += S.wwin[ww + st][d] <= r ? st : 0;
                        r -= S.wwin[ww][d];
                        const uint16_t* pr = &S.pre[ww][d][0];
                        int l = 0;                   // last even lane whose prefix is <= r, then maybe the next
#pragma unroll
                        for (int st = 8; st; st >>= 1) l += pr[l + st] <= r ? st : 0;
                        r -= pr[l];
                        l *= 2;
                        uint32_t m = S.msk[ww][d][l];
                        const uint32_t c0 = uint32_t(__popc(m));
                        if (r >= c0) {
                            r -= c0;
                            m = S.msk[ww][d][++l];
                        }
                        // a selection past the mask's bits leaves the change unplaced: the host then
                        // reports that not every change was placed
                        i = r < uint32_t(__popc(m)) ? ww * MP_SPAN + l * MP_RUN + int(nth_set_bit(m, r)) : -1;
                    } else {
                        i = order[S.estart[e] + r];
                    }
                    if (unsigned(i) < unsigned(n)) {
                        S.nz8[i] = uint8_t(tmin(z, 255u));
                        if (z >= 255u) esc[i] = uint16_t(int32_t(z >> 1) ^ -int32_t(z & 1));   // residual, mod 2^16
                        atomicOr(&S.mark[i >> 5], 1u << (i & 31));
                    }
                }
                const uint32_t m = __ballot_sync(FULL, valid);
                const int taken = __popc(~m) ? __ffs(~m) - 1 : 32;   // consumed changes are a prefix
                if (taken < 32) {
                    cur += uint32_t(taken);
                    next = __shfl_sync(FULL, lc, taken);   // local[cur], or ~0 past the group's end
                    break;
                }
                cur += 32u;
                lc = lcn;
                z = zn;
            }
            __syncwarp();
            if (lane == 0) {
                S.cursor[k] = cur;
                S.nextloc[k] = next;
                if (cur < ge) {   // the group's next changes, for a later sub-tile
                    const size_t nb = size_t(tmin(ge - cur, 128u));
                    prefetch_l2(lrel + cur, 4 * nb);
                    prefetch_l2(zrel + cur, 4 * nb);
                }
            }
            __syncwarp();
        };
#pragma unroll
        for (int j = 0; j < MP_PRE; ++j) {
            const int k = w + MP_WARPS * j;
            if (k < ngt) place_group(k, pl[j], pz[j]);
        }
        for (int k = w + MP_WARPS * MP_PRE; k < ngt; k += MP_WARPS) {
            const uint32_t c = S.cursor[k];
            uint32_t lc = 0xFFFFFFFFu, z = 0;
            if (uint32_t(lane) < S.gend[k] - c) { lc = lrel[c + lane]; z = zrel[c + lane]; }
            place_group(k, lc, z);
        }
        __syncthreads();
        // ---- stage this warp span's new values in position order, one atomic per warp: the
        //      span's changed positions are listed (in the warp's spent masks), then taken 32 at a time
        {
            static_assert(sizeof(S.msk[0]) >= MP_SPAN * sizeof(uint16_t), "a span's list fits in its masks");
            const uint32_t bits = S.mark[(span0 >> 5) + lane];
            const uint32_t c = __popc(bits);
            uint32_t incl = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(FULL, incl, o);
                if (lane >= o) incl += y;
            }
            const uint32_t total = __shfl_sync(FULL, incl, 31);
            unsigned long long sb = 0;
            if (lane == 31 && total) sb = atomicAdd(staged, (unsigned long long)total);
            sb = __shfl_sync(FULL, sb, 31);
            {   // the commit list: the span's changed-position bits and where its values start
                const int64_t st_i = s * (SUPER_N / MP_SUB) + (base - e_begin) / MP_SUB;   // sub-tile
                marks[st_i * (MP_SUB / 32) + (span0 >> 5) + lane] = bits;
                if (lane == 0) spanbase[st_i * MP_WARPS + w] = sb;
            }
            uint16_t* lst = reinterpret_cast<uint16_t*>(&S.msk[w][0][0]);
            uint32_t at = incl - c;
            for (uint32_t b = bits; b; b &= b - 1, ++at) lst[at] = uint16_t(lane * 32 + (__ffs(b) - 1));
            __syncwarp();
            int16_t* const pw = tt.w + base;
            for (uint32_t k = lane; k < total; k += 32) {
                const int i = span0 + lst[k];
                const uint32_t z8 = S.nz8[i];
                const uint32_t res = z8 < 255u ? uint32_t(int32_t(z8 >> 1) ^ -int32_t(z8 & 1)) : uint32_t(esc[i]);
                const uint32_t old = uint16_t(p[i]), nv = (old + res) & 0xFFFFu;
                if (sb + k < stage_cap) {
                    if (inplace) {   // written now; the list keeps the old value, to put back if the update fails
                        pw[i] = int16_t(nv);
                        cval[sb + k] = uint16_t(old);
                    } else {
                        cval[sb + k] = uint16_t(nv);
                    }
                }
                delta += (uint64_t(nv) - uint64_t(old)) * splitmix_weight(uint64_t(base + i));
                if (HNEW) {
                    const uint32_t eo = (old >> 7) & 0xFFu, en = (nv >> 7) & 0xFFu;
                    if (eo != en) {
                        atomicSub(&S.hdelta[eo], 1);
                        atomicAdd(&S.hdelta[en], 1);
                    }
                }
            }
        }
        S.pcur[tid] += S.tot[tid];
    }
    if (HNEW) {   // the weights' histogram after this update (the last span's moves are in)
        __syncthreads();
        HNEW[s * 256 + tid] = uint32_t(S.hdelta[tid]);
    }
    block_add_u64<MP_THREADS>(delta, &chk_delta[t], S.red);
}

// Writes the list's values at its positions: the new values for weights that k_map staged (host
// weights, after a passing verdict), the old ones to undo k_map's in-place writes after a failing
// one.  Slots at or past cap were never written by k_map (only a hostile update over-fills the
// list) and are skipped.  One CTA per sub-tile, a warp per span: each lane takes its 32-element
// run's mark word, its values start at the span's base plus the changed positions of the lanes
// before it.
__global__ void __launch_bounds__(MP_THREADS) k_commit(const AppTensor* __restrict__ T, int nT,
                                                       const uint32_t* __restrict__ marks,
                                                       const unsigned long long* __restrict__ spanbase,
                                                       const uint16_t* __restrict__ cval, int64_t st0, uint64_t cap) {
    const int64_t st_i = st0 + blockIdx.x;                // sub-tile
    const int64_t s = st_i / (SUPER_N / MP_SUB);
    const int t = tensor_of_super(T, nT, s);
    const AppTensor tt = T[t];
    const int64_t sub0 = (s - tt.super_begin) * SUPER_N + (st_i % (SUPER_N / MP_SUB)) * MP_SUB;
    if (sub0 >= tt.numel) return;                          // past the tensor's last sub-tile: nothing staged
    __shared__ uint16_t lst[MP_WARPS][MP_SPAN];   // a span's changed positions, in order
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const uint32_t bits = marks[st_i * (MP_SUB / 32) + w * 32 + lane];
    const uint32_t c = __popc(bits);
    uint32_t incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(FULL, incl, o);
        if (lane >= o) incl += y;
    }
    const uint32_t total = __shfl_sync(FULL, incl, 31);
    if (!total) return;
    uint32_t at = incl - c;
    for (uint32_t b = bits; b; b &= b - 1, ++at) lst[w][at] = uint16_t(lane * MP_RUN + (__ffs(b) - 1));
    __syncwarp();
    // consecutive lanes take consecutive changes: coalesced value reads, neighbouring writes
    const uint64_t vb = spanbase[st_i * MP_WARPS + w];
    const uint16_t* v = cval + vb;
    int16_t* dst = tt.w + sub0 + w * MP_SPAN;
    for (uint32_t k = lane; k < total; k += 32)
        if (vb + k < cap) dst[lst[w][k]] = int16_t(v[k]);   // slots past the list: never staged
}

// The same commit into host memory (weights the caller keeps on the host; the device copies the
// update was verified against are temporaries): the commit list comes down once, host threads
// scatter it.  `mk`, `sbase`, `vals` are host copies of marks, spanbase and cval.
void commit_host(const std::vector<AppTensor>& T, int16_t* const* host, const uint32_t* mk, const uint64_t* sbase,
                 const uint16_t* vals, int64_t n_super) {   // super-tiles [0, n_super)
    const int nt = int(T.size());
    parallel_for(size_t(n_super), [&](size_t si) {
        const int64_t s = int64_t(si);
        int t = 0;
        {
            int lo = 0, hi = nt - 1;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (T[size_t(mid)].super_begin <= s) lo = mid; else hi = mid - 1;
            }
            t = lo;
        }
        const AppTensor& tt = T[size_t(t)];
        for (int sub = 0; sub < int(SUPER_N / MP_SUB); ++sub) {
            const int64_t sub0 = (s - tt.super_begin) * SUPER_N + int64_t(sub) * MP_SUB;
            if (sub0 >= tt.numel) break;
            const int64_t st_i = s * (SUPER_N / MP_SUB) + sub;
            for (int w = 0; w < MP_WARPS; ++w) {
                const uint16_t* v = vals + sbase[st_i * MP_WARPS + w];
                const uint32_t* m = mk + st_i * (MP_SUB / 32) + w * 32;
                int16_t* dst = host[t] + sub0 + w * MP_SPAN;
                for (int l = 0; l < 32; ++l)
                    for (uint32_t b = m[l]; b; b &= b - 1) dst[l * MP_RUN + __builtin_ctz(b)] = int16_t(*v++);
            }
        }
    });
}

__global__ void k_widen(const uint32_t* __restrict__ a, uint64_t* __restrict__ b, int64_t n) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) b[i] = a[i];
}

__global__ void __launch_bounds__(512) k_checksum(const int16_t* __restrict__ p, int64_t n, unsigned long long* __restrict__ out) {
    __shared__ uint64_t red[16];
    uint64_t s = 0;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
        s += uint64_t(uint16_t(p[i])) * splitmix_weight(uint64_t(i));
    block_add_u64<512>(s, out, red);
}

template <class T>
T* dev(Ctx& c, Slot s) { return reinterpret_cast<T*>(c.b[s].p); }

void build_lut(const DecodeTable& d, const uint32_t* sorted_syms, uint32_t* lut) {
    for (uint32_t p = 0; p < (1u << LUT_BITS); ++p) {
        const uint32_t lo = p << (kMaxCodeLen - LUT_BITS);
        int L = 1;
        while (L <= kMaxCodeLen && lo >= d.limit[L]) ++L;
        if (L <= LUT_BITS) lut[p] = (uint32_t(L) << 24) | sorted_syms[d.base[L] + (lo >> (kMaxCodeLen - L)) - d.first[L]];
        else lut[p] = 0;
    }
}

}  // namespace

__global__ void k_hist_store(const uint32_t* __restrict__ src, uint32_t* const* __restrict__ dst,
                             const int64_t* __restrict__ row0, const int64_t* __restrict__ rows, int n) {
    const int t = blockIdx.y;
    if (t >= n) return;
    const int64_t cells = rows[t] * 256;
    for (int64_t k = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; k < cells; k += int64_t(gridDim.x) * blockDim.x)
        dst[t][k] = src[row0[t] * 256 + k];
}

Status apply_impl(Ctx& C, const Update& u, int16_t* const* weights, const uint64_t* old_chk, const uint8_t* has_chk,
                  cudaStream_t st, int64_t* changed, std::string* err, const uint64_t* versions,
                  const uint8_t* has_version, int16_t* const* host_weights) {
    *changed = 0;
    const int nt = int(u.tensors.size());
    if (u.payload_len && !u.payload && !u.payload_device) {
        *err = "the update was parsed from its head only; its payload is not at hand";
        return kValueError;
    }
    if (nt == 0) return kOk;
    trace_phase(C, "apply: start");
    // ---- host tables
    std::vector<AppTensor> T(static_cast<size_t>(nt));
    std::vector<AppGroup> G;
    std::vector<uint64_t> gblock(1, 0);
    std::vector<int64_t> row_begin(static_cast<size_t>(nt) + 1), chunk_begin(static_cast<size_t>(nt) + 1, 0);
    int64_t n_super = 0;
    uint64_t start = 0;
    for (int t = 0; t < nt; ++t) {
        const TensorHeader& h = u.tensors[size_t(t)];
        if (h.numel >= (int64_t(1) << 32)) { *err = "tensors of 2^32 or more elements are not supported"; return kValueError; }
        AppTensor& d = T[size_t(t)];
        d.w = weights[t];
        d.numel = h.numel;
        d.super_begin = n_super;
        d.want_full = has_chk && has_chk[t] ? 0 : 1;
        d.hcache = nullptr;
        if (versions && has_version && has_version[t] && !d.want_full) {   // histogram from the last apply?
            const auto it = C.hist_cache.find(reinterpret_cast<uintptr_t>(weights[t]));
            if (it != C.hist_cache.end() && it->second.numel == h.numel && it->second.tag == versions[t] &&
                it->second.checksum == old_chk[t]) {
                d.hcache = static_cast<const uint32_t*>(it->second.rows.p);
                ++C.hist_hits;
            }
        }
        d.g_begin = int32_t(G.size());
        for (const Group& g : h.groups) {
            AppGroup ag{};
            ag.start = start;
            ag.count = uint64_t(g.count);
            ag.tensor = t;
            ag.exp = g.exponent;
            ag.rice = g.rice;
            ag.table = u.table_of_exp[g.exponent];
            G.push_back(ag);
            start += uint64_t(g.count);
            gblock.push_back(gblock.back() + (uint64_t(g.count) + kBlock - 1) / kBlock);
        }
        d.g_end = int32_t(G.size());
        row_begin[size_t(t)] = n_super;
        const int64_t rows = (h.numel + SUPER_N - 1) / SUPER_N;
        n_super += rows;
        chunk_begin[size_t(t) + 1] = chunk_begin[size_t(t)] + (rows + SCAN_CHUNK - 1) / SCAN_CHUNK;
    }
    row_begin[size_t(nt)] = n_super;
    const int64_t n_chunks = chunk_begin[size_t(nt)];
    const int64_t ng = int64_t(G.size());
    const uint64_t total = start;
    const int64_t n_blocks = u.n_blocks;
    if (int64_t(gblock.back()) != n_blocks) { *err = "internal: block count mismatch"; return kCudaError; }
    // decode tables: their sizes now, their contents once the histogram pass and the copies run
    std::vector<size_t> toffs(u.tables.size() + 1, 0);
    for (size_t k = 0; k < u.tables.size(); ++k) toffs[k + 1] = toffs[k] + u.tables[k].symbols.size();
    const size_t n_tables = u.tables.size(), n_syms = toffs.back();
    trace_phase(C, "apply: host tables");
    // ---- device buffers
    const size_t cells = size_t(nt) * 256;
    const size_t payload_alloc = size_t(u.payload_len) + 64;
    CRX_CUDA(ensure_dev(C.b[S_A_TENS], sizeof(AppTensor) * size_t(nt), st));
    CRX_CUDA(ensure_dev(C.b[S_A_GROUPS], sizeof(AppGroup) * size_t(ng) + sizeof(uint64_t) * (size_t(ng) + 1), st));
    CRX_CUDA(ensure_dev(C.b[S_A_TABLES], sizeof(DecTable) * n_tables, st));
    CRX_CUDA(ensure_dev(C.b[S_A_SYMS], sizeof(uint32_t) * n_syms, st));
    CRX_CUDA(ensure_dev(C.b[S_A_PAYLOAD], payload_alloc, st));
    CRX_CUDA(ensure_dev(C.b[S_A_BB], sizeof(uint32_t) * size_t(n_blocks), st));
    CRX_CUDA(ensure_dev(C.b[S_A_BOFF], sizeof(uint64_t) * size_t(n_blocks), st));
    CRX_CUDA(ensure_dev(C.b[S_A_BSUM], sizeof(uint64_t) * size_t(n_blocks), st));
    CRX_CUDA(ensure_dev(C.b[S_A_SCAN_TMP], sizeof(uint64_t) * (exclusive_scan_tmp_elems(n_blocks) + 2), st));
    CRX_CUDA(ensure_dev(C.b[S_A_BGROUP], sizeof(int32_t) * size_t(n_blocks), st));
    CRX_CUDA(ensure_dev(C.b[S_A_ZZ], sizeof(uint32_t) * total, st));
    CRX_CUDA(ensure_dev(C.b[S_A_LOCAL], sizeof(uint32_t) * total, st));
    // commit list: a bit per element, the span's first value slot, the values in position order
    const size_t mark_words = size_t(n_super) * (SUPER_N / 32);
    const size_t span_slots = size_t(n_super) * (SUPER_N / MP_SUB) * MP_WARPS;
    CRX_CUDA(ensure_dev(C.b[S_A_CADDR], sizeof(uint32_t) * mark_words, st));
    CRX_CUDA(ensure_dev(C.b[S_A_SPANB], sizeof(uint64_t) * span_slots, st));
    CRX_CUDA(ensure_dev(C.b[S_A_CVAL], sizeof(uint16_t) * total, st));
    CRX_CUDA(ensure_dev(C.b[S_A_HS], sizeof(uint32_t) * 256 * size_t(n_super), st));
    bool keep_hist = false;   // some tensor asks for its histogram to be cached
    for (int t = 0; t < nt && versions && has_version; ++t) keep_hist |= has_version[t] != 0;
    if (keep_hist) CRX_CUDA(ensure_dev(C.b[S_A_HNEW], sizeof(uint32_t) * 256 * size_t(n_super), st));
    uint32_t* hnew = keep_hist ? dev<uint32_t>(C, S_A_HNEW) : nullptr;
    CRX_CUDA(ensure_dev(C.b[S_A_ORDER], sizeof(uint16_t) * MP_SUB * size_t(n_super), st));
    CRX_CUDA(ensure_dev(C.b[S_A_ESC], sizeof(uint16_t) * MP_SUB * size_t(n_super), st));
    CRX_CUDA(ensure_dev(C.b[S_A_TOT], sizeof(uint64_t) * cells, st));
    CRX_CUDA(ensure_dev(C.b[S_A_CHUNK_ROWS], sizeof(int64_t) * 2 * (size_t(nt) + 1), st));
    CRX_CUDA(ensure_dev(C.b[S_A_CHUNK_SUMS], sizeof(uint32_t) * 256 * size_t(n_chunks), st));
    CRX_CUDA(ensure_dev(C.b[S_A_COUNTERS], sizeof(uint64_t) * (16 + 2 * size_t(nt)), st));

    // ---- uploads: metadata through pinned staging, the payload straight from the caller's buffer
    const size_t up = sizeof(AppTensor) * nt + sizeof(AppGroup) * ng + 8 * (ng + 1) + sizeof(DecTable) * n_tables +
                      4 * n_syms + 16 * (nt + 1) + 256;
    CRX_CUDA(ensure_host(C, up, st));
    uint8_t* h = static_cast<uint8_t*>(C.host);
    size_t o = 0;
    auto upload = [&](void* dst, const void* src, size_t bytes) -> cudaError_t {
        if (!bytes) return cudaSuccess;
        std::memcpy(h + o, src, bytes);
        const cudaError_t e = cudaMemcpyAsync(dst, h + o, bytes, cudaMemcpyHostToDevice, st);
        o += (bytes + 15) & ~size_t(15);
        return e;
    };
    auto* dG = dev<AppGroup>(C, S_A_GROUPS);
    auto* dgblock = reinterpret_cast<uint64_t*>(dG + ng);
    auto* drows = dev<int64_t>(C, S_A_CHUNK_ROWS);
    CRX_CUDA(upload(C.b[S_A_TENS].p, T.data(), sizeof(AppTensor) * size_t(nt)));
    CRX_CUDA(upload(dG, G.data(), sizeof(AppGroup) * size_t(ng)));
    CRX_CUDA(upload(dgblock, gblock.data(), 8 * (size_t(ng) + 1)));
    CRX_CUDA(upload(drows, row_begin.data(), 8 * (size_t(nt) + 1)));
    CRX_CUDA(upload(drows + nt + 1, chunk_begin.data(), 8 * (size_t(nt) + 1)));
    CRX_CUDA(cudaMemsetAsync(static_cast<uint8_t*>(C.b[S_A_PAYLOAD].p) + u.payload_len, 0, 64, st));
    auto* counters = dev<unsigned long long>(C, S_A_COUNTERS);
    auto* chk_delta = counters + 16;
    auto* chk_full = chk_delta + nt;
    CRX_CUDA(cudaMemsetAsync(counters, 0, sizeof(uint64_t) * (16 + 2 * size_t(nt)), st));

    // ---- exponent histograms, per-super-tile offsets and group sizes
    const AppTensor* dT = dev<AppTensor>(C, S_A_TENS);
    { KernelScope ks_(C, "k_app_hist", st);
    k_app_hist<<<unsigned(n_super), HIST_THREADS, 0, st>>>(dT, nt, dev<uint32_t>(C, S_A_HS), chk_full);
    }
    CRX_CUDA(cudaGetLastError());
    launch_column_scan(C, dev<uint32_t>(C, S_A_HS), n_super, drows, nt, drows + nt + 1, n_chunks,
                       dev<uint32_t>(C, S_A_CHUNK_SUMS), dev<uint64_t>(C, S_A_TOT), st);
    trace_phase(C, "apply: uploads + hist launched");
    // ---- block table and payload: chunked multithreaded copies into pinned memory, each chunk's
    //      DMA overlapping the next chunk's copy (and the histogram pass already running)
    const size_t bt_bytes = 4 * size_t(n_blocks);
    CRX_CUDA(ensure_pinned(C.in_host, bt_bytes + size_t(u.payload_len) + 16, st));
    uint8_t* ih = static_cast<uint8_t*>(C.in_host.p);
    CRX_CUDA(ensure_copy_stream(C));
    CRX_CUDA(cudaEventRecord(C.ev_main, st));
    CRX_CUDA(cudaStreamWaitEvent(C.copy_stream, C.ev_main, 0));
    if (u.block_table)
        CRX_CUDA(upload_pipelined(C, C.b[S_A_BB].p, u.block_table, ih, bt_bytes, C.copy_stream));
    else if (bt_bytes)   // the update lives in device memory (its table at any byte offset)
        CRX_CUDA(cudaMemcpyAsync(C.b[S_A_BB].p, u.block_table_device, bt_bytes, cudaMemcpyDeviceToDevice, C.copy_stream));
    if (u.payload)
        CRX_CUDA(upload_pipelined(C, C.b[S_A_PAYLOAD].p, u.payload, ih + bt_bytes, size_t(u.payload_len), C.copy_stream));
    else if (u.payload_len)   // the update lives in device memory
        CRX_CUDA(cudaMemcpyAsync(C.b[S_A_PAYLOAD].p, u.payload_device, size_t(u.payload_len), cudaMemcpyDeviceToDevice,
                                 C.copy_stream));
    CRX_CUDA(cudaEventRecord(C.ev_copy, C.copy_stream));
    std::vector<DecTable> TB(n_tables);
    std::vector<uint32_t> syms;
    {   // decode tables and their lookup tables, independent per exponent: built on the host pool
        //  while the histogram pass and the update's copies run
        const std::vector<size_t>& offs = toffs;
        syms.resize(n_syms);
        auto one = [&](size_t k) {
            DecodeTable d;
            build_decode_table(u.tables[k], &d, syms.data() + offs[k]);
            DecTable& x = TB[k];
            std::memcpy(x.first, d.first, sizeof(x.first));
            std::memcpy(x.base, d.base, sizeof(x.base));
            std::memcpy(x.limit, d.limit, sizeof(x.limit));
            x.sym_off = uint32_t(offs[k]);
            x.nsym = uint32_t(u.tables[k].symbols.size());
            build_lut(d, syms.data() + offs[k], x.lut);
        };
        if (u.tables.size() > 4) parallel_for(u.tables.size(), one);
        else for (size_t k = 0; k < u.tables.size(); ++k) one(k);
    }
    CRX_CUDA(upload(C.b[S_A_TABLES].p, TB.data(), sizeof(DecTable) * n_tables));
    CRX_CUDA(upload(C.b[S_A_SYMS].p, syms.data(), 4 * n_syms));
    trace_phase(C, "apply: decode tables up");
    CRX_CUDA(cudaStreamWaitEvent(st, C.ev_copy, 0));
    // ---- block offsets and decode
    uint64_t* boff = dev<uint64_t>(C, S_A_BOFF);
    uint64_t* scan_tmp = dev<uint64_t>(C, S_A_SCAN_TMP);
    uint64_t* d_total = scan_tmp + exclusive_scan_tmp_elems(n_blocks);
    { KernelScope ks_(C, "k_widen", st);
    k_widen<<<unsigned((n_blocks + 255) / 256), 256, 0, st>>>(dev<uint32_t>(C, S_A_BB), boff, n_blocks);
    }
    launch_exclusive_scan_u64(C, boff, n_blocks, scan_tmp, d_total, st);
    { KernelScope ks_(C, "k_decode", st);
    k_decode<<<unsigned((n_blocks + DEC_THREADS - 1) / DEC_THREADS), DEC_THREADS, 0, st>>>(
        dev<uint64_t>(C, S_A_PAYLOAD), uint64_t(payload_alloc / 4), dev<uint32_t>(C, S_A_BB), boff, n_blocks, dG, dgblock, ng, dev<DecTable>(C, S_A_TABLES),
        dev<uint32_t>(C, S_A_SYMS), dev<uint64_t>(C, S_A_TOT), dev<uint32_t>(C, S_A_LOCAL), dev<uint32_t>(C, S_A_ZZ),
        dev<uint64_t>(C, S_A_BSUM), dev<int32_t>(C, S_A_BGROUP), counters);
    }
    CRX_CUDA(cudaGetLastError());
    launch_exclusive_scan_u64(C, dev<uint64_t>(C, S_A_BSUM), n_blocks, scan_tmp, d_total, st);
    { KernelScope ks_(C, "k_locals", st);
    k_locals<<<unsigned((n_blocks * 32 + 255) / 256), 256, 0, st>>>(dev<uint64_t>(C, S_A_BSUM), n_blocks, dG, dgblock,
                                                                   dev<int32_t>(C, S_A_BGROUP), dev<uint64_t>(C, S_A_TOT),
                                                                   dev<uint32_t>(C, S_A_LOCAL), counters);
    }
    CRX_CUDA(cudaGetLastError());
    // ---- positions, staged values, checksum deltas.  Device weights are written here, in place,
    //      with the old values kept in the list; the host's verdict then either keeps them or has
    //      k_commit put the old values back.  Host weights get the new values in the list.
    const bool inplace = host_weights == nullptr;
    const size_t map_smem = sizeof(MapSmem);
    CRX_CUDA(cudaFuncSetAttribute(k_map, cudaFuncAttributeMaxDynamicSharedMemorySize, int(map_smem)));
    { KernelScope ks_(C, "k_map", st);
    k_map<<<unsigned(n_super), MP_THREADS, map_smem, st>>>(dT, nt, dG, dev<uint32_t>(C, S_A_HS), dev<uint32_t>(C, S_A_LOCAL),
                                                            dev<uint32_t>(C, S_A_ZZ), dev<uint32_t>(C, S_A_CADDR),
                                                            dev<unsigned long long>(C, S_A_SPANB),
                                                            dev<uint16_t>(C, S_A_CVAL), total, chk_delta, counters + 2,
                                                            dev<uint64_t>(C, S_A_TOT), hnew, dev<uint16_t>(C, S_A_ORDER),
                                                            dev<uint16_t>(C, S_A_ESC), inplace ? 1 : 0);
    }
    CRX_CUDA(cudaGetLastError());
    // ---- verdict (one synchronisation for the whole update)
    uint64_t* hc = C.small;
    const size_t nsmall = 16 + 2 * size_t(nt);
    std::vector<uint64_t> hv(nsmall);
    if (nsmall < size_t(kEncStatusWord)) {
        CRX_CUDA(cudaMemcpyAsync(hc, counters, 8 * nsmall, cudaMemcpyDeviceToHost, st));
        CRX_CUDA(cudaStreamSynchronize(st));
        std::memcpy(hv.data(), hc, 8 * nsmall);
    } else {
        CRX_CUDA(ensure_host(C, 8 * nsmall, st));
        CRX_CUDA(cudaMemcpyAsync(C.host, counters, 8 * nsmall, cudaMemcpyDeviceToHost, st));
        CRX_CUDA(cudaStreamSynchronize(st));
        std::memcpy(hv.data(), C.host, 8 * nsmall);
    }
    trace_phase(C, "apply: verdict (sync)");
    // A failed verdict leaves the weights as they were: the old values go back over what k_map
    // wrote (each written element is listed once, with its old value in the slot k_map used).
    auto undo = [&](Status s) -> Status {
        if (!inplace) return s;
        { KernelScope ks_(C, "k_commit", st);
        k_commit<<<unsigned(n_super * (SUPER_N / MP_SUB)), MP_THREADS, 0, st>>>(
            dT, nt, dev<uint32_t>(C, S_A_CADDR), dev<unsigned long long>(C, S_A_SPANB), dev<uint16_t>(C, S_A_CVAL), 0, total);
        }
        const cudaError_t e1 = cudaGetLastError();
        const cudaError_t e2 = cudaStreamSynchronize(st);
        if (e1 != cudaSuccess || e2 != cudaSuccess) {
            *err += std::string("; restoring the weights failed: ") + cudaGetErrorString(e1 != cudaSuccess ? e1 : e2);
            return kCudaError;
        }
        return s;
    };
    if (hv[1] & (ERR_DECODE | ERR_RANGE)) {
        *err = "payload positions outside their exponent groups";
        return undo(kCorrupt);
    }
    if (hv[2] != total) {   // every in-range change lands in exactly one sub-tile
        *err = "internal: not every change was placed";
        return undo(kCudaError);
    }
    std::string bad_names;
    int n_bad = 0;
    for (int t = 0; t < nt; ++t) {
        const uint64_t base = T[size_t(t)].want_full ? hv[16 + size_t(nt) + size_t(t)] : old_chk[t];
        if (base + hv[16 + size_t(t)] != u.tensors[size_t(t)].checksum) {
            if (n_bad < 3) {
                if (n_bad) bad_names += ", ";
                bad_names.append(reinterpret_cast<const char*>(u.tensors[size_t(t)].name), size_t(u.tensors[size_t(t)].name_len));
            }
            ++n_bad;
        }
    }
    if (n_bad) {
        *err = "update does not verify (checksum mismatch: " + bad_names + ")";
        return undo(kCorrupt);
    }
    if (host_weights) {   // the weights live on the host
        // Two ways down, run at once.  The last tensors, while their host memory is pinned and up to
        // kDmaShare of the elements, are committed on the device and copied down whole by DMA (2 B
        // an element over PCIe); the others get the commit list (a bit an element + the changed
        // values) and are scattered by the host threads, which costs them the host's memory traffic
        // of every touched line.  Measured on a 16-core host at 7.6e9 elements and 5.8 % changed:
        // DMA ~35 ps an element, list + scatter ~29 ps, so about 45 % goes by DMA.
        constexpr double kDmaShare = 0.45;
        int64_t all = 0;
        for (int t = 0; t < nt; ++t) all += T[size_t(t)].numel;
        int t_split = nt;
        int64_t dma = 0;
        while (t_split > 0) {
            const int t = t_split - 1;
            cudaPointerAttributes pa{};
            const bool pinned = cudaPointerGetAttributes(&pa, host_weights[t]) == cudaSuccess && pa.type == cudaMemoryTypeHost;
            (void)cudaGetLastError();   // an unregistered pointer may leave an error behind
            if (!pinned || double(dma + T[size_t(t)].numel) > kDmaShare * double(all)) break;
            dma += T[size_t(t)].numel;
            t_split = t;
        }
        const int64_t s_split = t_split < nt ? T[size_t(t_split)].super_begin : n_super;
        const size_t mb = sizeof(uint32_t) * size_t(s_split) * (SUPER_N / 32);
        const size_t sb = sizeof(uint64_t) * size_t(s_split) * (SUPER_N / MP_SUB) * MP_WARPS;
        const size_t vb = s_split ? sizeof(uint16_t) * total : 0;   // value slots are spread over the whole list
        CRX_CUDA(ensure_pinned(C.in_host, mb + sb + vb + 16, st));
        uint8_t* hb = static_cast<uint8_t*>(C.in_host.p);
        if (mb) CRX_CUDA(cudaMemcpyAsync(hb, C.b[S_A_CADDR].p, mb, cudaMemcpyDeviceToHost, st));
        if (sb) CRX_CUDA(cudaMemcpyAsync(hb + mb, C.b[S_A_SPANB].p, sb, cudaMemcpyDeviceToHost, st));
        if (vb) CRX_CUDA(cudaMemcpyAsync(hb + mb + sb, C.b[S_A_CVAL].p, vb, cudaMemcpyDeviceToHost, st));
        cudaEvent_t list_down = nullptr;
        CRX_CUDA(cudaEventCreateWithFlags(&list_down, cudaEventDisableTiming));
        const cudaError_t rec = cudaEventRecord(list_down, st);
        if (rec != cudaSuccess) { cudaEventDestroy(list_down); CRX_CUDA(rec); }
        if (s_split < n_super) {   // the DMA share: commit on the device, then copy down tensors that changed
            const int64_t st0 = s_split * (SUPER_N / MP_SUB);
            { KernelScope ks_(C, "k_commit", st);
            k_commit<<<unsigned((n_super - s_split) * (SUPER_N / MP_SUB)), MP_THREADS, 0, st>>>(
                dT, nt, dev<uint32_t>(C, S_A_CADDR), dev<unsigned long long>(C, S_A_SPANB), dev<uint16_t>(C, S_A_CVAL), st0,
                total);
            }
            cudaError_t e = cudaGetLastError();
            for (int t = t_split; t < nt && e == cudaSuccess; ++t) {
                uint64_t cnt = 0;
                for (const Group& g : u.tensors[size_t(t)].groups) cnt += uint64_t(g.count);
                if (cnt) e = cudaMemcpyAsync(host_weights[t], weights[t], sizeof(int16_t) * size_t(T[size_t(t)].numel),
                                             cudaMemcpyDeviceToHost, st);
            }
            if (e != cudaSuccess) { cudaEventDestroy(list_down); CRX_CUDA(e); }
        }
        const cudaError_t ew = cudaEventSynchronize(list_down);
        cudaEventDestroy(list_down);
        CRX_CUDA(ew);
        trace_phase(C, "apply: commit list down");
        if (s_split) commit_host(T, host_weights, reinterpret_cast<const uint32_t*>(hb), reinterpret_cast<const uint64_t*>(hb + mb),
                                 reinterpret_cast<const uint16_t*>(hb + mb + sb), s_split);
        trace_phase(C, "apply: host scatter");
        CRX_CUDA(cudaStreamSynchronize(st));
        trace_phase(C, "apply: DMA share down");
        *changed = int64_t(total);
        return kOk;
    }
    // ---- the new weights' histograms for the next apply (tagged version + 1: the caller bumps it).
    //      Rows of dropped entries go to a free list and are reused; nothing is freed here (a
    //      cudaFree would synchronize the device and stall every other stream).
    auto retire = [&](DevBuf& b) {
        if (b.p) C.hist_free.push_back(b);
        b = DevBuf{};
    };
    for (int t = 0; t < nt; ++t) {
        const auto key = reinterpret_cast<uintptr_t>(weights[t]);
        if (!(keep_hist && has_version[t])) {   // written without a tag: forget what was cached
            const auto it = C.hist_cache.find(key);
            if (it != C.hist_cache.end()) {
                retire(it->second.rows);
                C.hist_cache.erase(it);
            }
        }
    }
    if (keep_hist) {
        constexpr size_t kHistBound = size_t(4) << 30;   // cached rows plus free rows
        size_t held = 0;
        for (auto& kv : C.hist_cache) held += kv.second.rows.cap;
        for (auto& d : C.hist_free) held += d.cap;
        std::vector<uint32_t*> dst;
        std::vector<int64_t> row0, rows;
        for (int t = 0; t < nt; ++t) {
            if (!has_version[t]) continue;
            auto& ent = C.hist_cache[reinterpret_cast<uintptr_t>(weights[t])];
            const int64_t nr = (T[size_t(t)].numel + SUPER_N - 1) / SUPER_N;
            const size_t need = sizeof(uint32_t) * 256 * size_t(nr);
            if (ent.rows.cap < need) {
                retire(ent.rows);
                size_t best = C.hist_free.size();   // the smallest free rows that fit
                for (size_t k = 0; k < C.hist_free.size(); ++k)
                    if (C.hist_free[k].cap >= need && (best == C.hist_free.size() || C.hist_free[k].cap < C.hist_free[best].cap))
                        best = k;
                if (best < C.hist_free.size()) {
                    ent.rows = C.hist_free[best];
                    C.hist_free.erase(C.hist_free.begin() + std::ptrdiff_t(best));
                } else if (held + need <= kHistBound) {
                    CRX_CUDA(ensure_dev(ent.rows, need, st));
                    held += ent.rows.cap;
                } else {   // over the bound: this tensor is not cached (its next apply reads the weights)
                    C.hist_cache.erase(reinterpret_cast<uintptr_t>(weights[t]));
                    continue;
                }
            }
            ent.numel = T[size_t(t)].numel;
            ent.tag = versions[t] + 1;
            ent.checksum = u.tensors[size_t(t)].checksum;
            dst.push_back(static_cast<uint32_t*>(ent.rows.p));
            row0.push_back(T[size_t(t)].super_begin);
            rows.push_back(nr);
        }
        const int ne = int(dst.size());
        if (ne) {
            const size_t tb = 8 * size_t(ne) * 3;
            CRX_CUDA(ensure_dev(C.b[S_A_HSTORE], tb, st));
            if (!C.hstore_ev) CRX_CUDA(cudaEventCreateWithFlags(&C.hstore_ev, cudaEventDisableTiming));
            CRX_CUDA(cudaEventSynchronize(C.hstore_ev));   // the previous store's copy has read the table
            CRX_CUDA(ensure_pinned(C.hstore_table, tb, st));
            uint8_t* hh = static_cast<uint8_t*>(C.hstore_table.p);
            std::memcpy(hh, dst.data(), 8 * size_t(ne));
            std::memcpy(hh + 8 * ne, row0.data(), 8 * size_t(ne));
            std::memcpy(hh + 16 * ne, rows.data(), 8 * size_t(ne));
            uint8_t* dd = static_cast<uint8_t*>(C.b[S_A_HSTORE].p);
            CRX_CUDA(cudaMemcpyAsync(dd, hh, tb, cudaMemcpyHostToDevice, st));
            { KernelScope ks_(C, "k_hist_store", st);
            k_hist_store<<<dim3(64, unsigned(ne)), 256, 0, st>>>(hnew, reinterpret_cast<uint32_t* const*>(dd),
                                                                reinterpret_cast<const int64_t*>(dd + 8 * ne),
                                                                reinterpret_cast<const int64_t*>(dd + 16 * ne), ne);
            }
            CRX_CUDA(cudaGetLastError());
            CRX_CUDA(cudaEventRecord(C.hstore_ev, st));
        }
    }
    *changed = int64_t(total);
    return kOk;
}

Status checksum_impl(Ctx& C, const int16_t* data, int64_t n, cudaStream_t st, uint64_t* out, std::string* err) {
    CRX_CUDA(ensure_dev(C.b[S_CHK], 64, st));
    auto* acc = dev<unsigned long long>(C, S_CHK);
    CRX_CUDA(cudaMemsetAsync(acc, 0, 8, st));
    if (n > 0) {
        const int64_t blocks = std::min<int64_t>((n + 511) / 512, 148 * 8);
        { KernelScope ks_(C, "k_checksum", st);
        k_checksum<<<unsigned(blocks), 512, 0, st>>>(data, n, acc);
        }
        CRX_CUDA(cudaGetLastError());
    }
    CRX_CUDA(cudaMemcpyAsync(C.small, acc, 8, cudaMemcpyDeviceToHost, st));
    CRX_CUDA(cudaStreamSynchronize(st));
    *out = C.small[0];
    return kOk;
}

}  // namespace crx
