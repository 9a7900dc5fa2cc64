// Per-device context: grow-only device workspace, pinned host staging and the lock that
// serializes calls on one context.  Library-owned scratch; callers own every weight buffer.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>
#include <unordered_map>
#include <string>
#include <vector>

#include "host_codec.h"

namespace crx {

struct DevBuf {
    void* p = nullptr;
    size_t cap = 0;
};

struct Ctx;

// Counts one device or pinned-host allocation or free made by this library (process-wide; read by
// crx_alloc_calls, so tests can check that an entry point allocates nothing).
void note_alloc();

// Grow `buf` to at least `bytes` (contents not preserved).  Synchronizes `s` before freeing.
cudaError_t ensure_dev(DevBuf& buf, size_t bytes, cudaStream_t s);
cudaError_t ensure_host(Ctx& c, size_t bytes, cudaStream_t s);
cudaError_t ensure_pinned(DevBuf& buf, size_t bytes, cudaStream_t s);
// memcpy split over threads (large copies; also spreads first-touch page faults)
void parallel_copy(void* dst, const void* src, size_t n);
// Touch every page of [dst, dst + n) from the worker threads, so that a freshly allocated
// destination takes its page faults in parallel (and ahead of the copy into it).
void prefault(void* dst, size_t n);
// host -> device through pinned staging, chunk by chunk: the host copy of chunk k+1 overlaps the
// DMA of chunk k.  `pinned` holds at least n bytes.
cudaError_t upload_pipelined(Ctx& c, void* dev_dst, const void* host_src, uint8_t* pinned, size_t n, cudaStream_t s);
// pipelined copies move kCopyChunk bytes per cudaMemcpyAsync; chunk_events makes sure the context
// holds at least n timing-free events (Ctx::copy_ev)
constexpr size_t kCopyChunk = size_t(32) << 20;
cudaError_t chunk_events(Ctx& c, size_t n);
// creates Ctx::copy_stream and its two events on first use (the context's device is current)
cudaError_t ensure_copy_stream(Ctx& c);
// word of Ctx::small that receives the error flags of an encode whose copies are still in flight
constexpr int kEncStatusWord = 511;

// Named slots of Ctx::b.
enum Slot : int {
    S_TENS = 0, S_HS, S_CS, S_CHUNK_ROWS, S_CHUNK_SUMS, S_TOTALS_A, S_TOTALS_C, S_COUNTERS, S_REC_KEY, S_REC_VAL,
    S_GIDX, S_GROUPS, S_LOCAL, S_VALS, S_COSTS, S_DENSE_HIST, S_RARE_HIST, S_RARE_FLAG, S_RARE_OUT,
    S_DENSE_CODE, S_BIG_CODE, S_BLOCK_BITS, S_SCAN_TMP, S_PAYLOAD, S_BB32, S_RARE_CODES,
    // apply
    S_A_TENS, S_A_GROUPS, S_A_TABLES, S_A_SYMS, S_A_PAYLOAD, S_A_BB, S_A_BOFF, S_A_ZZ, S_A_BSUM,
    S_A_LOCAL, S_A_CADDR, S_A_CVAL, S_A_HS, S_A_TOT, S_A_CHUNK_ROWS, S_A_CHUNK_SUMS, S_A_COUNTERS, S_A_SCAN_TMP,
    S_CHK, S_SUPER_T, S_A_HNEW, S_A_HSTORE, S_A_ORDER,
    // size statistics
    S_SZ_STATS, S_SZ_TILES,
    // apply: first value slot of every span of the commit list
    S_A_SPANB,
    // apply: k_map's large residuals, by sub-tile position, one sub-tile per super-tile at a time
    S_A_ESC,
    // apply: the group of every 256-change block (k_decode finds it, k_locals reads it)
    S_A_BGROUP,
    // encode: every block's bits, assembled from bit 0 in a fixed-size slot (k_pack_slots -> k_compact)
    S_PACK_SLOTS,
    S_NSLOTS
};

struct ProfMark {
    const char* name;
    cudaEvent_t a, b;
    cudaStream_t s = nullptr;   // the stream the kernel ran on
};

struct Encoded;

struct Ctx {
    int device = 0;
    std::mutex mu;
    DevBuf b[S_NSLOTS];
    void* host = nullptr;       // pinned host staging (metadata both ways, payload down)
    size_t host_cap = 0;
    uint64_t* small = nullptr;  // fixed pinned words for counters and verdicts (never moves)
    DevBuf out_host;            // pinned: block table + payload of the last encode (see Encoded)
    DevBuf in_host;             // pinned: block table + payload of the update being applied
    Encoded* live = nullptr;    // the encode result still reading out_host, if any
    uint64_t launches = 0;      // kernels launched by this context since creation
    // optional per-kernel timing with CUDA events on the caller's stream
    bool profile = false;
    bool trace = false;         // CRUKX_B200_TRACE=1: synchronize after every kernel and log its time
    std::vector<cudaEvent_t> ev_pool;
    size_t ev_used = 0;
    std::vector<ProfMark> marks;
    double phase_t = 0.0;
    std::vector<cudaEvent_t> copy_ev;   // chunk events of the pipelined host <-> device copies
    // apply's uploads run on their own stream so that the DMA overlaps the histogram pass;
    // ev_main orders them after the caller's stream, ev_copy the decode after them
    cudaStream_t copy_stream = nullptr;
    cudaEvent_t ev_main = nullptr, ev_copy = nullptr;
    // receiver: exponent histograms per super-tile of weights this context last wrote, keyed by the
    // weights' address, valid while the caller's version tag matches (crx_apply_versioned)
    struct HistEntry {
        int64_t numel = 0;
        uint64_t tag = 0;
        uint64_t checksum = 0;   // of the weights the rows describe: a hit also needs the caller's checksum to match
        DevBuf rows;   // [super-tiles of the tensor][256] u32
    };
    std::unordered_map<uintptr_t, HistEntry> hist_cache;
    // rows of evicted entries, reused by capacity for new ones: apply never calls cudaFree, which
    // would synchronize the whole device (freed only with the context)
    std::vector<DevBuf> hist_free;
    uint64_t hist_hits = 0;   // tensors whose histogram pass was skipped
    DevBuf hstore_table;      // pinned: the table of the last histogram store, read by an async copy
    cudaEvent_t hstore_ev = nullptr;   // recorded after that copy
    // device results (Encoded::write_device): the header and length varint go up from head_host on
    // the caller's stream; wd_ev is recorded after that call's copies.  Until it has passed, the
    // host does not rewrite head_host and the next encode's stream does not rewrite the workspace's
    // block table and payload, which those copies read.
    DevBuf head_host;
    cudaEvent_t wd_ev = nullptr;
    bool wd_busy = false;
    ~Ctx();
};

// Host-phase timestamps on stderr while tracing (CRUKX_B200_TRACE=1); no synchronisation.
void trace_phase(Ctx& c, const char* name);

// Brackets one kernel launch: counts it and, while profiling is on, records events around it.
struct KernelScope {
    Ctx& c;
    cudaStream_t s;
    ProfMark m{nullptr, nullptr, nullptr};
    double t0 = 0.0;
    KernelScope(Ctx& ctx, const char* name, cudaStream_t st);
    ~KernelScope();
};

#define CRX_CUDA(call)                                                               \
    do {                                                                             \
        cudaError_t e_ = (call);                                                     \
        if (e_ != cudaSuccess) {                                                     \
            if (err) *err = std::string(#call ": ") + cudaGetErrorString(e_);        \
            return kCudaError;                                                       \
        }                                                                            \
    } while (0)

}  // namespace crx
