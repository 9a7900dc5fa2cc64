// Internal interface between the C-ABI glue (capi.cu) and the encode/apply drivers.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "context.h"
#include "host_codec.h"

namespace crx {

// A serialized update, kept in pieces so the large part is copied once, straight into the
// caller's buffer: header bytes (host); the block table (in the context's pinned output buffer);
// the payload, still in device memory until write() streams it down chunk by chunk, overlapping
// each chunk's DMA with the host copy of the previous one.  The next encode on the same context
// first moves block table and payload into `own` (detach()).
// Collectives of one update encoded by several ranks (crx_encode_global); each returns 0 on
// success.  sum_u64: element-wise sum over ranks, in place.  allgather_bytes: every rank's bytes
// concatenated in rank order, in a buffer the caller's side keeps alive until the next call.
struct GlobalExchange {
    int (*sum_u64)(void* user, uint64_t* data, int64_t n);
    int (*allgather_bytes)(void* user, const uint8_t* mine, int64_t len, const uint8_t** all, int64_t* all_len);
    void* user;
    int rank, world;
};

struct Encoded {
    Ctx* ctx = nullptr;
    cudaStream_t stream = nullptr;
    std::vector<uint8_t> head;         // magic .. last group header
    const uint8_t* table = nullptr;    // 4 * n_blocks block-table bytes, then the payload (pinned, or own)
    bool pending = false;              // device -> host copies into `table` still in flight: ctx->copy_ev[0]
                                       // covers the block table and the error flags, copy_ev[1 + k] payload chunk k
    bool internal_error = false;       // the encoder's consistency check failed (seen once the copies landed)
    bool device = false;               // block table and payload stay in the context's device workspace
    const uint8_t* dtable = nullptr;   // (device) block table
    const uint8_t* dpay = nullptr;     // (device) payload
    std::vector<uint8_t> own;          // block table + payload after detach()
    // a rank's share of a global update: `head` is then the update's prefix (magic .. tensor count),
    // part_tensors this rank's tensor headers, and the payload starts bit_offset % 8 bits into its
    // first byte; total_bits counts the whole update's payload
    bool part = false;
    std::vector<uint8_t> part_tensors;
    uint64_t bit_offset = 0, total_bits = 0;
    int64_t n_blocks = 0;
    uint64_t payload_len = 0;
    std::vector<uint8_t> len_varint;   // payload_len as LEB128
    // a device result's header parsed up to its block table while the encoder's last kernels ran
    // (names point into `head`); crx_encoded_parse_device completes it once, then it is gone
    mutable std::unique_ptr<Update> pre;
    std::vector<uint64_t> checksums;   // per caller tensor: checksum of `cur` (when present)
    std::vector<uint8_t> present;      // per caller tensor: 1 when the tensor is in the update
    uint64_t changes = 0;

    size_t size() const { return head.size() + 4 * size_t(n_blocks) + len_varint.size() + payload_len; }
    // Serialized bytes into dst (size() bytes): cudaSuccess, a CUDA error, or cudaErrorUnknown when
    // the encoder's consistency check failed.  Pre-faults dst while the copies are in flight.
    cudaError_t write(uint8_t* dst) const;   // capi.cu
    // A part of a global update: its prefix, tensor headers, block table and payload (any may be null).
    cudaError_t write_part(uint8_t* prefix, uint8_t* tensors, uint8_t* table, uint8_t* payload) const;   // capi.cu
    // The same bytes into device memory on `s` (stream-ordered; nothing is read back).
    cudaError_t write_device(uint8_t* dst, cudaStream_t s) const;   // capi.cu
    cudaError_t detach();                    // capi.cu: wait for the copies and keep a private copy
};

// Encode n tensors (device pointers).  cache_chk/has_cache may be null.
Status encode_impl(Ctx& C, int n, const int16_t* const* prev, const int16_t* const* cur, const int64_t* numel,
                   const uint8_t* const* names, const int64_t* name_len, const uint64_t* cache_chk,
                   const uint8_t* has_cache, cudaStream_t st, Encoded* out, std::string* err,
                   bool device_result = false, const GlobalExchange* gx = nullptr);

// Verify `u` against `weights` (one device pointer per update tensor, same order) and commit on
// success.  old_chk/has_chk: the receiver's trusted checksum of each tensor's current contents.
Status apply_impl(Ctx& C, const Update& u, int16_t* const* weights, const uint64_t* old_chk, const uint8_t* has_chk,
                  cudaStream_t st, int64_t* changed, std::string* err, const uint64_t* versions = nullptr,
                  const uint8_t* has_version = nullptr, int16_t* const* host_weights = nullptr);

// Full checksum of one device tensor (reference codec.checksum).
Status checksum_impl(Ctx& C, const int16_t* data, int64_t n, cudaStream_t st, uint64_t* out, std::string* err);

// Histograms behind the size comparison (sizes.cu); `out` (host) receives size_stats_words() u64.
int size_stats_words();
Status size_stats_impl(Ctx& C, int n, const int16_t* const* prev, const int16_t* const* cur, const int64_t* numel,
                       cudaStream_t st, uint64_t* out, std::string* err);

}  // namespace crx
