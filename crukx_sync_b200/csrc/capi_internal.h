// Internal interface between the C-ABI glue (capi.cu) and the encode/apply drivers.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

#include "context.h"
#include "host_codec.h"

namespace crx {

struct Encoded {
    std::vector<uint8_t> bytes;        // the complete serialized update
    std::vector<uint64_t> checksums;   // per caller tensor: checksum of `cur` (when present)
    std::vector<uint8_t> present;      // per caller tensor: 1 when the tensor is in the update
    uint64_t changes = 0;
};

// Encode n tensors (device pointers).  cache_chk/has_cache may be null.
Status encode_impl(Ctx& C, int n, const int16_t* const* prev, const int16_t* const* cur, const int64_t* numel,
                   const uint8_t* const* names, const int64_t* name_len, const uint64_t* cache_chk,
                   const uint8_t* has_cache, cudaStream_t st, Encoded* out, std::string* err);

// Verify `u` against `weights` (one device pointer per update tensor, same order) and commit on
// success.  old_chk/has_chk: the receiver's trusted checksum of each tensor's current contents.
Status apply_impl(Ctx& C, const Update& u, int16_t* const* weights, const uint64_t* old_chk, const uint8_t* has_chk,
                  cudaStream_t st, int64_t* changed, std::string* err);

// Full checksum of one device tensor (reference codec.checksum).
Status checksum_impl(Ctx& C, const int16_t* data, int64_t n, cudaStream_t st, uint64_t* out, std::string* err);

}  // namespace crx
