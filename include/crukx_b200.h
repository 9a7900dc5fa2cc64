/*
 * crukx_b200.h -- C ABI of the B200-native crukx-sync encode/apply path.
 *
 * Plain pointers, sizes and an opaque CUDA stream (cudaStream_t passed as void*); no C++ or torch
 * types cross this boundary and no exceptions escape it.  Every call returns a status code:
 *
 *   CRX_OK            success
 *   CRX_VALUE_ERROR   caller mistake / unrepresentable update      -> Python ValueError
 *   CRX_CORRUPT       malformed update or one that does not verify -> Python CorruptUpdate
 *   CRX_CUDA_ERROR    CUDA runtime failure
 *   CRX_NO_MEMORY     host allocation failure
 *   CRX_BAD_ARGUMENT  null/negative arguments
 *
 * and writes a NUL-terminated message into err[0..errlen) on failure.
 *
 * Device pointers are owned by the caller; scratch memory is owned by the context (one per
 * device, grown on demand, reused across calls).  Calls on one context are serialized by an
 * internal lock; work is ordered on the caller's stream.  The reference interfaces each entry
 * point replaces are cited beside it (paths relative to the crukx-sync project).
 */
#ifndef CRUKX_B200_H
#define CRUKX_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CRX_OK 0
#define CRX_VALUE_ERROR 1
#define CRX_CORRUPT 2
#define CRX_CUDA_ERROR 3
#define CRX_NO_MEMORY 4
#define CRX_BAD_ARGUMENT 5
#define CRX_NEED_MORE 6      /* crx_parse_head: the head given is too short; *need is a lower bound */

typedef struct crx_ctx crx_ctx;
typedef struct crx_encoded crx_encoded;
typedef struct crx_update crx_update;

/* Wire format version produced and accepted (src/crukx_sync/wire.py:9: VERSION = 2). */
int crx_wire_version(void);

/* Per-device context.  No reference counterpart: the reference allocates through torch. */
int crx_ctx_create(int device, crx_ctx** out, char* err, size_t errlen);
void crx_ctx_destroy(crx_ctx* ctx);
/* Kernels launched by this context so far (no reference counterpart: instrumentation). */
uint64_t crx_ctx_launches(crx_ctx* ctx);
/* Device and pinned-host allocations and frees this library has made so far, process-wide
 * (instrumentation, no reference counterpart): a test reads it around calls of an entry point that
 * must allocate nothing. */
uint64_t crx_alloc_calls(void);
/* Kernels launched by crx_parse_device (its block-table check), process-wide: crx_parse_device
 * takes no context, so these are not in crx_ctx_launches. */
uint64_t crx_parse_device_launches(void);
/* Per-kernel timing with CUDA events on the caller's stream while enabled (instrumentation, no
 * reference counterpart).  Enabling clears earlier records.  crx_ctx_kernel_times returns the
 * number of distinct kernels, writes their names ('\n'-separated) and total ms / launch counts
 * for the first `max` of them. */
int crx_ctx_profile(crx_ctx* ctx, int enable);
int32_t crx_ctx_kernel_times(crx_ctx* ctx, char* names, size_t names_len, double* ms, int32_t* counts, int32_t max);
/* While profiling: per kernel, the total time its stream sat idle between the previous profiled
 * kernel's end and its start (host work, synchronisations and copies in between); names as for
 * crx_ctx_kernel_times.  Instrumentation, no reference counterpart. */
int32_t crx_ctx_kernel_gaps(crx_ctx* ctx, char* names, size_t names_len, double* gap_ms, int32_t max);

/*
 * Encode old -> new for n tensors of bf16/int16 bits on the context's device.
 * Replaces codec.encode + wire.serialize (src/crukx_sync/codec.py:278-420, wire.py:64-89) as
 * called by encode_update (src/crukx_sync/__init__.py:38-48).  Tensor order = update order;
 * names are UTF-8 (name_len bytes each).  cached_checksums/has_cached (may be NULL) hold the
 * sender's cached checksum of prev[i] (codec.py:345-352).  On success *out holds the update.
 */
int crx_encode(crx_ctx* ctx, int32_t n_tensors, const int16_t* const* prev, const int16_t* const* cur,
               const int64_t* numel, const uint8_t* const* names, const int64_t* name_len,
               const uint64_t* cached_checksums, const uint8_t* has_cached, void* stream,
               crx_encoded** out, char* err, size_t errlen);
int64_t crx_encoded_size(const crx_encoded* enc);
/* Copy the serialized update into dst (cap >= crx_encoded_size). */
int crx_encoded_copy(const crx_encoded* enc, uint8_t* dst, int64_t cap);
int64_t crx_encoded_changes(const crx_encoded* enc);
/* Per input tensor: the checksum of new[i] to commit to the sender cache, present[i] = 1 when
 * tensor i is in the update (the reference commits only those, __init__.py:46-47). */
void crx_encoded_checksums(const crx_encoded* enc, uint64_t* checksums, uint8_t* present);
void crx_encoded_free(crx_encoded* enc);

/*
 * Device-resident updates (no reference counterpart: the reference always returns host bytes).
 * crx_encode_device runs the same encoder but leaves the block table and payload in the context's
 * device workspace; crx_encoded_copy_device writes the complete update, byte-identical to
 * crx_encoded_copy's, into device memory `dst` (cap >= crx_encoded_size) on `stream`, ordered after
 * the encode; it returns without waiting for the device (the encoder's consistency checks were
 * read back before crx_encode_device returned).  Copy (or free) the result before the next encode
 * on the same context, which otherwise first moves it to host memory.  crx_encoded_copy also works
 * on such a result.
 */
int crx_encode_device(crx_ctx* ctx, int32_t n_tensors, const int16_t* const* prev, const int16_t* const* cur,
                      const int64_t* numel, const uint8_t* const* names, const int64_t* name_len,
                      const uint64_t* cached_checksums, const uint8_t* has_cached, void* stream,
                      crx_encoded** out, char* err, size_t errlen);
int crx_encoded_copy_device(const crx_encoded* enc, void* dst, int64_t cap, void* stream);
/*
 * The parsed form of the update that crx_encoded_copy_device wrote at device address `data`, built
 * from the encoder's own host-side header (no reference counterpart): what crx_parse_device would
 * return for those bytes, without copying the header down or checking the block table, so that a
 * receiver in the same process (the sender's own replica) applies it without waiting for the
 * encode to finish.  Only for a device result (crx_encode_device) whose bytes at `data` are
 * unchanged; free with crx_update_free.
 */
int crx_encoded_parse_device(const crx_encoded* enc, const uint8_t* data, crx_update** out, char* err, size_t errlen);

/*
 * One update encoded by several ranks (no reference counterpart; the single-GPU encode of the
 * whole dict is the reference's encode_update, and the result is byte-identical to it).  Rank r
 * passes its own tensors, which must be the r-th contiguous range of the update's tensor order.
 * Inside, the library calls the two collectives below on every rank in the same order (each
 * returns 0 on success; a rank that fails must still have taken every earlier call):
 *   sum_u64(user, data, n): element-wise sum over ranks of n u64 values, in place (wrapping);
 *   allgather(user, mine, len, &all, &all_len): every rank's bytes, concatenated in rank order, in
 *     a buffer the caller's side keeps valid until the next callback or until crx_encode_global
 *     returns.
 * The symbol histogram is summed over ranks so the Huffman tables are the whole update's, and
 * each rank packs its payload at its bit offset in the whole payload.  The result is a part:
 * crx_encoded_part gives the sizes of its pieces, crx_encoded_part_copy copies them.  The update
 * is prefix (rank-independent) + every rank's tensor headers + every rank's block table + LEB128
 * of (total_bits + 7) / 8 + the payloads OR-ed together, rank r's starting at byte
 * bit_offset / 8 (its first byte holds the previous rank's last bits when bit_offset % 8 != 0).
 * crx_encoded_size/_copy/_copy_device refuse a part.
 */
typedef int (*crx_sum_u64_fn)(void* user, uint64_t* data, int64_t n);
typedef int (*crx_allgather_fn)(void* user, const uint8_t* mine, int64_t len, const uint8_t** all, int64_t* all_len);
int crx_encode_global(crx_ctx* ctx, int32_t n_tensors, const int16_t* const* prev, const int16_t* const* cur,
                      const int64_t* numel, const uint8_t* const* names, const int64_t* name_len,
                      const uint64_t* cached_checksums, const uint8_t* has_cached, void* stream, int32_t rank,
                      int32_t world, crx_sum_u64_fn sum_u64, crx_allgather_fn allgather, void* user,
                      crx_encoded** out, char* err, size_t errlen);
int crx_encoded_part(const crx_encoded* enc, int64_t* prefix_len, int64_t* tensors_len, int64_t* table_len,
                     int64_t* payload_len, uint64_t* bit_offset, uint64_t* total_bits);
int crx_encoded_part_copy(const crx_encoded* enc, uint8_t* prefix, uint8_t* tensors, uint8_t* table, uint8_t* payload);

/*
 * Parse and validate an update on the host: every limit of wire.parse
 * (src/crukx_sync/wire.py:126-212).  The handle borrows data[0..len), which must outlive it.
 */
int crx_parse(const uint8_t* data, int64_t len, crx_update** out, char* err, size_t errlen);
/* The same validation from the update's head alone (wire.py:126-212 reads the payload only for its
 * length and final padding bits): head = the first head_len of the update's len bytes, last = its
 * final byte.  CRX_NEED_MORE when the header or block table reaches past head_len, with *need = a
 * length the head must at least have (grow it geometrically); otherwise the same verdict as
 * crx_parse.  The handle borrows `head` and has
 * no payload (crx_update_payload gives NULL), so it cannot be applied; it serves transports that
 * validate an update before its payload has arrived. */
int crx_parse_head(const uint8_t* head, int64_t head_len, int64_t len, uint8_t last, crx_update** out, int64_t* need,
                   char* err, size_t errlen);
/* Parse an update held in device memory (len bytes at `data`): its header is copied to the host on
 * `stream`, its block table is summed and checked on the device where it lies, and every check of
 * crx_parse is made with the same verdicts; the block table and payload stay where they are and
 * crx_apply reads them there (data must stay valid until crx_apply returns).  No reference
 * counterpart. */
int crx_parse_device(const uint8_t* data, int64_t len, void* stream, crx_update** out, char* err, size_t errlen);
int64_t crx_update_n_tensors(const crx_update* u);
int64_t crx_update_changes(const crx_update* u);
int crx_update_tensor(const crx_update* u, int64_t i, const uint8_t** name, int64_t* name_len, int64_t* numel,
                      uint64_t* checksum, int32_t* n_groups);
int crx_update_group(const crx_update* u, int64_t i, int32_t k, int32_t* exponent, int64_t* count, int32_t* rice);
/* All tensor headers at once (arrays of crx_update_n_tensors entries; any may be NULL). */
int crx_update_tensor_table(const crx_update* u, const uint8_t** names, int64_t* name_lens, int64_t* numels,
                            uint64_t* checksums);
int32_t crx_update_n_tables(const crx_update* u);
int crx_update_table(const crx_update* u, int32_t k, int32_t* exponent, int64_t* n_symbols);
int crx_update_table_entries(const crx_update* u, int32_t k, uint32_t* symbols, uint8_t* lengths);
int64_t crx_update_n_blocks(const crx_update* u);
int crx_update_block_bits(const crx_update* u, uint32_t* out);
/* The payload bytes at hand (NULL and 0 for an update parsed from its head or from device memory). */
int crx_update_payload(const crx_update* u, const uint8_t** data, int64_t* len);
void crx_update_free(crx_update* u);

/*
 * Verify a parsed update against the receiver's weights and write it in place, all or nothing.
 * Replaces codec.apply (src/crukx_sync/codec.py:578-717) as called by apply_update
 * (src/crukx_sync/__init__.py:51-57).  weights[i] is the device buffer of update tensor i (the
 * caller matched names and sizes first, codec.py:582-592).  cached_checksums/has_cached (may be
 * NULL): the receiver's trusted checksum of weights[i] (codec.py:457-460, 702-705).  On
 * CRX_CORRUPT nothing was written; on CRX_OK the commit is enqueued on `stream`.
 */
int crx_apply(crx_ctx* ctx, const crx_update* u, int16_t* const* weights, const uint64_t* cached_checksums,
              const uint8_t* has_cached, void* stream, int64_t* changed, char* err, size_t errlen);

/*
 * crx_apply with the context's exponent-histogram cache (the caching of per-super-tile exponent
 * tables across steps; no reference counterpart).  versions[i]/has_version[i] tag update tensor
 * i's weights with the caller's version counter (torch: tensor._version).  A tagged tensor whose
 * weights address, size and tag match what this context stored after its last apply, and whose
 * cached checksum (cached_checksums[i], required) equals the checksum that apply established,
 * skips the pass that histograms its exponents.  After a successful apply every tagged tensor's
 * histogram is stored with tag versions[i] + 1: the caller bumps its version counter by one for
 * the in-place write.  Untagged tensors that the update writes drop their entry.  A stale entry can
 * only make the update fail verification (CorruptUpdate, nothing written), never write wrong values.
 */
int crx_apply_versioned(crx_ctx* ctx, const crx_update* u, int16_t* const* weights, const uint64_t* cached_checksums,
                        const uint8_t* has_cached, const uint64_t* versions, const uint8_t* has_version, void* stream,
                        int64_t* changed, char* err, size_t errlen);
/*
 * crx_apply for weights the caller keeps in host memory (the reference accepts CPU tensors,
 * src/crukx_sync/codec.py:578-592, and writes them in place, :713-714).  device_copies[i] hold
 * the same bits as host_weights[i] (the caller uploaded them); the update is decoded, placed and
 * verified against the copies exactly as crx_apply does, and on success only the changed elements
 * are written into host_weights (the commit list -- a bit per element and the new values -- comes
 * down once and host threads scatter it; tensors whose host memory is pinned may instead be
 * committed into their device copy and copied down whole).  The device copies are scratch: after a
 * success some may hold the new values.  On any error nothing is written to either.
 * host_weights[i] must stay valid and unused by others until it returns.
 */
int crx_apply_to_host(crx_ctx* ctx, const crx_update* u, int16_t* const* device_copies, int16_t* const* host_weights,
                      const uint64_t* cached_checksums, const uint8_t* has_cached, void* stream, int64_t* changed,
                      char* err, size_t errlen);
/* Tensors whose histogram pass was skipped by the cache so far (instrumentation). */
uint64_t crx_ctx_hist_cache_hits(crx_ctx* ctx);

/* Length-limited canonical Huffman code lengths for n symbol counts, with the reference's tie
 * order (src/crukx_sync/codec.py:71-98).  Host only; the encoder uses the same routine. */
int crx_huffman_lengths(const uint64_t* counts, int64_t n, uint8_t* lengths);

/* Full checksum of n int16 elements on the device (src/crukx_sync/codec.py:61-68). */
int crx_checksum(crx_ctx* ctx, const int16_t* data, int64_t n, void* stream, uint64_t* out, char* err, size_t errlen);

/* The same checksum for callers that must not allocate device memory; no counterpart in the
 * reference.  Examples: a serving process whose HBM is reserved up front for weights and
 * KV-cache (a cudaMalloc in steady state fails or breaks the budget), code inside an allocator
 * callback or out-of-memory handler (re-entering the allocator can deadlock), or a loop that must
 * not stall other streams (cudaFree synchronizes the device).  It needs no crx_ctx, allocates
 * nothing and does not synchronize: data (n int16 elements, 2-byte aligned) and out (8 bytes,
 * 8-byte aligned) are device memory on the current device (or managed memory), and the result is
 * in *out once the work on `stream` is done.  A misaligned pointer, or one that is not device
 * memory of the current device, returns CRX_BAD_ARGUMENT before anything is launched.
 *
 * Limit: n <= CRX_CHECKSUM_NOALLOC_MAX (2^30 elements); larger n returns CRX_VALUE_ERROR — use
 * crx_checksum.  Its scratch is one fixed 128 KiB device array per device: the first call on a
 * device (with it current) looks the array up, which loads this library on that device, so make
 * one call before capturing a stream.  Nothing has to start at zero.  Calls that overlap on one
 * device (two streams or unordered host threads) race on the scratch; order them. */
#define CRX_CHECKSUM_NOALLOC_MAX (INT64_C(1) << 30)
int crx_checksum_noalloc(const int16_t* data, int64_t n, void* stream, uint64_t* out, char* err, size_t errlen);

/*
 * Histograms behind the update-size comparison of the reference's bench/compare.py (:56-100, its
 * raw, sparserl and ctxfree columns), over n tensors of old/new bits on the context's device, in
 * one pass.  out (host) receives CRX_SIZE_STATS_WORDS u64: [0] changed elements, [1] changes
 * whose position delta needs more than 16 bits, [2] the sum over changes of
 * max(bit_length(gap) - 1, 0), [3, 67) changes per gap bit length, then 65536 counts of the new
 * values' bit patterns and 65536 counts of old ^ new.  The gap of a change is its distance to the
 * tensor's previous change minus one; the tensor's first change has gap = delta = its index.
 * crukx_sync_b200.sizes turns these into the three sizes with compare.py's formulas.
 */
#define CRX_SIZE_STATS_WORDS (3 + 64 + 2 * 65536)
int crx_size_stats(crx_ctx* ctx, int32_t n_tensors, const int16_t* const* prev, const int16_t* const* cur,
                   const int64_t* numel, void* stream, uint64_t* out, char* err, size_t errlen);

#ifdef __cplusplus
}
#endif

#endif /* CRUKX_B200_H */
