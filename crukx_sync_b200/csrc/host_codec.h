// Host-side pieces of the crukx-sync wire format (version 2): bounds-checked parsing,
// serialization and the length-limited canonical Huffman builder.  Plain C++17, no CUDA.
//
// Reference behaviour restated here (paths relative to the crukx-sync project):
//   src/crukx_sync/wire.py:8-13    constants
//   src/crukx_sync/wire.py:55-61   LEB128 writer
//   src/crukx_sync/wire.py:64-89   serialize
//   src/crukx_sync/wire.py:92-212  _Reader / parse and every receiver limit
//   src/crukx_sync/codec.py:71-111 huffman_lengths / _huffman_unlimited / canonical_codes
//   src/crukx_sync/codec.py:434-454 canonical decode tables
#pragma once

#include <cstddef>
#include <cstdint>
#include <functional>
#include <string>
#include <vector>

namespace crx {

// fn(0 .. n-1) on the calling thread and a pool of worker threads; returns when all are done
// (host_util.cpp)
void parallel_for(size_t n, const std::function<void(size_t)>& fn);

constexpr int kMaxCodeLen = 17;
constexpr uint32_t kMaxSymbol = 131070;
constexpr uint32_t kSymSpace = kMaxSymbol + 1;
constexpr int kMaxRice = 30;
constexpr int kBlock = 256;

enum Status : int { kOk = 0, kValueError = 1, kCorrupt = 2, kCudaError = 3, kNoMemory = 4, kBadArgument = 5, kNeedMore = 6 };

struct Table {
    int exponent = 0;
    std::vector<uint32_t> symbols;
    std::vector<uint8_t> lengths;
};

struct Group {
    int exponent = 0;
    int64_t count = 0;
    int rice = 0;
};

struct TensorHeader {
    const uint8_t* name = nullptr;  // borrowed from the parsed buffer (or owned_names)
    int64_t name_len = 0;
    int64_t numel = 0;
    uint64_t checksum = 0;
    std::vector<Group> groups;
};

struct Update {
    std::vector<Table> tables;
    int table_of_exp[256];
    std::vector<TensorHeader> tensors;
    const uint8_t* block_table = nullptr;  // n_blocks little-endian u32 words, borrowed
    int64_t block_table_offset = -1;       // of the block table within the update (parse_head_device_table)
    const uint8_t* block_table_device = nullptr;  // the block table in device memory (not 4-byte aligned)
    int64_t n_blocks = 0;
    const uint8_t* payload = nullptr;      // borrowed; null when only the head was parsed
    int64_t payload_offset = 0;            // of the payload within the update
    const uint8_t* payload_device = nullptr;  // the payload in device memory (update parsed from its head)
    int64_t payload_len = 0;
    uint64_t total_bits = 0;
    int64_t total_changes = 0;
};

// Parse and validate `data` exactly as the reference's wire.parse does; the result borrows
// `data`, which must outlive it.  Returns kOk or kCorrupt (message in *err).
Status parse_update(const uint8_t* data, int64_t len, Update* out, std::string* err);

// The same parse from the update's head only: `head` holds its first head_len of len bytes and
// `last` is its final byte.  Every check is the same as parse_update's (the payload bytes are
// never inspected except the last, for the padding bits).  Returns kNeedMore with *need = a length
// the head must at least have when the header or block table reaches past head_len.
Status parse_head(const uint8_t* head, int64_t head_len, int64_t len, uint8_t last, Update* out, int64_t* need,
                  std::string* err);

// parse_head for an update whose block table stays where it is (device memory): the table's bytes
// are neither needed in `head` nor read; u->block_table_offset is set once the parse reaches it,
// and a kNeedMore past that offset asks only for the bytes after the table.  On kOk every check
// but the block table's is done: the caller sums the table and finishes with
// finish_block_table_checks.
Status parse_head_device_table(const uint8_t* head, int64_t head_len, int64_t len, uint8_t last, Update* out,
                               int64_t* need, std::string* err);
// Resumes a parse_head_device_table that stopped with kNeedMore past the block table (every check
// before it done, u->block_table_offset and u->n_blocks set): reads what follows the table from
// `head`, which now holds bytes [0, head_len) at least where they are needed, and gives the verdict
// the whole parse would give.  `u` must still point into `head` (its names do).
Status resume_head_device_table(const uint8_t* head, int64_t head_len, int64_t len, Update* u, int64_t* need,
                                std::string* err);
// The same completion from the bytes right after the block table alone (`after`, after_len of them,
// the update being len bytes): for a header whose names point elsewhere.
Status resume_after_table(const uint8_t* after, int64_t after_len, int64_t len, Update* u, std::string* err);
// The block table's checks from its bit total and whether some block is shorter than its symbols
// could be (same messages and order as parse_update's); sets u->total_bits on kOk.
Status finish_block_table_checks(Update* u, uint64_t total_bits, bool short_block, uint8_t last, std::string* err);
// Per group in update order: its first block, and its change count << 8 | rice (the short-block check)
void block_spans(const Update& u, std::vector<uint64_t>* first_block, std::vector<uint64_t>* count_rice);

// Length-limited Huffman code lengths with the reference's tie order.
void huffman_lengths(const uint64_t* counts, int64_t n, uint8_t* lengths);
// Canonical codes in order of (length, table position).
void canonical_codes(const uint8_t* lengths, int64_t n, uint32_t* codes);

// Decode tables of one canonical code: for each length L, the first code, the number of codes and
// the index of its first symbol in (length, position) order; plus left-justified interval limits.
struct DecodeTable {
    uint32_t first[kMaxCodeLen + 1];
    uint32_t count[kMaxCodeLen + 1];
    uint32_t base[kMaxCodeLen + 1];
    uint32_t limit[kMaxCodeLen + 1];  // (first+count) << (17-L): codes of length <= L lie below
};
void build_decode_table(const Table& t, DecodeTable* d, uint32_t* sorted_syms /* n_sym */);

// Little helpers for the serializer.
inline void put_varint(std::vector<uint8_t>& out, uint64_t v) {
    while (v >= 0x80) { out.push_back(uint8_t((v & 0x7F) | 0x80)); v >>= 7; }
    out.push_back(uint8_t(v));
}
inline size_t varint_size(uint64_t v) { size_t n = 1; while (v >= 0x80) { v >>= 7; ++n; } return n; }

}  // namespace crx
