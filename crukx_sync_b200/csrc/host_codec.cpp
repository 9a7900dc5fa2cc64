// Host-side wire-format code: parse (with every receiver limit), Huffman lengths with the
// reference's tie order, canonical codes and decode tables.  See host_codec.h for the
// reference lines each function restates.
#include "host_codec.h"

#include <algorithm>
#include <cstring>
#include <string_view>
#include <unordered_set>

namespace crx {

namespace {

// Sequential reader over an update of n bytes of which the first `avail` are at hand: reading
// past n is a corrupt update (wire.py:92-123); reading past `avail` fails too but records in
// `need` how many bytes the read wanted, so the caller can fetch more and parse again.
struct Reader {
    const uint8_t* d;
    int64_t n;
    int64_t avail;
    int64_t pos = 0;
    int64_t need = 0;
    bool have(int64_t k) {
        if (k < 0 || k > n - pos) return false;
        if (k > avail - pos) {
            need = std::max(need, pos + k);
            return false;
        }
        return true;
    }
    bool take(int64_t k, const uint8_t** p) {
        if (!have(k)) return false;
        *p = d + pos;
        pos += k;
        return true;
    }
    bool skip(int64_t k) {   // bytes the parser does not look at (the payload)
        if (k < 0 || k > n - pos) return false;
        pos += k;
        return true;
    }
    bool u8(int* v) {
        if (!have(1)) return false;
        *v = d[pos++];
        return true;
    }
    // LEB128 below 2^63 and at most 10 bytes (wire.py:109-120): a set bit at or above bit 63 is
    // corrupt as soon as it is read, a continuation past shift 63 likewise.
    bool varint(int64_t* out) {
        uint64_t v = 0;
        int shift = 0;
        for (;;) {
            int b;
            if (!u8(&b)) return false;
            uint64_t part = uint64_t(b & 0x7F);
            if (part) {
                if (shift >= 63) return false;
                if (shift > 56 && (part >> (63 - shift)) != 0) return false;
                v |= part << shift;
            }
            if (!(b & 0x80)) { *out = int64_t(v); return true; }
            shift += 7;
            if (shift > 63) return false;
        }
    }
    int64_t remaining() const { return n - pos; }
};

// Strict UTF-8 as Python decodes it: no overlong forms, no surrogates, at most U+10FFFF.
bool valid_utf8(const uint8_t* s, int64_t n) {
    int64_t i = 0;
    while (i < n) {
        const uint32_t c = s[i];
        if (c < 0x80) { ++i; continue; }
        int extra;
        uint32_t cp, lo;
        if (c >= 0xC2 && c <= 0xDF) { extra = 1; cp = c & 0x1F; lo = 0x80; }
        else if (c >= 0xE0 && c <= 0xEF) { extra = 2; cp = c & 0x0F; lo = 0x800; }
        else if (c >= 0xF0 && c <= 0xF4) { extra = 3; cp = c & 0x07; lo = 0x10000; }
        else return false;
        if (n - i <= extra) return false;
        for (int k = 1; k <= extra; ++k) {
            const uint32_t cc = s[i + k];
            if ((cc & 0xC0) != 0x80) return false;
            cp = (cp << 6) | (cc & 0x3F);
        }
        if (cp < lo || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) return false;
        i += extra + 1;
    }
    return true;
}

}  // namespace

namespace {

// The whole parse over the first `avail` of `len` bytes; `last` is the update's final byte (the
// padding check needs it).  kNeedMore with *need set when the head does not fit in `avail`.
// What follows a block table kept elsewhere: the payload length, the payload's place, nothing after
// it.  `r` stands just past the table.
template <class Bad>
Status parse_after_table(Reader& r, const uint8_t* data, int64_t avail, Update* u, Bad& bad) {
    int64_t pl;
    if (!r.varint(&pl)) return bad("update is truncated");
    u->payload_offset = r.pos;
    if (!r.skip(pl)) return bad("update is truncated");
    u->payload = r.pos <= avail ? data + u->payload_offset : nullptr;
    u->payload_len = pl;
    if (r.remaining() != 0) return bad("trailing bytes after the payload");
    int64_t changes = 0;
    for (const TensorHeader& h : u->tensors)
        for (const Group& g : h.groups) changes += g.count;
    u->total_changes = changes;
    u->total_bits = 0;
    return kOk;
}

Status parse_core(const uint8_t* data, int64_t avail, int64_t len, uint8_t last, Update* u, int64_t* need,
                  std::string* err, bool table_elsewhere = false) {
    Reader r{data, len, avail};
    auto bad = [&](const char* m) {
        if (r.need > 0) {   // ran out of the bytes at hand, not out of the update
            if (need) *need = r.need;
            return kNeedMore;
        }
        if (err) *err = m;
        return kCorrupt;
    };
    const uint8_t* p;
    int v;
    int64_t x;
    for (int e = 0; e < 256; ++e) u->table_of_exp[e] = -1;
    if (!r.take(4, &p)) return bad("update is truncated");
    if (std::memcmp(p, "CRXS", 4) != 0) return bad("not a crukx-sync update");
    if (!r.u8(&v)) return bad("update is truncated");
    if (v != 2) return bad("unsupported format version");

    int64_t n_tables;
    if (!r.varint(&n_tables)) return bad("update is truncated or has a bad varint");
    if (n_tables > 256) return bad("too many tables");
    u->tables.resize(size_t(n_tables));
    std::vector<uint8_t> seen_sym;
    for (int64_t t = 0; t < n_tables; ++t) {
        int e;
        int64_t n_sym;
        if (!r.u8(&e) || !r.varint(&n_sym)) return bad("update is truncated or has a bad varint");
        const int64_t cap = std::min<int64_t>(kMaxSymbol + 1, r.remaining() / 2);
        if (u->table_of_exp[e] >= 0 || !(n_sym > 0 && n_sym <= cap)) return bad("bad table header");
        u->table_of_exp[e] = int(t);
        Table& tb = u->tables[size_t(t)];
        tb.exponent = e;
        tb.symbols.resize(size_t(n_sym));
        tb.lengths.resize(size_t(n_sym));
        bool sym_range_ok = true;
        int64_t k = 0;
        // fast path while 4 bytes are at hand: a symbol of at most 3 varint bytes and its length
        // byte, read straight from the buffer (the same values and verdicts as the reader below,
        // which takes over at the first longer varint or near the end of the bytes)
        while (k < n_sym && r.avail - r.pos >= 4) {
            const uint8_t* q = r.d + r.pos;
            uint32_t v = q[0], nb = 1;
            if (v & 0x80) {
                v = (v & 0x7Fu) | (uint32_t(q[1] & 0x7F) << 7);
                nb = 2;
                if (q[1] & 0x80) {
                    if (q[2] & 0x80) break;
                    v |= uint32_t(q[2]) << 14;
                    nb = 3;
                }
            }
            if (v > kMaxSymbol) sym_range_ok = false;
            tb.symbols[size_t(k)] = std::min<uint32_t>(v, kMaxSymbol + 1);
            tb.lengths[size_t(k)] = q[nb];
            r.pos += nb + 1;
            ++k;
        }
        for (; k < n_sym; ++k) {
            int64_t s;
            int L;
            if (!r.varint(&s) || !r.u8(&L)) return bad("update is truncated or has a bad varint");
            if (s > int64_t(kMaxSymbol)) sym_range_ok = false;
            tb.symbols[size_t(k)] = uint32_t(std::min<int64_t>(s, kMaxSymbol + 1));
            tb.lengths[size_t(k)] = uint8_t(L);
        }
        // symbols unique and <= MAX_SYMBOL (either failure is the same error)
        if (!sym_range_ok) return bad("bad table symbols");
        if (seen_sym.empty()) seen_sym.assign(kSymSpace, 0);
        bool dup = false;
        for (uint32_t s : tb.symbols) { dup |= seen_sym[s] != 0; seen_sym[s] = 1; }
        for (uint32_t s : tb.symbols) seen_sym[s] = 0;
        if (dup) return bad("bad table symbols");
        // lengths 1..17 and Kraft sum <= 1; each term is a multiple of 2^-17, so the float test
        // with its 1e-12 slack (wire.py:149) is this exact integer test
        uint64_t kraft = 0;
        for (uint8_t L : tb.lengths) {
            if (L < 1 || L > kMaxCodeLen) return bad("bad Huffman code lengths");
            kraft += uint64_t(1) << (kMaxCodeLen - L);
        }
        if (kraft > (uint64_t(1) << kMaxCodeLen)) return bad("bad Huffman code lengths");
    }

    int64_t n_tensors;
    if (!r.varint(&n_tensors)) return bad("update is truncated or has a bad varint");
    if (n_tensors > r.remaining()) return bad("too many tensors");
    u->tensors.resize(size_t(n_tensors));
    std::unordered_set<std::string_view> names_seen;   // a tensor named twice is corrupt (wire.py's check)
    names_seen.reserve(size_t(n_tensors) * 2);
    unsigned __int128 total_blocks = 0;
    unsigned __int128 per_exp[256] = {};
    for (int64_t t = 0; t < n_tensors; ++t) {
        TensorHeader& h = u->tensors[size_t(t)];
        int64_t nl;
        if (!r.varint(&nl) || !r.take(nl, &p)) return bad("update is truncated");
        if (!valid_utf8(p, nl)) return bad("tensor name is not valid UTF-8");
        h.name = p;
        h.name_len = nl;
        if (!names_seen.emplace(reinterpret_cast<const char*>(p), size_t(nl)).second) return bad("tensor appears twice");
        if (!r.varint(&h.numel)) return bad("update is truncated or has a bad varint");
        if (!r.take(8, &p)) return bad("update is truncated");
        h.checksum = 0;
        for (int k = 7; k >= 0; --k) h.checksum = (h.checksum << 8) | p[k];
        int64_t ng;
        if (!r.varint(&ng)) return bad("update is truncated or has a bad varint");
        if (!(ng > 0 && ng <= 256)) return bad("bad group count");
        h.groups.resize(size_t(ng));
        bool used[256] = {};
        unsigned __int128 sum = 0;
        for (int64_t k = 0; k < ng; ++k) {
            int e, rice;
            int64_t c;
            if (!r.u8(&e) || !r.varint(&c) || !r.u8(&rice)) return bad("update is truncated or has a bad varint");
            if (used[e] || u->table_of_exp[e] < 0) return bad("bad group exponent");
            if (!(c > 0 && c <= h.numel) || rice > kMaxRice) return bad("bad group header");
            used[e] = true;
            h.groups[size_t(k)] = Group{e, c, rice};
            total_blocks += (unsigned __int128)((c + kBlock - 1) / kBlock);
            sum += (unsigned __int128)c;
            per_exp[e] += (unsigned __int128)c;
        }
        if (sum > (unsigned __int128)h.numel) return bad("more changes than elements");
    }
    for (const Table& tb : u->tables)
        if ((unsigned __int128)tb.symbols.size() > per_exp[tb.exponent]) return bad("table unused or larger than its changes");
    if (total_blocks * 4 > (unsigned __int128)r.remaining()) return bad("block table longer than the update");
    u->n_blocks = int64_t(total_blocks);
    if (table_elsewhere) {   // the table's bytes are not here: only its place and length
        u->block_table_offset = r.pos;
        u->block_table = nullptr;
        if (!r.skip(4 * u->n_blocks)) return bad("update is truncated");
    } else if (!r.take(4 * u->n_blocks, &u->block_table)) {
        return bad("update is truncated");
    }
    if (table_elsewhere) return parse_after_table(r, data, avail, u, bad);
    int64_t pl;
    if (!r.varint(&pl)) return bad("update is truncated");
    u->payload_offset = r.pos;
    if (!r.skip(pl)) return bad("update is truncated");
    u->payload = r.pos <= avail ? data + u->payload_offset : nullptr;
    u->payload_len = pl;
    if (r.remaining() != 0) return bad("trailing bytes after the payload");
    // block table, one pass split over the worker threads: the bit total, and every change costs
    // at least 2 + rice bits (wire.py:204-211)
    struct Span { int64_t b0, count; int rice; };
    std::vector<Span> spans;
    int64_t changes = 0;
    {
        int64_t b = 0;
        for (const TensorHeader& h : u->tensors)
            for (const Group& g : h.groups) {
                spans.push_back(Span{b, g.count, g.rice});
                b += (g.count + kBlock - 1) / kBlock;
                changes += g.count;
            }
    }
    const uint8_t* bt = u->block_table;
    constexpr int64_t kPer = int64_t(1) << 16;   // blocks per task
    const size_t n_tasks = size_t((u->n_blocks + kPer - 1) / kPer);
    std::vector<uint64_t> part_bits(n_tasks, 0);
    std::vector<uint8_t> part_bad(n_tasks, 0);
    auto task = [&](size_t k) {
        const int64_t lo = int64_t(k) * kPer, hi = std::min(u->n_blocks, lo + kPer);
        // the span holding block lo, then walk forward
        size_t sp = size_t(std::upper_bound(spans.begin(), spans.end(), lo,
                                            [](int64_t v, const Span& x) { return v < x.b0; }) - spans.begin()) - 1;
        uint64_t bits = 0;
        bool bad_block = false;
        for (int64_t b = lo; b < hi; ++b) {
            while (sp + 1 < spans.size() && spans[sp + 1].b0 <= b) ++sp;
            uint32_t w;
            std::memcpy(&w, bt + 4 * b, 4);
            bits += w;
            const Span& x = spans[sp];
            const int64_t m = std::min<int64_t>(kBlock, x.count - (b - x.b0) * kBlock);
            bad_block |= uint64_t(w) < uint64_t(m) * uint64_t(2 + x.rice);
        }
        part_bits[k] = bits;
        part_bad[k] = bad_block;
    };
    if (n_tasks > 1) parallel_for(n_tasks, task);
    else if (n_tasks == 1) task(0);
    uint64_t total_bits = 0;
    bool short_block = false;
    for (size_t k = 0; k < n_tasks; ++k) { total_bits += part_bits[k]; short_block |= part_bad[k] != 0; }
    u->total_changes = changes;
    return finish_block_table_checks(u, total_bits, short_block, last, err);
}

}  // namespace

Status parse_update(const uint8_t* data, int64_t len, Update* u, std::string* err) {
    return parse_core(data, len, len, len > 0 ? data[len - 1] : 0, u, nullptr, err);
}

Status parse_head(const uint8_t* head, int64_t head_len, int64_t len, uint8_t last, Update* u, int64_t* need,
                  std::string* err) {
    return parse_core(head, std::min(head_len, len), len, last, u, need, err);
}

Status parse_head_device_table(const uint8_t* head, int64_t head_len, int64_t len, uint8_t last, Update* u,
                               int64_t* need, std::string* err) {
    return parse_core(head, std::min(head_len, len), len, last, u, need, err, true);
}

Status resume_head_device_table(const uint8_t* head, int64_t head_len, int64_t len, Update* u, int64_t* need,
                                std::string* err) {
    Reader r{head, len, std::min(head_len, len)};
    r.pos = u->block_table_offset + 4 * u->n_blocks;
    auto bad = [&](const char* m) {
        if (r.need > 0) {
            if (need) *need = r.need;
            return kNeedMore;
        }
        if (err) *err = m;
        return kCorrupt;
    };
    return parse_after_table(r, head, r.avail, u, bad);
}

Status resume_after_table(const uint8_t* after, int64_t after_len, int64_t len, Update* u, std::string* err) {
    const int64_t t1 = u->block_table_offset + 4 * u->n_blocks;
    if (t1 > len) {
        if (err) *err = "update is truncated";
        return kCorrupt;
    }
    Reader r{after, len - t1, std::min(after_len, len - t1)};   // offsets relative to t1
    auto bad = [&](const char* m) {
        if (err) *err = m;
        return kCorrupt;
    };
    const Status s = parse_after_table(r, after, r.avail, u, bad);
    if (s == kOk) {
        u->payload_offset += t1;
        u->payload = nullptr;
    }
    return s;
}

Status finish_block_table_checks(Update* u, uint64_t total_bits, bool short_block, uint8_t last, std::string* err) {
    auto bad = [&](const char* m) {
        if (err) *err = m;
        return kCorrupt;
    };
    if ((total_bits + 7) / 8 != uint64_t(u->payload_len)) return bad("payload length does not match its block table");
    if ((total_bits & 7) && (last & ((1u << (8 - (total_bits & 7))) - 1))) return bad("non-zero padding bits");
    if (short_block) return bad("block shorter than its symbols could be");
    u->total_bits = total_bits;
    return kOk;
}

void block_spans(const Update& u, std::vector<uint64_t>* first_block, std::vector<uint64_t>* count_rice) {
    first_block->clear();
    count_rice->clear();
    uint64_t b = 0;
    for (const TensorHeader& h : u.tensors)
        for (const Group& g : h.groups) {
            first_block->push_back(b);
            count_rice->push_back((uint64_t(g.count) << 8) | uint64_t(g.rice & 0xFF));
            b += (uint64_t(g.count) + kBlock - 1) / kBlock;
        }
}

// ---------------------------------------------------------------- Huffman

namespace {

struct Item {
    uint64_t count;
    int64_t id;
    bool operator<(const Item& o) const { return count != o.count ? count < o.count : id < o.id; }
};

// Code lengths of an unlimited Huffman code, popping (count, id) pairs in the order a binary
// min-heap would (codec.py:81-98): leaves are ids 0..n-1, merged nodes n, n+1, ...  Merged
// counts never decrease, so two FIFO queues (sorted leaves, merged nodes) reproduce the heap.
void huffman_unlimited(const std::vector<uint64_t>& counts, std::vector<int>& depth_out) {
    const int64_t n = int64_t(counts.size());
    depth_out.assign(size_t(n), 1);
    if (n == 1) return;
    std::vector<Item> leaves(static_cast<size_t>(n));
    for (int64_t i = 0; i < n; ++i) leaves[size_t(i)] = Item{counts[size_t(i)], i};
    std::sort(leaves.begin(), leaves.end());
    std::vector<Item> merged;
    merged.reserve(size_t(n));
    std::vector<int64_t> parent(static_cast<size_t>(2 * n - 1), 0);
    size_t li = 0, mi = 0;
    int64_t next_id = n;
    auto pop = [&]() -> Item {
        if (li < leaves.size() && (mi >= merged.size() || leaves[li] < merged[mi])) return leaves[li++];
        return merged[mi++];
    };
    for (int64_t k = 0; k < n - 1; ++k) {
        const Item a = pop(), b = pop();
        parent[size_t(a.id)] = next_id;
        parent[size_t(b.id)] = next_id;
        merged.push_back(Item{a.count + b.count, next_id});
        ++next_id;
    }
    std::vector<int> depth(static_cast<size_t>(2 * n - 1), 0);
    for (int64_t node = 2 * n - 3; node >= 0; --node) depth[size_t(node)] = depth[size_t(parent[size_t(node)])] + 1;
    for (int64_t i = 0; i < n; ++i) depth_out[size_t(i)] = depth[size_t(i)];
}

// huffman_unlimited with the leaves sorted as packed 64-bit keys (count << 24 | id): the same
// (count, id) order, an order of magnitude cheaper to sort than Items; needs every count < 2^40 and
// n <= 2^24 (the caller checks).  Scratch buffers are reused across the length-limit rounds.
struct HuffScratch {
    std::vector<uint64_t> keys, mcount, tmp;
    std::vector<int32_t> parent, depth;
};

// Ascending sort of distinct keys (count << 24 | id) that arrive in id order: an LSD radix sort
// over the count bytes only, a byte per pass (the passes over the id bytes would keep the order the
// keys already have, and each later pass is stable); bytes that are the same in every key are
// skipped (the length-limit rounds shrink the counts, so fewer bytes vary).
void radix_sort_keys(std::vector<uint64_t>& a, std::vector<uint64_t>& tmp) {
    const size_t n = a.size();
    if (n < 256) {
        std::sort(a.begin(), a.end());
        return;
    }
    uint64_t diff = 0;
    for (const uint64_t x : a) diff |= x ^ a[0];
    tmp.resize(n);
    for (int sh = 24; sh < 64; sh += 8) {
        if (((diff >> sh) & 0xFFu) == 0) continue;
        size_t cnt[257] = {};
        for (const uint64_t x : a) ++cnt[((x >> sh) & 0xFFu) + 1];
        for (int i = 0; i < 256; ++i) cnt[i + 1] += cnt[i];
        for (const uint64_t x : a) tmp[cnt[(x >> sh) & 0xFFu]++] = x;
        a.swap(tmp);
    }
}

void huffman_unlimited_packed(const std::vector<uint64_t>& counts, std::vector<int>& depth_out, HuffScratch& w) {
    const int64_t n = int64_t(counts.size());
    depth_out.assign(size_t(n), 1);
    if (n == 1) return;
    w.keys.resize(size_t(n));
    for (int64_t i = 0; i < n; ++i) w.keys[size_t(i)] = (counts[size_t(i)] << 24) | uint64_t(i);   // in id order
    radix_sort_keys(w.keys, w.tmp);
    w.mcount.clear();
    w.mcount.reserve(size_t(n));
    w.parent.assign(size_t(2 * n - 1), 0);
    size_t li = 0, mi = 0;
    // a leaf and a merged node of equal count: the leaf first (leaf ids are below merged ids)
    auto pop = [&](uint64_t& c) -> int64_t {
        if (li < size_t(n) && (mi >= w.mcount.size() || (w.keys[li] >> 24) <= w.mcount[mi])) {
            c = w.keys[li] >> 24;
            return int64_t(w.keys[li++] & 0xFFFFFFu);
        }
        c = w.mcount[mi];
        return n + int64_t(mi++);
    };
    for (int64_t k = 0; k < n - 1; ++k) {
        uint64_t ca, cb;
        const int64_t a = pop(ca), b = pop(cb);
        const int64_t id = n + int64_t(w.mcount.size());
        w.parent[size_t(a)] = int32_t(id);
        w.parent[size_t(b)] = int32_t(id);
        w.mcount.push_back(ca + cb);
    }
    w.depth.assign(size_t(2 * n - 1), 0);
    for (int64_t node = 2 * n - 3; node >= 0; --node) w.depth[size_t(node)] = w.depth[size_t(w.parent[size_t(node)])] + 1;
    for (int64_t i = 0; i < n; ++i) depth_out[size_t(i)] = w.depth[size_t(i)];
}

}  // namespace

void huffman_lengths(const uint64_t* counts_in, int64_t n, uint8_t* lengths) {
    std::vector<uint64_t> c(counts_in, counts_in + n);
    std::vector<int> d;
    bool packed = n <= (int64_t(1) << 24);
    for (int64_t i = 0; i < n && packed; ++i) packed = counts_in[i] < (uint64_t(1) << 40);
    HuffScratch w;
    for (int round = 0; round < 8; ++round) {          // codec.py:71-78
        if (packed) huffman_unlimited_packed(c, d, w);
        else huffman_unlimited(c, d);
        if (*std::max_element(d.begin(), d.end()) <= kMaxCodeLen) {
            for (int64_t i = 0; i < n; ++i) lengths[i] = uint8_t(d[size_t(i)]);
            return;
        }
        for (auto& x : c) x = std::max<uint64_t>(1, x >> 2);
    }
    int bl = 0;
    for (uint64_t v = uint64_t(n - 1); v; v >>= 1) ++bl;
    bl = std::max(bl, 1);
    for (int64_t i = 0; i < n; ++i) lengths[i] = uint8_t(bl);
}

void canonical_codes(const uint8_t* lengths, int64_t n, uint32_t* codes) {
    uint32_t per[kMaxCodeLen + 1] = {};
    for (int64_t i = 0; i < n; ++i) per[lengths[i]]++;
    // first code of each length in canonical order; codes of one length follow table position
    uint32_t next[kMaxCodeLen + 1] = {};
    uint32_t code = 0;
    for (int L = 1; L <= kMaxCodeLen; ++L) {
        next[L] = code;
        code = (code + per[L]) << 1;
    }
    for (int64_t i = 0; i < n; ++i) codes[i] = next[lengths[i]]++;
}

void build_decode_table(const Table& t, DecodeTable* d, uint32_t* sorted_syms) {
    uint32_t per[kMaxCodeLen + 1] = {};
    for (uint8_t L : t.lengths) per[L]++;
    uint32_t code = 0, idx = 0;
    d->first[0] = d->count[0] = d->base[0] = d->limit[0] = 0;
    for (int L = 1; L <= kMaxCodeLen; ++L) {
        d->first[L] = code;
        d->count[L] = per[L];
        d->base[L] = idx;
        d->limit[L] = (code + per[L]) << (kMaxCodeLen - L);
        code = (code + per[L]) << 1;
        idx += per[L];
    }
    uint32_t fill[kMaxCodeLen + 1];
    for (int L = 1; L <= kMaxCodeLen; ++L) fill[L] = d->base[L];
    for (size_t k = 0; k < t.symbols.size(); ++k) sorted_syms[fill[t.lengths[k]]++] = t.symbols[k];
}

}  // namespace crx
