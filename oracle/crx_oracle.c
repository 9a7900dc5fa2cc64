/*
 * crx_oracle.c -- TEST INFRASTRUCTURE ONLY: a sequential CPU restatement of crukx-sync's
 * encode/apply path (wire format version 2).  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg may load this library, and only as a checker or as the timed
 * CPU baseline.  The product (crukx_sync_b200) never links or calls it.
 *
 * Each function cites the reference code it restates (paths relative to the crukx-sync
 * project):
 *   src/crukx_sync/codec.py   encode (:278-420), apply (:578-717), checksum (:53-68),
 *                             huffman_lengths (:71-98), canonical_codes (:101-111),
 *                             _rice_params (:268-275), _pack_bits (:218-257),
 *                             _canonical_tables (:434-454), block decode (:504-575)
 *   src/crukx_sync/wire.py    serialize (:64-89), varint (:55-61), _Reader/parse (:92-212)
 *   docs/FORMAT.md            grammar (:10-14), groups (:19-31), symbols/blocks (:33-44),
 *                             limits (:46-57), checksum (:59-68)
 *
 * The algorithm is written from the format description, element by element, with no
 * batching: the reference's slabs, batches and small-tensor sort sharing do not change the
 * bytes (codec.py:214, :303-342 only bound memory).  Stable sort by old exponent is realised
 * as one walk over the tensor with 256 running counters.
 *
 * Status codes: 0 ok, 1 ValueError, 2 CorruptUpdate, 3 internal (allocation) error.
 */
#define _GNU_SOURCE
#include <pthread.h>
#include <sched.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdlib.h>
#include <unistd.h>
#include <string.h>
#include <stdio.h>
#include <math.h>

#define ORC_OK 0
#define ORC_VALUE 1
#define ORC_CORRUPT 2
#define ORC_NOMEM 3

#define MAX_CODE_LEN 17
#define MAX_SYMBOL 131070
#define SYM_SPACE (MAX_SYMBOL + 1)
#define MAX_RICE 30
#define BLOCK 256

static void set_err(char *err, size_t n, const char *msg) {
    if (err && n) { snprintf(err, n, "%s", msg); }
}

/* Threads of the per-tensor and per-exponent passes (0 = every processor this process may run
 * on).  The passes split independent tensors or exponents only, so the bytes never depend on it. */
static int g_threads = 0;
void orc_set_threads(int n) { g_threads = n > 0 ? n : 0; }
static int orc_threads(void) {
    if (g_threads) return g_threads;
    cpu_set_t set;
    if (sched_getaffinity(0, sizeof(set), &set) == 0) return CPU_COUNT(&set) > 0 ? CPU_COUNT(&set) : 1;
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

/* fn(ctx, i) for i in [0, n) on up to orc_threads() threads, indices handed out one at a time */
typedef void (*orc_task_fn)(void *ctx, int64_t i);
typedef struct { orc_task_fn fn; void *ctx; int64_t n; atomic_llong next; } pfor_t;
static void *pfor_worker(void *arg) {
    pfor_t *p = arg;
    for (;;) {
        int64_t i = atomic_fetch_add(&p->next, 1);
        if (i >= p->n) break;
        p->fn(p->ctx, i);
    }
    return NULL;
}
static void parallel_for(int64_t n, orc_task_fn fn, void *ctx) {
    int nt = orc_threads();
    if (nt > 256) nt = 256;
    if (n < nt) nt = (int)n;
    pfor_t p = {fn, ctx, n, 0};
    atomic_init(&p.next, 0);
    pthread_t th[256];
    int started = 0;
    for (int k = 1; k < nt; k++)
        if (pthread_create(&th[started], NULL, pfor_worker, &p) == 0) started++;
    pfor_worker(&p);   /* this thread works too; with no extra thread it does everything */
    for (int k = 0; k < started; k++) pthread_join(th[k], NULL);
}

/* ------------------------------------------------------------------ checksum (FORMAT.md:59-68) */

static inline uint64_t splitmix_weight(uint64_t i) {
    /* codec.py:53-58: z = (i+1)*G, two xor-shift-multiply rounds, final xor-shift, | 1 */
    uint64_t z = (i + 1) * 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return (z ^ (z >> 31)) | 1ULL;
}

uint64_t orc_weight(uint64_t i) { return splitmix_weight(i); }

uint64_t orc_checksum(const int16_t *a, int64_t n) {
    /* codec.py:61-68: sum over i of uint16(a_i) * w_i, mod 2^64 */
    uint64_t s = 0;
    for (int64_t i = 0; i < n; i++) s += (uint64_t)(uint16_t)a[i] * splitmix_weight((uint64_t)i);
    return s;
}

/* ------------------------------------------------------------------ Huffman (codec.py:71-111) */

typedef struct { uint64_t c; int64_t id; } node_t;

static int cmp_node(const void *x, const void *y) {
    const node_t *a = x, *b = y;
    if (a->c != b->c) return a->c < b->c ? -1 : 1;
    return a->id < b->id ? -1 : (a->id > b->id);
}

/* Unlimited Huffman lengths with the tie order of a min-heap on (count, id): leaves have
 * ids 0..n-1, merged nodes get n, n+1, ... in creation order (codec.py:81-98).  Merged
 * weights come out non-decreasing, so a sorted leaf queue plus a FIFO of merged nodes pops
 * exactly the same sequence as the heap. */
static int huff_unlimited(const uint64_t *counts, int64_t n, int32_t *len_out) {
    if (n == 1) { len_out[0] = 1; return 0; }
    node_t *leaves = malloc(sizeof(node_t) * n);
    node_t *merged = malloc(sizeof(node_t) * n);
    int64_t *parent = malloc(sizeof(int64_t) * (2 * n - 1));
    int32_t *depth = malloc(sizeof(int32_t) * (2 * n - 1));
    if (!leaves || !merged || !parent || !depth) { free(leaves); free(merged); free(parent); free(depth); return -1; }
    for (int64_t i = 0; i < n; i++) { leaves[i].c = counts[i]; leaves[i].id = i; }
    qsort(leaves, n, sizeof(node_t), cmp_node);
    int64_t li = 0, mi = 0, mn = 0, nxt = n;
    for (int64_t k = 0; k < n - 1; k++) {
        node_t pick[2];
        for (int t = 0; t < 2; t++) {
            int take_leaf;
            if (li >= n) take_leaf = 0;
            else if (mi >= mn) take_leaf = 1;
            else take_leaf = cmp_node(&leaves[li], &merged[mi]) < 0;
            pick[t] = take_leaf ? leaves[li++] : merged[mi++];
        }
        parent[pick[0].id] = nxt;
        parent[pick[1].id] = nxt;
        merged[mn].c = pick[0].c + pick[1].c;
        merged[mn].id = nxt;
        mn++; nxt++;
    }
    depth[2 * n - 2] = 0;
    for (int64_t node = 2 * n - 3; node >= 0; node--) depth[node] = depth[parent[node]] + 1;
    for (int64_t i = 0; i < n; i++) len_out[i] = depth[i];
    free(leaves); free(merged); free(parent); free(depth);
    return 0;
}

/* codec.py:71-78: up to 8 rounds of counts = max(1, c >> 2) while any length exceeds 17,
 * then equal lengths bit_length(n - 1) (at least 1). */
int orc_huffman_lengths(const uint64_t *counts_in, int64_t n, int32_t *lengths) {
    uint64_t *c = malloc(sizeof(uint64_t) * n);
    if (!c) return -1;
    memcpy(c, counts_in, sizeof(uint64_t) * n);
    for (int round = 0; round < 8; round++) {
        if (huff_unlimited(c, n, lengths)) { free(c); return -1; }
        int32_t mx = 0;
        for (int64_t i = 0; i < n; i++) if (lengths[i] > mx) mx = lengths[i];
        if (mx <= MAX_CODE_LEN) { free(c); return 0; }
        for (int64_t i = 0; i < n; i++) { uint64_t v = c[i] >> 2; c[i] = v ? v : 1; }
    }
    int32_t bl = 0;
    for (uint64_t v = (uint64_t)(n - 1); v; v >>= 1) bl++;
    if (bl < 1) bl = 1;
    for (int64_t i = 0; i < n; i++) lengths[i] = bl;
    free(c);
    return 0;
}

/* codec.py:101-111: canonical codes in order of (length, position). */
static void canonical_codes(const int32_t *len, int64_t n, uint32_t *codes) {
    /* counting order by length, positions ascending within a length */
    int64_t per[MAX_CODE_LEN + 2] = {0};
    for (int64_t i = 0; i < n; i++) per[len[i]]++;
    uint32_t next[MAX_CODE_LEN + 2] = {0};
    uint32_t code = 0;
    int first = 1; int prev = 0;
    for (int L = 1; L <= MAX_CODE_LEN; L++) {
        if (!per[L]) continue;
        if (first) { code = 0; first = 0; }
        else code = (code + 1) << (L - prev);
        next[L] = code;
        code += (uint32_t)per[L] - 1;
        prev = L;
    }
    for (int64_t i = 0; i < n; i++) codes[i] = next[len[i]]++;
}

/* ------------------------------------------------------------------ byte/bit writers */

typedef struct { uint8_t *p; size_t n, cap; int fail; } buf_t;

static void buf_reserve(buf_t *b, size_t extra) {
    if (b->fail) return;
    if (b->n + extra <= b->cap) return;
    size_t cap = b->cap ? b->cap : 256;
    while (cap < b->n + extra) cap *= 2;
    uint8_t *np = realloc(b->p, cap);
    if (!np) { b->fail = 1; return; }
    b->p = np; b->cap = cap;
}
static void buf_put(buf_t *b, const void *src, size_t n) {
    buf_reserve(b, n); if (b->fail) return;
    memcpy(b->p + b->n, src, n); b->n += n;
}
static void buf_u8(buf_t *b, uint8_t v) { buf_put(b, &v, 1); }
static void buf_varint(buf_t *b, uint64_t v) {  /* wire.py:55-61 (v < 2^63 by construction) */
    while (v >= 0x80) { buf_u8(b, (uint8_t)((v & 0x7F) | 0x80)); v >>= 7; }
    buf_u8(b, (uint8_t)v);
}
static void buf_le(buf_t *b, uint64_t v, int nbytes) {
    for (int k = 0; k < nbytes; k++) buf_u8(b, (uint8_t)(v >> (8 * k)));
}

typedef struct { uint8_t *p; uint64_t nbits, capbytes; int fail; } bits_t;

static void bits_reserve(bits_t *w, uint64_t extra_bits) {
    if (w->fail) return;
    uint64_t need = (w->nbits + extra_bits + 7) / 8 + 8;
    if (need <= w->capbytes) return;
    uint64_t cap = w->capbytes ? w->capbytes : 1024;
    while (cap < need) cap *= 2;
    uint8_t *np = realloc(w->p, cap);
    if (!np) { w->fail = 1; return; }
    memset(np + w->capbytes, 0, cap - w->capbytes);
    w->p = np; w->capbytes = cap;
}
/* MSB-first: the first written bit is bit 7 of byte 0 (FORMAT.md:39-44). */
static void bits_put(bits_t *w, uint64_t v, int n) {
    bits_reserve(w, (uint64_t)n); if (w->fail) return;
    for (int k = n - 1; k >= 0; k--) {
        if ((v >> k) & 1) w->p[w->nbits >> 3] |= (uint8_t)(0x80 >> (w->nbits & 7));
        w->nbits++;
    }
}
static void bits_ones(bits_t *w, uint64_t q) {
    bits_reserve(w, q); if (w->fail) return;
    while (q && (w->nbits & 7)) { w->p[w->nbits >> 3] |= (uint8_t)(0x80 >> (w->nbits & 7)); w->nbits++; q--; }
    uint64_t whole = q / 8;
    memset(w->p + (w->nbits >> 3), 0xFF, whole);
    w->nbits += whole * 8; q -= whole * 8;
    while (q) { w->p[w->nbits >> 3] |= (uint8_t)(0x80 >> (w->nbits & 7)); w->nbits++; q--; }
}

/* ------------------------------------------------------------------ encoder (codec.py:278-420) */

typedef struct {
    int exp; int64_t count; int rice;
    int64_t *local;   /* rank among same-exponent elements, index order */
    int16_t *va, *vb; /* old / new bits */
    int64_t cap;
} group_t;

typedef struct { group_t g[256]; int present; int64_t numel; } tstate_t;

static int group_push(group_t *g, int64_t local, int16_t va, int16_t vb) {
    if (g->count == g->cap) {
        int64_t cap = g->cap ? g->cap * 2 : 64;
        int64_t *l = realloc(g->local, sizeof(int64_t) * cap);
        if (!l) return -1;
        g->local = l;
        int16_t *a = realloc(g->va, sizeof(int16_t) * cap);
        if (!a) return -1;
        g->va = a;
        int16_t *b = realloc(g->vb, sizeof(int16_t) * cap);
        if (!b) return -1;
        g->vb = b;
        g->cap = cap;
    }
    g->local[g->count] = local; g->va[g->count] = va; g->vb[g->count] = vb; g->count++;
    return 0;
}

static inline uint32_t zigzag_res(int16_t va, int16_t vb) {
    int64_t res = (int64_t)vb - (int64_t)va;   /* signed int16 values, no wrap (FORMAT.md:27-29) */
    return (uint32_t)((res << 1) ^ (res >> 63));
}

static inline int64_t gap_at(const group_t *g, int64_t j) {
    return j ? g->local[j] - g->local[j - 1] - 1 : g->local[0];
}

/* codec.py:268-275: three candidates around floor(log2(mean gap)), first cheapest wins. */
static int rice_param(const group_t *g) {
    int64_t sum = 0;
    for (int64_t j = 0; j < g->count; j++) sum += gap_at(g, j);
    double mean = (double)sum / (double)g->count;
    if (mean < 1.0) mean = 1.0;
    int64_t r0 = (int64_t)floor(log2(mean));
    if (r0 < 0) r0 = 0;
    if (r0 > MAX_RICE) r0 = MAX_RICE;
    int64_t cand[3] = { r0 - 1 < 0 ? 0 : r0 - 1, r0, r0 + 1 > MAX_RICE ? MAX_RICE : r0 + 1 };
    int64_t best = -1; int bi = 0;
    for (int k = 0; k < 3; k++) {
        int64_t cost = 0, c = cand[k];
        for (int64_t j = 0; j < g->count; j++) cost += (gap_at(g, j) >> c) + 1 + c;
        if (best < 0 || cost < best) { best = cost; bi = k; }
    }
    return (int)cand[bi];
}

typedef struct { uint64_t *count; uint32_t *code; int32_t *len; int64_t nsym; int32_t *syms; } etab_t;

static void free_tstate(tstate_t *ts, int n) {
    if (!ts) return;
    for (int t = 0; t < n; t++)
        for (int e = 0; e < 256; e++) { free(ts[t].g[e].local); free(ts[t].g[e].va); free(ts[t].g[e].vb); }
    free(ts);
}

typedef struct {
    tstate_t *ts;
    etab_t *tabs;
    const int16_t *const *prev, *const *cur;
    const int64_t *numel;
    const uint64_t *cache_chk;
    const uint8_t *has_cache;
    uint64_t *new_chk;
    uint8_t *chk_present;
    int n;
    bits_t *tbits;
    const int64_t *tblock;
    uint32_t *block_bits;
    atomic_int fail, too_long;
} enc_ctx_t;

/* pass 1 for tensor t: its changes per old exponent, the new checksum, the Rice parameters */
static void enc_pass1(void *vc, int64_t t) {
    enc_ctx_t *c = vc;
    tstate_t *ts = &c->ts[t];
    c->chk_present[t] = 0;
    ts->numel = c->numel[t];
    int64_t counter[256] = {0};
    const int16_t *a = c->prev[t], *b = c->cur[t];
    for (int64_t i = 0; i < c->numel[t]; i++) {
        int e = ((uint16_t)a[i] >> 7) & 0xFF;
        if (a[i] != b[i]) {
            if (group_push(&ts->g[e], counter[e], a[i], b[i])) { atomic_store(&c->fail, 1); return; }
            ts->present = 1;
        }
        counter[e]++;
    }
    if (!ts->present) return;
    /* checksum of the new tensor: cached + delta, else a full pass (codec.py:344-352) */
    uint64_t chk;
    if (c->has_cache && c->has_cache[t]) {
        uint64_t d = 0;
        for (int64_t i = 0; i < c->numel[t]; i++)
            if (a[i] != b[i])
                d += ((uint64_t)(uint16_t)b[i] - (uint64_t)(uint16_t)a[i]) * splitmix_weight((uint64_t)i);
        chk = c->cache_chk[t] + d;
    } else {
        chk = orc_checksum(b, c->numel[t]);
    }
    c->new_chk[t] = chk;
    c->chk_present[t] = 1;
    for (int e = 0; e < 256; e++) {
        group_t *g = &ts->g[e];
        g->exp = e;
        if (g->count) g->rice = rice_param(g);
    }
}

/* pass 2 for exponent e: its symbol counts over every tensor of the update */
static void enc_pass2(void *vc, int64_t e) {
    enc_ctx_t *c = vc;
    for (int t = 0; t < c->n; t++) {
        if (!c->ts[t].present) continue;
        const group_t *g = &c->ts[t].g[e];
        if (!g->count) continue;
        if (!c->tabs[e].count) {
            c->tabs[e].count = calloc(SYM_SPACE, sizeof(uint64_t));
            if (!c->tabs[e].count) { atomic_store(&c->fail, 1); return; }
        }
        for (int64_t j = 0; j < g->count; j++) c->tabs[e].count[zigzag_res(g->va[j], g->vb[j])]++;
    }
}

/* pass 3 for tensor t: its bits from bit 0 of its own buffer, its blocks' bit counts */
static void enc_pass3(void *vc, int64_t t) {
    enc_ctx_t *c = vc;
    bits_t *tw = &c->tbits[t];
    int64_t bi = c->tblock[t];
    for (int e = 0; e < 256; e++) {
        const group_t *g = &c->ts[t].g[e];
        if (!g->count) continue;
        const etab_t *tb = &c->tabs[e];
        for (int64_t k0 = 0; k0 < g->count; k0 += BLOCK) {
            uint64_t start = tw->nbits;
            int64_t k1 = k0 + BLOCK < g->count ? k0 + BLOCK : g->count;
            for (int64_t j = k0; j < k1; j++) {
                uint64_t gap = (uint64_t)gap_at(g, j);
                uint64_t q = gap >> g->rice;
                bits_ones(tw, q);
                bits_put(tw, 0, 1);
                if (g->rice) bits_put(tw, gap & ((1ULL << g->rice) - 1), g->rice);
                uint32_t z = zigzag_res(g->va[j], g->vb[j]);
                bits_put(tw, tb->code[z], tb->len[z]);
            }
            uint64_t nb = tw->nbits - start;
            if (nb >= (1ULL << 32)) atomic_store(&c->too_long, 1);
            c->block_bits[bi++] = (uint32_t)nb;
        }
    }
}

/*
 * Encode n tensors (old = prev[t], new = cur[t], numel[t] elements, names[t] of name_len[t]
 * bytes).  cache_chk/has_cache: the sender's cached checksum of prev[t] (codec.py:345-352).
 * On success *out (malloc'd) holds the serialized update; new_chk[t] and chk_present[t]
 * report the checksums the caller commits (only tensors present in the update).
 */
int orc_encode(int n, const int16_t *const *prev, const int16_t *const *cur, const int64_t *numel,
               const char *const *names, const int64_t *name_len,
               const uint64_t *cache_chk, const uint8_t *has_cache,
               uint8_t **out, size_t *out_len, uint64_t *new_chk, uint8_t *chk_present,
               char *err, size_t errlen) {
    *out = NULL; *out_len = 0;
    tstate_t *ts = calloc(n > 0 ? n : 1, sizeof(tstate_t));
    etab_t *tabs = calloc(256, sizeof(etab_t));
    int status = ORC_NOMEM;
    buf_t b = {0};
    bits_t w = {0};
    bits_t *tbits = NULL;
    uint32_t *block_bits = NULL;
    if (!ts || !tabs) goto done;

    /* pass 1: changed elements per (tensor, old exponent) in index order = stable rank order.
     * Tensors are independent until the Huffman tables: one task per tensor. */
    enc_ctx_t ec = {ts, tabs, prev, cur, numel, cache_chk, has_cache, new_chk, chk_present, n, NULL, NULL, NULL, 0, 0};
    parallel_for(n, enc_pass1, &ec);
    if (ec.fail) goto done;

    /* pass 2: one Huffman table per exponent over the whole update (codec.py:355-392); the
     * exponents are independent: one task per exponent */
    parallel_for(256, enc_pass2, &ec);
    if (ec.fail) goto done;
    for (int e = 0; e < 256; e++) {
        etab_t *tb = &tabs[e];
        if (!tb->count) continue;
        int64_t ns = 0;
        for (int64_t s = 0; s < SYM_SPACE; s++) ns += tb->count[s] != 0;
        tb->nsym = ns;
        tb->syms = malloc(sizeof(int32_t) * ns);
        uint64_t *cnt = malloc(sizeof(uint64_t) * ns);
        tb->len = calloc(SYM_SPACE, sizeof(int32_t));
        tb->code = calloc(SYM_SPACE, sizeof(uint32_t));
        int32_t *ln = malloc(sizeof(int32_t) * ns);
        uint32_t *cd = malloc(sizeof(uint32_t) * ns);
        if (!tb->syms || !cnt || !tb->len || !tb->code || !ln || !cd) { free(cnt); free(ln); free(cd); goto done; }
        int64_t k = 0;
        for (int64_t s = 0; s < SYM_SPACE; s++) if (tb->count[s]) { tb->syms[k] = (int32_t)s; cnt[k] = tb->count[s]; k++; }
        if (orc_huffman_lengths(cnt, ns, ln)) { free(cnt); free(ln); free(cd); goto done; }
        canonical_codes(ln, ns, cd);
        for (k = 0; k < ns; k++) { tb->len[tb->syms[k]] = ln[k]; tb->code[tb->syms[k]] = cd[k]; }
        free(cnt); free(ln); free(cd);
    }

    /* pass 3: bits, in (tensor, group, element) order; block sizes per 256-run of a group.  Each
     * tensor's bits are written by one task into its own buffer from bit 0; the buffers are then
     * joined in tensor order at their running bit offsets (the reference's carry, codec.py:405-410). */
    int64_t n_blocks = 0;
    int64_t *tblock = calloc((size_t)n + 1, sizeof(int64_t));   /* first block of each tensor */
    tbits = calloc(n > 0 ? (size_t)n : 1, sizeof(bits_t));
    if (!tblock || !tbits) { free(tblock); goto done; }
    for (int t = 0; t < n; t++) {
        tblock[t] = n_blocks;
        for (int e = 0; e < 256; e++) n_blocks += (ts[t].g[e].count + BLOCK - 1) / BLOCK;
    }
    tblock[n] = n_blocks;
    block_bits = malloc(sizeof(uint32_t) * (n_blocks ? n_blocks : 1));
    if (!block_bits) { free(tblock); goto done; }
    ec.tbits = tbits;
    ec.tblock = tblock;
    ec.block_bits = block_bits;
    parallel_for(n, enc_pass3, &ec);
    const int too_long = ec.too_long;
    free(tblock);
    for (int t = 0; t < n; t++) if (tbits[t].fail) goto done;
    if (too_long) {
        status = ORC_VALUE;
        set_err(err, errlen, "a block exceeds 2^32 bits; the update cannot be represented");
        goto done;
    }
    {   /* join: tensor t's bits start at bit w.nbits of the whole payload */
        uint64_t total = 0;
        for (int t = 0; t < n; t++) total += tbits[t].nbits;
        bits_reserve(&w, total);
        if (w.fail) goto done;
        for (int t = 0; t < n; t++) {
            const bits_t *tw = &tbits[t];
            uint64_t nbytes = (tw->nbits + 7) / 8;
            uint64_t at = w.nbits >> 3;
            int sh = (int)(w.nbits & 7);
            if (sh == 0) {
                if (nbytes) memcpy(w.p + at, tw->p, nbytes);
            } else {
                for (uint64_t k = 0; k < nbytes; k++) {
                    w.p[at + k] |= (uint8_t)(tw->p[k] >> sh);
                    w.p[at + k + 1] |= (uint8_t)(tw->p[k] << (8 - sh));
                }
            }
            w.nbits += tw->nbits;
        }
    }

    /* serialize (wire.py:64-89) */
    buf_put(&b, "CRXS", 4);
    buf_u8(&b, 2);
    int64_t nt = 0;
    for (int e = 0; e < 256; e++) nt += tabs[e].nsym > 0;
    buf_varint(&b, (uint64_t)nt);
    for (int e = 0; e < 256; e++) {
        etab_t *tb = &tabs[e];
        if (!tb->nsym) continue;
        buf_u8(&b, (uint8_t)e);
        buf_varint(&b, (uint64_t)tb->nsym);
        for (int64_t k = 0; k < tb->nsym; k++) { buf_varint(&b, (uint64_t)tb->syms[k]); buf_u8(&b, (uint8_t)tb->len[tb->syms[k]]); }
    }
    int64_t ntens = 0;
    for (int t = 0; t < n; t++) ntens += ts[t].present;
    buf_varint(&b, (uint64_t)ntens);
    for (int t = 0; t < n; t++) {
        if (!ts[t].present) continue;
        buf_varint(&b, (uint64_t)name_len[t]);
        buf_put(&b, names[t], (size_t)name_len[t]);
        buf_varint(&b, (uint64_t)numel[t]);
        buf_le(&b, new_chk[t], 8);
        int ng = 0;
        for (int e = 0; e < 256; e++) ng += ts[t].g[e].count > 0;
        buf_varint(&b, (uint64_t)ng);
        for (int e = 0; e < 256; e++) {
            group_t *g = &ts[t].g[e];
            if (!g->count) continue;
            buf_u8(&b, (uint8_t)e);
            buf_varint(&b, (uint64_t)g->count);
            buf_u8(&b, (uint8_t)g->rice);
        }
    }
    for (int64_t k = 0; k < n_blocks; k++) buf_le(&b, block_bits[k], 4);
    uint64_t plen = (w.nbits + 7) / 8;
    buf_varint(&b, plen);
    if (plen) buf_put(&b, w.p, plen);
    if (b.fail) goto done;
    *out = b.p; *out_len = b.n; b.p = NULL;
    status = ORC_OK;
done:
    if (status == ORC_NOMEM) set_err(err, errlen, "oracle: out of memory");
    free(b.p); free(w.p); free(block_bits);
    if (tbits) { for (int t = 0; t < n; t++) free(tbits[t].p); free(tbits); }
    free_tstate(ts, n);
    if (tabs) for (int e = 0; e < 256; e++) { free(tabs[e].count); free(tabs[e].code); free(tabs[e].len); free(tabs[e].syms); }
    free(tabs);
    return status;
}

void orc_free(void *p) { free(p); }

/* ------------------------------------------------------------------ parser (wire.py:92-212) */

typedef struct { int exp; int64_t nsym; int64_t *syms; int32_t *lens; } ptable_t;
typedef struct { int exp; int64_t count; int rice; } pgroup_t;
typedef struct { const uint8_t *name; int64_t name_len; int64_t numel; uint64_t chk; int ng; pgroup_t g[256]; } ptensor_t;

typedef struct {
    int n_tables; ptable_t tab[256];
    int64_t n_tensors; ptensor_t *tens;
    int64_t n_blocks; uint32_t *block_bits;
    const uint8_t *payload; int64_t payload_len;
} pupdate_t;

typedef struct { const uint8_t *d; int64_t n, pos; } rd_t;

static int rd_take(rd_t *r, int64_t k, const uint8_t **p) {
    if (k < 0 || r->pos + k > r->n) return -1;
    *p = r->d + r->pos; r->pos += k; return 0;
}
static int rd_u8(rd_t *r, int *v) { const uint8_t *p; if (rd_take(r, 1, &p)) return -1; *v = p[0]; return 0; }
static int rd_varint(rd_t *r, int64_t *out) {
    /* wire.py:109-120: LEB128, any value >= 2^63 or more than 10 bytes is corrupt */
    unsigned __int128 v = 0; int shift = 0;
    for (;;) {
        int b; if (rd_u8(r, &b)) return -1;
        v |= (unsigned __int128)(b & 0x7F) << shift;
        if (v >= ((unsigned __int128)1 << 63)) return -1;
        if (!(b & 0x80)) { *out = (int64_t)v; return 0; }
        shift += 7;
        if (shift > 63) return -1;
    }
}

/* Python's strict UTF-8 decoder: no overlongs, no surrogates, nothing above U+10FFFF. */
static int utf8_ok(const uint8_t *s, int64_t n) {
    int64_t i = 0;
    while (i < n) {
        uint8_t c = s[i];
        if (c < 0x80) { i++; continue; }
        int need; uint32_t cp;
        if (c >= 0xC2 && c <= 0xDF) { need = 1; cp = c & 0x1F; }
        else if (c >= 0xE0 && c <= 0xEF) { need = 2; cp = c & 0x0F; }
        else if (c >= 0xF0 && c <= 0xF4) { need = 3; cp = c & 0x07; }
        else return 0;
        if (i + need >= n) return 0;
        for (int k = 1; k <= need; k++) {
            uint8_t cc = s[i + k];
            if ((cc & 0xC0) != 0x80) return 0;
            cp = (cp << 6) | (cc & 0x3F);
        }
        if (need == 2 && (cp < 0x800 || (cp >= 0xD800 && cp <= 0xDFFF))) return 0;
        if (need == 3 && (cp < 0x10000 || cp > 0x10FFFF)) return 0;
        i += need + 1;
    }
    return 1;
}

static void free_update(pupdate_t *u) {
    if (!u) return;
    for (int t = 0; t < u->n_tables; t++) { free(u->tab[t].syms); free(u->tab[t].lens); }
    free(u->tens); free(u->block_bits); free(u);
}

static int parse_update(const uint8_t *data, int64_t len, pupdate_t **out, char *err, size_t errlen) {
#define BAD(msg) do { set_err(err, errlen, msg); free_update(u); return ORC_CORRUPT; } while (0)
    pupdate_t *u = calloc(1, sizeof(pupdate_t));
    if (!u) return ORC_NOMEM;
    rd_t r = { data, len, 0 };
    const uint8_t *p; int v; int64_t x;
    if (rd_take(&r, 4, &p)) BAD("update is truncated");
    if (memcmp(p, "CRXS", 4)) BAD("not a crukx-sync update");
    if (rd_u8(&r, &v)) BAD("update is truncated");
    if (v != 2) BAD("unsupported format version");
    if (rd_varint(&r, &x)) BAD("bad varint");
    if (x > 256) BAD("too many tables");
    int seen[256] = {0};
    for (int64_t t = 0; t < x; t++) {
        int e; int64_t ns;
        if (rd_u8(&r, &e) || rd_varint(&r, &ns)) BAD("update is truncated");
        int64_t lim = (r.n - r.pos) / 2;
        if (lim > MAX_SYMBOL + 1) lim = MAX_SYMBOL + 1;
        if (seen[e] || !(ns > 0 && ns <= lim)) BAD("bad table header");
        seen[e] = 1;
        ptable_t *tb = &u->tab[u->n_tables++];
        tb->exp = e; tb->nsym = ns;
        tb->syms = malloc(sizeof(int64_t) * ns); tb->lens = malloc(sizeof(int32_t) * ns);
        if (!tb->syms || !tb->lens) { free_update(u); return ORC_NOMEM; }
        for (int64_t k = 0; k < ns; k++) {
            int L;
            if (rd_varint(&r, &tb->syms[k]) || rd_u8(&r, &L)) BAD("update is truncated");
            tb->lens[k] = L;
        }
        /* symbols unique and <= MAX_SYMBOL */
        int64_t mx = 0;
        for (int64_t k = 0; k < ns; k++) if (tb->syms[k] > mx) mx = tb->syms[k];
        uint8_t *mark = NULL;
        int dup = 0;
        if (mx <= MAX_SYMBOL) {
            mark = calloc(MAX_SYMBOL + 1, 1);
            if (!mark) { free_update(u); return ORC_NOMEM; }
            for (int64_t k = 0; k < ns; k++) { if (mark[tb->syms[k]]) dup = 1; mark[tb->syms[k]] = 1; }
            free(mark);
        } else {
            /* uniqueness is checked first in wire.py, but either failure is the same error */
            dup = 1;
        }
        if (dup || mx > MAX_SYMBOL) BAD("bad table symbols");
        int32_t mn = 99, mxl = 0; uint64_t kraft = 0;
        for (int64_t k = 0; k < ns; k++) { if (tb->lens[k] < mn) mn = tb->lens[k]; if (tb->lens[k] > mxl) mxl = tb->lens[k]; }
        if (mn < 1 || mxl > MAX_CODE_LEN) BAD("bad Huffman code lengths");
        /* the float Kraft sum of wire.py:149 is exact here: every term is a multiple of 2^-17 */
        for (int64_t k = 0; k < ns; k++) kraft += 1ULL << (MAX_CODE_LEN - tb->lens[k]);
        if (kraft > (1ULL << MAX_CODE_LEN)) BAD("bad Huffman code lengths");
    }
    int64_t nt;
    if (rd_varint(&r, &nt)) BAD("update is truncated");
    if (nt > r.n - r.pos) BAD("too many tensors");
    u->n_tensors = nt;
    u->tens = calloc(nt ? nt : 1, sizeof(ptensor_t));
    if (!u->tens) { free_update(u); return ORC_NOMEM; }
    unsigned __int128 total_blocks = 0;
    for (int64_t t = 0; t < nt; t++) {
        ptensor_t *h = &u->tens[t];
        int64_t nl;
        if (rd_varint(&r, &nl) || rd_take(&r, nl, &p)) BAD("update is truncated");
        if (!utf8_ok(p, nl)) BAD("tensor name is not valid UTF-8");
        for (int64_t s = 0; s < t; s++)
            if (u->tens[s].name_len == nl && !memcmp(u->tens[s].name, p, (size_t)nl)) BAD("tensor appears twice");
        h->name = p; h->name_len = nl;
        if (rd_varint(&r, &h->numel)) BAD("update is truncated");
        if (rd_take(&r, 8, &p)) BAD("update is truncated");
        h->chk = 0;
        for (int k = 7; k >= 0; k--) h->chk = (h->chk << 8) | p[k];
        int64_t ng;
        if (rd_varint(&r, &ng)) BAD("update is truncated");
        if (!(ng > 0 && ng <= 256)) BAD("bad group count");
        int exps[256] = {0};
        unsigned __int128 sum = 0;
        for (int64_t k = 0; k < ng; k++) {
            int e, rr; int64_t c;
            if (rd_u8(&r, &e) || rd_varint(&r, &c) || rd_u8(&r, &rr)) BAD("update is truncated");
            if (exps[e] || !seen[e]) BAD("bad group exponent");
            if (!(c > 0 && c <= h->numel) || rr > MAX_RICE) BAD("bad group header");
            exps[e] = 1;
            h->g[k].exp = e; h->g[k].count = c; h->g[k].rice = rr;
            total_blocks += (unsigned __int128)((c + BLOCK - 1) / BLOCK);
            sum += (unsigned __int128)c;   /* exact, like the Python sum */
        }
        h->ng = (int)ng;
        if (sum > (unsigned __int128)h->numel) BAD("more changes than elements");
    }
    /* every table used, and no larger than its changes (wire.py:184-191) */
    {
        unsigned __int128 per[256] = {0};
        for (int64_t t = 0; t < nt; t++) for (int k = 0; k < u->tens[t].ng; k++) per[u->tens[t].g[k].exp] += (unsigned __int128)u->tens[t].g[k].count;
        for (int t = 0; t < u->n_tables; t++) if ((unsigned __int128)u->tab[t].nsym > per[u->tab[t].exp]) BAD("table unused or larger than its changes");
    }
    if (4 * total_blocks > (unsigned __int128)(r.n - r.pos)) BAD("block table longer than the update");
    if (rd_take(&r, 4 * (int64_t)total_blocks, &p)) BAD("update is truncated");
    u->n_blocks = (int64_t)total_blocks;
    u->block_bits = malloc(sizeof(uint32_t) * (u->n_blocks ? u->n_blocks : 1));
    if (!u->block_bits) { free_update(u); return ORC_NOMEM; }
    uint64_t total_bits = 0;
    for (int64_t k = 0; k < u->n_blocks; k++) {
        u->block_bits[k] = (uint32_t)p[4 * k] | ((uint32_t)p[4 * k + 1] << 8) | ((uint32_t)p[4 * k + 2] << 16) | ((uint32_t)p[4 * k + 3] << 24);
        total_bits += u->block_bits[k];
    }
    int64_t pl;
    if (rd_varint(&r, &pl) || rd_take(&r, pl, &p)) BAD("update is truncated");
    u->payload = p; u->payload_len = pl;
    if (r.pos != r.n) BAD("trailing bytes after the payload");
    if ((total_bits + 7) / 8 != (uint64_t)pl) BAD("payload length does not match its block table");
    if ((total_bits % 8) && (p[pl - 1] & ((1u << (8 - total_bits % 8)) - 1))) BAD("non-zero padding bits");
    int64_t b = 0;
    for (int64_t t = 0; t < nt; t++)
        for (int k = 0; k < u->tens[t].ng; k++) {
            pgroup_t *g = &u->tens[t].g[k];
            for (int64_t j = 0; j * BLOCK < g->count; j++) {
                int64_t m = g->count - j * BLOCK; if (m > BLOCK) m = BLOCK;
                if ((uint64_t)u->block_bits[b] < (uint64_t)m * (uint64_t)(2 + g->rice)) BAD("block shorter than its symbols could be");
                b++;
            }
        }
    *out = u;
    return ORC_OK;
#undef BAD
}

/* Parse only: returns status; on success fills per-tensor name offsets so the caller can run
 * the receiver checks (names, numel) before apply, as codec.apply does first (codec.py:582-592). */
typedef struct { pupdate_t *u; } orc_update_t;

int orc_parse(const uint8_t *data, int64_t len, void **handle, char *err, size_t errlen) {
    pupdate_t *u = NULL;
    int st = parse_update(data, len, &u, err, errlen);
    *handle = u;
    return st;
}
int64_t orc_update_n_tensors(void *h) { return ((pupdate_t *)h)->n_tensors; }
void orc_update_tensor(void *h, int64_t t, const uint8_t **name, int64_t *name_len, int64_t *numel, uint64_t *chk, int *n_groups) {
    ptensor_t *x = &((pupdate_t *)h)->tens[t];
    *name = x->name; *name_len = x->name_len; *numel = x->numel; *chk = x->chk; *n_groups = x->ng;
}
void orc_update_group(void *h, int64_t t, int k, int *exp, int64_t *count, int *rice) {
    pgroup_t *g = &((pupdate_t *)h)->tens[t].g[k];
    *exp = g->exp; *count = g->count; *rice = g->rice;
}
void orc_update_free(void *h) { free_update((pupdate_t *)h); }

/* ------------------------------------------------------------------ decoder + apply (codec.py:578-717) */

typedef struct {
    uint64_t first[MAX_CODE_LEN + 1], cnt[MAX_CODE_LEN + 1], base[MAX_CODE_LEN + 1];
    int64_t *sorted;   /* symbols in (length, table position) order */
    int64_t nsym;
} dtab_t;

static int build_dtab(const ptable_t *tb, dtab_t *d) {   /* codec.py:434-454 */
    memset(d, 0, sizeof(*d));
    d->nsym = tb->nsym;
    d->sorted = malloc(sizeof(int64_t) * tb->nsym);
    if (!d->sorted) return -1;
    int64_t per[MAX_CODE_LEN + 1] = {0};
    for (int64_t k = 0; k < tb->nsym; k++) per[tb->lens[k]]++;
    uint64_t code = 0; int64_t idx = 0;
    for (int L = 1; L <= MAX_CODE_LEN; L++) {
        d->first[L] = code; d->cnt[L] = (uint64_t)per[L]; d->base[L] = (uint64_t)idx;
        code = (code + (uint64_t)per[L]) << 1;
        idx += per[L];
    }
    int64_t fill[MAX_CODE_LEN + 1];
    for (int L = 1; L <= MAX_CODE_LEN; L++) fill[L] = (int64_t)d->base[L];
    for (int64_t k = 0; k < tb->nsym; k++) d->sorted[fill[tb->lens[k]]++] = tb->syms[k];
    return 0;
}

static inline int bit_at(const uint8_t *p, int64_t nbytes, uint64_t pos) {
    uint64_t byte = pos >> 3;
    if (byte >= (uint64_t)nbytes) return 0;   /* zero padding past the payload (codec.py:478-482) */
    return (p[byte] >> (7 - (pos & 7))) & 1;
}
static inline uint64_t read_bits(const uint8_t *p, int64_t nbytes, uint64_t pos, int n) {
    uint64_t v = 0;
    for (int k = 0; k < n; k++) v = (v << 1) | (uint64_t)bit_at(p, nbytes, pos + k);
    return v;
}

typedef struct {
    pupdate_t *u;
    int16_t *const *weights;
    const uint64_t *old_chk;
    const uint8_t *has_chk;
    const dtab_t *dt;
    const int *tab_of;
    const int64_t *tb0;
    const uint64_t *tbit0;
    int64_t **pos;
    int16_t **val;
    int *tbad;
    int64_t *tchanged;
    atomic_int nomem;
} app_ctx_t;

/* decode, place and verify tensor t (nothing is written to the weights here) */
static void app_tensor(void *vc, int64_t t) {
    app_ctx_t *c = vc;
    pupdate_t *u = c->u;
    int bad = 0;
    uint64_t bitpos = c->tbit0[t];
    int64_t b = c->tb0[t];
    ptensor_t *h = &u->tens[t];
    const int16_t *a = c->weights[t];
    int64_t size[256] = {0};
    for (int64_t i = 0; i < h->numel; i++) size[((uint16_t)a[i] >> 7) & 0xFF]++;
    int64_t tot = 0;
    for (int k = 0; k < h->ng; k++) tot += h->g[k].count;
    c->pos[t] = malloc(sizeof(int64_t) * (tot ? tot : 1));
    c->val[t] = malloc(sizeof(int16_t) * (tot ? tot : 1));
    int64_t *local = malloc(sizeof(int64_t) * (tot ? tot : 1));
    uint32_t *zz = malloc(sizeof(uint32_t) * (tot ? tot : 1));
    int *gexp = malloc(sizeof(int) * (tot ? tot : 1));
    if (!c->pos[t] || !c->val[t] || !local || !zz || !gexp) {
        free(local); free(zz); free(gexp);
        atomic_store(&c->nomem, 1);
        return;
    }
    int64_t o = 0;
    for (int k = 0; k < h->ng && !bad; k++) {
        pgroup_t *g = &h->g[k];
        const dtab_t *d = &c->dt[c->tab_of[g->exp]];
        int64_t gsize = size[g->exp];
        uint64_t qmax = (uint64_t)gsize >> g->rice;
        int64_t prev_local = -1;
        for (int64_t j0 = 0; j0 < g->count && !bad; j0 += BLOCK, b++) {
            uint64_t cur = bitpos, end = bitpos + u->block_bits[b];
            bitpos = end;
            int64_t j1 = j0 + BLOCK < g->count ? j0 + BLOCK : g->count;
            for (int64_t j = j0; j < j1; j++) {
                if (cur >= end) { bad = 1; break; }
                /* unary run, bounded by the block's own end and by qmax (_triton.py:54-62) */
                uint64_t q = 0;
                while (bit_at(u->payload, u->payload_len, cur + q)) {
                    q++;
                    if (q > qmax || cur + q >= end) break;
                }
                if (q > qmax || cur + q >= end) { bad = 1; break; }
                uint64_t c = cur + q + 1;
                uint64_t rem = g->rice ? read_bits(u->payload, u->payload_len, c, g->rice) : 0;
                uint64_t peek = read_bits(u->payload, u->payload_len, c + g->rice, MAX_CODE_LEN);
                int L = 0;
                for (int ln = 1; ln <= MAX_CODE_LEN; ln++) {
                    uint64_t code = peek >> (MAX_CODE_LEN - ln);
                    if (code >= d->first[ln] && code < d->first[ln] + d->cnt[ln]) { L = ln; break; }
                }
                if (!L) { bad = 1; break; }
                uint64_t code = peek >> (MAX_CODE_LEN - L);
                int64_t sym = d->sorted[d->base[L] + code - d->first[L]];
                uint64_t gap = (q << g->rice) | rem;
                if ((int64_t)gap >= gsize) { bad = 1; break; }
                int64_t loc = prev_local + (int64_t)gap + 1;
                if (loc >= gsize) { bad = 1; break; }
                prev_local = loc;
                local[o] = loc; zz[o] = (uint32_t)sym; gexp[o] = g->exp; o++;
                cur = c + g->rice + L;
            }
            if (!bad && cur != end) bad = 1;
        }
    }
    if (!bad) {
        /* (exponent, rank) -> position: one walk with running counters (codec.py:636-694) */
        int64_t counter[256] = {0};
        int64_t ptr[256], gend[256], gbeg[256];
        for (int e = 0; e < 256; e++) { ptr[e] = -1; gend[e] = -1; }
        int64_t oo = 0;
        for (int k = 0; k < h->ng; k++) { gbeg[h->g[k].exp] = oo; ptr[h->g[k].exp] = oo; oo += h->g[k].count; gend[h->g[k].exp] = oo; }
        uint64_t delta = 0;
        for (int64_t i = 0; i < h->numel; i++) {
            int e = ((uint16_t)a[i] >> 7) & 0xFF;
            if (ptr[e] >= 0 && ptr[e] < gend[e] && local[ptr[e]] == counter[e]) {
                int64_t j = ptr[e]++;
                uint32_t z = zz[j];
                int64_t res = (int64_t)(z >> 1) ^ -(int64_t)(z & 1);
                uint64_t old_u = (uint16_t)a[i];
                uint64_t new_u = (old_u + (uint64_t)res) & 0xFFFF;
                delta += (new_u - old_u) * splitmix_weight((uint64_t)i);
                c->pos[t][j] = i; c->val[t][j] = (int16_t)(uint16_t)new_u;
            }
            counter[e]++;
        }
        (void)gbeg;
        uint64_t base = (c->has_chk && c->has_chk[t]) ? c->old_chk[t] : orc_checksum(a, h->numel);
        if (base + delta != h->chk) { bad = 2; }
    }
    free(local); free(zz); free(gexp);
    c->tbad[t] = bad;
    c->tchanged[t] = tot;
}

/* the verified changes of tensor t into its weights */
static void app_commit(void *vc, int64_t t) {
    app_ctx_t *c = vc;
    int64_t tot = 0;
    for (int k = 0; k < c->u->tens[t].ng; k++) tot += c->u->tens[t].g[k].count;
    for (int64_t j = 0; j < tot; j++) c->weights[t][c->pos[t][j]] = c->val[t][j];
}

/*
 * Apply a parsed update.  weights[t] / old_chk[t] / has_chk[t] are given per update tensor
 * (the caller matched names and numel).  Writes nothing unless every block decodes exactly,
 * every change lies inside its exponent group and every checksum matches; *changed = the
 * number of changed elements.
 */
int orc_apply(void *handle, int16_t *const *weights, const uint64_t *old_chk, const uint8_t *has_chk,
              int64_t *changed, char *err, size_t errlen) {
    pupdate_t *u = handle;
    *changed = 0;
    int status = ORC_NOMEM;
    int tab_of[256]; for (int e = 0; e < 256; e++) tab_of[e] = -1;
    dtab_t *dt = calloc(u->n_tables ? u->n_tables : 1, sizeof(dtab_t));
    int64_t **pos = calloc(u->n_tensors ? u->n_tensors : 1, sizeof(int64_t *));
    int16_t **val = calloc(u->n_tensors ? u->n_tensors : 1, sizeof(int16_t *));
    int bad = 0;
    if (!dt || !pos || !val) goto done;
    for (int t = 0; t < u->n_tables; t++) { tab_of[u->tab[t].exp] = t; if (build_dtab(&u->tab[t], &dt[t])) goto done; }

    /* blocks are consecutive in the payload (FORMAT.md:39-44): each tensor's first block and bit,
     * so that tensors decode independently (one thread per tensor) */
    int64_t *tb0 = malloc(sizeof(int64_t) * (size_t)(u->n_tensors + 1));
    uint64_t *tbit0 = malloc(sizeof(uint64_t) * (size_t)(u->n_tensors + 1));
    int *tbad = calloc((size_t)(u->n_tensors + 1), sizeof(int));
    int64_t *tchanged = calloc((size_t)(u->n_tensors + 1), sizeof(int64_t));
    if (!tb0 || !tbit0 || !tbad || !tchanged) { free(tb0); free(tbit0); free(tbad); free(tchanged); goto done; }
    {
        int64_t bb = 0;
        uint64_t bits = 0;
        for (int64_t t = 0; t < u->n_tensors; t++) {
            tb0[t] = bb;
            tbit0[t] = bits;
            for (int k = 0; k < u->tens[t].ng; k++) {
                int64_t nbk = (u->tens[t].g[k].count + BLOCK - 1) / BLOCK;
                for (int64_t q = 0; q < nbk; q++) bits += u->block_bits[bb + q];
                bb += nbk;
            }
        }
    }
    app_ctx_t ac = {u, weights, old_chk, has_chk, dt, tab_of, tb0, tbit0, pos, val, tbad, tchanged, 0};
    parallel_for(u->n_tensors, app_tensor, &ac);
    const int nomem = ac.nomem;
    for (int64_t t = 0; t < u->n_tensors; t++) {   /* a decode or range error outranks a checksum one */
        if (tbad[t] == 1 || (tbad[t] == 2 && bad == 0)) bad = tbad[t];
        *changed += tchanged[t];
    }
    free(tb0); free(tbit0); free(tbad); free(tchanged);
    if (nomem) goto done;
    if (bad) {
        status = ORC_CORRUPT;
        set_err(err, errlen, bad == 2 ? "update does not verify (checksum mismatch)" : "payload positions outside their exponent groups");
        *changed = 0;
        goto done;
    }
    /* commit only now (codec.py:713-714) */
    parallel_for(u->n_tensors, app_commit, &ac);
    status = ORC_OK;
done:
    if (status == ORC_NOMEM) set_err(err, errlen, "oracle: out of memory");
    if (dt) for (int t = 0; t < u->n_tables; t++) free(dt[t].sorted);
    free(dt);
    if (pos) for (int64_t t = 0; t < u->n_tensors; t++) free(pos[t]);
    if (val) for (int64_t t = 0; t < u->n_tensors; t++) free(val[t]);
    free(pos); free(val);
    return status;
}
