// extern "C" entry points (include/crukx_b200.h) over the C++ drivers; no exception crosses.
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <new>
#include <unordered_map>
#include <string>

#include "../../include/crukx_b200.h"
#include "capi_internal.h"
#include "common.cuh"

struct crx_ctx {
    crx::Ctx c;
};
struct crx_encoded {
    crx::Encoded e;
};
struct crx_update {
    crx::Update u;
    std::vector<uint8_t> head;   // the update's head copied from device memory (crx_parse_device)
    ~crx_update();
};

namespace crx {

std::atomic<uint64_t> g_alloc_calls{0};
void note_alloc() { g_alloc_calls.fetch_add(1, std::memory_order_relaxed); }

static cudaEvent_t pooled_event(Ctx& c) {
    if (c.ev_used == c.ev_pool.size()) {
        cudaEvent_t e = nullptr;
        if (cudaEventCreate(&e) != cudaSuccess) { cudaGetLastError(); return nullptr; }
        c.ev_pool.push_back(e);
    }
    return c.ev_pool[c.ev_used++];
}

static double now_ms() {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

void trace_phase(Ctx& c, const char* name) {
    if (!c.trace) return;
    const double t = now_ms();
    std::fprintf(stderr, "[crx-host] %-28s +%9.3f ms\n", name, c.phase_t > 0 ? t - c.phase_t : 0.0);
    c.phase_t = t;
}

KernelScope::KernelScope(Ctx& ctx, const char* name, cudaStream_t st) : c(ctx), s(st) {
    ++c.launches;
    m.name = name;
    if (c.trace) {
        cudaStreamSynchronize(s);
        t0 = now_ms();
    }
    if (c.profile) {
        m.name = name;
        m.s = s;
        m.a = pooled_event(c);
        m.b = pooled_event(c);
        if (m.a) cudaEventRecord(m.a, s);
    }
}

KernelScope::~KernelScope() {
    if (c.profile && m.a && m.b) {
        cudaEventRecord(m.b, s);
        c.marks.push_back(m);
    }
    if (c.trace) {
        const cudaError_t e = cudaStreamSynchronize(s);
        std::fprintf(stderr, "[crx] %-16s %10.3f ms  %s\n", m.name, now_ms() - t0, cudaGetErrorString(e));
    }
}

Ctx::~Ctx() {
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    cudaDeviceSynchronize();
    for (cudaEvent_t e : ev_pool) cudaEventDestroy(e);
    for (cudaEvent_t e : copy_ev) cudaEventDestroy(e);
    if (ev_main) cudaEventDestroy(ev_main);
    if (hstore_ev) cudaEventDestroy(hstore_ev);
    if (hstore_table.p) cudaFreeHost(hstore_table.p);
    if (wd_ev) cudaEventDestroy(wd_ev);
    if (head_host.p) cudaFreeHost(head_host.p);
    if (ev_copy) cudaEventDestroy(ev_copy);
    if (copy_stream) cudaStreamDestroy(copy_stream);
    for (auto& d : b)
        if (d.p) cudaFree(d.p);
    for (auto& kv : hist_cache)
        if (kv.second.rows.p) cudaFree(kv.second.rows.p);
    for (auto& d : hist_free)
        if (d.p) cudaFree(d.p);
    if (host) cudaFreeHost(host);
    if (out_host.p) cudaFreeHost(out_host.p);
    if (in_host.p) cudaFreeHost(in_host.p);
    if (small) cudaFreeHost(small);
    if (prev >= 0) cudaSetDevice(prev);
}

cudaError_t ensure_dev(DevBuf& buf, size_t bytes, cudaStream_t s) {
    if (bytes <= buf.cap) return cudaSuccess;
    size_t cap = buf.cap ? buf.cap : 4096;
    while (cap < bytes) cap += cap / 2 + 4096;
    if (buf.p) {
        cudaError_t e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return e;
        note_alloc();
        cudaFree(buf.p);
        buf.p = nullptr;
        buf.cap = 0;
    }
    note_alloc();
    cudaError_t e = cudaMalloc(&buf.p, cap);
    if (e != cudaSuccess) {
        cudaGetLastError();
        note_alloc();
        e = cudaMalloc(&buf.p, bytes);   // retry without headroom
        if (e != cudaSuccess) { buf.p = nullptr; return e; }
        cap = bytes;
    }
    buf.cap = cap;
    return cudaSuccess;
}

cudaError_t ensure_host(Ctx& c, size_t bytes, cudaStream_t s) {
    if (bytes <= c.host_cap) return cudaSuccess;
    size_t cap = c.host_cap ? c.host_cap : (1 << 20);
    while (cap < bytes) cap *= 2;
    if (c.host) {
        cudaError_t e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return e;
        note_alloc();
        cudaFreeHost(c.host);
        c.host = nullptr;
        c.host_cap = 0;
    }
    note_alloc();
    cudaError_t e = cudaMallocHost(&c.host, cap);
    if (e != cudaSuccess) { c.host = nullptr; return e; }
    c.host_cap = cap;
    return cudaSuccess;
}

cudaError_t ensure_pinned(DevBuf& buf, size_t bytes, cudaStream_t s) {
    if (bytes <= buf.cap) return cudaSuccess;
    size_t cap = buf.cap ? buf.cap : (size_t(1) << 20);
    while (cap < bytes) cap += cap / 2;
    if (buf.p) {
        cudaError_t e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return e;
        note_alloc();
        cudaFreeHost(buf.p);
        buf.p = nullptr;
        buf.cap = 0;
    }
    note_alloc();
    cudaError_t e = cudaMallocHost(&buf.p, cap);
    if (e != cudaSuccess) { buf.p = nullptr; return e; }
    buf.cap = cap;
    return cudaSuccess;
}

cudaError_t ensure_copy_stream(Ctx& c) {
    if (c.copy_stream) return cudaSuccess;
    cudaError_t e = cudaEventCreateWithFlags(&c.ev_main, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c.ev_copy, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c.copy_stream, cudaStreamNonBlocking);
    return e;
}

cudaError_t chunk_events(Ctx& c, size_t n_chunks) {
    while (c.copy_ev.size() < n_chunks) {
        cudaEvent_t e = nullptr;
        const cudaError_t r = cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
        if (r != cudaSuccess) return r;
        c.copy_ev.push_back(e);
    }
    return cudaSuccess;
}

cudaError_t upload_pipelined(Ctx& c, void* dev_dst, const void* host_src, uint8_t* pinned, size_t n, cudaStream_t s) {
    for (size_t off = 0; off < n; off += kCopyChunk) {
        const size_t len = std::min(kCopyChunk, n - off);
        parallel_copy(pinned + off, static_cast<const uint8_t*>(host_src) + off, len);
        const cudaError_t e = cudaMemcpyAsync(static_cast<uint8_t*>(dev_dst) + off, pinned + off, len, cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t Encoded::write(uint8_t* dst) const {
    if (device) {   // from the device workspace, synchronously
        cudaError_t e = cudaEventSynchronize(ctx->copy_ev[0]);
        if (e != cudaSuccess) return e;
        if (ctx->small[kEncStatusWord] & ERR_INTERNAL) return cudaErrorUnknown;
        std::memcpy(dst, head.data(), head.size());
        dst += head.size();
        const size_t bt = 4 * size_t(n_blocks);
        if (bt) e = cudaMemcpyAsync(dst, dtable, bt, cudaMemcpyDeviceToHost, stream);
        dst += bt;
        std::memcpy(dst, len_varint.data(), len_varint.size());
        dst += len_varint.size();
        if (e == cudaSuccess && payload_len) e = cudaMemcpyAsync(dst, dpay, payload_len, cudaMemcpyDeviceToHost, stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
        return e;
    }
    if (pending) prefault(dst, size());   // the GPU is still packing and copying meanwhile
    std::memcpy(dst, head.data(), head.size());
    dst += head.size();
    const size_t bt = 4 * size_t(n_blocks);
    if (pending) {
        const cudaError_t e = cudaEventSynchronize(ctx->copy_ev[0]);
        if (e != cudaSuccess) return e;
        if (ctx->small[kEncStatusWord] & ERR_INTERNAL) return cudaErrorUnknown;
    } else if (internal_error) {
        return cudaErrorUnknown;
    }
    if (bt) parallel_copy(dst, table, bt);
    dst += bt;
    std::memcpy(dst, len_varint.data(), len_varint.size());
    dst += len_varint.size();
    if (!pending) {
        if (payload_len) parallel_copy(dst, table + bt, payload_len);
        return cudaSuccess;
    }
    for (uint64_t off = 0, k = 0; off < payload_len; off += kCopyChunk, ++k) {
        const size_t len = size_t(std::min<uint64_t>(kCopyChunk, payload_len - off));
        const cudaError_t e = cudaEventSynchronize(ctx->copy_ev[1 + k]);
        if (e != cudaSuccess) return e;
        parallel_copy(dst + off, table + bt + off, len);
    }
    return cudaSuccess;
}

cudaError_t Encoded::write_part(uint8_t* prefix, uint8_t* tensors, uint8_t* tbl, uint8_t* pay) const {
    const size_t bt = 4 * size_t(n_blocks);
    if (pending) {
        const cudaError_t e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess) return e;
        if (ctx->small[kEncStatusWord] & ERR_INTERNAL) return cudaErrorUnknown;
    } else if (internal_error) {
        return cudaErrorUnknown;
    }
    if (prefix) std::memcpy(prefix, head.data(), head.size());
    if (tensors && !part_tensors.empty()) std::memcpy(tensors, part_tensors.data(), part_tensors.size());
    if (tbl && bt) std::memcpy(tbl, table, bt);
    if (pay && payload_len) parallel_copy(pay, table + bt, payload_len);
    return cudaSuccess;
}

cudaError_t Encoded::write_device(uint8_t* dst, cudaStream_t s) const {
    const size_t bt = 4 * size_t(n_blocks);
    cudaError_t e = cudaSuccess;
    if (device) {   // stream-ordered: nothing waits for the device here
        // after the encoder's last kernel (its stream may not be `s`); its consistency checks were
        // read back before the encode returned
        e = cudaStreamWaitEvent(s, ctx->copy_ev[0], 0);
        if (e != cudaSuccess) return e;
        // the header and the length varint are a few KB of host bytes, sent from pinned memory that
        // the previous call's copies have finished reading; the rest moves on the device
        if (ctx->wd_busy) {
            e = cudaEventSynchronize(ctx->wd_ev);
            if (e != cudaSuccess) return e;
            ctx->wd_busy = false;
        }
        if (!ctx->wd_ev && (e = cudaEventCreateWithFlags(&ctx->wd_ev, cudaEventDisableTiming)) != cudaSuccess) return e;
        if ((e = ensure_pinned(ctx->head_host, head.size() + len_varint.size(), s)) != cudaSuccess) return e;
        uint8_t* hh = static_cast<uint8_t*>(ctx->head_host.p);
        std::memcpy(hh, head.data(), head.size());
        std::memcpy(hh + head.size(), len_varint.data(), len_varint.size());
        e = cudaMemcpyAsync(dst, hh, head.size(), cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess && bt) e = cudaMemcpyAsync(dst + head.size(), dtable, bt, cudaMemcpyDeviceToDevice, s);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(dst + head.size() + bt, hh + head.size(), len_varint.size(), cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess && payload_len)
            e = cudaMemcpyAsync(dst + head.size() + bt + len_varint.size(), dpay, payload_len, cudaMemcpyDeviceToDevice, s);
        if (e == cudaSuccess) e = cudaEventRecord(ctx->wd_ev, s);
        if (e == cudaSuccess) ctx->wd_busy = true;
        return e;
    }
    if (pending) {
        e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess) return e;
        if (ctx->small[kEncStatusWord] & ERR_INTERNAL) return cudaErrorUnknown;
    } else if (internal_error) {
        return cudaErrorUnknown;
    }
    std::vector<uint8_t> all(size());
    e = write(all.data());
    if (e == cudaSuccess) e = cudaMemcpyAsync(dst, all.data(), all.size(), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    return e;
}

cudaError_t Encoded::detach() {
    if (device) {   // keep a host copy: the next encode reuses the device workspace
        const cudaError_t e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess) return e;
        internal_error = (ctx->small[kEncStatusWord] & ERR_INTERNAL) != 0;
        const size_t bt = 4 * size_t(n_blocks);
        std::vector<uint8_t> tmp(bt + payload_len);
        cudaError_t r = cudaSuccess;
        if (bt) r = cudaMemcpy(tmp.data(), dtable, bt, cudaMemcpyDeviceToHost);
        if (r == cudaSuccess && payload_len) r = cudaMemcpy(tmp.data() + bt, dpay, payload_len, cudaMemcpyDeviceToHost);
        if (r != cudaSuccess) return r;
        own.swap(tmp);
        table = own.data();
        device = false;
        return cudaSuccess;
    }
    if (!pending) return cudaSuccess;
    const cudaError_t e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return e;
    internal_error = (ctx->small[kEncStatusWord] & ERR_INTERNAL) != 0;
    const size_t n = 4 * size_t(n_blocks) + payload_len;
    std::vector<uint8_t> tmp(n);
    if (n) std::memcpy(tmp.data(), table, n);
    own.swap(tmp);
    table = own.data();
    pending = false;
    return cudaSuccess;
}

}  // namespace crx

namespace {

void put_err(char* err, size_t n, const std::string& m) {
    if (err && n) std::snprintf(err, n, "%s", m.c_str());
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

}  // namespace

extern "C" {

int crx_wire_version(void) { return 2; }

uint64_t crx_alloc_calls(void) { return crx::g_alloc_calls.load(std::memory_order_relaxed); }

int crx_ctx_create(int device, crx_ctx** out, char* err, size_t errlen) {
    if (!out) return CRX_BAD_ARGUMENT;
    *out = nullptr;
    crx_ctx* c = new (std::nothrow) crx_ctx;
    if (!c) return CRX_NO_MEMORY;
    c->c.device = device;
    const char* tr = std::getenv("CRUKX_B200_TRACE");
    c->c.trace = tr && *tr && *tr != '0';
    DeviceGuard g(device);
    cudaError_t e = cudaSetDevice(device);
    crx::note_alloc();
    if (e == cudaSuccess) e = cudaMallocHost(reinterpret_cast<void**>(&c->c.small), 4096);
    if (e != cudaSuccess) {
        put_err(err, errlen, std::string("crx_ctx_create: ") + cudaGetErrorString(e));
        cudaGetLastError();
        c->c.small = nullptr;
        delete c;
        return CRX_CUDA_ERROR;
    }
    *out = c;
    return CRX_OK;
}

void crx_ctx_destroy(crx_ctx* ctx) { delete ctx; }

int crx_encode(crx_ctx* ctx, int32_t n_tensors, const int16_t* const* prev, const int16_t* const* cur,
               const int64_t* numel, const uint8_t* const* names, const int64_t* name_len,
               const uint64_t* cached_checksums, const uint8_t* has_cached, void* stream,
               crx_encoded** out, char* err, size_t errlen) {
    if (!ctx || !out || n_tensors < 0 || (n_tensors && (!prev || !cur || !numel || !names || !name_len))) {
        put_err(err, errlen, "crx_encode: bad argument");
        return CRX_BAD_ARGUMENT;
    }
    *out = nullptr;
    try {
        std::lock_guard<std::mutex> lock(ctx->c.mu);
        DeviceGuard g(ctx->c.device);
        crx_encoded* e = new crx_encoded;
        std::string msg;
        const crx::Status s = crx::encode_impl(ctx->c, n_tensors, prev, cur, numel, names, name_len, cached_checksums,
                                               has_cached, static_cast<cudaStream_t>(stream), &e->e, &msg);
        if (s != crx::kOk) {
            delete e;
            put_err(err, errlen, msg);
            return int(s);
        }
        *out = e;
        return CRX_OK;
    } catch (const std::bad_alloc&) {
        put_err(err, errlen, "crx_encode: out of host memory");
        return CRX_NO_MEMORY;
    } catch (const std::exception& ex) {
        put_err(err, errlen, std::string("crx_encode: ") + ex.what());
        return CRX_CUDA_ERROR;
    }
}

int crx_encode_device(crx_ctx* ctx, int32_t n_tensors, const int16_t* const* prev, const int16_t* const* cur,
                      const int64_t* numel, const uint8_t* const* names, const int64_t* name_len,
                      const uint64_t* cached_checksums, const uint8_t* has_cached, void* stream,
                      crx_encoded** out, char* err, size_t errlen) {
    if (!ctx || !out || n_tensors < 0 || (n_tensors && (!prev || !cur || !numel || !names || !name_len))) {
        put_err(err, errlen, "crx_encode_device: bad argument");
        return CRX_BAD_ARGUMENT;
    }
    *out = nullptr;
    try {
        std::lock_guard<std::mutex> lock(ctx->c.mu);
        DeviceGuard g(ctx->c.device);
        crx_encoded* e = new crx_encoded;
        std::string msg;
        const crx::Status s = crx::encode_impl(ctx->c, n_tensors, prev, cur, numel, names, name_len, cached_checksums,
                                               has_cached, static_cast<cudaStream_t>(stream), &e->e, &msg, true);
        if (s != crx::kOk) {
            delete e;
            put_err(err, errlen, msg);
            return int(s);
        }
        *out = e;
        return CRX_OK;
    } catch (const std::bad_alloc&) {
        put_err(err, errlen, "crx_encode_device: out of host memory");
        return CRX_NO_MEMORY;
    } catch (const std::exception& ex) {
        put_err(err, errlen, std::string("crx_encode_device: ") + ex.what());
        return CRX_CUDA_ERROR;
    }
}

namespace {

struct CallbackExchange {   // adapts the C callbacks to crx::GlobalExchange
    crx_sum_u64_fn sum;
    crx_allgather_fn gather;
    void* user;
};

int cb_sum(void* u, uint64_t* d, int64_t n) {
    auto* x = static_cast<CallbackExchange*>(u);
    return x->sum(x->user, d, n);
}

int cb_gather(void* u, const uint8_t* mine, int64_t len, const uint8_t** all, int64_t* all_len) {
    auto* x = static_cast<CallbackExchange*>(u);
    return x->gather(x->user, mine, len, all, all_len);
}

}  // namespace

int crx_encode_global(crx_ctx* ctx, int32_t n_tensors, const int16_t* const* prev, const int16_t* const* cur,
                      const int64_t* numel, const uint8_t* const* names, const int64_t* name_len,
                      const uint64_t* cached_checksums, const uint8_t* has_cached, void* stream, int32_t rank,
                      int32_t world, crx_sum_u64_fn sum_u64, crx_allgather_fn allgather, void* user,
                      crx_encoded** out, char* err, size_t errlen) {
    if (!ctx || !out || n_tensors < 0 || (n_tensors && (!prev || !cur || !numel || !names || !name_len)) ||
        world < 1 || rank < 0 || rank >= world || !sum_u64 || !allgather) {
        put_err(err, errlen, "crx_encode_global: bad argument");
        return CRX_BAD_ARGUMENT;
    }
    *out = nullptr;
    try {
        std::lock_guard<std::mutex> lock(ctx->c.mu);
        DeviceGuard g(ctx->c.device);
        CallbackExchange cx{sum_u64, allgather, user};
        const crx::GlobalExchange gx{cb_sum, cb_gather, &cx, rank, world};
        crx_encoded* e = new crx_encoded;
        std::string msg;
        const crx::Status s = crx::encode_impl(ctx->c, n_tensors, prev, cur, numel, names, name_len, cached_checksums,
                                               has_cached, static_cast<cudaStream_t>(stream), &e->e, &msg, false, &gx);
        if (s != crx::kOk) {
            delete e;
            put_err(err, errlen, msg);
            return int(s);
        }
        *out = e;
        return CRX_OK;
    } catch (const std::bad_alloc&) {
        put_err(err, errlen, "crx_encode_global: out of host memory");
        return CRX_NO_MEMORY;
    } catch (const std::exception& ex) {
        put_err(err, errlen, std::string("crx_encode_global: ") + ex.what());
        return CRX_CUDA_ERROR;
    }
}

int crx_encoded_part(const crx_encoded* enc, int64_t* prefix_len, int64_t* tensors_len, int64_t* table_len,
                     int64_t* payload_len, uint64_t* bit_offset, uint64_t* total_bits) {
    if (!enc || !enc->e.part) return CRX_BAD_ARGUMENT;
    if (prefix_len) *prefix_len = int64_t(enc->e.head.size());
    if (tensors_len) *tensors_len = int64_t(enc->e.part_tensors.size());
    if (table_len) *table_len = 4 * enc->e.n_blocks;
    if (payload_len) *payload_len = int64_t(enc->e.payload_len);
    if (bit_offset) *bit_offset = enc->e.bit_offset;
    if (total_bits) *total_bits = enc->e.total_bits;
    return CRX_OK;
}

int crx_encoded_part_copy(const crx_encoded* enc, uint8_t* prefix, uint8_t* tensors, uint8_t* table, uint8_t* payload) {
    if (!enc || !enc->e.part) return CRX_BAD_ARGUMENT;
    cudaError_t e;
    if (enc->e.ctx) {
        std::lock_guard<std::mutex> lock(enc->e.ctx->mu);
        DeviceGuard g(enc->e.ctx->device);
        e = enc->e.write_part(prefix, tensors, table, payload);
    } else {
        e = enc->e.write_part(prefix, tensors, table, payload);
    }
    return e == cudaSuccess ? CRX_OK : CRX_CUDA_ERROR;
}

int crx_encoded_copy_device(const crx_encoded* enc, void* dst, int64_t cap, void* stream) {
    if (!enc || !dst || enc->e.part || cap < int64_t(enc->e.size())) return CRX_BAD_ARGUMENT;
    cudaError_t e;
    if (enc->e.ctx) {
        std::lock_guard<std::mutex> lock(enc->e.ctx->mu);
        DeviceGuard g(enc->e.ctx->device);
        e = enc->e.write_device(static_cast<uint8_t*>(dst), static_cast<cudaStream_t>(stream));
    } else {
        e = enc->e.write_device(static_cast<uint8_t*>(dst), static_cast<cudaStream_t>(stream));
    }
    return e == cudaSuccess ? CRX_OK : CRX_CUDA_ERROR;
}

int64_t crx_encoded_size(const crx_encoded* enc) { return enc && !enc->e.part ? int64_t(enc->e.size()) : -1; }

int crx_encoded_copy(const crx_encoded* enc, uint8_t* dst, int64_t cap) {
    if (!enc || !dst || enc->e.part || cap < int64_t(enc->e.size())) return CRX_BAD_ARGUMENT;
    cudaError_t e;
    if (enc->e.ctx) {   // the context lock keeps the next encode from reusing the buffers meanwhile
        std::lock_guard<std::mutex> lock(enc->e.ctx->mu);
        DeviceGuard g(enc->e.ctx->device);
        e = enc->e.write(dst);
    } else {
        e = enc->e.write(dst);
    }
    return e == cudaSuccess ? CRX_OK : CRX_CUDA_ERROR;
}

int64_t crx_encoded_changes(const crx_encoded* enc) { return enc ? int64_t(enc->e.changes) : -1; }

void crx_encoded_checksums(const crx_encoded* enc, uint64_t* checksums, uint8_t* present) {
    if (!enc) return;
    for (size_t i = 0; i < enc->e.checksums.size(); ++i) {
        if (checksums) checksums[i] = enc->e.checksums[i];
        if (present) present[i] = enc->e.present[i];
    }
}

void crx_encoded_free(crx_encoded* enc) {
    if (!enc) return;
    if (enc->e.ctx) {
        std::lock_guard<std::mutex> lock(enc->e.ctx->mu);
        // copies still landing in the context's pinned buffer must finish before it is reused (a
        // device result's copies are ordered by the context's wd_ev instead)
        if (enc->e.pending) {
            DeviceGuard g(enc->e.ctx->device);
            cudaStreamSynchronize(enc->e.stream);
        }
        if (enc->e.ctx->live == &enc->e) enc->e.ctx->live = nullptr;
    }
    delete enc;
}

int crx_parse(const uint8_t* data, int64_t len, crx_update** out, char* err, size_t errlen) {
    if (!out || len < 0 || (len && !data)) return CRX_BAD_ARGUMENT;
    *out = nullptr;
    try {
        crx_update* u = new crx_update;
        std::string msg;
        const crx::Status s = crx::parse_update(data, len, &u->u, &msg);
        if (s != crx::kOk) {
            delete u;
            put_err(err, errlen, msg);
            return int(s);
        }
        *out = u;
        return CRX_OK;
    } catch (const std::bad_alloc&) {
        put_err(err, errlen, "crx_parse: out of host memory");
        return CRX_NO_MEMORY;
    }
}

int crx_parse_head(const uint8_t* head, int64_t head_len, int64_t len, uint8_t last, crx_update** out, int64_t* need,
                   char* err, size_t errlen) {
    if (!out || len < 0 || head_len < 0 || (head_len && !head)) return CRX_BAD_ARGUMENT;
    *out = nullptr;
    if (need) *need = 0;
    try {
        crx_update* u = new crx_update;
        std::string msg;
        int64_t nd = 0;
        const crx::Status s = crx::parse_head(head, head_len, len, last, &u->u, &nd, &msg);
        if (s != crx::kOk) {
            delete u;
            if (s == crx::kNeedMore) {
                if (need) *need = nd;
                return CRX_NEED_MORE;
            }
            put_err(err, errlen, msg);
            return int(s);
        }
        *out = u;
        return CRX_OK;
    } catch (const std::bad_alloc&) {
        put_err(err, errlen, "crx_parse_head: out of host memory");
        return CRX_NO_MEMORY;
    }
}

namespace {

// What crx_parse_device keeps per device: its lock (the block-table check's accumulators below are
// per device, so parses on different devices run concurrently), pinned staging for the heads it
// copies back (device -> pageable copies run at a fraction of the link's bandwidth) and the group
// spans of the last checked table, both grown on demand and kept for the process.
struct DevParse {
    std::mutex mu;
    uint8_t* pinned = nullptr;
    size_t cap = 0;
    void* spans = nullptr;
    size_t spans_cap = 0;
    uint8_t* res = nullptr;     // pinned: the block-table check's results (bit total, short flag)
    uint8_t* spin = nullptr;    // pinned: the group spans going up for the check
    size_t spin_cap = 0;
    int64_t last_head = 0;      // header length of the last update parsed here: the next first copy's size
};
std::mutex g_devparse_mu;                                   // guards the map only
std::unordered_map<int, std::unique_ptr<DevParse>> g_devparse;

DevParse& dev_parse(int dev) {
    std::lock_guard<std::mutex> lock(g_devparse_mu);
    auto& p = g_devparse[dev];
    if (!p) p.reset(new DevParse);
    return *p;
}

// host buffers of freed device-update heads, reused: a fresh multi-megabyte vector costs its
// zero fill and page faults on every parse
std::mutex g_pool_mu;
std::vector<std::vector<uint8_t>> g_head_pool;
constexpr size_t kHeadPoolMax = 8;
std::atomic<uint64_t> g_parse_launches{0};   // kernels crx_parse_device launched

}  // namespace

crx_update::~crx_update() {
    if (head.capacity() == 0) return;
    std::lock_guard<std::mutex> lock(g_pool_mu);
    if (g_head_pool.size() < kHeadPoolMax) g_head_pool.push_back(std::move(head));
}

namespace {

// The block table of a device update, checked where it lies: its bit total and whether some block
// is shorter than its symbols could be (every change costs at least 2 + rice bits).  The table
// starts at any byte offset, so its words are read bytewise.
__device__ unsigned long long g_bt_total;
__device__ unsigned int g_bt_short;

__global__ void __launch_bounds__(256) k_check_block_table(const uint8_t* __restrict__ table, int64_t n_blocks,
                                                           const uint64_t* __restrict__ first_block,
                                                           const uint64_t* __restrict__ count_rice, int64_t ns) {
    uint64_t bits = 0;
    bool bad = false;
    for (int64_t b = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; b < n_blocks; b += int64_t(gridDim.x) * blockDim.x) {
        const uint8_t* p = table + 4 * b;
        const uint32_t w = uint32_t(p[0]) | (uint32_t(p[1]) << 8) | (uint32_t(p[2]) << 16) | (uint32_t(p[3]) << 24);
        int64_t lo = 0, hi = ns - 1;   // the group of block b: the last one starting at or before it
        while (lo < hi) {
            const int64_t mid = (lo + hi + 1) >> 1;
            if (first_block[mid] <= uint64_t(b)) lo = mid; else hi = mid - 1;
        }
        const uint64_t cr = count_rice[lo];
        const uint64_t m = crx::tmin<uint64_t>(crx::kBlock, (cr >> 8) - (uint64_t(b) - first_block[lo]) * crx::kBlock);
        bad |= uint64_t(w) < m * (2 + (cr & 0xFF));
        bits += w;
    }
    for (int o = 16; o; o >>= 1) bits += __shfl_xor_sync(0xffffffffu, bits, o);
    const bool any_bad = __any_sync(0xffffffffu, bad);
    if ((threadIdx.x & 31) == 0) {
        if (bits) atomicAdd(&g_bt_total, (unsigned long long)bits);
        if (any_bad) atomicOr(&g_bt_short, 1u);
    }
}

// pinned staging of at least `bytes` in P (the caller holds P.mu)
bool stage_pinned(DevParse& P, size_t bytes) {
    if (bytes <= P.cap) return true;
    crx::note_alloc();
    if (P.pinned) cudaFreeHost(P.pinned);
    P.pinned = nullptr;
    P.cap = 0;
    const size_t cap = std::max(bytes, size_t(1) << 20);
    crx::note_alloc();
    if (cudaMallocHost(reinterpret_cast<void**>(&P.pinned), cap) != cudaSuccess) return false;
    P.cap = cap;
    return true;
}

// queues the check of u's block table at `table` in device memory: its bit total and whether some
// block is shorter than its symbols could be, into P.res (read after the caller's next
// synchronisation of `st`); the caller holds P.mu
int issue_block_table_check(DevParse& P, const crx::Update& u, const uint8_t* table, cudaStream_t st) {
    if (!P.res) {
        crx::note_alloc();
        if (cudaMallocHost(reinterpret_cast<void**>(&P.res), 64) != cudaSuccess) { P.res = nullptr; return CRX_CUDA_ERROR; }
    }
    std::memset(P.res, 0, 16);
    if (u.n_blocks <= 0) return CRX_OK;
    std::vector<uint64_t> fb, cr;
    crx::block_spans(u, &fb, &cr);
    const int64_t ns = int64_t(fb.size());
    const size_t span_bytes = 16 * size_t(ns);
    if (P.spans_cap < span_bytes + 16) {
        crx::note_alloc();
        if (P.spans && cudaFree(P.spans) != cudaSuccess) return CRX_CUDA_ERROR;
        P.spans = nullptr;
        P.spans_cap = 0;
        const size_t cap = std::max(span_bytes + 16, size_t(1) << 20);
        crx::note_alloc();
        if (cudaMalloc(&P.spans, cap) != cudaSuccess) return CRX_CUDA_ERROR;
        P.spans_cap = cap;
    }
    // the spans go up from their own pinned buffer (a pageable source would synchronise the stream;
    // head and window copies use P.pinned); it is reused only after the caller's synchronisation
    if (P.spin_cap < span_bytes) {
        crx::note_alloc();
        if (P.spin) cudaFreeHost(P.spin);
        P.spin = nullptr;
        P.spin_cap = 0;
        const size_t cap = std::max(span_bytes, size_t(1) << 20);
        crx::note_alloc();
        if (cudaMallocHost(reinterpret_cast<void**>(&P.spin), cap) != cudaSuccess) { P.spin = nullptr; return CRX_CUDA_ERROR; }
        P.spin_cap = cap;
    }
    std::memcpy(P.spin, fb.data(), 8 * size_t(ns));
    std::memcpy(P.spin + 8 * size_t(ns), cr.data(), 8 * size_t(ns));
    const uint64_t* dfb = static_cast<const uint64_t*>(P.spans);
    const uint64_t* dcr = dfb + ns;
    void* dtot = nullptr;
    void* dshort = nullptr;
    bool ok = cudaMemcpyAsync(P.spans, P.spin, span_bytes, cudaMemcpyHostToDevice, st) == cudaSuccess &&
              cudaGetSymbolAddress(&dtot, g_bt_total) == cudaSuccess &&
              cudaGetSymbolAddress(&dshort, g_bt_short) == cudaSuccess &&
              cudaMemsetAsync(dtot, 0, 8, st) == cudaSuccess && cudaMemsetAsync(dshort, 0, 4, st) == cudaSuccess;
    if (ok) {
        const int64_t grid = crx::tmin<int64_t>((u.n_blocks + 255) / 256, 148 * 8);
        k_check_block_table<<<unsigned(grid), 256, 0, st>>>(table, u.n_blocks, dfb, dcr, ns);
        ++g_parse_launches;
        ok = cudaGetLastError() == cudaSuccess &&
             cudaMemcpyAsync(P.res, dtot, 8, cudaMemcpyDeviceToHost, st) == cudaSuccess &&
             cudaMemcpyAsync(P.res + 8, dshort, 4, cudaMemcpyDeviceToHost, st) == cudaSuccess;
    }
    return ok ? CRX_OK : CRX_CUDA_ERROR;
}

// after the synchronisation that follows issue_block_table_check: the table's verdict
int finish_block_table_check(DevParse& P, crx::Update* u, uint8_t last, std::string* msg) {
    uint64_t total = 0;
    uint32_t sh = 0;
    std::memcpy(&total, P.res, 8);
    std::memcpy(&sh, P.res + 8, 4);
    return int(crx::finish_block_table_checks(u, total, sh != 0, last, msg));
}

}  // namespace

int crx_parse_device(const uint8_t* data, int64_t len, void* stream, crx_update** out, char* err, size_t errlen) {
    if (!out || len < 0 || (len && !data)) return CRX_BAD_ARGUMENT;
    *out = nullptr;
    try {
        const cudaStream_t st = static_cast<cudaStream_t>(stream);
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) return CRX_CUDA_ERROR;
        DevParse& P = dev_parse(dev);
        std::lock_guard<std::mutex> lock(P.mu);
        std::vector<uint8_t> head;
        {
            std::lock_guard<std::mutex> pl(g_pool_mu);
            if (!g_head_pool.empty()) {
                head.swap(g_head_pool.back());
                g_head_pool.pop_back();
            }
        }
        auto keep = [&]() {
            std::lock_guard<std::mutex> pl(g_pool_mu);
            if (g_head_pool.size() < kHeadPoolMax) g_head_pool.push_back(std::move(head));
        };
        auto stage = [&](size_t bytes) { return stage_pinned(P, bytes); };
        uint8_t last = 0;
        // the first copy: as long as the last header parsed here (updates of one model are alike)
        int64_t have = std::min<int64_t>(len, std::max<int64_t>(int64_t(1) << 16, P.last_head + 4096));
        int64_t got = 0;      // bytes [0, got) of the update are in `head`
        int64_t avail = 0;    // what the parser may read: [0, got), and past the block table a window after it
        bool checked = false; // the block table's check is queued (its results land with the window)
        crx_update* held = nullptr;         // a parse that stopped just past the block table
        const uint8_t* held_at = nullptr;   // the head buffer its names point into
        for (;;) {   // copy a head, parse it, copy more when the header reaches past it
            if (have > got) {
                delete held;   // a new head: parse from the start
                held = nullptr;
                if (!stage(size_t(have - got) + 1)) return CRX_CUDA_ERROR;
                if (cudaMemcpyAsync(P.pinned, data + got, size_t(have - got), cudaMemcpyDeviceToHost, st) != cudaSuccess)
                    return CRX_CUDA_ERROR;
                if (got == 0 && len &&
                    cudaMemcpyAsync(P.pinned + (have - got), data + len - 1, 1, cudaMemcpyDeviceToHost, st) != cudaSuccess)
                    return CRX_CUDA_ERROR;
                if (cudaStreamSynchronize(st) != cudaSuccess) return CRX_CUDA_ERROR;
                if (got == 0 && len) last = P.pinned[have];
                if (head.size() < size_t(have)) head.resize(size_t(have));   // a reused buffer keeps its size
                crx::parallel_copy(head.data() + got, P.pinned, size_t(have - got));
                got = have;
                avail = std::max(avail, got);
            }
            crx_update* u;
            std::string msg;
            int64_t nd = 0;
            crx::Status s;
            if (held && held_at == head.data()) {   // only the bytes after the table were missing
                u = held;
                s = crx::resume_head_device_table(head.data(), avail, len, &u->u, &nd, &msg);
            } else {
                delete held;
                u = new crx_update;
                s = crx::parse_head_device_table(head.data(), avail, len, last, &u->u, &nd, &msg);
            }
            held = nullptr;
            if (s == crx::kOk) {
                const int64_t t0 = u->u.block_table_offset;
                P.last_head = t0;
                int rc = CRX_OK;
                if (!checked) {
                    rc = issue_block_table_check(P, u->u, data + t0, st);
                    if (rc == CRX_OK && cudaStreamSynchronize(st) != cudaSuccess) rc = CRX_CUDA_ERROR;
                }
                if (rc == CRX_OK) rc = finish_block_table_check(P, &u->u, last, &msg);
                if (rc != CRX_OK) {
                    delete u;
                    keep();
                    if (rc == int(crx::kCorrupt)) put_err(err, errlen, msg);
                    return rc;
                }
                u->u.block_table_device = data + t0;
                u->u.payload_device = data + u->u.payload_offset;
                u->u.payload = nullptr;
                u->head.swap(head);   // the header's pointers stay valid: the vector's buffer moves with it
                *out = u;
                return CRX_OK;
            }
            const int64_t t0 = u->u.block_table_offset;
            const int64_t t1 = t0 >= 0 ? t0 + 4 * u->u.n_blocks : -1;
            if (s == crx::kNeedMore && t0 >= 0 && nd > t0 && got >= t0 && !checked) {
                // the header is complete: queue the block table's check now, so that its results
                // come back with the window copied below (one synchronisation for both)
                const int rc = issue_block_table_check(P, u->u, data + t0, st);
                if (rc != CRX_OK) {
                    delete u;
                    keep();
                    return rc;
                }
                checked = true;
            }
            if (s != crx::kNeedMore) {
                delete u;
                keep();
                put_err(err, errlen, msg);
                return int(s);
            }
            if (t0 >= 0 && nd > t0 && got >= t0) {
                // the header is here; past the table comes at most a 10-byte length varint: copy
                // that window only (the table itself is checked on the device), then resume the
                // parse there (it is redone from the start only if the head buffer moved)
                const int64_t w1 = std::min(len, t1 + 16);
                const bool failed = w1 <= avail || !stage(size_t(w1 - t1)) ||
                                   cudaMemcpyAsync(P.pinned, data + t1, size_t(w1 - t1), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
                                   cudaStreamSynchronize(st) != cudaSuccess;
                if (failed) {   // no progress (cannot happen) or a failed copy
                    delete u;
                    return CRX_CUDA_ERROR;
                }
                held = u;
                held_at = head.data();   // the buffer the parse read (and its names point into)
                if (head.size() < size_t(w1)) head.resize(size_t(w1));   // may move it: then parse anew
                std::memcpy(head.data() + t1, P.pinned, size_t(w1 - t1));
                avail = w1;
                continue;
            }
            delete u;
            have = std::min(len, std::max(nd + 16, 4 * have));
        }
    } catch (const std::bad_alloc&) {
        put_err(err, errlen, "crx_parse_device: out of host memory");
        return CRX_NO_MEMORY;
    }
}

int crx_encoded_parse_device(const crx_encoded* enc, const uint8_t* data, crx_update** out, char* err, size_t errlen) {
    if (!enc || !out || !data || enc->e.part || !enc->e.device) return CRX_BAD_ARGUMENT;
    *out = nullptr;
    const crx::Encoded& E = enc->e;
    try {
        // the prepared parse is taken once; the context lock orders calls on one result
        std::unique_lock<std::mutex> lock;
        if (E.ctx) lock = std::unique_lock<std::mutex>(E.ctx->mu);
        const int64_t len = int64_t(E.size());
        if (E.pre) {   // parsed up to the block table while the encoder's last kernels ran
            crx_update* u = new crx_update;
            u->u = std::move(*E.pre);
            E.pre.reset();
            u->head = E.head;   // the names move to this copy of the header
            for (crx::TensorHeader& h : u->u.tensors) h.name = u->head.data() + (h.name - E.head.data());
            std::string msg;
            if (crx::resume_after_table(E.len_varint.data(), int64_t(E.len_varint.size()), len, &u->u, &msg) != crx::kOk ||
                uint64_t(u->u.payload_len) != E.payload_len) {
                delete u;
                put_err(err, errlen, "crx_encoded_parse_device: internal: the encoder's header does not parse (" + msg + ")");
                return CRX_CUDA_ERROR;
            }
            u->u.total_bits = E.total_bits;
            u->u.block_table_device = data + E.head.size();
            u->u.payload_device = data + u->u.payload_offset;
            *out = u;
            return CRX_OK;
        }
        // the update's bytes as the host parser sees them in a device parse: the header, then (past
        // the block table, which it does not read) the length varint
        const int64_t t0 = int64_t(E.head.size()), t1 = t0 + 4 * E.n_blocks;
        const int64_t w1 = t1 + int64_t(E.len_varint.size());
        std::vector<uint8_t> head;
        {
            std::lock_guard<std::mutex> pl(g_pool_mu);
            if (!g_head_pool.empty()) {
                head.swap(g_head_pool.back());
                g_head_pool.pop_back();
            }
        }
        if (head.size() < size_t(w1)) head.resize(size_t(w1));
        std::memcpy(head.data(), E.head.data(), size_t(t0));
        std::memcpy(head.data() + t1, E.len_varint.data(), E.len_varint.size());
        crx_update* u = new crx_update;
        std::string msg;
        int64_t nd = 0;
        crx::Status s = crx::parse_head_device_table(head.data(), t0, len, 0, &u->u, &nd, &msg);
        if (s == crx::kNeedMore && u->u.block_table_offset == t0)
            s = crx::resume_head_device_table(head.data(), w1, len, &u->u, &nd, &msg);
        if (s != crx::kOk || u->u.payload_offset != w1 || uint64_t(u->u.payload_len) != E.payload_len) {
            delete u;
            std::lock_guard<std::mutex> pl(g_pool_mu);
            if (g_head_pool.size() < kHeadPoolMax) g_head_pool.push_back(std::move(head));
            put_err(err, errlen, "crx_encoded_parse_device: internal: the encoder's header does not parse (" + msg + ")");
            return CRX_CUDA_ERROR;
        }
        u->u.total_bits = E.total_bits;
        u->u.block_table_device = data + t0;
        u->u.payload_device = data + w1;
        u->u.payload = nullptr;
        u->head.swap(head);   // the header's pointers stay valid: the vector's buffer moves with it
        *out = u;
        return CRX_OK;
    } catch (const std::bad_alloc&) {
        put_err(err, errlen, "crx_encoded_parse_device: out of host memory");
        return CRX_NO_MEMORY;
    }
}

int64_t crx_update_n_tensors(const crx_update* u) { return u ? int64_t(u->u.tensors.size()) : -1; }
int64_t crx_update_changes(const crx_update* u) { return u ? u->u.total_changes : -1; }

int crx_update_tensor(const crx_update* u, int64_t i, const uint8_t** name, int64_t* name_len, int64_t* numel,
                      uint64_t* checksum, int32_t* n_groups) {
    if (!u || i < 0 || i >= int64_t(u->u.tensors.size())) return CRX_BAD_ARGUMENT;
    const crx::TensorHeader& h = u->u.tensors[size_t(i)];
    if (name) *name = h.name;
    if (name_len) *name_len = h.name_len;
    if (numel) *numel = h.numel;
    if (checksum) *checksum = h.checksum;
    if (n_groups) *n_groups = int32_t(h.groups.size());
    return CRX_OK;
}

int crx_update_tensor_table(const crx_update* u, const uint8_t** names, int64_t* name_lens, int64_t* numels,
                            uint64_t* checksums) {
    if (!u) return CRX_BAD_ARGUMENT;
    for (size_t i = 0; i < u->u.tensors.size(); ++i) {
        const crx::TensorHeader& h = u->u.tensors[i];
        if (names) names[i] = h.name;
        if (name_lens) name_lens[i] = h.name_len;
        if (numels) numels[i] = h.numel;
        if (checksums) checksums[i] = h.checksum;
    }
    return CRX_OK;
}

int crx_update_group(const crx_update* u, int64_t i, int32_t k, int32_t* exponent, int64_t* count, int32_t* rice) {
    if (!u || i < 0 || i >= int64_t(u->u.tensors.size())) return CRX_BAD_ARGUMENT;
    const auto& gs = u->u.tensors[size_t(i)].groups;
    if (k < 0 || k >= int32_t(gs.size())) return CRX_BAD_ARGUMENT;
    if (exponent) *exponent = gs[size_t(k)].exponent;
    if (count) *count = gs[size_t(k)].count;
    if (rice) *rice = gs[size_t(k)].rice;
    return CRX_OK;
}

int32_t crx_update_n_tables(const crx_update* u) { return u ? int32_t(u->u.tables.size()) : -1; }

int crx_update_table(const crx_update* u, int32_t k, int32_t* exponent, int64_t* n_symbols) {
    if (!u || k < 0 || k >= int32_t(u->u.tables.size())) return CRX_BAD_ARGUMENT;
    if (exponent) *exponent = u->u.tables[size_t(k)].exponent;
    if (n_symbols) *n_symbols = int64_t(u->u.tables[size_t(k)].symbols.size());
    return CRX_OK;
}

int crx_update_table_entries(const crx_update* u, int32_t k, uint32_t* symbols, uint8_t* lengths) {
    if (!u || k < 0 || k >= int32_t(u->u.tables.size())) return CRX_BAD_ARGUMENT;
    const crx::Table& t = u->u.tables[size_t(k)];
    if (symbols) std::memcpy(symbols, t.symbols.data(), 4 * t.symbols.size());
    if (lengths) std::memcpy(lengths, t.lengths.data(), t.lengths.size());
    return CRX_OK;
}

int64_t crx_update_n_blocks(const crx_update* u) { return u ? u->u.n_blocks : -1; }

int crx_update_block_bits(const crx_update* u, uint32_t* out) {
    if (!u || !out) return CRX_BAD_ARGUMENT;
    if (u->u.block_table) {
        std::memcpy(out, u->u.block_table, 4 * size_t(u->u.n_blocks));
    } else if (u->u.n_blocks) {   // the table stayed in device memory
        if (!u->u.block_table_device ||
            cudaMemcpy(out, u->u.block_table_device, 4 * size_t(u->u.n_blocks), cudaMemcpyDeviceToHost) != cudaSuccess)
            return CRX_CUDA_ERROR;
    }
    return CRX_OK;
}

int crx_update_payload(const crx_update* u, const uint8_t** data, int64_t* len) {
    if (!u) return CRX_BAD_ARGUMENT;
    if (data) *data = u->u.payload;
    if (len) *len = u->u.payload ? u->u.payload_len : 0;   // none at hand: head-only or device update
    return CRX_OK;
}

void crx_update_free(crx_update* u) { delete u; }

int crx_apply(crx_ctx* ctx, const crx_update* u, int16_t* const* weights, const uint64_t* cached_checksums,
              const uint8_t* has_cached, void* stream, int64_t* changed, char* err, size_t errlen) {
    if (!ctx || !u || !changed || (!u->u.tensors.empty() && !weights)) {
        put_err(err, errlen, "crx_apply: bad argument");
        return CRX_BAD_ARGUMENT;
    }
    if (has_cached && !cached_checksums) {
        put_err(err, errlen, "crx_apply: has_cached without cached_checksums");
        return CRX_BAD_ARGUMENT;
    }
    try {
        std::lock_guard<std::mutex> lock(ctx->c.mu);
        DeviceGuard g(ctx->c.device);
        std::string msg;
        const crx::Status s = crx::apply_impl(ctx->c, u->u, weights, cached_checksums, has_cached,
                                              static_cast<cudaStream_t>(stream), changed, &msg);
        if (s != crx::kOk) {
            put_err(err, errlen, msg);
            return int(s);
        }
        return CRX_OK;
    } catch (const std::bad_alloc&) {
        put_err(err, errlen, "crx_apply: out of host memory");
        return CRX_NO_MEMORY;
    } catch (const std::exception& ex) {
        put_err(err, errlen, std::string("crx_apply: ") + ex.what());
        return CRX_CUDA_ERROR;
    }
}

int crx_apply_to_host(crx_ctx* ctx, const crx_update* u, int16_t* const* device_copies, int16_t* const* host_weights,
                      const uint64_t* cached_checksums, const uint8_t* has_cached, void* stream, int64_t* changed,
                      char* err, size_t errlen) {
    if (!ctx || !u || !changed || (!u->u.tensors.empty() && (!device_copies || !host_weights))) {
        put_err(err, errlen, "crx_apply_to_host: bad argument");
        return CRX_BAD_ARGUMENT;
    }
    if (has_cached && !cached_checksums) {
        put_err(err, errlen, "crx_apply_to_host: has_cached without cached_checksums");
        return CRX_BAD_ARGUMENT;
    }
    try {
        std::lock_guard<std::mutex> lock(ctx->c.mu);
        DeviceGuard g(ctx->c.device);
        std::string msg;
        const crx::Status s = crx::apply_impl(ctx->c, u->u, device_copies, cached_checksums, has_cached,
                                              static_cast<cudaStream_t>(stream), changed, &msg, nullptr, nullptr,
                                              host_weights);
        if (s != crx::kOk) {
            put_err(err, errlen, msg);
            return int(s);
        }
        return CRX_OK;
    } catch (const std::bad_alloc&) {
        put_err(err, errlen, "crx_apply_to_host: out of host memory");
        return CRX_NO_MEMORY;
    } catch (const std::exception& ex) {
        put_err(err, errlen, std::string("crx_apply_to_host: ") + ex.what());
        return CRX_CUDA_ERROR;
    }
}

int crx_apply_versioned(crx_ctx* ctx, const crx_update* u, int16_t* const* weights, const uint64_t* cached_checksums,
                        const uint8_t* has_cached, const uint64_t* versions, const uint8_t* has_version, void* stream,
                        int64_t* changed, char* err, size_t errlen) {
    if (!ctx || !u || !changed || (!u->u.tensors.empty() && !weights) || (has_version && !versions)) {
        put_err(err, errlen, "crx_apply_versioned: bad argument");
        return CRX_BAD_ARGUMENT;
    }
    if (has_cached && !cached_checksums) {
        put_err(err, errlen, "crx_apply_versioned: has_cached without cached_checksums");
        return CRX_BAD_ARGUMENT;
    }
    try {
        std::lock_guard<std::mutex> lock(ctx->c.mu);
        DeviceGuard g(ctx->c.device);
        std::string msg;
        const crx::Status s = crx::apply_impl(ctx->c, u->u, weights, cached_checksums, has_cached,
                                              static_cast<cudaStream_t>(stream), changed, &msg, versions, has_version);
        if (s != crx::kOk) {
            put_err(err, errlen, msg);
            return int(s);
        }
        return CRX_OK;
    } catch (const std::bad_alloc&) {
        put_err(err, errlen, "crx_apply_versioned: out of host memory");
        return CRX_NO_MEMORY;
    } catch (const std::exception& ex) {
        put_err(err, errlen, std::string("crx_apply_versioned: ") + ex.what());
        return CRX_CUDA_ERROR;
    }
}

uint64_t crx_ctx_hist_cache_hits(crx_ctx* ctx) { return ctx ? ctx->c.hist_hits : 0; }

int crx_huffman_lengths(const uint64_t* counts, int64_t n, uint8_t* lengths) {
    if (n <= 0 || !counts || !lengths) return CRX_BAD_ARGUMENT;
    try {
        crx::huffman_lengths(counts, n, lengths);
        return CRX_OK;
    } catch (const std::bad_alloc&) {
        return CRX_NO_MEMORY;
    }
}

uint64_t crx_ctx_launches(crx_ctx* ctx) { return ctx ? ctx->c.launches : 0; }
uint64_t crx_parse_device_launches(void) { return g_parse_launches.load(); }

int crx_ctx_profile(crx_ctx* ctx, int enable) {
    if (!ctx) return CRX_BAD_ARGUMENT;
    std::lock_guard<std::mutex> lock(ctx->c.mu);
    ctx->c.profile = enable != 0;
    if (enable) {
        ctx->c.marks.clear();
        ctx->c.ev_used = 0;
    }
    return CRX_OK;
}

int32_t crx_ctx_kernel_times(crx_ctx* ctx, char* names, size_t names_len, double* ms, int32_t* counts, int32_t max) {
    if (!ctx) return -1;
    std::lock_guard<std::mutex> lock(ctx->c.mu);
    DeviceGuard g(ctx->c.device);
    std::vector<std::string> order;
    std::vector<double> tot;
    std::vector<int32_t> cnt;
    for (const crx::ProfMark& m : ctx->c.marks) {
        float t = 0.f;
        if (cudaEventSynchronize(m.b) != cudaSuccess || cudaEventElapsedTime(&t, m.a, m.b) != cudaSuccess) {
            cudaGetLastError();
            continue;
        }
        size_t k = 0;
        while (k < order.size() && order[k] != m.name) ++k;
        if (k == order.size()) { order.push_back(m.name); tot.push_back(0.0); cnt.push_back(0); }
        tot[k] += t;
        cnt[k] += 1;
    }
    std::string joined;
    for (size_t k = 0; k < order.size(); ++k) {
        if (int32_t(k) < max) {
            if (ms) ms[k] = tot[k];
            if (counts) counts[k] = cnt[k];
        }
        joined += order[k];
        joined += '\n';
    }
    if (names && names_len) std::snprintf(names, names_len, "%s", joined.c_str());
    return int32_t(order.size());
}

int32_t crx_ctx_kernel_gaps(crx_ctx* ctx, char* names, size_t names_len, double* gap_ms, int32_t max) {
    if (!ctx) return -1;
    std::lock_guard<std::mutex> lock(ctx->c.mu);
    DeviceGuard g(ctx->c.device);
    std::vector<std::string> order;
    std::vector<double> tot;
    const crx::ProfMark* prev = nullptr;
    for (const crx::ProfMark& m : ctx->c.marks) {
        float t = 0.f;
        const bool ok = prev && prev->s == m.s && cudaEventSynchronize(m.a) == cudaSuccess &&
                        cudaEventElapsedTime(&t, prev->b, m.a) == cudaSuccess;
        if (!ok) cudaGetLastError();
        prev = &m;
        if (!ok) continue;
        size_t k = 0;
        while (k < order.size() && order[k] != m.name) ++k;
        if (k == order.size()) { order.push_back(m.name); tot.push_back(0.0); }
        tot[k] += t > 0.f ? t : 0.f;
    }
    std::string joined;
    for (size_t k = 0; k < order.size(); ++k) {
        if (int32_t(k) < max && gap_ms) gap_ms[k] = tot[k];
        joined += order[k];
        joined += '\n';
    }
    if (names && names_len) std::snprintf(names, names_len, "%s", joined.c_str());
    return int32_t(order.size());
}

int crx_checksum(crx_ctx* ctx, const int16_t* data, int64_t n, void* stream, uint64_t* out, char* err, size_t errlen) {
    if (!ctx || !out || n < 0 || (n && !data)) return CRX_BAD_ARGUMENT;
    try {
        std::lock_guard<std::mutex> lock(ctx->c.mu);
        DeviceGuard g(ctx->c.device);
        std::string msg;
        const crx::Status s = crx::checksum_impl(ctx->c, data, n, static_cast<cudaStream_t>(stream), out, &msg);
        if (s != crx::kOk) {
            put_err(err, errlen, msg);
            return int(s);
        }
        return CRX_OK;
    } catch (const std::exception& ex) {
        put_err(err, errlen, std::string("crx_checksum: ") + ex.what());
        return CRX_CUDA_ERROR;
    }
}

int crx_size_stats(crx_ctx* ctx, int32_t n_tensors, const int16_t* const* prev, const int16_t* const* cur,
                   const int64_t* numel, void* stream, uint64_t* out, char* err, size_t errlen) {
    if (!ctx || !out || n_tensors < 0 || (n_tensors && (!prev || !cur || !numel))) return CRX_BAD_ARGUMENT;
    static_assert(CRX_SIZE_STATS_WORDS == 3 + 64 + 2 * 65536, "stats layout");
    try {
        if (crx::size_stats_words() != CRX_SIZE_STATS_WORDS) return CRX_CUDA_ERROR;
        std::lock_guard<std::mutex> lock(ctx->c.mu);
        DeviceGuard g(ctx->c.device);
        std::string msg;
        const crx::Status s = crx::size_stats_impl(ctx->c, n_tensors, prev, cur, numel, static_cast<cudaStream_t>(stream),
                                                   out, &msg);
        if (s != crx::kOk) {
            put_err(err, errlen, msg);
            return int(s);
        }
        return CRX_OK;
    } catch (const std::exception& ex) {
        put_err(err, errlen, std::string("crx_size_stats: ") + ex.what());
        return CRX_CUDA_ERROR;
    }
}

}  // extern "C"
