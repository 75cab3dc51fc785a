// runtime.cu -- device contexts, stream-ordered pool, staging, errors.
// See runtime.h for the mapping to the reference's Vulkan runtime.
#include "runtime.h"

#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <map>
#include <tuple>

namespace nxv {

std::atomic<unsigned long> g_launches{0};

namespace {

constexpr int kMaxDevices = 64;
constexpr size_t kPoolCapPerSize = 64;  // c_src/nx_vulkan_shim.cpp:47

std::mutex g_init_mu;
Device* g_devices[kMaxDevices] = {};
int g_default_device = -1;
std::atomic<bool> g_inited{false};
bool g_sync_mode = false;

std::atomic<unsigned long> g_hits{0}, g_misses{0}, g_freed{0};

thread_local int tl_device = -1;
thread_local cudaStream_t tl_stream = nullptr;
thread_local bool tl_stream_set = false;
thread_local int tl_cuda_current = -1;
thread_local char tl_err[512] = {0};

std::mutex g_scratch_mu;
// (device, stream, slot) -> (region, bytes)
std::map<std::tuple<int, cudaStream_t, int>, std::pair<void*, size_t>> g_scratch;

int init_one(int id) {
    if (id < 0 || id >= kMaxDevices) {
        set_error("device id %d out of range", id);
        return E_ARG;
    }
    if (g_devices[id]) return OK;
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0) {
        set_error("no CUDA device: %s", cudaGetErrorString(e));
        return E_INIT;
    }
    if (id >= count) {
        set_error("device %d not present (%d devices)", id, count);
        return E_INIT;
    }
    NXV_CK(cudaSetDevice(id));
    Device* d = new Device();
    d->id = id;
    cudaDeviceProp prop;
    NXV_CK(cudaGetDeviceProperties(&prop, id));
    d->name = prop.name;
    d->sm_count = prop.multiProcessorCount;
    d->l2_bytes = (size_t)prop.l2CacheSize;
    NXV_CK(cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking));
    cudaMemPool_t mp;
    NXV_CK(cudaDeviceGetDefaultMemPool(&mp, id));
    uint64_t thr = UINT64_MAX;
    NXV_CK(cudaMemPoolSetAttribute(mp, cudaMemPoolAttrReleaseThreshold, &thr));
    for (int s = 0; s < Device::kSlots; s++) {
        NXV_CK(cudaMallocHost(&d->staging[s], Device::kSlotBytes));
        NXV_CK(cudaEventCreateWithFlags(&d->slot_ev[s], cudaEventDisableTiming));
    }
    g_devices[id] = d;
    tl_cuda_current = id;
    return OK;
}

int make_current(int id) {
    if (tl_cuda_current != id) {
        NXV_CK(cudaSetDevice(id));
        tl_cuda_current = id;
    }
    return OK;
}

}  // namespace

bool fast_f32() {
    const char* v = getenv("NXV_EXACT_F32");
    return !(v && atoi(v) != 0);
}

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(tl_err, sizeof(tl_err), fmt, ap);
    va_end(ap);
}

int cuda_fail(cudaError_t e, const char* what) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return E_CUDA;
}

const char* last_error() { return tl_err; }

bool is_initialised() { return g_inited.load(); }

int init_default() {
    std::lock_guard<std::mutex> lk(g_init_mu);
    if (g_inited.load()) return OK;
    const char* env = getenv("NXV_DEVICES");
    g_sync_mode = getenv("NXV_SYNC") && atoi(getenv("NXV_SYNC")) != 0;
    std::vector<int> ids;
    if (env && *env) {
        const char* p = env;
        while (*p) {
            char* end;
            long v = strtol(p, &end, 10);
            if (end == p) break;
            ids.push_back((int)v);
            p = (*end == ',') ? end + 1 : end;
        }
    }
    if (ids.empty()) ids.push_back(0);
    for (int id : ids) {
        int rc = init_one(id);
        if (rc != OK) return rc;
    }
    g_default_device = ids[0];
    g_inited.store(true);
    return OK;
}

int init_devices(const int* ids, int n) {
    if (!ids || n <= 0) return E_NULL;
    std::lock_guard<std::mutex> lk(g_init_mu);
    g_sync_mode = getenv("NXV_SYNC") && atoi(getenv("NXV_SYNC")) != 0;
    for (int i = 0; i < n; i++) {
        int rc = init_one(ids[i]);
        if (rc != OK) return rc;
    }
    g_default_device = ids[0];
    tl_device = ids[0];
    g_inited.store(true);
    return OK;
}

void destroy_all() {
    std::lock_guard<std::mutex> lk(g_init_mu);
    if (!g_inited.load()) return;
    pool_clear();
    {
        std::lock_guard<std::mutex> sk(g_scratch_mu);
        for (auto& kv : g_scratch) {
            cudaSetDevice(std::get<0>(kv.first));
            cudaFree(kv.second.first);
        }
        g_scratch.clear();
    }
    for (int i = 0; i < kMaxDevices; i++) {
        Device* d = g_devices[i];
        if (!d) continue;
        cudaSetDevice(i);
        cudaStreamSynchronize(d->stream);
        for (int s = 0; s < Device::kSlots; s++) {
            if (d->staging[s]) cudaFreeHost(d->staging[s]);
            if (d->slot_ev[s]) cudaEventDestroy(d->slot_ev[s]);
        }
        cudaStreamDestroy(d->stream);
        delete d;
        g_devices[i] = nullptr;
    }
    g_default_device = -1;
    tl_device = -1;
    tl_cuda_current = -1;
    tl_stream_set = false;
    g_inited.store(false);
}

Device* device(int id) {
    if (id < 0 || id >= kMaxDevices) return nullptr;
    return g_devices[id];
}

static Device* current_device() {
    int id = (tl_device >= 0) ? tl_device : g_default_device;
    return device(id);
}

int set_current(int id) {
    if (!g_inited.load()) return E_INIT;
    if (!device(id)) {
        set_error("device %d not initialised", id);
        return E_ARG;
    }
    tl_device = id;
    tl_stream_set = false;
    return make_current(id);
}

int set_stream(cudaStream_t s) {
    if (!g_inited.load()) return E_INIT;
    tl_stream = s;
    tl_stream_set = (s != nullptr);
    return OK;
}

Buf* as_buf(const void* h) {
    Buf* b = (Buf*)h;
    if (!b || b->magic != kBufMagic) return nullptr;
    return b;
}

int begin(Ctx& c, std::initializer_list<const void*> bufs) {
    if (!g_inited.load()) {
        set_error("nxv_init has not run");
        return E_INIT;
    }
    Device* d = current_device();
    if (!d) {
        set_error("no current device");
        return E_INIT;
    }
    int rc = make_current(d->id);
    if (rc) return rc;
    for (const void* h : bufs) {
        if (!h) continue;
        Buf* b = as_buf(h);
        if (!b) {
            set_error("not an nxv buffer handle");
            return E_ARG;
        }
        if (b->device != d->id) {
            set_error("buffer lives on device %d, current device is %d", b->device, d->id);
            return E_ARG;
        }
    }
    c.dev = d;
    c.stream = tl_stream_set ? tl_stream : d->stream;
    return OK;
}

int finish(Ctx& c) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "kernel launch");
    if (g_sync_mode) NXV_CK(cudaStreamSynchronize(c.stream));
    return OK;
}

int sync(Ctx& c) {
    NXV_CK(cudaStreamSynchronize(c.stream));
    return OK;
}

void* scratch(Ctx& c, size_t bytes, int slot) {
    if (bytes == 0) bytes = 256;
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    auto key = std::make_tuple(c.dev->id, c.stream, slot);
    auto it = g_scratch.find(key);
    if (it != g_scratch.end() && it->second.second >= bytes) return it->second.first;
    if (it != g_scratch.end()) {
        cudaFreeAsync(it->second.first, c.stream);
        g_scratch.erase(it);
    }
    size_t sz = 1 << 20;
    while (sz < bytes) sz <<= 1;
    void* p = nullptr;
    if (cudaMallocAsync(&p, sz, c.stream) != cudaSuccess) {
        set_error("scratch allocation of %zu bytes failed", sz);
        return nullptr;
    }
    g_scratch[key] = std::make_pair(p, sz);
    return p;
}

// True when none of the inputs [p, p + bytes) overlaps the output of the last
// programmatic launch on c.stream; then records [out, out + bytes) as that
// output (kernels with a smaller output record more than they write, which
// only makes a later early load less likely).
bool pdl_independent_and_record(Ctx& c, const void* const* ins, int nin, size_t bytes,
                                const void* out) {
    std::lock_guard<std::mutex> lk(c.dev->pdl_mu);
    auto it = c.dev->pdl_last.find(c.stream);
    bool indep = true;
    if (it != c.dev->pdl_last.end()) {
        const uintptr_t lo = it->second.first, hi = lo + it->second.second;
        for (int q = 0; q < nin; q++) {
            const uintptr_t a = (uintptr_t)ins[q], b = a + bytes;
            if (a < hi && lo < b) indep = false;
        }
    }
    c.dev->pdl_last[c.stream] = {(uintptr_t)out, bytes};
    return indep;
}

// A programmatic launch that keeps no record of its output (its kernel lets
// the next kernel start before it completes): no later kernel may load early.
void pdl_record_all(Ctx& c) {
    std::lock_guard<std::mutex> lk(c.dev->pdl_mu);
    c.dev->pdl_last[c.stream] = {(uintptr_t)0, ~(size_t)0};
}

std::string spv_base(const char* spv_path) {
    if (!spv_path) return std::string();
    const char* s = strrchr(spv_path, '/');
    return std::string(s ? s + 1 : spv_path);
}

// ---- pool -----------------------------------------------------------------

void* buf_alloc(size_t n_bytes) {
    Ctx c;
    if (begin(c, {}) != OK) return nullptr;
    Device* d = c.dev;
    {
        std::lock_guard<std::mutex> lk(d->pool_mu);
        auto it = d->pool.find(n_bytes);
        if (it != d->pool.end() && !it->second.empty()) {
            Buf* b = it->second.back();
            it->second.pop_back();
            if (it->second.empty()) d->pool.erase(it);
            g_hits++;
            return b;
        }
    }
    g_misses++;
    Buf* b = new Buf{kBufMagic, d->id, nullptr, n_bytes, true};
    if (n_bytes > 0) {
        cudaError_t e = cudaMallocAsync(&b->ptr, n_bytes, c.stream);
        if (e != cudaSuccess) {
            cuda_fail(e, "cudaMallocAsync");
            cudaGetLastError();
            delete b;
            return nullptr;
        }
    }
    return b;
}

static void release(Buf* b, cudaStream_t s) {
    if (b->owned && b->ptr) cudaFreeAsync(b->ptr, s);
    b->magic = 0;
    delete b;
}

void buf_free(void* h) {
    Buf* b = as_buf(h);
    if (!b) return;
    if (!b->owned) {
        b->magic = 0;
        delete b;
        return;
    }
    Device* d = device(b->device);
    if (!d) return;
    {
        std::lock_guard<std::mutex> lk(d->pool_mu);
        auto& slot = d->pool[b->n_bytes];
        if (slot.size() < kPoolCapPerSize) {
            slot.push_back(b);
            return;
        }
    }
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(d->id);
    release(b, d->stream);
    if (prev >= 0 && prev != d->id) cudaSetDevice(prev);
    g_freed++;
}

void pool_clear() {
    for (int i = 0; i < kMaxDevices; i++) {
        Device* d = g_devices[i];
        if (!d) continue;
        cudaSetDevice(i);
        std::lock_guard<std::mutex> lk(d->pool_mu);
        for (auto& kv : d->pool)
            for (Buf* b : kv.second) {
                release(b, d->stream);
                g_freed++;
            }
        d->pool.clear();
        cudaStreamSynchronize(d->stream);
        cudaMemPool_t mp;
        if (cudaDeviceGetDefaultMemPool(&mp, i) == cudaSuccess) cudaMemPoolTrimTo(mp, 0);
    }
    if (tl_cuda_current >= 0) cudaSetDevice(tl_cuda_current);
}

void pool_stats(unsigned long* hits, unsigned long* misses, unsigned long* freed,
                unsigned long* size_classes, unsigned long* total_pooled) {
    if (hits) *hits = g_hits.load();
    if (misses) *misses = g_misses.load();
    if (freed) *freed = g_freed.load();
    unsigned long sc = 0, tp = 0;
    for (int i = 0; i < kMaxDevices; i++) {
        Device* d = g_devices[i];
        if (!d) continue;
        std::lock_guard<std::mutex> lk(d->pool_mu);
        for (auto& kv : d->pool) {
            if (kv.second.empty()) continue;
            sc++;
            tp += kv.second.size();
        }
    }
    if (size_classes) *size_classes = sc;
    if (total_pooled) *total_pooled = tp;
}

void* buf_wrap(void* p, size_t n) {
    Ctx c;
    if (begin(c, {}) != OK) return nullptr;
    return new Buf{kBufMagic, c.dev->id, p, n, false};
}

// ---- transfers --------------------------------------------------------------

static bool is_pinned(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost || a.type == cudaMemoryTypeManaged;
}

int buf_upload(void* h, const void* data, size_t n) {
    Ctx c;
    int rc = begin(c, {h});
    if (rc) return rc;
    Buf* b = as_buf(h);
    if (n > b->n_bytes) {
        set_error("upload of %zu bytes into a %zu-byte buffer", n, b->n_bytes);
        return E_ARG;
    }
    if (n == 0) return OK;
    if (is_pinned(data)) {
        NXV_CK(cudaMemcpyAsync(b->ptr, data, n, cudaMemcpyHostToDevice, c.stream));
        return sync(c);  // the caller may reuse `data` on return
    }
    // Pageable: pipeline through the pinned staging ring.  Each slot is
    // reused only after its previous copy has completed (slot event).
    Device* d = c.dev;
    std::lock_guard<std::mutex> lk(d->xfer_mu);
    size_t off = 0;
    int slot = 0;
    while (off < n) {
        size_t len = n - off < Device::kSlotBytes ? n - off : Device::kSlotBytes;
        NXV_CK(cudaEventSynchronize(d->slot_ev[slot]));
        memcpy(d->staging[slot], (const char*)data + off, len);
        NXV_CK(cudaMemcpyAsync((char*)b->ptr + off, d->staging[slot], len,
                               cudaMemcpyHostToDevice, c.stream));
        NXV_CK(cudaEventRecord(d->slot_ev[slot], c.stream));
        off += len;
        slot = (slot + 1) % Device::kSlots;
    }
    // Staging slots stay busy until their events fire; the host data has
    // been consumed already.  Wait anyway so the handle's bytes are ready
    // for any stream the caller uses next.
    return sync(c);
}

int buf_download(void* h, void* data, size_t n) {
    Ctx c;
    int rc = begin(c, {h});
    if (rc) return rc;
    Buf* b = as_buf(h);
    if (n > b->n_bytes) {
        set_error("download of %zu bytes from a %zu-byte buffer", n, b->n_bytes);
        return E_ARG;
    }
    if (n == 0) return sync(c);
    if (is_pinned(data)) {
        NXV_CK(cudaMemcpyAsync(data, b->ptr, n, cudaMemcpyDeviceToHost, c.stream));
        return sync(c);
    }
    Device* d = c.dev;
    std::lock_guard<std::mutex> lk(d->xfer_mu);
    size_t nchunks = (n + Device::kSlotBytes - 1) / Device::kSlotBytes;
    size_t issued = 0;
    auto issue = [&](size_t i) -> int {
        size_t off = i * Device::kSlotBytes;
        size_t len = n - off < Device::kSlotBytes ? n - off : Device::kSlotBytes;
        int s = (int)(i % Device::kSlots);
        NXV_CK(cudaMemcpyAsync(d->staging[s], (const char*)b->ptr + off, len,
                               cudaMemcpyDeviceToHost, c.stream));
        NXV_CK(cudaEventRecord(d->slot_ev[s], c.stream));
        return OK;
    };
    for (; issued < nchunks && issued < (size_t)Device::kSlots; issued++) {
        int r = issue(issued);
        if (r) return r;
    }
    for (size_t i = 0; i < nchunks; i++) {
        int s = (int)(i % Device::kSlots);
        NXV_CK(cudaEventSynchronize(d->slot_ev[s]));
        size_t off = i * Device::kSlotBytes;
        size_t len = n - off < Device::kSlotBytes ? n - off : Device::kSlotBytes;
        memcpy((char*)data + off, d->staging[s], len);
        if (issued < nchunks) {
            int r = issue(issued++);
            if (r) return r;
        }
    }
    return OK;
}

}  // namespace nxv
