// runtime.h -- CUDA runtime layer under the nxv_* C ABI.
//
// Replaces the reference's Vulkan runtime (c_src/spirit/.../
// Backend_par_vulkan.cpp: vk_init 67-168, buf_alloc 189-215, staging
// upload/download 240-304, synchronous dispatch 436-481) and the shim's
// buffer pool (c_src/nx_vulkan_shim.cpp:47-77, 174-240):
//   - one Device per initialised GPU: a non-blocking stream, the device's
//     default cudaMemPool (release threshold = max, so freed memory stays
//     mapped), a pinned staging ring for pageable host transfers;
//   - an exact-size free-list pool in front of cudaMallocAsync with the
//     reference's cap of 64 buffers per size class and its counters;
//   - a per-thread current device and optional caller stream.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <atomic>
#include <map>
#include <mutex>
#include <string>
#include <vector>

namespace nxv {

constexpr uint32_t kBufMagic = 0x4E585642u;  // "NXVB"

struct Buf {
    uint32_t magic;
    int device;
    void* ptr;
    size_t n_bytes;
    bool owned;  // false for nxv_buf_wrap views
};

struct Device {
    int id = -1;
    cudaStream_t stream = nullptr;
    std::string name;
    int sm_count = 0;
    size_t l2_bytes = 0;
    std::mutex pool_mu;
    std::map<size_t, std::vector<Buf*>> pool;
    // pinned staging ring for pageable transfers
    static constexpr int kSlots = 4;
    static constexpr size_t kSlotBytes = size_t(8) << 20;
    void* staging[kSlots] = {nullptr, nullptr, nullptr, nullptr};
    cudaEvent_t slot_ev[kSlots] = {nullptr, nullptr, nullptr, nullptr};
    std::mutex xfer_mu;
    // Held by an op from its scratch() call until its last launch is
    // enqueued, so two host threads sharing a stream cannot interleave
    // their multi-launch ops on the same scratch region.
    std::recursive_mutex scratch_mu;
    // Per stream: the output range [ptr, ptr + bytes) of the last kernel
    // this library launched with programmatic dependent launch
    // (k_elementwise.cu); the next such kernel may read its inputs before the
    // previous one completes only when they do not overlap this range.
    std::mutex pdl_mu;
    std::map<cudaStream_t, std::pair<uintptr_t, size_t>> pdl_last;
};

// Error codes of the C ABI.
enum : int { OK = 0, E_NULL = -1, E_KERNEL = -2, E_ARG = -3, E_CUDA = -4, E_INIT = -5 };

// Per-call context: the current device and the stream to launch on.
struct Ctx {
    Device* dev;
    cudaStream_t stream;
};

// Library state.
bool is_initialised();
int init_default();
int init_devices(const int* ids, int n);
void destroy_all();
Device* device(int id);
int set_current(int id);
int set_stream(cudaStream_t s);

// Begin an op: check init, resolve the current device, make it current on
// this thread and validate that every non-null buffer belongs to it.
int begin(Ctx& c, std::initializer_list<const void*> bufs);
// After launches: check for launch errors; in NXV_SYNC mode also wait.
int finish(Ctx& c);
int sync(Ctx& c);

Buf* as_buf(const void* h);
inline void* dptr(const void* h) { return h ? static_cast<const Buf*>(h)->ptr : nullptr; }
inline size_t nbytes(const void* h) { return h ? static_cast<const Buf*>(h)->n_bytes : 0; }

// Scratch memory: returns a device region of at least `bytes`, valid for
// work queued on c.stream until the next scratch() call with the same slot
// on this device.  Callers hold a ScratchGuard for the whole op (see
// Device::scratch_mu).  Slot 0 belongs to the op entry points; slot 1 to the
// GEMM (its stream-K workspace), which ops holding slot 0 may call; slot 2
// to the one-call NUTS transition (its tree state and leaf store), which
// calls the chain launcher (slot 0) between its own kernels.
enum { kScratchOp = 0, kScratchGemm = 1, kScratchNuts = 2 };
void* scratch(Ctx& c, size_t bytes, int slot = kScratchOp);
struct ScratchGuard {
    std::lock_guard<std::recursive_mutex> lk;
    explicit ScratchGuard(Ctx& c) : lk(c.dev->scratch_mu) {}
};

// Error reporting.
void set_error(const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* what);
const char* last_error();

// Launch accounting (every kernel launch of this library bumps it).
extern std::atomic<unsigned long> g_launches;
inline void count_launch(unsigned long k = 1) { g_launches.fetch_add(k, std::memory_order_relaxed); }

// Programmatic dependent launch bookkeeping (Device::pdl_last): true when
// none of the nin inputs [p, p + bytes) overlaps the output of the last
// kernel launched with programmatic serialization on c.stream; records
// [out, out + bytes) as the output of the launch being made.
bool pdl_independent_and_record(Ctx& c, const void* const* ins, int nin, size_t bytes,
                                const void* out);
// For programmatic launches whose outputs are not tracked: marks all memory
// as the last output, so the next programmatic launch loads only after its
// wait.
void pdl_record_all(Ctx& c);

// spv basename helpers.
std::string spv_base(const char* spv_path);

// Pool API.
void* buf_alloc(size_t n_bytes);
void buf_free(void* h);
void pool_clear();
void pool_stats(unsigned long* hits, unsigned long* misses, unsigned long* freed,
                unsigned long* size_classes, unsigned long* total_pooled);
int buf_upload(void* h, const void* data, size_t n);
int buf_download(void* h, void* data, size_t n);
void* buf_wrap(void* p, size_t n);

}  // namespace nxv

#define NXV_CK(call)                                                      \
    do {                                                                  \
        cudaError_t e_ = (call);                                          \
        if (e_ != cudaSuccess) return ::nxv::cuda_fail(e_, #call);        \
    } while (0)
