// allocator.cpp -- caching device allocator of the kunlun backend on
// stream-ordered CUDA memory pools, plus a pinned host allocator.
//
// Counterpart of the reference's csrc/allocator.cpp (KunlunCachingAllocator,
// :72-465).  The reference keeps its own best-fit free list, waits on events
// with host-blocking synchronisation before reusing a block, and enforces a
// per-device budget and a 2 GiB single-allocation cap (:41-48, :131-145)
// because K200 xpu_malloc can hang.  Here each device has a cudaMemPool with
// an unlimited release threshold, so freed memory stays cached in the pool;
// a block is allocated and freed in stream order on the stream that was
// current at allocation, and record_stream() makes that free wait (on the
// device, not the host) for every other stream that used the block.  There
// is no size cap.  KUNLUN_MEMORY_FRACTION optionally bounds the pool.
#include <atomic>
#include <cstdlib>
#include <mutex>
#include <vector>

#include "kunlun.h"

namespace torch_kunlun {

void check_cuda(cudaError_t e, const char* what);

namespace {

constexpr int kMaxDevices = 64;

struct Block {
    void* ptr;
    size_t size;
    int device;
    cudaStream_t stream;             // allocation (and free) stream
    std::vector<cudaStream_t> uses;  // other streams recorded via record_stream
    std::mutex mu;
};

struct DeviceState {
    std::once_flag init;
    cudaMemPool_t pool = nullptr;
    std::atomic<size_t> allocated{0};
    std::atomic<size_t> peak{0};
    size_t limit = 0;  // 0 = no limit
};

DeviceState g_dev[kMaxDevices];

double env_fraction() {
    const char* v = std::getenv("KUNLUN_MEMORY_FRACTION");
    if (v == nullptr || *v == '\0') return 0.0;
    char* end = nullptr;
    const double f = std::strtod(v, &end);
    return (end == v || f <= 0.0 || f > 1.0) ? 0.0 : f;
}

DeviceState& state(int device) {
    TORCH_CHECK(device >= 0 && device < kMaxDevices, "kunlun: bad device ", device);
    DeviceState& s = g_dev[device];
    std::call_once(s.init, [&] {
        cudaMemPoolProps props = {};
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = device;
        check_cuda(cudaMemPoolCreate(&s.pool, &props), "cudaMemPoolCreate");
        uint64_t threshold = UINT64_MAX;  // never return cached memory implicitly
        check_cuda(cudaMemPoolSetAttribute(s.pool, cudaMemPoolAttrReleaseThreshold, &threshold),
                   "cudaMemPoolSetAttribute");
        const double f = env_fraction();
        if (f > 0.0) {
            size_t free_b = 0, total_b = 0;
            int prev = 0;
            cudaGetDevice(&prev);
            cudaSetDevice(device);
            cudaMemGetInfo(&free_b, &total_b);
            cudaSetDevice(prev);
            s.limit = static_cast<size_t>(f * static_cast<double>(total_b));
        }
    });
    return s;
}

size_t reserved_bytes(DeviceState& s) {
    uint64_t v = 0;
    cudaMemPoolGetAttribute(s.pool, cudaMemPoolAttrReservedMemCurrent, &v);
    return static_cast<size_t>(v);
}

void free_block(void* ctx) {
    Block* b = static_cast<Block*>(ctx);
    if (b == nullptr) return;
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != b->device) cudaSetDevice(b->device);
    cudaStream_t fs = b->stream;
    if (!stream_is_live(fs)) fs = nullptr;  // its stream was destroyed (and drained)
    {
        std::lock_guard<std::mutex> lk(b->mu);
        for (cudaStream_t u : b->uses) {
            if (u == fs || !stream_is_live(u)) continue;
            cudaEvent_t ev = nullptr;
            if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) == cudaSuccess) {
                cudaEventRecord(ev, u);
                cudaStreamWaitEvent(fs, ev, 0);
                cudaEventDestroy(ev);
            } else {
                cudaStreamSynchronize(u);
            }
        }
    }
    cudaFreeAsync(b->ptr, fs);
    g_dev[b->device].allocated.fetch_sub(b->size);
    if (prev != b->device) cudaSetDevice(prev);
    delete b;
}

class PoolAllocator final : public c10::Allocator {
   public:
    c10::DataPtr allocate(size_t n) override {
        const int device = current_device();
        const c10::Device dev(c10::DeviceType::PrivateUse1, static_cast<c10::DeviceIndex>(device));
        if (n == 0) return c10::DataPtr(nullptr, nullptr, &free_block, dev);
        DeviceState& s = state(device);
        if (s.limit != 0 && s.allocated.load() + n > s.limit) {
            TORCH_CHECK_WITH(OutOfMemoryError, false, "kunlun out of memory: request of ", n,
                             " bytes exceeds KUNLUN_MEMORY_FRACTION limit (", s.limit,
                             " bytes, ", s.allocated.load(), " allocated)");
        }
        cudaStream_t stream = current_stream(device);
        void* p = nullptr;
        cudaError_t e = cudaMallocFromPoolAsync(&p, n, s.pool, stream);
        if (e == cudaErrorMemoryAllocation) {
            cudaGetLastError();
            // Release everything cached in this pool and retry once.
            cudaDeviceSynchronize();
            cudaMemPoolTrimTo(s.pool, 0);
            e = cudaMallocFromPoolAsync(&p, n, s.pool, stream);
        }
        if (e != cudaSuccess) {
            cudaGetLastError();
            TORCH_CHECK_WITH(OutOfMemoryError, false, "kunlun out of memory allocating ", n,
                             " bytes on device ", device, ": ", cudaGetErrorString(e), " (",
                             s.allocated.load(), " bytes allocated, ", reserved_bytes(s),
                             " reserved)");
        }
        Block* b = new Block();
        b->ptr = p;
        b->size = n;
        b->device = device;
        b->stream = stream;
        const size_t now = s.allocated.fetch_add(n) + n;
        size_t peak = s.peak.load();
        while (now > peak && !s.peak.compare_exchange_weak(peak, now)) {
        }
        return c10::DataPtr(p, b, &free_block, dev);
    }

    c10::DeleterFnPtr raw_deleter() const override { return nullptr; }

    void copy_data(void* dest, const void* src, std::size_t count) const override {
        check_cuda(cudaMemcpy(dest, src, count, cudaMemcpyDeviceToDevice), "cudaMemcpy(copy_data)");
    }
};

PoolAllocator g_allocator;

// Pinned host memory: page-locked buffers DMA-able by every device.
void free_pinned(void* p) {
    if (p) cudaFreeHost(p);
}

class PinnedAllocator final : public c10::Allocator {
   public:
    c10::DataPtr allocate(size_t n) override {
        void* p = nullptr;
        if (n > 0) {
            check_cuda(cudaHostAlloc(&p, n, cudaHostAllocPortable), "cudaHostAlloc");
        }
        return c10::DataPtr(p, p, &free_pinned, c10::Device(c10::DeviceType::CPU));
    }
    c10::DeleterFnPtr raw_deleter() const override { return &free_pinned; }
    void copy_data(void* dest, const void* src, std::size_t count) const override {
        std::memcpy(dest, src, count);
    }
};

PinnedAllocator g_pinned;

}  // namespace

c10::Allocator* get_allocator() { return &g_allocator; }
c10::Allocator* get_pinned_allocator() { return &g_pinned; }

size_t memory_allocated(int device) {
    return g_dev[device < 0 ? current_device() : device].allocated.load();
}

size_t max_memory_allocated(int device) {
    return g_dev[device < 0 ? current_device() : device].peak.load();
}

void reset_peak_memory_stats(int device) {
    DeviceState& s = g_dev[device < 0 ? current_device() : device];
    s.peak.store(s.allocated.load());
}

size_t memory_reserved(int device) {
    device = device < 0 ? current_device() : device;
    if (g_dev[device].pool == nullptr) return 0;
    return reserved_bytes(g_dev[device]);
}

void empty_cache() {
    int prev = current_device();
    for (int d = 0; d < kMaxDevices; ++d) {
        if (g_dev[d].pool == nullptr) continue;
        cudaSetDevice(d);
        cudaDeviceSynchronize();
        cudaMemPoolTrimTo(g_dev[d].pool, 0);
    }
    cudaSetDevice(prev);
}

void record_data_ptr_on_stream(const c10::DataPtr& data_ptr, const c10::Stream& stream) {
    if (data_ptr.get_deleter() != &free_block) return;
    Block* b = static_cast<Block*>(data_ptr.get_context());
    if (b == nullptr) return;
    cudaStream_t s = stream_handle(stream.id());
    std::lock_guard<std::mutex> lk(b->mu);
    if (s == b->stream) return;
    for (cudaStream_t u : b->uses)
        if (u == s) return;
    b->uses.push_back(s);
}

int device_of_ptr(void* ptr) {
    if (ptr == nullptr) return -1;
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, ptr) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    return attr.type == cudaMemoryTypeDevice ? attr.device : -1;
}

bool is_pinned_ptr(const void* ptr) {
    if (ptr == nullptr) return false;
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, ptr) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return attr.type == cudaMemoryTypeHost;
}

}  // namespace torch_kunlun
