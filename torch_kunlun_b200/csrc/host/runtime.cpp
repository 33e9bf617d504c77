// runtime.cpp -- devices, streams, events, device guard, PrivateUse1 hooks,
// CPU-fallback policy and the `_C` Python module of the kunlun backend.
//
// Counterpart of the reference's csrc/kunlun.cpp.  Differences by design:
// streams/events are CUDA streams/events (event query is non-blocking and
// elapsed_time works, unlike csrc/kunlun.cpp:573-582 and :752-755); there is
// no per-device launch mutex or stream-switch drain (csrc/kunlun.cpp:624-637);
// the XDNN version scan and cluster scheduling (csrc/kunlun.cpp:35-221) have no
// B200 equivalent -- set_cluster_budget is kept as an API-compatible no-op.
#include <ATen/detail/PrivateUse1HooksInterface.h>
#include <ATen/native/CPUFallback.h>
#include <c10/core/impl/DeviceGuardImplInterface.h>
#include <torch/csrc/Device.h>
#include <torch/library.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <mutex>
#include <unordered_set>
#include <vector>

#include "kunlun.h"

namespace torch_kunlun {

void check_cuda(cudaError_t e, const char* what) {
    TORCH_CHECK(e == cudaSuccess, "kunlun: ", what, " failed: ", cudaGetErrorString(e));
}

void check_tk(int rc, const char* what) {
    TORCH_CHECK(rc == TK_OK, "kunlun: ", what, " failed (status ", rc, "): ",
                tk_last_error_string());
}

// ---- devices ---------------------------------------------------------------

int device_count() {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

int current_device() {
    int d = 0;
    check_cuda(cudaGetDevice(&d), "cudaGetDevice");
    return d;
}

void set_device(int device) {
    TORCH_CHECK(device >= 0 && device < device_count(), "kunlun: invalid device index ", device);
    check_cuda(cudaSetDevice(device), "cudaSetDevice");
}

namespace {

struct DeviceRestore {
    int prev;
    explicit DeviceRestore(int dev) : prev(current_device()) {
        if (dev != prev) check_cuda(cudaSetDevice(dev), "cudaSetDevice");
    }
    ~DeviceRestore() { cudaSetDevice(prev); }
};

std::mutex g_stream_mu;
std::unordered_set<cudaStream_t> g_live_streams;
thread_local std::vector<int64_t> t_current;  // per device, 0 = default

}  // namespace

// ---- streams ---------------------------------------------------------------

cudaStream_t stream_handle(int64_t id) { return reinterpret_cast<cudaStream_t>(id); }

int64_t default_stream_id(int) { return 0; }

int64_t current_stream_id(int device) {
    if (device < 0) device = current_device();
    if (static_cast<size_t>(device) >= t_current.size()) return 0;
    return t_current[device];
}

cudaStream_t current_stream(int device) { return stream_handle(current_stream_id(device)); }

int64_t create_stream(int device, int priority) {
    DeviceRestore g(device);
    int lo = 0, hi = 0;
    cudaDeviceGetStreamPriorityRange(&lo, &hi);
    const int prio = std::max(hi, std::min(lo, lo - priority));
    cudaStream_t s = nullptr;
    check_cuda(cudaStreamCreateWithPriority(&s, cudaStreamNonBlocking, prio), "cudaStreamCreate");
    std::lock_guard<std::mutex> lk(g_stream_mu);
    g_live_streams.insert(s);
    return reinterpret_cast<int64_t>(s);
}

bool stream_is_live(cudaStream_t s) {
    if (s == nullptr) return true;
    std::lock_guard<std::mutex> lk(g_stream_mu);
    return g_live_streams.count(s) != 0;
}

void destroy_stream(int device, int64_t id) {
    if (id == 0) return;
    cudaStream_t s = stream_handle(id);
    {
        std::lock_guard<std::mutex> lk(g_stream_mu);
        if (g_live_streams.erase(s) == 0) return;
    }
    if (static_cast<size_t>(device) < t_current.size() && t_current[device] == id)
        t_current[device] = 0;
    DeviceRestore g(device);
    cudaStreamSynchronize(s);  // blocks freed on it must not be reused early
    cudaStreamDestroy(s);
}

void require_live(int64_t id) {
    TORCH_CHECK(stream_is_live(stream_handle(id)), "kunlun: stream ", id,
                " was destroyed or was not created by this backend");
}

void set_current_stream(int device, int64_t id) {
    if (device < 0) device = current_device();
    if (static_cast<size_t>(device) >= t_current.size()) t_current.resize(device + 1, 0);
    t_current[device] = id;
}

void synchronize_stream(int device, int64_t id) {
    require_live(id);
    DeviceRestore g(device);
    check_cuda(cudaStreamSynchronize(stream_handle(id)), "cudaStreamSynchronize");
}

bool stream_query(int device, int64_t id) {
    require_live(id);
    DeviceRestore g(device);
    cudaError_t e = cudaStreamQuery(stream_handle(id));
    if (e == cudaErrorNotReady) {
        cudaGetLastError();
        return false;
    }
    check_cuda(e, "cudaStreamQuery");
    return true;
}

void synchronize_all() {
    const int n = device_count();
    for (int d = 0; d < n; ++d) {
        DeviceRestore g(d);
        check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    }
}

// ---- events ----------------------------------------------------------------

int64_t event_create(int device, bool timing) {
    DeviceRestore g(device < 0 ? current_device() : device);
    cudaEvent_t e = nullptr;
    check_cuda(cudaEventCreateWithFlags(&e, timing ? cudaEventDefault : cudaEventDisableTiming),
               "cudaEventCreate");
    return reinterpret_cast<int64_t>(e);
}

void event_destroy(int64_t id) {
    if (id != 0) cudaEventDestroy(reinterpret_cast<cudaEvent_t>(id));
}

void event_record(int64_t ev, int device, int64_t stream_id) {
    require_live(stream_id);
    DeviceRestore g(device);
    check_cuda(cudaEventRecord(reinterpret_cast<cudaEvent_t>(ev), stream_handle(stream_id)),
               "cudaEventRecord");
}

void stream_wait_event(int device, int64_t stream_id, int64_t ev) {
    require_live(stream_id);
    DeviceRestore g(device);
    check_cuda(cudaStreamWaitEvent(stream_handle(stream_id), reinterpret_cast<cudaEvent_t>(ev), 0),
               "cudaStreamWaitEvent");
}

void event_synchronize(int64_t ev) {
    check_cuda(cudaEventSynchronize(reinterpret_cast<cudaEvent_t>(ev)), "cudaEventSynchronize");
}

bool event_query(int64_t ev) {
    cudaError_t e = cudaEventQuery(reinterpret_cast<cudaEvent_t>(ev));
    if (e == cudaErrorNotReady) {
        cudaGetLastError();
        return false;
    }
    check_cuda(e, "cudaEventQuery");
    return true;
}

double event_elapsed_ms(int64_t a, int64_t b) {
    float ms = 0.f;
    check_cuda(cudaEventElapsedTime(&ms, reinterpret_cast<cudaEvent_t>(a),
                                    reinterpret_cast<cudaEvent_t>(b)),
               "cudaEventElapsedTime");
    return ms;
}

// ---- fallback policy (same contract as the reference's KUNLUN_CPU_FALLBACK) --

namespace {
enum class FallbackPolicy { Default, Error, Warn, Silent };

FallbackPolicy fallback_policy() {
    static const FallbackPolicy p = [] {
        const char* v = std::getenv("KUNLUN_CPU_FALLBACK");
        const std::string s = v ? v : "";
        if (s == "silent") return FallbackPolicy::Silent;
        if (s == "warn") return FallbackPolicy::Warn;
        if (s == "error") return FallbackPolicy::Error;
        return FallbackPolicy::Default;
    }();
    return p;
}

bool first_notice(const char* op) {
    static std::mutex mu;
    static std::unordered_set<std::string> seen;
    std::lock_guard<std::mutex> lk(mu);
    return seen.insert(op ? op : "").second;
}
}  // namespace

void note_cpu_fallback(const char* op) {
    const FallbackPolicy p = fallback_policy();
    TORCH_CHECK(p != FallbackPolicy::Error, "kunlun operator '", op,
                "' is implemented by staging tensors through the CPU, which "
                "KUNLUN_CPU_FALLBACK=error rejects.");
    if (p != FallbackPolicy::Silent && first_notice(op))
        std::fprintf(stderr, "kunlun host-staged implementation: %s "
                             "(KUNLUN_CPU_FALLBACK=silent hides this)\n", op);
}

void check_generic_fallback(const char* op) {
    const FallbackPolicy p = fallback_policy();
    if (p == FallbackPolicy::Silent) return;
    if (p == FallbackPolicy::Warn) {
        std::fprintf(stderr, "kunlun CPU fallback: %s\n", op);
        return;
    }
    TORCH_CHECK(false, "kunlun has no device implementation for '", op,
                "'; the generic CPU fallback is disabled by default. Set "
                "KUNLUN_CPU_FALLBACK=warn (or silent) to allow it.");
}

// ---- helpers ---------------------------------------------------------------

at::Tensor workspace(size_t bytes, const at::Device& device) {
    return at::empty({static_cast<int64_t>(bytes + 1024)},
                     at::TensorOptions().dtype(at::kByte).device(device));
}

void* aligned_base(const at::Tensor& ws) {
    const uintptr_t p = reinterpret_cast<uintptr_t>(ws.data_ptr());
    return reinterpret_cast<void*>((p + 1023) & ~static_cast<uintptr_t>(1023));
}

int tk_scalar_code(at::ScalarType t) {
    switch (t) {
        case at::kBool: return TK_T_BOOL;
        case at::kByte: return TK_T_U8;
        case at::kChar: return TK_T_I8;
        case at::kShort: return TK_T_I16;
        case at::kInt: return TK_T_I32;
        case at::kLong: return TK_T_I64;
        case at::kHalf: return TK_T_F16;
        case at::kBFloat16: return TK_T_BF16;
        case at::kFloat: return TK_T_F32;
        case at::kDouble: return TK_T_F64;
        default: TORCH_CHECK(false, "kunlun: unsupported dtype ", t);
    }
}

// ---- device guard ------------------------------------------------------------

namespace {

struct KunlunGuardImpl final : c10::impl::DeviceGuardImplInterface {
    static constexpr c10::DeviceType static_type = c10::DeviceType::PrivateUse1;
    c10::DeviceType type() const override { return static_type; }
    c10::Device exchangeDevice(c10::Device d) const override {
        const int old = current_device();
        if (d.index() >= 0 && d.index() != old) set_device(d.index());
        return c10::Device(static_type, static_cast<c10::DeviceIndex>(old));
    }
    c10::Device getDevice() const override {
        return c10::Device(static_type, static_cast<c10::DeviceIndex>(current_device()));
    }
    void setDevice(c10::Device d) const override { set_device(d.index()); }
    void uncheckedSetDevice(c10::Device d) const noexcept override { cudaSetDevice(d.index()); }
    c10::Stream getStream(c10::Device d) const noexcept override {
        return c10::Stream(c10::Stream::UNSAFE, d, current_stream_id(d.index()));
    }
    c10::Stream getDefaultStream(c10::Device d) const override {
        return c10::Stream(c10::Stream::UNSAFE, d, 0);
    }
    c10::Stream getStreamFromGlobalPool(c10::Device d, bool = false) const override {
        static std::mutex mu;
        static std::vector<int64_t> pool(64, 0);
        std::lock_guard<std::mutex> lk(mu);
        const int i = d.index() < 0 ? current_device() : d.index();
        if (pool[i] == 0) pool[i] = create_stream(i, 0);
        return c10::Stream(c10::Stream::UNSAFE, d, pool[i]);
    }
    c10::Stream getNewStream(c10::Device d, int priority = 0) const override {
        return c10::Stream(c10::Stream::UNSAFE, d, create_stream(d.index(), priority));
    }
    c10::Stream exchangeStream(c10::Stream s) const noexcept override {
        const c10::Stream old = getStream(s.device());
        set_current_stream(s.device_index(), s.id());
        return old;
    }
    c10::DeviceIndex deviceCount() const noexcept override {
        return static_cast<c10::DeviceIndex>(device_count());
    }
    void synchronizeDevice(c10::DeviceIndex d) const override {
        DeviceRestore g(d < 0 ? current_device() : d);
        check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    }
    void synchronizeStream(const c10::Stream& s) const override {
        synchronize_stream(s.device_index(), s.id());
    }
    bool queryStream(const c10::Stream& s) const override {
        return stream_query(s.device_index(), s.id());
    }
    void record(void** event, const c10::Stream& s, const c10::DeviceIndex,
                const c10::EventFlag flag) const override {
        if (*event == nullptr) {
            *event = reinterpret_cast<void*>(
                event_create(s.device_index(), flag == c10::EventFlag::BACKEND_DEFAULT));
        }
        event_record(reinterpret_cast<int64_t>(*event), s.device_index(), s.id());
    }
    void block(void* event, const c10::Stream& s) const override {
        if (event == nullptr) return;
        stream_wait_event(s.device_index(), s.id(), reinterpret_cast<int64_t>(event));
    }
    bool queryEvent(void* event) const override {
        return event == nullptr || event_query(reinterpret_cast<int64_t>(event));
    }
    void synchronizeEvent(void* event) const override {
        if (event) event_synchronize(reinterpret_cast<int64_t>(event));
    }
    void destroyEvent(void* event, const c10::DeviceIndex) const noexcept override {
        event_destroy(reinterpret_cast<int64_t>(event));
    }
    double elapsedTime(void* a, void* b, const c10::DeviceIndex) const override {
        return event_elapsed_ms(reinterpret_cast<int64_t>(a), reinterpret_cast<int64_t>(b));
    }
    void recordDataPtrOnStream(const c10::DataPtr& p, const c10::Stream& s) const override {
        record_data_ptr_on_stream(p, s);
    }
};

struct KunlunHooks final : at::PrivateUse1HooksInterface {
    bool isBuilt() const override { return true; }
    bool isAvailable() const override { return device_count() > 0; }
    bool hasPrimaryContext(c10::DeviceIndex) const override { return true; }
    void init() const override {}
    at::Device getDeviceFromPtr(void* ptr) const override {
        const int d = device_of_ptr(ptr);
        TORCH_CHECK(d >= 0, "kunlun getDeviceFromPtr: pointer is not device memory");
        return at::Device(at::DeviceType::PrivateUse1, static_cast<c10::DeviceIndex>(d));
    }
    bool isPinnedPtr(const void* ptr) const override { return is_pinned_ptr(ptr); }
    c10::Allocator* getPinnedMemoryAllocator() const override { return get_pinned_allocator(); }
    c10::DeviceIndex deviceCount() const override {
        return static_cast<c10::DeviceIndex>(device_count());
    }
    c10::DeviceIndex getCurrentDevice() const override {
        return static_cast<c10::DeviceIndex>(current_device());
    }
    void setCurrentDevice(c10::DeviceIndex d) const override { set_device(d); }
    c10::DeviceIndex exchangeDevice(c10::DeviceIndex d) const override {
        const int old = current_device();
        if (d >= 0 && d != old) set_device(d);
        return static_cast<c10::DeviceIndex>(old);
    }
    c10::DeviceIndex maybeExchangeDevice(c10::DeviceIndex d) const override {
        return exchangeDevice(d);
    }
    void resizePrivateUse1Bytes(const c10::Storage& storage, size_t newsize) const override;
};

void KunlunHooks::resizePrivateUse1Bytes(const c10::Storage& storage, size_t newsize) const {
    c10::StorageImpl* impl = storage.unsafeGetStorageImpl();
    TORCH_CHECK(impl->resizable(), "kunlun: trying to resize storage that is not resizable");
    const size_t old = impl->nbytes();
    if (newsize == old) return;
    at::DataPtr fresh = get_allocator()->allocate(newsize);
    const size_t keep = std::min(old, newsize);
    if (keep > 0) {
        check_cuda(cudaMemcpyAsync(fresh.get(), impl->data(), keep, cudaMemcpyDeviceToDevice,
                                   current_stream(current_device())),
                   "cudaMemcpyAsync(resize)");
    }
    impl->set_data_ptr_noswap(std::move(fresh));
    impl->set_nbytes(newsize);
}

}  // namespace
}  // namespace torch_kunlun

C10_REGISTER_GUARD_IMPL(PrivateUse1, torch_kunlun::KunlunGuardImpl);

namespace torch_kunlun {
namespace {

void cpu_fallback(const c10::OperatorHandle& op, torch::jit::Stack* stack) {
    const std::string name = op.schema().name();
    check_generic_fallback(name.c_str());
    at::native::cpu_fallback(op, stack);
}

const bool kRegistered = [] {
    c10::register_privateuse1_backend("kunlun");
    c10::SetAllocator(c10::DeviceType::PrivateUse1, get_allocator());
    at::RegisterPrivateUse1HooksInterface(new KunlunHooks());
    return true;
}();

}  // namespace
}  // namespace torch_kunlun

TORCH_LIBRARY_IMPL(_, PrivateUse1, m) {
    m.fallback(torch::CppFunction::makeFromBoxedFunction<&torch_kunlun::cpu_fallback>());
}
