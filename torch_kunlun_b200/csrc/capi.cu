// capi.cu -- library-level entry points of libtk_kernels.so: ABI version,
// per-thread error strings, device attributes and the device error word.
#include <atomic>
#include <mutex>

#include "tk_internal.h"

namespace tk {

namespace {
thread_local std::string t_last_error;
constexpr int kMaxDevices = 64;

// One error word per device.  A kernel whose bounded wait times out writes a
// DeviceError code here (first writer wins) and unwinds.
__device__ unsigned g_tk_error_word;

std::mutex g_dev_mu;
int g_sm_count[kMaxDevices];
unsigned* g_err_addr[kMaxDevices];
}  // namespace

void set_error(const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
}

int current_device() {
    int d = 0;
    cudaGetDevice(&d);
    return d;
}

int sm_count(int device) {
    if (device < 0 || device >= kMaxDevices) return 148;
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (g_sm_count[device] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
            n <= 0) {
            n = 148;
        }
        g_sm_count[device] = n;
    }
    return g_sm_count[device];
}

unsigned* device_error_word(int device) {
    if (device < 0 || device >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (g_err_addr[device] == nullptr) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_tk_error_word) == cudaSuccess) {
            g_err_addr[device] = static_cast<unsigned*>(p);
        }
    }
    return g_err_addr[device];
}

}  // namespace tk

extern "C" {

int tk_abi_version(void) { return TK_ABI_VERSION; }

const char* tk_last_error_string(void) { return tk::t_last_error.c_str(); }

int tk_device_error(int device, unsigned* code_out) {
    TK_CHECK_ARG(code_out != nullptr, "tk_device_error: code_out is NULL");
    int prev = 0;
    TK_CUDA_TRY(cudaGetDevice(&prev));
    TK_CUDA_TRY(cudaSetDevice(device));
    unsigned* w = tk::device_error_word(device);
    if (w == nullptr) {
        cudaSetDevice(prev);
        TK_FAIL(TK_ERR_CUDA, "tk_device_error: error word unavailable on device %d", device);
    }
    unsigned v = 0;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(&v, w, sizeof(v), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemset(w, 0, sizeof(unsigned));
    cudaSetDevice(prev);
    if (e != cudaSuccess) TK_FAIL(TK_ERR_CUDA, "tk_device_error: %s", cudaGetErrorString(e));
    *code_out = v;
    return TK_OK;
}

}  // extern "C"
