// noalloc.cu -- tk_qgemm_noalloc: the quantised GEMM of tk_qgemm for callers
// that cannot allocate device memory.
//
// Some callers own every byte of device memory themselves: a host
// application or inference server that hands this library its input and
// output buffers but gives it no allocator, or that forbids allocation after
// start-up so that its memory footprint stays fixed.  Such a caller cannot
// provide (or let us obtain) the scratch that tk_qgemm needs for the amax
// values and the int8 limb planes.  tk_qgemm_noalloc instead uses a fixed
// scratch array that is part of this library's device image, so a call
// allocates nothing: no cudaMalloc, no cudaFree, no allocating library call.
//
// Limits and sharing:
//   * the scratch is kNoAllocScratchBytes (64 MiB) per GPU, held by every
//     GPU that loads the library until the process exits;
//   * a problem whose workspace (tk_qgemm_workspace_size) exceeds that size
//     is rejected with TK_ERR_WORKSPACE -- for fp16/fp32 operands this is
//     roughly batch*(m + n)*round_up(k, 16)*2 bytes plus a few KiB;
//   * every call shares the one array: calls that overlap on the GPU (on
//     different streams, or from different threads without ordering) race
//     and corrupt each other's results; calls ordered on one stream are
//     safe.  The array keeps the previous call's contents; the amax slots
//     that must start at zero are cleared by each call before use and the
//     limb planes are fully rewritten;
//   * the first call on a device performs a one-time set-up (it looks up the
//     array's device address with cudaGetSymbolAddress while that device is
//     current); make that first call before any stream capture;
//   * `stream` must belong to the current device: the scratch used is the
//     current device's copy, so a stream of another GPU is rejected with
//     TK_ERR_INVALID_ARG instead of running with another GPU's scratch.
#include <mutex>

#include "tk_internal.h"

namespace tk {
namespace {

constexpr size_t kNoAllocScratchBytes = 64ull << 20;
constexpr int kMaxDevices = 64;

// The scratch itself.  In host code this name is only a host-side stand-in
// for the device array: its device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
void* g_addr[kMaxDevices];

// Device address of the scratch on the current device (set up once).
int scratch_address(int device, void** out) {
    TK_CHECK_ARG(device >= 0 && device < kMaxDevices, "tk_qgemm_noalloc: bad device %d", device);
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_addr[device] == nullptr) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr)
            TK_FAIL(TK_ERR_CUDA, "tk_qgemm_noalloc: cudaGetSymbolAddress failed on device %d: %s",
                    device, cudaGetErrorString(e));
        g_addr[device] = p;
    }
    *out = g_addr[device];
    return TK_OK;
}

}  // namespace
}  // namespace tk

extern "C" int tk_qgemm_noalloc(const tk_qgemm_desc_t* desc, void* stream) {
    using namespace tk;
    TK_CHECK_ARG(desc != nullptr, "tk_qgemm_noalloc: desc is NULL");
    // the same argument checks as tk_qgemm, before any size arithmetic
    int rc = qgemm_validate(*desc);
    if (rc) return rc;
    const size_t need = tk_qgemm_workspace_size(desc);
    // tk_qgemm wants a 1024-byte-aligned workspace; the array is 256-aligned.
    const size_t slack = 1024;
    if (need + slack > kNoAllocScratchBytes) {
        TK_FAIL(TK_ERR_WORKSPACE,
                "tk_qgemm_noalloc: problem needs %zu bytes of scratch but the built-in scratch "
                "holds %zu bytes (%zu usable); use tk_qgemm with a caller workspace",
                need, kNoAllocScratchBytes, kNoAllocScratchBytes - slack);
    }
    const int dev = current_device();
    if (stream != nullptr) {
        int sdev = -1;
        TK_CUDA_TRY(cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &sdev));
        TK_CHECK_ARG(sdev == dev,
                     "tk_qgemm_noalloc: the stream belongs to device %d but device %d is current; "
                     "make the stream's device current first", sdev, dev);
    }
    void* base = nullptr;
    rc = scratch_address(dev, &base);
    if (rc) return rc;
    const uintptr_t b = reinterpret_cast<uintptr_t>(base);
    void* aligned = reinterpret_cast<void*>((b + 1023) & ~static_cast<uintptr_t>(1023));
    const size_t avail = kNoAllocScratchBytes - (reinterpret_cast<uintptr_t>(aligned) - b);
    return tk_qgemm(desc, aligned, avail, stream);
}
