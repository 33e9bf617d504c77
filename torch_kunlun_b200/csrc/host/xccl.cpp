// xccl.cpp -- collectives of the kunlun backend on NCCL over NVLink/NVSwitch.
//
// Counterpart of the reference's csrc/xccl.cpp (one BKCL context per process,
// :10-91; all_reduce / broadcast / all_gather / reduce_scatter on the current
// stream, :111-163; barrier as a host rendezvous after draining the stream,
// :165-175).  The communicator is created non-blocking so that
// initialisation and enqueue are bounded by KUNLUN_XCCL_TIMEOUT_S (default
// 300 s): a rank that never arrives turns into an error (after
// ncclCommAbort) instead of a hang.  Work is enqueued on the caller's current
// stream; nothing here synchronises the device except barrier().
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>

#include "kunlun.h"

namespace torch_kunlun {

void check_cuda(cudaError_t e, const char* what);

namespace {

std::mutex g_mu;
ncclComm_t g_comm = nullptr;
int g_rank = -1;
int g_nranks = 0;
int g_device = -1;
void* g_barrier_buf = nullptr;

double timeout_s() {
    const char* v = std::getenv("KUNLUN_XCCL_TIMEOUT_S");
    if (v == nullptr || *v == '\0') return 300.0;
    const double t = std::atof(v);
    return t > 0 ? t : 300.0;
}

// Waits (bounded) until a non-blocking NCCL call leaves ncclInProgress.
void settle(ncclResult_t rc, const char* what) {
    const auto t0 = std::chrono::steady_clock::now();
    while (rc == ncclInProgress) {
        std::this_thread::sleep_for(std::chrono::microseconds(20));
        ncclCommGetAsyncError(g_comm, &rc);
        const double el =
            std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (rc == ncclInProgress && el > timeout_s()) {
            ncclCommAbort(g_comm);
            g_comm = nullptr;
            TORCH_CHECK(false, "kunlun xccl: ", what, " timed out after ", timeout_s(),
                        " s; communicator aborted");
        }
    }
    TORCH_CHECK(rc == ncclSuccess, "kunlun xccl: ", what, " failed: ", ncclGetErrorString(rc));
}

ncclDataType_t to_nccl(at::ScalarType t) {
    switch (t) {
        case at::kFloat: return ncclFloat32;
        case at::kHalf: return ncclFloat16;
        case at::kBFloat16: return ncclBfloat16;
        case at::kDouble: return ncclFloat64;
        case at::kInt: return ncclInt32;
        case at::kLong: return ncclInt64;
        case at::kChar: return ncclInt8;
        case at::kByte:
        case at::kBool: return ncclUint8;
        default:
            TORCH_CHECK(false, "kunlun xccl unsupported dtype ", t);
    }
}

ncclRedOp_t to_op(const std::string& op) {
    if (op == "sum" || op == "add") return ncclSum;
    if (op == "prod" || op == "product" || op == "mul") return ncclProd;
    if (op == "min") return ncclMin;
    if (op == "max") return ncclMax;
    if (op == "avg") return ncclAvg;
    TORCH_CHECK(false, "kunlun xccl unsupported reduction op: ", op);
}

void check_tensor(const at::Tensor& t, const char* what) {
    TORCH_CHECK(t.device().type() == c10::DeviceType::PrivateUse1, what,
                " requires a kunlun tensor");
    TORCH_CHECK(t.is_contiguous(), what, " requires a contiguous tensor");
}

void require_comm() { TORCH_CHECK(g_comm != nullptr, "kunlun xccl is not initialized"); }

struct DeviceScope {
    int prev;
    explicit DeviceScope(int dev) : prev(current_device()) {
        if (dev >= 0 && dev != prev) cudaSetDevice(dev);
    }
    ~DeviceScope() { cudaSetDevice(prev); }
};

}  // namespace

std::string xccl_get_unique_id() {
    ncclUniqueId id;
    const ncclResult_t rc = ncclGetUniqueId(&id);
    TORCH_CHECK(rc == ncclSuccess, "ncclGetUniqueId failed: ", ncclGetErrorString(rc));
    return std::string(id.internal, NCCL_UNIQUE_ID_BYTES);
}

void xccl_init_rank(int rank, int nranks, const std::string& uid, int device) {
    TORCH_CHECK(nranks > 0 && rank >= 0 && rank < nranks,
                "kunlun xccl requires 0 <= rank < nranks, got rank=", rank, " nranks=", nranks);
    TORCH_CHECK(uid.size() == NCCL_UNIQUE_ID_BYTES, "kunlun xccl unique id must be ",
                NCCL_UNIQUE_ID_BYTES, " bytes");
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_comm != nullptr) {
        ncclCommDestroy(g_comm);
        g_comm = nullptr;
    }
    set_device(device);
    ncclUniqueId id;
    std::memcpy(id.internal, uid.data(), NCCL_UNIQUE_ID_BYTES);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    const ncclResult_t rc = ncclCommInitRankConfig(&g_comm, nranks, id, rank, &cfg);
    TORCH_CHECK(rc == ncclSuccess || rc == ncclInProgress,
                "ncclCommInitRankConfig failed: ", ncclGetErrorString(rc));
    settle(rc, "communicator init");
    g_rank = rank;
    g_nranks = nranks;
    g_device = device;
    if (g_barrier_buf == nullptr) check_cuda(cudaMalloc(&g_barrier_buf, 16), "cudaMalloc(barrier)");
}

void xccl_destroy() {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_comm != nullptr) {
        ncclCommFinalize(g_comm);
        ncclResult_t rc = ncclInProgress;
        const auto t0 = std::chrono::steady_clock::now();
        while (rc == ncclInProgress) {
            ncclCommGetAsyncError(g_comm, &rc);
            if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > 30.0)
                break;
            std::this_thread::sleep_for(std::chrono::microseconds(50));
        }
        if (rc == ncclSuccess)
            ncclCommDestroy(g_comm);
        else
            ncclCommAbort(g_comm);
        g_comm = nullptr;
    }
    if (g_barrier_buf != nullptr) {
        cudaFree(g_barrier_buf);
        g_barrier_buf = nullptr;
    }
    g_rank = -1;
    g_nranks = 0;
}

int xccl_rank() { return g_rank; }
int xccl_nranks() { return g_nranks; }

void xccl_all_reduce(const at::Tensor& t, const std::string& op, int device) {
    check_tensor(t, "all_reduce");
    require_comm();
    DeviceScope g(device);
    settle(ncclAllReduce(t.data_ptr(), t.data_ptr(), t.numel(), to_nccl(t.scalar_type()), to_op(op),
                         g_comm, current_stream(device)),
           "all_reduce");
}

void xccl_broadcast(const at::Tensor& t, int root, int device) {
    check_tensor(t, "broadcast");
    require_comm();
    DeviceScope g(device);
    settle(ncclBroadcast(t.data_ptr(), t.data_ptr(), t.numel(), to_nccl(t.scalar_type()), root,
                         g_comm, current_stream(device)),
           "broadcast");
}

void xccl_all_gather(const at::Tensor& out, const at::Tensor& input, int device) {
    check_tensor(out, "all_gather out");
    check_tensor(input, "all_gather input");
    TORCH_CHECK(out.scalar_type() == input.scalar_type(), "all_gather dtype mismatch");
    require_comm();
    TORCH_CHECK(out.numel() >= input.numel() * static_cast<int64_t>(g_nranks),
                "all_gather output is too small");
    DeviceScope g(device);
    settle(ncclAllGather(input.data_ptr(), out.data_ptr(), input.numel(),
                         to_nccl(input.scalar_type()), g_comm, current_stream(device)),
           "all_gather");
}

void xccl_reduce_scatter(const at::Tensor& out, const at::Tensor& input, const std::string& op,
                         int device) {
    check_tensor(out, "reduce_scatter out");
    check_tensor(input, "reduce_scatter input");
    TORCH_CHECK(out.scalar_type() == input.scalar_type(), "reduce_scatter dtype mismatch");
    require_comm();
    TORCH_CHECK(input.numel() >= out.numel() * static_cast<int64_t>(g_nranks),
                "reduce_scatter input is too small");
    DeviceScope g(device);
    settle(ncclReduceScatter(input.data_ptr(), out.data_ptr(), out.numel(),
                             to_nccl(out.scalar_type()), to_op(op), g_comm, current_stream(device)),
           "reduce_scatter");
}

void xccl_barrier(int device) {
    require_comm();
    DeviceScope g(device);
    cudaStream_t s = current_stream(device);
    // Drain this rank's stream, rendezvous with a 1-element all-reduce, and
    // wait for it: no rank leaves before every rank has arrived.
    check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize(barrier)");
    settle(ncclAllReduce(g_barrier_buf, g_barrier_buf, 1, ncclFloat32, ncclSum, g_comm, s),
           "barrier");
    check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize(barrier)");
}

}  // namespace torch_kunlun
