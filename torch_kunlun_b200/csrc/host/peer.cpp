// peer.cpp -- device memory shared between the ranks of one node, and the
// row-parallel linear that writes its output rows straight into the rank
// that owns them.
//
// The reference reduces a row-parallel linear's partial sums with a separate
// bkcl collective after the fc (csrc/xccl.cpp:111-163, torch_kunlun/xccl.py:
// 158-213).  Here each rank allocates a receive buffer, exports it with a
// CUDA IPC handle (exchanged through the c10d store by the Python layer), and
// opens the peers' buffers; tk_qgemm_scatter_rows then stores every output
// tile of rank r into slot r of the row block's owner over NVLink while the
// GEMM runs, and the owner sums its slots in a fixed order.
#include <cuda_runtime.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <torch/extension.h>

#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

#include "kunlun.h"

namespace py = pybind11;

namespace torch_kunlun {

void check_cuda(cudaError_t e, const char* what);

namespace {

struct DeviceScope {
    int prev;
    explicit DeviceScope(int dev) : prev(current_device()) {
        if (dev >= 0 && dev != prev) check_cuda(cudaSetDevice(dev), "cudaSetDevice");
    }
    ~DeviceScope() { cudaSetDevice(prev); }
};

std::mutex g_mu;
std::unordered_map<uintptr_t, int> g_owned;   // buffers this process allocated -> device
std::unordered_map<uintptr_t, int> g_opened;  // peers' buffers opened here -> device

}  // namespace

// A device buffer of `bytes` on `device` that other processes may open:
// returns (pointer, IPC handle bytes).  Memory comes from cudaMalloc so that
// the handle covers exactly this buffer.
py::tuple peer_alloc(int64_t bytes, int device) {
    TORCH_CHECK(bytes > 0, "peer_alloc: size must be positive");
    DeviceScope g(device);
    void* p = nullptr;
    check_cuda(cudaMalloc(&p, static_cast<size_t>(bytes)), "cudaMalloc(peer buffer)");
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        check_cuda(e, "cudaIpcGetMemHandle");
    }
    {
        std::lock_guard<std::mutex> lk(g_mu);
        g_owned[reinterpret_cast<uintptr_t>(p)] = device;
    }
    return py::make_tuple(reinterpret_cast<int64_t>(p),
                          py::bytes(reinterpret_cast<const char*>(&h), sizeof(h)));
}

// Open another process's buffer on `device`; returns the local pointer.
int64_t peer_open(const py::bytes& handle, int device) {
    const std::string s = handle;
    TORCH_CHECK(s.size() == sizeof(cudaIpcMemHandle_t), "peer_open: bad handle size");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, s.data(), sizeof(h));
    DeviceScope g(device);
    void* p = nullptr;
    check_cuda(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
    std::lock_guard<std::mutex> lk(g_mu);
    g_opened[reinterpret_cast<uintptr_t>(p)] = device;
    return reinterpret_cast<int64_t>(p);
}

// Close a peer buffer opened here, or free a buffer allocated here (after
// every peer has closed it).
void peer_release(int64_t ptr) {
    void* p = reinterpret_cast<void*>(ptr);
    int dev = -1;
    bool opened = false;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_opened.find(reinterpret_cast<uintptr_t>(p));
        if (it != g_opened.end()) {
            dev = it->second;
            opened = true;
            g_opened.erase(it);
        } else {
            auto jt = g_owned.find(reinterpret_cast<uintptr_t>(p));
            TORCH_CHECK(jt != g_owned.end(), "peer_release: unknown pointer");
            dev = jt->second;
            g_owned.erase(jt);
        }
    }
    DeviceScope g(dev);
    check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize(peer release)");
    if (opened)
        check_cuda(cudaIpcCloseMemHandle(p), "cudaIpcCloseMemHandle");
    else
        check_cuda(cudaFree(p), "cudaFree(peer buffer)");
}

// act(h @ W^T) with the given per-tensor scales, its rows
// [q*rows_per_dest, (q+1)*rows_per_dest) stored at dests[q] (row-major, row
// stride = W's row count).  dests are device pointers valid on h's device.
void linear_scatter_rows(const at::Tensor& input, const at::Tensor& weight, const at::Tensor& amax_x,
                         const at::Tensor& amax_w, const std::vector<int64_t>& dests, int64_t rows_per_dest) {
    TORCH_CHECK(input.dim() == 2 && weight.dim() == 2 && input.size(1) == weight.size(1),
                "linear_scatter_rows: input [M, K] and weight [N, K]");
    TORCH_CHECK(input.device() == weight.device() && input.scalar_type() == weight.scalar_type(),
                "linear_scatter_rows: operands on one device with one dtype");
    for (const at::Tensor* t : {&amax_x, &amax_w})
        TORCH_CHECK(t->scalar_type() == at::kFloat && t->numel() >= 1 && t->device() == input.device(),
                    "linear_scatter_rows: scales must be fp32 tensors on the input's device");
    TORCH_CHECK(!dests.empty() && static_cast<int64_t>(dests.size()) * rows_per_dest == input.size(0),
                "linear_scatter_rows: M must equal len(dests) * rows_per_dest");
    at::Tensor a = input.contiguous(), b = weight.contiguous();
    tk_qgemm_desc_t d = {};
    d.dtype = tk_dtype(a.scalar_type());
    d.batch = 1;
    d.m = a.size(0);
    d.n = b.size(0);
    d.k = a.size(1);
    d.a = a.data_ptr();
    d.a_sb = d.m * d.k;
    d.a_sm = d.k;
    d.a_sk = 1;
    d.b = b.data_ptr();
    d.b_sb = d.n * d.k;
    d.b_sn = d.k;
    d.b_sk = 1;
    d.out_sb = rows_per_dest * d.n;
    d.out_sm = d.n;
    d.alpha = 1.0f;
    d.beta = 0.0f;
    d.act = TK_ACT_NONE;
    d.per_slice_scales = 0;
    d.amax_a = amax_x.data_ptr<float>();
    d.amax_b = amax_w.data_ptr<float>();
    std::vector<void*> ptrs;
    for (int64_t p : dests) ptrs.push_back(reinterpret_cast<void*>(p));
    const int dev = a.device().index();
    DeviceScope g(dev);
    const size_t ws_bytes = tk_qgemm_workspace_size(&d);
    at::Tensor ws = workspace(ws_bytes, a.device());
    check_tk(tk_qgemm_scatter_rows(&d, ptrs.data(), static_cast<int>(ptrs.size()), rows_per_dest,
                                   aligned_base(ws), ws_bytes, current_stream(dev)),
             "tk_qgemm_scatter_rows");
}

// out = T(sum over s of slots[s]) for slots [S, ...] in slot order, fp32
// accumulation, one rounding (tk_reduce_sum).
at::Tensor sum_slots(const at::Tensor& slots) {
    TORCH_CHECK(slots.dim() >= 2, "sum_slots: [slots, ...]");
    at::Tensor x = slots.contiguous();
    std::vector<int64_t> shape(x.sizes().begin() + 1, x.sizes().end());
    at::Tensor out = at::empty(shape, x.options());
    const int64_t inner = out.numel();
    if (inner == 0) return out;
    const int dev = x.device().index();
    DeviceScope g(dev);
    check_tk(tk_reduce_sum(tk_dtype(x.scalar_type()), tk_dtype(x.scalar_type()), x.data_ptr(), 1, x.size(0),
                           inner, out.data_ptr(), current_stream(dev)),
             "tk_reduce_sum");
    return out;
}

// nbytes from src to dst on the current stream; either may be another GPU's
// memory opened here, so this is a copy-engine transfer over NVLink.
void copy_bytes(int64_t dst, int64_t src, int64_t nbytes) {
    TORCH_CHECK(nbytes >= 0 && dst != 0 && src != 0, "copy_bytes: bad arguments");
    if (nbytes == 0) return;
    const int dev = current_device();
    check_cuda(cudaMemcpyAsync(reinterpret_cast<void*>(dst), reinterpret_cast<const void*>(src),
                               static_cast<size_t>(nbytes), cudaMemcpyDefault, current_stream(dev)),
               "cudaMemcpyAsync(peer)");
}

// A kunlun tensor viewing `bytes` of device memory at `ptr` (no ownership).
at::Tensor tensor_at(int64_t ptr, std::vector<int64_t> shape, at::ScalarType dtype, int device) {
    return at::from_blob(reinterpret_cast<void*>(ptr), shape,
                         at::TensorOptions().dtype(dtype).device(c10::Device(c10::DeviceType::PrivateUse1,
                                                                             static_cast<int8_t>(device))));
}

void register_peer(py::module& m) {
    m.def("peer_alloc", &peer_alloc);
    m.def("peer_open", &peer_open);
    m.def("peer_release", &peer_release);
    m.def("linear_scatter_rows", &linear_scatter_rows);
    m.def("sum_slots", &sum_slots);
    m.def("tensor_at", &tensor_at);
    m.def("copy_bytes", &copy_bytes);
}

}  // namespace torch_kunlun
