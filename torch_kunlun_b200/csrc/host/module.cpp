// module.cpp -- the `_C` Python module of the kunlun backend.
//
// Same function names and argument meaning as the reference's pybind module
// (csrc/kunlun.cpp:828-897), with the device index made explicit on stream
// and event calls (the reference encodes it in its handle objects).
// xdnn_version / cluster budget calls exist for API compatibility only: there
// is no XDNN library and no cluster partitioning on B200.
#include <torch/extension.h>

#include <atomic>

#include "kunlun.h"

namespace {

std::atomic<int> g_cluster_budget{4};
std::atomic<int> g_sdnn_budget{4};

py::dict device_properties(int device) {
    cudaDeviceProp p;
    torch_kunlun::check_cuda(cudaGetDeviceProperties(&p, device), "cudaGetDeviceProperties");
    py::dict d;
    d["name"] = std::string(p.name);
    d["total_memory"] = static_cast<uint64_t>(p.totalGlobalMem);
    d["multi_processor_count"] = p.multiProcessorCount;
    d["warp_size"] = p.warpSize;
    d["major"] = p.major;
    d["minor"] = p.minor;
    d["model"] = p.major * 10 + p.minor;
    return d;
}

}  // namespace

namespace torch_kunlun {
void register_peer(pybind11::module& m);
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    using namespace torch_kunlun;
    // The blocking waits release the GIL, so other Python threads (a clock
    // sampler, a data loader) keep running while the host waits on the GPU.
    m.def("device_count", &device_count);
    m.def("current_device", &current_device);
    m.def("set_device", &set_device);
    m.def("synchronize", &synchronize_all, py::call_guard<py::gil_scoped_release>());
    m.def("memory_allocated", [](int d) { return memory_allocated(d); }, py::arg("device") = -1);
    m.def("max_memory_allocated", [](int d) { return max_memory_allocated(d); },
          py::arg("device") = -1);
    m.def("memory_reserved", [](int d) { return memory_reserved(d); }, py::arg("device") = -1);
    m.def("reset_peak_memory_stats", [](int d) { reset_peak_memory_stats(d); },
          py::arg("device") = -1);
    m.def("empty_cache", &empty_cache);
    m.def("set_cluster_budget", [](int nc, int ns) {
        TORCH_CHECK(nc >= 1 && nc <= 4 && ns >= 1 && ns <= 4,
                    "cluster budget must be in 1..4");
        g_cluster_budget = nc;
        g_sdnn_budget = ns;
        return nc;
    });
    m.def("cluster_budget", [] { return g_cluster_budget.load(); });
    m.def("sdnn_budget", [] { return g_sdnn_budget.load(); });
    m.def("xdnn_version", [] { return std::string("none (B200 sm_100a kernels)"); });
    m.def("is_pinned_ptr", [](uint64_t p) { return is_pinned_ptr(reinterpret_cast<const void*>(p)); });
    m.def("get_device_properties", &device_properties);

    m.def("current_stream", [](int d) { return current_stream_id(d); });
    m.def("default_stream", [](int d) { return default_stream_id(d); });
    m.def("create_stream", &create_stream, py::arg("device"), py::arg("priority") = 0);
    m.def("destroy_stream", &destroy_stream);
    m.def("set_stream", &set_current_stream);
    m.def("synchronize_stream", &synchronize_stream, py::call_guard<py::gil_scoped_release>());
    m.def("stream_query", &stream_query);
    m.def("event_create", &event_create, py::arg("device"), py::arg("timing") = false);
    m.def("event_destroy", &event_destroy);
    m.def("event_record", &event_record);
    m.def("stream_wait_event", &stream_wait_event);
    m.def("event_synchronize", &event_synchronize, py::call_guard<py::gil_scoped_release>());
    m.def("event_query", &event_query);
    m.def("event_elapsed_time", &event_elapsed_ms);

    m.def("xccl_get_unique_id", [] { return py::bytes(xccl_get_unique_id()); });
    m.def("xccl_init_rank", [](int rank, int nranks, py::bytes uid, int device) {
        xccl_init_rank(rank, nranks, uid.cast<std::string>(), device);
    });
    m.def("xccl_destroy", &xccl_destroy);
    m.def("xccl_rank", &xccl_rank);
    m.def("xccl_nranks", &xccl_nranks);
    m.def("xccl_all_reduce", &xccl_all_reduce);
    m.def("xccl_broadcast", &xccl_broadcast);
    m.def("xccl_all_gather", &xccl_all_gather);
    m.def("xccl_reduce_scatter", &xccl_reduce_scatter);
    m.def("xccl_barrier", &xccl_barrier);

    m.def("linear_act", &linear_act, py::arg("input"), py::arg("weight"),
          py::arg("bias") = py::none(), py::arg("act") = 0, py::arg("residual") = py::none(),
          py::arg("amax_x") = py::none(), py::arg("amax_out") = py::none());
    m.def("silu_mul", &silu_mul);
    m.def("silu_mul_amax", &silu_mul_amax);
    m.def("quantize_limbs", &quantize_limbs);
    m.def("linear_from_limbs", &linear_from_limbs, py::arg("a_limbs"), py::arg("b_limbs"), py::arg("k"),
          py::arg("amax_a"), py::arg("amax_b"), py::arg("bias") = py::none(), py::arg("act") = 0,
          py::arg("out") = py::none(), py::arg("dtype") = at::kHalf, py::arg("gate") = py::none(),
          py::arg("amax_out") = py::none());
    m.def("amax", &amax);
    m.def("linear_scaled", &linear_scaled, py::arg("input"), py::arg("weight"),
          py::arg("bias") = py::none(), py::arg("act") = 0, py::arg("amax_x") = py::none(),
          py::arg("amax_w") = py::none(), py::arg("out") = py::none());
    m.def("sdpa", &sdpa, py::arg("query"), py::arg("key"), py::arg("value"),
          py::arg("attn_mask") = py::none(), py::arg("is_causal") = false,
          py::arg("scale") = py::none(), py::arg("fused") = true);
    m.def("abi_version", [] { return tk_abi_version(); });
    torch_kunlun::register_peer(m);
}
