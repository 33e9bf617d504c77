// kunlun.h -- host runtime of the `kunlun` PrivateUse1 backend on B200.
//
// Mirrors the runtime API of the reference's csrc/kunlun.h:19-124 (device,
// stream and event management, allocator, fallback policy) with CUDA
// underneath: a kunlun device is a CUDA device, a kunlun stream is a CUDA
// stream, and every op enqueues work on the current stream of its device.
// There is no per-device launch mutex (the reference's ContextGuard,
// csrc/kunlun.h:113-124): kernels are launched directly on the caller's
// stream, so ops on different streams overlap.
#pragma once

#include <c10/core/Allocator.h>
#include <c10/core/Stream.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <cstdint>

#include "../../../include/tk_kernels.h"

namespace torch_kunlun {

// ---- devices (reference csrc/kunlun.h:21-26) ----
int device_count();
int current_device();
void set_device(int device);
void synchronize_all();

// ---- streams (reference csrc/kunlun.h:27-35) ----
// Stream ids: 0 is the device's default stream (the CUDA legacy default
// stream, so kunlun work is ordered with torch.cuda work on the same GPU);
// any other id is a cudaStream_t created by create_stream().
int64_t current_stream_id(int device);
int64_t default_stream_id(int device);
int64_t create_stream(int device, int priority);
void destroy_stream(int device, int64_t stream_id);
void set_current_stream(int device, int64_t stream_id);
void synchronize_stream(int device, int64_t stream_id);
bool stream_query(int device, int64_t stream_id);
cudaStream_t stream_handle(int64_t stream_id);
cudaStream_t current_stream(int device);
bool stream_is_live(cudaStream_t s);

// ---- events (reference csrc/kunlun.h:36-41; query and elapsed_time are real) ----
int64_t event_create(int device, bool timing);
void event_destroy(int64_t event_id);
void event_record(int64_t event_id, int device, int64_t stream_id);
void stream_wait_event(int device, int64_t stream_id, int64_t event_id);
void event_synchronize(int64_t event_id);
bool event_query(int64_t event_id);
double event_elapsed_ms(int64_t start_id, int64_t end_id);

// ---- allocator (reference csrc/allocator.cpp) ----
c10::Allocator* get_allocator();
size_t memory_allocated(int device);
size_t max_memory_allocated(int device);
size_t memory_reserved(int device);
void reset_peak_memory_stats(int device);
void empty_cache();
void record_data_ptr_on_stream(const c10::DataPtr& data_ptr, const c10::Stream& stream);
int device_of_ptr(void* ptr);
c10::Allocator* get_pinned_allocator();
bool is_pinned_ptr(const void* ptr);

// ---- CPU fallback policy (reference csrc/kunlun.cpp:313-375) ----
void note_cpu_fallback(const char* op);
void check_generic_fallback(const char* op);

// ---- helpers for op implementations ----
void check_cuda(cudaError_t e, const char* what);  // throws on a CUDA error
void check_tk(int rc, const char* what);  // throws with tk_last_error_string()
at::Tensor workspace(size_t bytes, const at::Device& device);  // 1024-aligned base
void* aligned_base(const at::Tensor& ws);
inline tk_dtype_t tk_dtype(at::ScalarType t) {
    TORCH_CHECK(t == at::kHalf || t == at::kFloat,
                "kunlun: only float16/float32 are supported here, got ", t);
    return t == at::kHalf ? TK_DTYPE_F16 : TK_DTYPE_F32;
}
int tk_scalar_code(at::ScalarType t);

// Host->device / device->host / device->device copies used by copy_.
at::Tensor& copy_impl(at::Tensor& self, const at::Tensor& src, bool non_blocking);

// ---- collectives (reference csrc/xccl.cpp; NCCL underneath) ----
std::string xccl_get_unique_id();
void xccl_init_rank(int rank, int nranks, const std::string& unique_id, int device);
void xccl_destroy();
int xccl_rank();
int xccl_nranks();
void xccl_all_reduce(const at::Tensor& tensor, const std::string& op, int device);
void xccl_broadcast(const at::Tensor& tensor, int root, int device);
void xccl_all_gather(const at::Tensor& out, const at::Tensor& input, int device);
void xccl_reduce_scatter(const at::Tensor& out, const at::Tensor& input, const std::string& op,
                         int device);
void xccl_barrier(int device);

// ---- fused ops exposed to Python ----
at::Tensor linear_act(const at::Tensor& input, const at::Tensor& weight,
                      const std::optional<at::Tensor>& bias, int64_t act,
                      const std::optional<at::Tensor>& residual,
                      const std::optional<at::Tensor>& amax_x,
                      const std::optional<at::Tensor>& amax_out);
at::Tensor silu_mul(const at::Tensor& gate, const at::Tensor& up);
std::tuple<at::Tensor, at::Tensor> silu_mul_amax(const at::Tensor& gate, const at::Tensor& up);
at::Tensor quantize_limbs(const at::Tensor& x, const at::Tensor& amax);
at::Tensor linear_from_limbs(const at::Tensor& a_limbs, const at::Tensor& b_limbs, int64_t k,
                             const at::Tensor& amax_a, const at::Tensor& amax_b,
                             const std::optional<at::Tensor>& bias, int64_t act,
                             const std::optional<at::Tensor>& out, at::ScalarType dtype,
                             const std::optional<at::Tensor>& gate, const std::optional<at::Tensor>& amax_out);
at::Tensor amax(const at::Tensor& x);
at::Tensor linear_scaled(const at::Tensor& input, const at::Tensor& weight,
                         const std::optional<at::Tensor>& bias, int64_t act,
                         const std::optional<at::Tensor>& amax_x,
                         const std::optional<at::Tensor>& amax_w,
                         const std::optional<at::Tensor>& out);
at::Tensor sdpa(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                const std::optional<at::Tensor>& mask, bool is_causal, std::optional<double> scale,
                bool fused);

}  // namespace torch_kunlun
