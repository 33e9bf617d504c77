// ops_core.cpp -- tensor creation, views, copies and fills of the kunlun
// backend (TORCH_LIBRARY_IMPL(aten, PrivateUse1)).
//
// Counterpart of the reference's csrc/ops.cpp:289-476 and :496-578 (empty,
// empty_strided, copy_, clone, fill_, zero_).  The reference moves every
// transfer synchronously through XPURT's default stream and stages
// non-contiguous views through host memory (materialize_private_contiguous,
// csrc/ops.cpp:289-350).  Here transfers are cudaMemcpyAsync on the current
// stream (non_blocking is honoured for pinned host memory) and strided or
// dtype-converting copies run on the device (tk_copy_strided).
#include <ATen/EmptyTensor.h>
#include <ATen/native/Resize.h>
#include <ATen/native/TensorFactories.h>
#include <ATen/ops/as_strided_native.h>
#include <ATen/ops/view_native.h>
#include <ATen/ops/_reshape_alias_native.h>
#include <torch/library.h>

#include <cstring>

#include "kunlun.h"

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

int dev_index(const c10::optional<at::Device>& d) {
    if (!d.has_value() || d->index() < 0) return current_device();
    TORCH_CHECK(d->type() == c10::DeviceType::PrivateUse1, "kunlun: expected a kunlun device, got ",
                *d);
    return d->index();
}

at::Tensor empty_memory_format(c10::SymIntArrayRef size, std::optional<at::ScalarType> dtype,
                               std::optional<at::Layout> layout, std::optional<at::Device> device,
                               std::optional<bool> pin_memory,
                               std::optional<at::MemoryFormat> memory_format) {
    TORCH_CHECK(!layout.has_value() || *layout == at::Layout::Strided,
                "kunlun empty only supports strided layout");
    TORCH_CHECK(!pin_memory.value_or(false), "kunlun empty does not support pin_memory");
    const int d = dev_index(device);
    DeviceScope g(d);
    return at::detail::empty_generic_symint(size, get_allocator(),
                                            c10::DispatchKeySet(c10::DispatchKey::PrivateUse1),
                                            c10::dtype_or_default(dtype), memory_format);
}

at::Tensor empty_strided(c10::SymIntArrayRef size, c10::SymIntArrayRef stride,
                         std::optional<at::ScalarType> dtype, std::optional<at::Layout> layout,
                         std::optional<at::Device> device, std::optional<bool> pin_memory) {
    TORCH_CHECK(!layout.has_value() || *layout == at::Layout::Strided,
                "kunlun empty_strided only supports strided layout");
    TORCH_CHECK(!pin_memory.value_or(false), "kunlun empty_strided does not support pin_memory");
    const int d = dev_index(device);
    DeviceScope g(d);
    return at::detail::empty_strided_symint_generic(
        size, stride, get_allocator(), c10::DispatchKeySet(c10::DispatchKey::PrivateUse1),
        c10::dtype_or_default(dtype));
}

const at::Tensor& resize_(const at::Tensor& self, c10::SymIntArrayRef size,
                          std::optional<at::MemoryFormat> memory_format) {
    auto* impl = self.unsafeGetTensorImpl();
    std::vector<int64_t> sizes;
    for (const auto& s : size) sizes.push_back(s.expect_int());
    const int64_t old_numel = self.numel();
    int64_t numel = 1;
    for (auto s : sizes) numel *= s;
    const size_t need = static_cast<size_t>(numel + self.storage_offset()) * self.itemsize();
    if (need > self.storage().nbytes()) {
        DeviceScope g(self.device().index());
        at::DataPtr fresh = get_allocator()->allocate(need);
        const size_t keep = self.storage().nbytes();
        if (keep > 0 && old_numel > 0) {
            check_cuda(cudaMemcpyAsync(fresh.get(), self.storage().data(), keep,
                                       cudaMemcpyDeviceToDevice, current_stream(self.device().index())),
                       "cudaMemcpyAsync(resize_)");
        }
        self.storage().unsafeGetStorageImpl()->set_data_ptr_noswap(std::move(fresh));
        self.storage().unsafeGetStorageImpl()->set_nbytes(need);
    }
    impl->set_sizes_contiguous(sizes);
    if (memory_format.has_value() && *memory_format != at::MemoryFormat::Preserve) {
        impl->empty_tensor_restride(*memory_format);
    }
    return self;
}

at::Scalar local_scalar_dense(const at::Tensor& self) {
    TORCH_CHECK(self.numel() == 1, "kunlun: a Tensor with ", self.numel(),
                " elements cannot be converted to Scalar");
    uint8_t buf[16] = {0};
    const int d = self.device().index();
    DeviceScope g(d);
    cudaStream_t s = current_stream(d);
    check_cuda(cudaMemcpyAsync(buf, self.data_ptr(), self.itemsize(), cudaMemcpyDeviceToHost, s),
               "cudaMemcpyAsync(item)");
    check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize(item)");
    switch (self.scalar_type()) {
        case at::kHalf: return at::Scalar(static_cast<double>(*reinterpret_cast<at::Half*>(buf)));
        case at::kBFloat16:
            return at::Scalar(static_cast<double>(*reinterpret_cast<at::BFloat16*>(buf)));
        case at::kFloat: return at::Scalar(static_cast<double>(*reinterpret_cast<float*>(buf)));
        case at::kDouble: return at::Scalar(*reinterpret_cast<double*>(buf));
        case at::kBool: return at::Scalar(static_cast<bool>(buf[0]));
        case at::kByte: return at::Scalar(static_cast<int64_t>(buf[0]));
        case at::kChar: return at::Scalar(static_cast<int64_t>(*reinterpret_cast<int8_t*>(buf)));
        case at::kShort: return at::Scalar(static_cast<int64_t>(*reinterpret_cast<int16_t*>(buf)));
        case at::kInt: return at::Scalar(static_cast<int64_t>(*reinterpret_cast<int32_t*>(buf)));
        case at::kLong: return at::Scalar(*reinterpret_cast<int64_t*>(buf));
        default: TORCH_CHECK(false, "kunlun item(): unsupported dtype ", self.scalar_type());
    }
}

// Strided device copy of `src` into `dst` (same device), with conversion.
void device_copy(const at::Tensor& dst, const at::Tensor& src) {
    TORCH_CHECK(dst.dim() <= 8, "kunlun copy_: at most 8 dims");
    const int d = dst.device().index();
    DeviceScope g(d);
    at::Tensor s = src.expand(dst.sizes());
    std::vector<int64_t> sizes = dst.sizes().vec(), ds = dst.strides().vec(), ss = s.strides().vec();
    check_tk(tk_copy_strided(dst.data_ptr(), tk_scalar_code(dst.scalar_type()), s.data_ptr(),
                             tk_scalar_code(s.scalar_type()), static_cast<int>(sizes.size()),
                             sizes.data(), ds.data(), ss.data(), current_stream(d)),
             "tk_copy_strided");
}

bool overlaps(const at::Tensor& a, const at::Tensor& b) {
    if (!a.has_storage() || !b.has_storage()) return false;
    if (a.storage().data() != b.storage().data()) return false;
    return true;
}

}  // namespace

at::Tensor& copy_impl(at::Tensor& self, const at::Tensor& src, bool non_blocking) {
    if (self.numel() == 0) return self;
    TORCH_CHECK(at::is_expandable_to(src.sizes(), self.sizes()),
                "kunlun copy_: source of shape ", src.sizes(), " cannot be broadcast to ",
                self.sizes());
    const bool self_dev = self.device().type() == c10::DeviceType::PrivateUse1;
    const bool src_dev = src.device().type() == c10::DeviceType::PrivateUse1;
    if (self_dev && src.device().is_cuda() && src.device().index() == self.device().index()) {
        // torch.cuda memory of the same GPU: an ordinary device copy on the
        // kunlun stream once the cuda stream's pending work is done.
        const int d = self.device().index();
        DeviceScope g(d);
        check_cuda(cudaStreamSynchronize(nullptr), "cudaStreamSynchronize(cuda src)");
        at::Tensor sc = src.contiguous();
        at::Tensor view = at::from_blob(sc.data_ptr(), sc.sizes(), sc.strides(),
                                        self.options().dtype(sc.scalar_type()));
        device_copy(self, view);
        check_cuda(cudaStreamSynchronize(current_stream(d)), "cudaStreamSynchronize(kunlun)");
        return self;
    }
    if (self_dev && src_dev) {
        if (self.device() == src.device()) {
            if (self.is_same(src)) return self;
            if (overlaps(self, src) && !self.is_same(src)) {
                // Partially overlapping views (x[1:].copy_(x[:-1])): go through a temporary.
                at::Tensor tmp = at::empty(src.sizes(), src.options());
                device_copy(tmp, src);
                device_copy(self, tmp);
            } else {
                device_copy(self, src);
            }
            return self;
        }
        // Cross-device: bring the source onto the destination device with a
        // peer copy of a contiguous version, then convert/scatter there.
        at::Tensor sc = src.contiguous();
        at::Tensor staged;
        {
            DeviceScope g(self.device().index());
            staged = at::empty(sc.sizes(), sc.options().device(self.device()));
        }
        {
            DeviceScope g(src.device().index());
            check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize(peer src)");
        }
        {
            DeviceScope g(self.device().index());
            check_cuda(cudaMemcpyPeerAsync(staged.data_ptr(), self.device().index(), sc.data_ptr(),
                                           src.device().index(), sc.nbytes(),
                                           current_stream(self.device().index())),
                       "cudaMemcpyPeerAsync");
        }
        device_copy(self, staged);
        return self;
    }
    if (self_dev && !src_dev) {
        // host -> device
        TORCH_CHECK(src.device().is_cpu(), "kunlun copy_: unsupported source device ", src.device());
        const int d = self.device().index();
        DeviceScope g(d);
        at::Tensor hs = src.expand(self.sizes()).contiguous();
        const bool direct = self.is_contiguous() && hs.scalar_type() == self.scalar_type();
        at::Tensor target = direct ? self : at::empty(hs.sizes(), self.options().dtype(hs.scalar_type()));
        cudaStream_t s = current_stream(d);
        check_cuda(cudaMemcpyAsync(target.data_ptr(), hs.data_ptr(), hs.nbytes(),
                                   cudaMemcpyHostToDevice, s),
                   "cudaMemcpyAsync(H2D)");
        if (!direct) device_copy(self, target);
        if (!(non_blocking && is_pinned_ptr(hs.data_ptr()))) {
            check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize(H2D)");
        }
        return self;
    }
    if (!self_dev && src_dev) {
        // device -> host
        TORCH_CHECK(self.device().is_cpu(), "kunlun copy_: unsupported destination device ",
                    self.device());
        const int d = src.device().index();
        DeviceScope g(d);
        at::Tensor ds = src;
        if (!src.is_contiguous() || src.scalar_type() != self.scalar_type() ||
            !src.sizes().equals(self.sizes())) {
            ds = at::empty(self.sizes(), src.options().dtype(self.scalar_type()));
            device_copy(ds, src);
        }
        cudaStream_t s = current_stream(d);
        const bool direct = self.is_contiguous();
        at::Tensor host = direct ? self : at::empty(self.sizes(), self.options().memory_format(at::MemoryFormat::Contiguous));
        check_cuda(cudaMemcpyAsync(host.data_ptr(), ds.data_ptr(), ds.nbytes(),
                                   cudaMemcpyDeviceToHost, s),
                   "cudaMemcpyAsync(D2H)");
        const bool async_ok = non_blocking && direct && is_pinned_ptr(host.data_ptr());
        if (!async_ok) check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize(D2H)");
        if (!direct) self.copy_(host);
        return self;
    }
    TORCH_CHECK(false, "kunlun copy_: unsupported device combination");
}

namespace {

at::Tensor& copy_(at::Tensor& self, const at::Tensor& src, bool non_blocking) {
    return copy_impl(self, src, non_blocking);
}

at::Tensor _copy_from(const at::Tensor& self, const at::Tensor& dst, bool non_blocking) {
    at::Tensor d = dst;
    copy_impl(d, self, non_blocking);
    return dst;
}

at::Tensor _copy_from_and_resize(const at::Tensor& self, const at::Tensor& dst) {
    if (!dst.sizes().equals(self.sizes())) dst.resize_(self.sizes());
    at::Tensor d = dst;
    copy_impl(d, self, false);
    return dst;
}

at::Tensor clone(const at::Tensor& self, std::optional<at::MemoryFormat> memory_format) {
    at::Tensor out;
    const auto mf = memory_format.value_or(at::MemoryFormat::Preserve);
    if (mf == at::MemoryFormat::Preserve && self.is_non_overlapping_and_dense()) {
        out = at::empty_strided(self.sizes(), self.strides(), self.options());
    } else {
        out = at::empty(self.sizes(), self.options().memory_format(
                                          mf == at::MemoryFormat::Preserve ? at::MemoryFormat::Contiguous : mf));
    }
    device_copy(out, self);
    return out;
}

at::Tensor& fill_impl(at::Tensor& self, const at::Scalar& value) {
    if (self.numel() == 0) return self;
    const at::ScalarType t = self.scalar_type();
    double fv = 0.0;
    int64_t iv = 0;
    if (at::isFloatingType(t)) {
        fv = value.toDouble();
    } else if (t == at::kBool) {
        iv = value.toBool() ? 1 : 0;
    } else {
        TORCH_CHECK(!value.isFloatingPoint() || std::trunc(value.toDouble()) == value.toDouble(),
                    "kunlun fill_ value ", value.toDouble(), " is not an integer");
        iv = value.toLong();
        const int64_t bits = static_cast<int64_t>(self.itemsize()) * 8;
        if (bits < 64) {
            const bool is_unsigned = t == at::kByte;
            const int64_t lo = is_unsigned ? 0 : -(int64_t(1) << (bits - 1));
            const int64_t hi = is_unsigned ? (int64_t(1) << bits) - 1 : (int64_t(1) << (bits - 1)) - 1;
            TORCH_CHECK(iv >= lo && iv <= hi, "kunlun fill_ value ", iv, " overflows ", bits,
                        "-bit dtype");
        }
    }
    TORCH_CHECK(self.dim() <= 8, "kunlun fill_: at most 8 dims");
    const int d = self.device().index();
    DeviceScope g(d);
    std::vector<int64_t> sizes = self.sizes().vec(), strides = self.strides().vec();
    check_tk(tk_fill_strided(self.data_ptr(), tk_scalar_code(t), fv, iv,
                             static_cast<int>(sizes.size()), sizes.data(), strides.data(),
                             current_stream(d)),
             "tk_fill_strided");
    return self;
}

at::Tensor& zero_impl(at::Tensor& self) { return fill_impl(self, at::Scalar(0)); }

void record_stream(at::Tensor& self, c10::Stream stream) {
    record_data_ptr_on_stream(self.storage().data_ptr(), stream);
}

// Concatenation along `dim`: each input is a device copy into its slice of
// the output (converting to the promoted dtype).  Legacy 1-D empty inputs
// are skipped as in aten.  Used by DDP's coalesced broadcast
// (flatten_dense_tensors) and by user code.
at::Tensor cat(const at::ITensorListRef& tensors, int64_t dim) {
    std::vector<at::Tensor> ts;
    for (const at::Tensor& t : tensors) ts.push_back(t);
    TORCH_CHECK(!ts.empty(), "kunlun cat: expected a non-empty list of tensors");
    auto skip = [](const at::Tensor& t) { return t.dim() == 1 && t.size(0) == 0; };
    const at::Tensor* ref = nullptr;
    at::ScalarType rt = ts[0].scalar_type();
    bool first = true;
    for (const at::Tensor& t : ts) {
        TORCH_CHECK(t.device().type() == c10::DeviceType::PrivateUse1, "kunlun cat: tensor on ",
                    t.device());
        rt = first ? t.scalar_type() : c10::promoteTypes(rt, t.scalar_type());
        first = false;
        if (!skip(t) && ref == nullptr) ref = &t;
    }
    if (ref == nullptr) return at::empty({0}, ts[0].options().dtype(rt));
    const int64_t nd = ref->dim();
    TORCH_CHECK(nd > 0, "kunlun cat: zero-dimensional tensor cannot be concatenated");
    dim = c10::maybe_wrap_dim(dim, nd);
    std::vector<int64_t> shape = ref->sizes().vec();
    int64_t total = 0;
    for (const at::Tensor& t : ts) {
        if (skip(t)) continue;
        TORCH_CHECK(t.dim() == nd, "kunlun cat: tensors must have the same number of dimensions");
        for (int64_t d = 0; d < nd; ++d)
            TORCH_CHECK(d == dim || t.size(d) == shape[d], "kunlun cat: sizes of tensors must match except in dimension ",
                        dim);
        TORCH_CHECK(t.device() == ref->device(), "kunlun cat: tensors on different devices");
        total += t.size(dim);
    }
    shape[dim] = total;
    at::Tensor out = at::empty(shape, ref->options().dtype(rt));
    int64_t off = 0;
    for (const at::Tensor& t : ts) {
        if (skip(t) || t.size(dim) == 0) continue;
        at::Tensor slice = out.narrow(dim, off, t.size(dim));
        device_copy(slice, t);
        off += t.size(dim);
    }
    return out;
}

}  // namespace
}  // namespace torch_kunlun

TORCH_LIBRARY_IMPL(aten, PrivateUse1, m) {
    m.impl("record_stream", TORCH_FN(torch_kunlun::record_stream));
    m.impl("empty.memory_format", TORCH_FN(torch_kunlun::empty_memory_format));
    m.impl("empty_strided", TORCH_FN(torch_kunlun::empty_strided));
    m.impl("as_strided", TORCH_FN(at::native::as_strided_tensorimpl));
    m.impl("view", TORCH_FN(at::native::view));
    m.impl("_reshape_alias", TORCH_FN(at::native::_reshape_alias));
    m.impl("resize_", TORCH_FN(torch_kunlun::resize_));
    m.impl("_local_scalar_dense", TORCH_FN(torch_kunlun::local_scalar_dense));
    m.impl("copy_", TORCH_FN(torch_kunlun::copy_));
    m.impl("_copy_from", TORCH_FN(torch_kunlun::_copy_from));
    m.impl("_copy_from_and_resize", TORCH_FN(torch_kunlun::_copy_from_and_resize));
    m.impl("clone", TORCH_FN(torch_kunlun::clone));
    m.impl("fill_.Scalar", TORCH_FN(torch_kunlun::fill_impl));
    m.impl("zero_", TORCH_FN(torch_kunlun::zero_impl));
    m.impl("cat", TORCH_FN(torch_kunlun::cat));
}
