// ops_nn.cpp -- row ops, activations, elementwise arithmetic and the fused
// attention of the kunlun backend.
//
// Counterparts in the reference: softmax / layer_norm / gelu
// (csrc/ops_nn.cpp:73-147, :309-345), add (csrc/ops.cpp:117-149), relu
// (csrc/ops.cpp:151-160), sub / mul / mul.Scalar / add_ / mul_
// (csrc/autograd.cpp:40-100, :586-601), silu (csrc/ops_extra.cpp:71) and the
// attention composition of torch_kunlun/kunlun/attention.py:36-107.
#include <torch/library.h>

#include <algorithm>
#include <cmath>

#include "kunlun.h"

namespace torch_kunlun {

namespace {

struct DeviceScope {
    int prev;
    explicit DeviceScope(int dev) : prev(current_device()) {
        if (dev >= 0 && dev != prev) cudaSetDevice(dev);
    }
    ~DeviceScope() { cudaSetDevice(prev); }
};

bool is_kunlun(const at::Tensor& t) { return t.device().type() == c10::DeviceType::PrivateUse1; }

at::Tensor softmax_lastdim(const at::Tensor& x, at::ScalarType out_t) {
    at::Tensor xc = x.contiguous();
    at::Tensor out = at::empty(xc.sizes(), xc.options().dtype(out_t));
    if (xc.numel() == 0) return out;
    const int64_t cols = xc.size(-1);
    const int64_t rows = xc.numel() / cols;
    const int dev = xc.device().index();
    DeviceScope g(dev);
    check_tk(tk_softmax(tk_dtype(xc.scalar_type()), tk_dtype(out_t), xc.data_ptr(), out.data_ptr(),
                        rows, cols, current_stream(dev)),
             "tk_softmax");
    return out;
}

at::Tensor _softmax(const at::Tensor& self, int64_t dim, bool half_to_float) {
    TORCH_CHECK(!half_to_float || self.scalar_type() == at::kHalf,
                "kunlun _softmax: half_to_float requires float16 input");
    const at::ScalarType out_t = half_to_float ? at::kFloat : self.scalar_type();
    if (self.dim() == 0) return softmax_lastdim(self.reshape({1}), out_t).reshape({});
    const int64_t d = c10::maybe_wrap_dim(dim, self.dim());
    if (d == self.dim() - 1) return softmax_lastdim(self, out_t);
    at::Tensor moved = self.movedim(d, -1);
    return softmax_lastdim(moved, out_t).movedim(-1, d).contiguous();
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> native_layer_norm(
    const at::Tensor& input, at::IntArrayRef normalized_shape,
    const std::optional<at::Tensor>& weight, const std::optional<at::Tensor>& bias, double eps) {
    int64_t n = 1;
    for (auto s : normalized_shape) n *= s;
    TORCH_CHECK(n > 0 && input.numel() % n == 0, "kunlun layer_norm: normalized_shape mismatch");
    at::Tensor x = input.contiguous();
    const int64_t rows = x.numel() / n;
    at::Tensor out = at::empty(x.sizes(), x.options());
    std::vector<int64_t> stat_shape = x.sizes().vec();
    for (size_t i = 0; i < normalized_shape.size(); ++i) stat_shape[x.dim() - 1 - i] = 1;
    at::Tensor mean = at::empty(stat_shape, x.options().dtype(at::kFloat));
    at::Tensor rstd = at::empty(stat_shape, x.options().dtype(at::kFloat));
    at::Tensor w, b;
    tk_dtype_t wdt = tk_dtype(x.scalar_type());
    if (weight.has_value() && weight->defined()) {
        w = weight->contiguous();
        wdt = tk_dtype(w.scalar_type());
    }
    if (bias.has_value() && bias->defined()) {
        b = bias->contiguous();
        if (!w.defined()) wdt = tk_dtype(b.scalar_type());
        TORCH_CHECK(tk_dtype(b.scalar_type()) == wdt, "kunlun layer_norm: weight/bias dtype mismatch");
    }
    if (rows > 0) {
        const int dev = x.device().index();
        DeviceScope g(dev);
        check_tk(tk_layer_norm(tk_dtype(x.scalar_type()), wdt, x.data_ptr(),
                               w.defined() ? w.data_ptr() : nullptr,
                               b.defined() ? b.data_ptr() : nullptr, out.data_ptr(),
                               mean.data_ptr<float>(), rstd.data_ptr<float>(), rows, n,
                               static_cast<float>(eps), current_stream(dev)),
                 "tk_layer_norm");
    }
    return {out, mean, rstd};
}

at::Tensor unary(const at::Tensor& self, int op, float p0 = 0.f, float p1 = 0.f) {
    at::Tensor x = self.contiguous();
    at::Tensor out = at::empty(x.sizes(), x.options());
    if (x.numel() == 0) return out;
    const int dev = x.device().index();
    DeviceScope g(dev);
    check_tk(tk_unary(op, tk_dtype(x.scalar_type()), x.data_ptr(), out.data_ptr(), x.numel(), p0,
                      p1, current_stream(dev)),
             "tk_unary");
    return out;
}

at::Tensor gelu(const at::Tensor& self, c10::string_view approximate) {
    return unary(self, approximate == "tanh" ? TK_UN_GELU_TANH : TK_UN_GELU);
}

at::Tensor silu(const at::Tensor& self) { return unary(self, TK_UN_SILU); }

at::Tensor relu(const at::Tensor& self) { return unary(self, TK_UN_RELU); }

at::Tensor& relu_(at::Tensor& self) {
    at::Tensor r = unary(self, TK_UN_RELU);
    self.copy_(r);
    return self;
}

// Elementwise binary op with broadcasting; a CPU 0-dim operand (a wrapped
// Python number) is applied as a scalar.
at::Tensor binary(const at::Tensor& a_in, const at::Tensor& b_in, int op, double alpha) {
    const bool a_scalar = !is_kunlun(a_in) && a_in.dim() == 0;
    const bool b_scalar = !is_kunlun(b_in) && b_in.dim() == 0;
    TORCH_CHECK(!(a_scalar && b_scalar), "kunlun binary op needs a kunlun tensor");
    const at::ScalarType rt = at::result_type(a_in, b_in);
    TORCH_CHECK(rt == at::kHalf || rt == at::kFloat,
                "kunlun arithmetic supports float16/float32, got ", rt);
    if (b_scalar || a_scalar) {
        const at::Tensor& t = b_scalar ? a_in : b_in;
        const double v = (b_scalar ? b_in : a_in).item<double>();
        at::Tensor x = t.scalar_type() == rt ? t : t.to(rt);
        switch (op) {
            case TK_BIN_ADD:
                return unary(x, TK_UN_SCALE, 1.f, static_cast<float>(b_scalar ? alpha * v : v));
            case TK_BIN_MUL: return unary(x, TK_UN_SCALE, static_cast<float>(v), 0.f);
            case TK_BIN_SUB:
                if (b_scalar) return unary(x, TK_UN_SCALE, 1.f, static_cast<float>(-alpha * v));
                return unary(x, TK_UN_SCALE, static_cast<float>(-alpha), static_cast<float>(v));
            case TK_BIN_DIV:
                // tensor / scalar multiplies by the reciprocal, as torch's CUDA
                // division by a CPU scalar does
                if (b_scalar) return unary(x, TK_UN_SCALE, static_cast<float>(1.0 / v), 0.f);
                break;  // scalar / tensor: the tensor path
            default:
                break;
        }
    }
    at::Tensor a = is_kunlun(a_in) ? a_in : a_in.to(b_in.device());
    at::Tensor b = is_kunlun(b_in) ? b_in : b_in.to(a_in.device());
    TORCH_CHECK(a.device() == b.device(), "kunlun binary op: tensors on different devices");
    if (a.scalar_type() != rt) a = a.to(rt);
    if (b.scalar_type() != rt) b = b.to(rt);
    const auto shape = at::infer_size(a.sizes(), b.sizes());
    TORCH_CHECK(shape.size() <= 8, "kunlun binary op: at most 8 dims");
    at::Tensor ae = a.expand(shape), be = b.expand(shape);
    at::Tensor out = at::empty(shape, a.options());
    if (out.numel() == 0) return out;
    std::vector<int64_t> sizes(shape.begin(), shape.end());
    std::vector<int64_t> sa = ae.strides().vec(), sb = be.strides().vec();
    const int dev = out.device().index();
    DeviceScope g(dev);
    check_tk(tk_binary(op, tk_dtype(rt), ae.data_ptr(), sa.data(), be.data_ptr(), sb.data(),
                       out.data_ptr(), static_cast<int>(sizes.size()), sizes.data(),
                       static_cast<float>(alpha), current_stream(dev)),
             "tk_binary");
    return out;
}

at::Tensor add(const at::Tensor& self, const at::Tensor& other, const at::Scalar& alpha) {
    return binary(self, other, TK_BIN_ADD, alpha.toDouble());
}
at::Tensor sub(const at::Tensor& self, const at::Tensor& other, const at::Scalar& alpha) {
    return binary(self, other, TK_BIN_SUB, alpha.toDouble());
}
at::Tensor mul(const at::Tensor& self, const at::Tensor& other) {
    return binary(self, other, TK_BIN_MUL, 1.0);
}
at::Tensor div(const at::Tensor& self, const at::Tensor& other) {
    return binary(self, other, TK_BIN_DIV, 1.0);
}
at::Tensor mul_scalar(const at::Tensor& self, const at::Scalar& other) {
    return unary(self, TK_UN_SCALE, static_cast<float>(other.toDouble()), 0.f);
}
at::Tensor& add_(at::Tensor& self, const at::Tensor& other, const at::Scalar& alpha) {
    self.copy_(binary(self, other, TK_BIN_ADD, alpha.toDouble()));
    return self;
}
at::Tensor& mul_(at::Tensor& self, const at::Tensor& other) {
    self.copy_(binary(self, other, TK_BIN_MUL, 1.0));
    return self;
}
at::Tensor& sub_(at::Tensor& self, const at::Tensor& other, const at::Scalar& alpha) {
    self.copy_(binary(self, other, TK_BIN_SUB, alpha.toDouble()));
    return self;
}
at::Tensor& div_(at::Tensor& self, const at::Tensor& other) {
    self.copy_(binary(self, other, TK_BIN_DIV, 1.0));
    return self;
}

// out= variants write through copy_, so `out` may be any strided view (DDP's
// reducer multiplies each gradient by 1/world_size straight into its bucket
// view: at::mul_out(bucket_view, grad, wrapped_scalar)).
at::Tensor& out_result(at::Tensor& out, const at::Tensor& r) {
    if (!out.sizes().equals(r.sizes())) {
        TORCH_CHECK(out.numel() == 0 || out.is_contiguous(), "kunlun out=: cannot resize a non-contiguous output");
        out.resize_(r.sizes());
    }
    out.copy_(r);
    return out;
}
at::Tensor& mul_out(const at::Tensor& self, const at::Tensor& other, at::Tensor& out) {
    return out_result(out, binary(self, other, TK_BIN_MUL, 1.0));
}
at::Tensor& add_out(const at::Tensor& self, const at::Tensor& other, const at::Scalar& alpha, at::Tensor& out) {
    return out_result(out, binary(self, other, TK_BIN_ADD, alpha.toDouble()));
}
at::Tensor& div_out(const at::Tensor& self, const at::Tensor& other, at::Tensor& out) {
    return out_result(out, binary(self, other, TK_BIN_DIV, 1.0));
}

// ---- backward support: relu gradient, sums, MSE loss --------------------------

// relu's backward (torch's threshold_backward): grad where self > threshold.
at::Tensor threshold_backward(const at::Tensor& grad_output, const at::Tensor& self,
                              const at::Scalar& threshold) {
    return binary(grad_output, self, TK_BIN_THRESHOLD_BACKWARD, threshold.toDouble());
}

// Sum over `dims` (all when empty) in fp32 with one rounding to the output
// dtype (fp16 input may sum into fp32).  Reduced dims that form one block of
// the shape are summed in place; otherwise they are moved last first.
at::Tensor sum_dim(const at::Tensor& self, at::OptionalIntArrayRef dim, bool keepdim,
                   std::optional<at::ScalarType> dtype) {
    const at::ScalarType in_t = self.scalar_type();
    const at::ScalarType out_t = dtype.value_or(in_t);
    TORCH_CHECK((in_t == at::kHalf && (out_t == at::kHalf || out_t == at::kFloat)) ||
                    (in_t == at::kFloat && out_t == at::kFloat),
                "kunlun sum supports float16 -> float16/float32 and float32 -> float32, got ", in_t,
                " -> ", out_t);
    const int64_t nd = self.dim();
    std::vector<bool> red(std::max<int64_t>(nd, 1), false);
    if (!dim.has_value() || dim->empty()) {
        std::fill(red.begin(), red.end(), true);
    } else {
        for (int64_t d : *dim) red[c10::maybe_wrap_dim(d, std::max<int64_t>(nd, 1))] = true;
    }
    std::vector<int64_t> out_shape, kept_dims, red_dims;
    for (int64_t d = 0; d < nd; ++d) {
        if (red[d]) {
            red_dims.push_back(d);
            if (keepdim) out_shape.push_back(1);
        } else {
            kept_dims.push_back(d);
            out_shape.push_back(self.size(d));
        }
    }
    at::Tensor out = at::empty(out_shape, self.options().dtype(out_t));
    if (out.numel() == 0) return out;
    at::Tensor x;
    int64_t outer = 1, rcount = 1, inner = 1;
    const bool block = red_dims.empty() || red_dims.back() - red_dims.front() + 1 ==
                                               static_cast<int64_t>(red_dims.size());
    if (nd == 0) {
        x = self.reshape({1});
    } else if (block) {
        x = self.contiguous();
        const int64_t lo = red_dims.empty() ? nd : red_dims.front();
        const int64_t hi = red_dims.empty() ? nd - 1 : red_dims.back();
        for (int64_t d = 0; d < lo; ++d) outer *= self.size(d);
        for (int64_t d = lo; d <= hi; ++d) rcount *= self.size(d);
        for (int64_t d = hi + 1; d < nd; ++d) inner *= self.size(d);
    } else {
        std::vector<int64_t> perm(kept_dims);
        perm.insert(perm.end(), red_dims.begin(), red_dims.end());
        x = self.permute(perm).contiguous();
        for (int64_t d : kept_dims) outer *= self.size(d);
        for (int64_t d : red_dims) rcount *= self.size(d);
    }
    if (rcount == 0) return out.zero_();
    const int dev = self.device().index();
    DeviceScope g(dev);
    check_tk(tk_reduce_sum(tk_dtype(in_t), tk_dtype(out_t), x.data_ptr(), outer, rcount, inner,
                           out.data_ptr(), current_stream(dev)),
             "tk_reduce_sum");
    return out;
}

at::Tensor sum_all(const at::Tensor& self, std::optional<at::ScalarType> dtype) {
    return sum_dim(self, std::nullopt, false, dtype);
}

// MSE loss with the reference's reduction codes (0 none, 1 mean, 2 sum): the
// difference and its square rounded to T, the reduction summed in fp32.
at::Tensor mse_loss(const at::Tensor& self, const at::Tensor& target, int64_t reduction) {
    at::Tensor d = binary(self, target, TK_BIN_SUB, 1.0);
    at::Tensor sq = binary(d, d, TK_BIN_MUL, 1.0);
    if (reduction == 0) return sq;
    at::Tensor s = sum_dim(sq, std::nullopt, false, at::kFloat);
    if (reduction == 1) s = unary(s, TK_UN_SCALE, static_cast<float>(1.0 / std::max<int64_t>(1, sq.numel())), 0.f);
    return s.to(self.scalar_type());
}

at::Tensor mse_loss_backward(const at::Tensor& grad_output, const at::Tensor& self,
                             const at::Tensor& target, int64_t reduction) {
    const double norm = reduction == 1 ? 2.0 / std::max<int64_t>(1, self.numel()) : 2.0;
    at::Tensor d = binary(self, target, TK_BIN_SUB, 1.0);
    at::Tensor g = binary(d, grad_output, TK_BIN_MUL, 1.0);
    return unary(g, TK_UN_SCALE, static_cast<float>(norm), 0.f);
}

}  // namespace

at::Tensor silu_mul(const at::Tensor& gate, const at::Tensor& up) {
    TORCH_CHECK(gate.sizes().equals(up.sizes()) && gate.scalar_type() == up.scalar_type(),
                "kunlun silu_mul: shape/dtype mismatch");
    at::Tensor g = gate.contiguous(), u = up.contiguous();
    at::Tensor out = at::empty(g.sizes(), g.options());
    if (g.numel() == 0) return out;
    const int dev = g.device().index();
    DeviceScope s(dev);
    check_tk(tk_silu_mul(tk_dtype(g.scalar_type()), g.data_ptr(), u.data_ptr(), out.data_ptr(),
                         g.numel(), current_stream(dev)),
             "tk_silu_mul");
    return out;
}

// (T(silu(gate)) * up, max |result| as a 1-element fp32 tensor) in one pass:
// the gate of a SiLU-gated MLP and the scale the next quantised GEMM takes.
std::tuple<at::Tensor, at::Tensor> silu_mul_amax(const at::Tensor& gate, const at::Tensor& up) {
    TORCH_CHECK(gate.sizes().equals(up.sizes()) && gate.scalar_type() == up.scalar_type(),
                "kunlun silu_mul_amax: shape/dtype mismatch");
    at::Tensor g = gate.contiguous(), u = up.contiguous();
    at::Tensor out = at::empty(g.sizes(), g.options());
    at::Tensor amax = at::empty({1}, g.options().dtype(at::kFloat));
    const int dev = g.device().index();
    DeviceScope s(dev);
    check_tk(tk_silu_mul_amax(tk_dtype(g.scalar_type()), g.data_ptr(), u.data_ptr(), out.data_ptr(), g.numel(),
                              amax.data_ptr<float>(), current_stream(dev)),
             "tk_silu_mul_amax");
    return {out, amax};
}

}  // namespace torch_kunlun

TORCH_LIBRARY_IMPL(aten, PrivateUse1, m) {
    m.impl("_softmax", TORCH_FN(torch_kunlun::_softmax));
    m.impl("native_layer_norm", TORCH_FN(torch_kunlun::native_layer_norm));
    m.impl("gelu", TORCH_FN(torch_kunlun::gelu));
    m.impl("silu", TORCH_FN(torch_kunlun::silu));
    m.impl("relu", TORCH_FN(torch_kunlun::relu));
    m.impl("relu_", TORCH_FN(torch_kunlun::relu_));
    m.impl("add.Tensor", TORCH_FN(torch_kunlun::add));
    m.impl("sub.Tensor", TORCH_FN(torch_kunlun::sub));
    m.impl("mul.Tensor", TORCH_FN(torch_kunlun::mul));
    m.impl("div.Tensor", TORCH_FN(torch_kunlun::div));
    m.impl("mul.Scalar", TORCH_FN(torch_kunlun::mul_scalar));
    m.impl("add_.Tensor", TORCH_FN(torch_kunlun::add_));
    m.impl("mul_.Tensor", TORCH_FN(torch_kunlun::mul_));
    m.impl("sub_.Tensor", TORCH_FN(torch_kunlun::sub_));
    m.impl("div_.Tensor", TORCH_FN(torch_kunlun::div_));
    m.impl("mul.out", TORCH_FN(torch_kunlun::mul_out));
    m.impl("add.out", TORCH_FN(torch_kunlun::add_out));
    m.impl("div.out", TORCH_FN(torch_kunlun::div_out));
    m.impl("threshold_backward", TORCH_FN(torch_kunlun::threshold_backward));
    m.impl("sum.dim_IntList", TORCH_FN(torch_kunlun::sum_dim));
    m.impl("sum", TORCH_FN(torch_kunlun::sum_all));
    m.impl("mse_loss", TORCH_FN(torch_kunlun::mse_loss));
    m.impl("mse_loss_backward", TORCH_FN(torch_kunlun::mse_loss_backward));
}
