// ops_dense.cpp -- the quantised dense-op hot path of the kunlun backend:
// mm, addmm, bmm, baddbmm, linear and conv2d (TORCH_LIBRARY_IMPL(aten,
// PrivateUse1)), plus the fused linear+activation and SiLU-gate helpers.
//
// Counterparts in the reference: fc_impl / mm / linear (csrc/ops.cpp:210-230,
// :480-495, :579-588), conv2d_impl (csrc/ops.cpp:237-285), bmm_impl
// (csrc/ops_nn.cpp:199-221), addmm (csrc/autograd.cpp:192-218) and baddbmm
// (csrc/linalg_extra.cpp:85-93).  Where the reference issues one XDNN fc per
// batch slice and separate scale/add launches, each op here is one call of
// the C ABI (tk_qgemm / tk_conv2d_q16) whose epilogue applies alpha, bias,
// beta*self and the activation in the reference's order and rounding.
#include <torch/library.h>

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

void check_operand(const at::Tensor& t, const at::Tensor& ref, const char* what) {
    TORCH_CHECK(t.device().type() == c10::DeviceType::PrivateUse1, what,
                " requires kunlun tensors, got ", t.device());
    TORCH_CHECK(t.device() == ref.device(), what, " requires tensors on one device");
    TORCH_CHECK(t.scalar_type() == ref.scalar_type(), what, " requires matching dtypes, got ",
                ref.scalar_type(), " and ", t.scalar_type());
}

// A [B, R, C] operand whose every slice is a dense row- or column-major block
// (what the quantiser reads directly); anything else is made contiguous on
// the device first.
at::Tensor dense_slices(const at::Tensor& t, bool whole_block) {
    const int64_t R = t.size(1), C = t.size(2);
    const int64_t sr = t.stride(1), sc = t.stride(2);
    bool ok = (R <= 1 || C <= 1) || (sr == C && sc == 1) || (sr == 1 && sc == R);
    if (ok && t.size(0) > 1) ok = t.stride(0) == R * C || (!whole_block && t.stride(0) >= R * C);
    if (ok && t.size(0) > 1 && !whole_block) {
        // per-slice scales only need each slice dense; overlapping slices are fine too
        ok = true;
    }
    return ok ? t : t.contiguous();
}

// out[b] = epilogue(q(a[b]) @ q(b_nk[b])^T); a [B,M,K], b_nk [B,N,K] views,
// out [B,M,N] with unit stride along N.
void run_qgemm(const at::Tensor& a_in, const at::Tensor& b_in, at::Tensor& out,
               const std::optional<at::Tensor>& bias, const at::Tensor* addend, double alpha,
               double beta, int act, bool per_slice, const float* amax_a = nullptr,
               const float* amax_b = nullptr) {
    const int dev = out.device().index();
    DeviceScope g(dev);
    const bool whole = !per_slice;
    at::Tensor a = dense_slices(a_in, whole);
    at::Tensor b = dense_slices(b_in, whole);
    if (whole) {
        // one scale for the whole operand: it must be one dense block
        if (a.size(0) > 1 && a.stride(0) != a.size(1) * a.size(2)) a = a.contiguous();
        if (b.size(0) > 1 && b.stride(0) != b.size(1) * b.size(2)) b = b.contiguous();
    }
    tk_qgemm_desc_t d = {};
    d.dtype = tk_dtype(a.scalar_type());
    d.batch = a.size(0);
    d.m = a.size(1);
    d.n = b.size(1);
    d.k = a.size(2);
    d.a = a.data_ptr();
    d.a_sb = a.stride(0);
    d.a_sm = a.stride(1);
    d.a_sk = a.stride(2);
    d.b = b.data_ptr();
    d.b_sb = b.stride(0);
    d.b_sn = b.stride(1);
    d.b_sk = b.stride(2);
    d.out = out.data_ptr();
    d.out_sb = out.stride(0);
    d.out_sm = out.stride(1);
    at::Tensor bias_c;
    if (bias.has_value() && bias->defined()) {
        bias_c = bias->contiguous();
        TORCH_CHECK(bias_c.numel() == d.n, "kunlun: bias size mismatch");
        check_operand(bias_c, a, "bias");
        d.bias = bias_c.data_ptr();
    }
    at::Tensor add_v;
    if (addend != nullptr && beta != 0.0) {
        add_v = addend->expand({d.batch, d.m, d.n});
        check_operand(add_v, a, "addend");
        d.addend = add_v.data_ptr();
        d.add_sb = add_v.stride(0);
        d.add_sm = add_v.stride(1);
        d.add_sn = add_v.stride(2);
    }
    d.alpha = static_cast<float>(alpha);
    d.beta = static_cast<float>(beta);
    d.act = static_cast<tk_act_t>(act);
    d.per_slice_scales = per_slice ? 1 : 0;
    d.amax_a = amax_a;
    d.amax_b = amax_b;
    const size_t ws_bytes = tk_qgemm_workspace_size(&d);
    at::Tensor ws = workspace(ws_bytes, out.device());
    check_tk(tk_qgemm(&d, aligned_base(ws), ws_bytes, current_stream(dev)), "tk_qgemm");
}

at::Tensor mm(const at::Tensor& self, const at::Tensor& mat2) {
    TORCH_CHECK(self.dim() == 2 && mat2.dim() == 2, "kunlun mm requires 2-D tensors");
    check_operand(mat2, self, "mm");
    TORCH_CHECK(self.size(1) == mat2.size(0), "kunlun mm inner dimensions mismatch: ",
                self.sizes(), " @ ", mat2.sizes());
    at::Tensor out = at::empty({self.size(0), mat2.size(1)}, self.options());
    if (out.numel() == 0) return out;
    at::Tensor o3 = out.unsqueeze(0);
    run_qgemm(self.unsqueeze(0), mat2.t().unsqueeze(0), o3, std::nullopt, nullptr, 1.0, 0.0,
              TK_ACT_NONE, true);
    return out;
}

at::Tensor addmm(const at::Tensor& self, const at::Tensor& mat1, const at::Tensor& mat2,
                 const at::Scalar& beta, const at::Scalar& alpha) {
    TORCH_CHECK(mat1.dim() == 2 && mat2.dim() == 2, "kunlun addmm requires 2-D matrices");
    check_operand(mat2, mat1, "addmm");
    TORCH_CHECK(mat1.size(1) == mat2.size(0), "kunlun addmm inner dimensions mismatch");
    at::Tensor out = at::empty({mat1.size(0), mat2.size(1)}, mat1.options());
    if (out.numel() == 0) return out;
    at::Tensor o3 = out.unsqueeze(0);
    const double b = beta.toDouble();
    at::Tensor add3;
    if (b != 0.0) {
        check_operand(self, mat1, "addmm self");
        add3 = self.expand({mat1.size(0), mat2.size(1)}).unsqueeze(0);
    }
    run_qgemm(mat1.unsqueeze(0), mat2.t().unsqueeze(0), o3, std::nullopt,
              b != 0.0 ? &add3 : nullptr, alpha.toDouble(), b, TK_ACT_NONE, true);
    return out;
}

at::Tensor bmm(const at::Tensor& self, const at::Tensor& mat2) {
    TORCH_CHECK(self.dim() == 3 && mat2.dim() == 3, "kunlun bmm requires 3-D tensors");
    check_operand(mat2, self, "bmm");
    TORCH_CHECK(self.size(0) == mat2.size(0) && self.size(2) == mat2.size(1),
                "kunlun bmm shape mismatch: ", self.sizes(), " @ ", mat2.sizes());
    at::Tensor out = at::empty({self.size(0), self.size(1), mat2.size(2)}, self.options());
    if (out.numel() == 0) return out;
    run_qgemm(self, mat2.transpose(1, 2), out, std::nullopt, nullptr, 1.0, 0.0, TK_ACT_NONE, true);
    return out;
}

at::Tensor baddbmm(const at::Tensor& self, const at::Tensor& batch1, const at::Tensor& batch2,
                   const at::Scalar& beta, const at::Scalar& alpha) {
    TORCH_CHECK(batch1.dim() == 3 && batch2.dim() == 3, "kunlun baddbmm requires 3-D tensors");
    check_operand(batch2, batch1, "baddbmm");
    at::Tensor out = at::empty({batch1.size(0), batch1.size(1), batch2.size(2)}, batch1.options());
    if (out.numel() == 0) return out;
    const double b = beta.toDouble();
    at::Tensor add3;
    if (b != 0.0) {
        check_operand(self, batch1, "baddbmm self");
        add3 = self.expand(out.sizes());
    }
    run_qgemm(batch1, batch2.transpose(1, 2), out, std::nullopt, b != 0.0 ? &add3 : nullptr,
              alpha.toDouble(), b, TK_ACT_NONE, true);
    return out;
}

std::vector<int64_t> pair_of(at::IntArrayRef v, int64_t dflt) {
    if (v.empty()) return {dflt, dflt};
    if (v.size() == 1) return {v[0], v[0]};
    TORCH_CHECK(v.size() == 2, "kunlun conv2d expects 1 or 2 element arrays");
    return {v[0], v[1]};
}

at::Tensor conv2d_impl(const at::Tensor& input, const at::Tensor& weight,
                       const std::optional<at::Tensor>& bias, at::IntArrayRef stride,
                       at::IntArrayRef padding, at::IntArrayRef dilation, int64_t groups) {
    check_operand(weight, input, "conv2d");
    const bool batched = input.dim() == 4;
    TORCH_CHECK((input.dim() == 4 || input.dim() == 3) && weight.dim() == 4,
                "kunlun conv2d requires NCHW (or CHW) input and OIHW weight");
    at::Tensor x = (batched ? input : input.unsqueeze(0)).contiguous();
    at::Tensor w = weight.contiguous();
    const auto s = pair_of(stride, 1), p = pair_of(padding, 0), dl = pair_of(dilation, 1);
    tk_conv2d_desc_t d = {};
    d.dtype = tk_dtype(x.scalar_type());
    d.n = x.size(0);
    d.c = x.size(1);
    d.h = x.size(2);
    d.w = x.size(3);
    d.f = w.size(0);
    d.kh = w.size(2);
    d.kw = w.size(3);
    d.stride_h = s[0];
    d.stride_w = s[1];
    d.pad_h = p[0];
    d.pad_w = p[1];
    d.dil_h = dl[0];
    d.dil_w = dl[1];
    d.groups = groups;
    TORCH_CHECK(groups > 0 && d.c % groups == 0 && w.size(1) == d.c / groups,
                "kunlun conv2d: weight/input channel mismatch");
    const int64_t oh = (d.h + 2 * d.pad_h - d.dil_h * (d.kh - 1) - 1) / d.stride_h + 1;
    const int64_t ow = (d.w + 2 * d.pad_w - d.dil_w * (d.kw - 1) - 1) / d.stride_w + 1;
    TORCH_CHECK(oh > 0 && ow > 0, "kunlun conv2d produced non-positive output shape");
    at::Tensor out = at::empty({d.n, d.f, oh, ow}, x.options());
    at::Tensor b;
    if (bias.has_value() && bias->defined()) {
        b = bias->contiguous();
        check_operand(b, x, "conv2d bias");
        TORCH_CHECK(b.numel() == d.f, "kunlun conv2d bias size mismatch");
        d.bias = b.data_ptr();
    }
    d.x = x.data_ptr();
    d.weight = w.data_ptr();
    d.out = out.data_ptr();
    const int dev = x.device().index();
    DeviceScope g(dev);
    if (out.numel() > 0) {
        const size_t ws_bytes = tk_conv2d_workspace_size(&d);
        at::Tensor ws = workspace(ws_bytes, x.device());
        check_tk(tk_conv2d_q16(&d, aligned_base(ws), ws_bytes, current_stream(dev)), "tk_conv2d_q16");
    }
    return batched ? out : out.squeeze(0);
}

at::Tensor conv2d(const at::Tensor& input, const at::Tensor& weight,
                  const std::optional<at::Tensor>& bias, at::IntArrayRef stride,
                  at::IntArrayRef padding, at::IntArrayRef dilation, int64_t groups) {
    return conv2d_impl(input, weight, bias, stride, padding, dilation, groups);
}

// aten::convolution_overrideable is where aten::convolution sends backends
// that are not built in (F.conv2d on a kunlun tensor with autograd active).
at::Tensor convolution_overrideable(const at::Tensor& input, const at::Tensor& weight,
                                    const std::optional<at::Tensor>& bias, at::IntArrayRef stride,
                                    at::IntArrayRef padding, at::IntArrayRef dilation,
                                    bool transposed, at::IntArrayRef output_padding,
                                    int64_t groups) {
    TORCH_CHECK(!transposed, "kunlun: transposed convolution is not implemented");
    TORCH_CHECK(input.dim() == 4 || input.dim() == 3, "kunlun: only 2-D convolution is implemented");
    return conv2d_impl(input, weight, bias, stride, padding, dilation, groups);
}

}  // namespace

// y = act(x @ W^T + b) for x [..., K], W [N, K] in one call.
at::Tensor linear_act(const at::Tensor& input, const at::Tensor& weight,
                      const std::optional<at::Tensor>& bias, int64_t act,
                      const std::optional<at::Tensor>& residual) {
    TORCH_CHECK(input.dim() >= 1 && weight.dim() == 2, "kunlun linear: bad ranks");
    check_operand(weight, input, "linear");
    const int64_t K = input.size(-1);
    TORCH_CHECK(weight.size(1) == K, "kunlun linear: in_features mismatch (", K, " vs ",
                weight.size(1), ")");
    const int64_t N = weight.size(0);
    at::Tensor x2 = input.reshape({-1, K});
    std::vector<int64_t> out_shape = input.sizes().vec();
    out_shape.back() = N;
    at::Tensor out = at::empty({x2.size(0), N}, input.options());
    if (out.numel() > 0) {
        at::Tensor o3 = out.unsqueeze(0);
        at::Tensor r3;
        if (residual.has_value() && residual->defined()) {
            TORCH_CHECK(residual->numel() == out.numel() && residual->size(-1) == N,
                        "kunlun linear: residual shape mismatch");
            r3 = residual->reshape({1, x2.size(0), N});
        }
        run_qgemm(x2.unsqueeze(0), weight.unsqueeze(0), o3, bias, r3.defined() ? &r3 : nullptr,
                  1.0, r3.defined() ? 1.0 : 0.0, static_cast<int>(act), true);
    }
    return out.view(out_shape);
}

// max |x| over the whole tensor as a 1-element fp32 kunlun tensor (the
// per-tensor quantisation scale source).
at::Tensor amax(const at::Tensor& x_in) {
    TORCH_CHECK(x_in.device().type() == c10::DeviceType::PrivateUse1, "kunlun amax: kunlun tensor");
    at::Tensor x = x_in.contiguous();
    at::Tensor out = at::empty({1}, x.options().dtype(at::kFloat));
    const int dev = x.device().index();
    DeviceScope g(dev);
    check_tk(tk_amax(tk_dtype(x.scalar_type()), x.data_ptr(), 1, 0, x.numel(),
                     out.data_ptr<float>(), current_stream(dev)),
             "tk_amax");
    return out;
}

// act(x @ W^T + b) with the per-tensor scales given (1-element fp32 tensors
// from amax(); None computes that operand's amax).  Splitting x into row
// blocks and passing the whole tensor's amax gives exactly the values of
// one unsplit call.
at::Tensor linear_scaled(const at::Tensor& input, const at::Tensor& weight,
                         const std::optional<at::Tensor>& bias, int64_t act,
                         const std::optional<at::Tensor>& amax_x,
                         const std::optional<at::Tensor>& amax_w,
                         const std::optional<at::Tensor>& out_opt) {
    TORCH_CHECK(input.dim() == 2 && weight.dim() == 2, "kunlun linear_scaled: 2-D operands");
    check_operand(weight, input, "linear_scaled");
    TORCH_CHECK(weight.size(1) == input.size(1), "kunlun linear_scaled: in_features mismatch");
    auto scale_ptr = [&](const std::optional<at::Tensor>& t) -> const float* {
        if (!t.has_value() || !t->defined()) return nullptr;
        TORCH_CHECK(t->scalar_type() == at::kFloat && t->numel() >= 1 && t->device() == input.device(),
                    "kunlun linear_scaled: scales must be fp32 kunlun tensors");
        return t->data_ptr<float>();
    };
    at::Tensor out;
    if (out_opt.has_value() && out_opt->defined()) {
        out = *out_opt;  // e.g. a row block of a larger output
        TORCH_CHECK(out.dim() == 2 && out.size(0) == input.size(0) && out.size(1) == weight.size(0) &&
                        out.stride(1) == 1 && out.scalar_type() == input.scalar_type() &&
                        out.device() == input.device(),
                    "kunlun linear_scaled: out must be a row-major [M, N] block of the input dtype");
    } else {
        out = at::empty({input.size(0), weight.size(0)}, input.options());
    }
    if (out.numel() > 0) {
        at::Tensor o3 = out.unsqueeze(0);
        run_qgemm(input.unsqueeze(0), weight.unsqueeze(0), o3, bias, nullptr, 1.0, 0.0,
                  static_cast<int>(act), true, scale_ptr(amax_x), scale_ptr(amax_w));
    }
    return out;
}

namespace {

at::Tensor linear_fwd(const at::Tensor& input, const at::Tensor& weight,
                      const std::optional<at::Tensor>& bias) {
    return linear_act(input, weight, bias, TK_ACT_NONE, std::nullopt);
}

// Autograd entry for linear: without gradients the fused kernel runs below
// autograd; with gradients torch's own decomposition (addmm / matmul) records
// the graph on the same quantised kernels, with identical forward values.
at::Tensor linear_autograd(const at::Tensor& input, const at::Tensor& weight,
                           const std::optional<at::Tensor>& bias) {
    const bool needs_grad = at::GradMode::is_enabled() &&
                            (input.requires_grad() || weight.requires_grad() ||
                             (bias.has_value() && bias->defined() && bias->requires_grad()));
    if (needs_grad) return at::native::linear(input, weight, bias);
    at::AutoDispatchBelowADInplaceOrView guard;
    return linear_fwd(input, weight, bias);
}

}  // namespace
}  // namespace torch_kunlun

TORCH_LIBRARY_IMPL(aten, PrivateUse1, m) {
    m.impl("mm", TORCH_FN(torch_kunlun::mm));
    m.impl("addmm", TORCH_FN(torch_kunlun::addmm));
    m.impl("bmm", TORCH_FN(torch_kunlun::bmm));
    m.impl("baddbmm", TORCH_FN(torch_kunlun::baddbmm));
    m.impl("linear", TORCH_FN(torch_kunlun::linear_fwd));
    m.impl("conv2d", TORCH_FN(torch_kunlun::conv2d));
    m.impl("convolution_overrideable", TORCH_FN(torch_kunlun::convolution_overrideable));
}

TORCH_LIBRARY_IMPL(aten, AutogradPrivateUse1, m) {
    m.impl("linear", TORCH_FN(torch_kunlun::linear_autograd));
}
