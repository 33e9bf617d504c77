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
               const float* amax_b = nullptr, float* amax_out = nullptr) {
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
    d.amax_out = amax_out;
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

// 1-D products on the quantised mm, each vector one per-tensor scale: the
// matmul cases the reference stages through the CPU
// (csrc/linalg_extra.cpp:232-236) -- torch's matmul sends 1-D x 1-D to dot
// and a (folded) matrix x vector to mv.
at::Tensor dot(const at::Tensor& self, const at::Tensor& other) {
    TORCH_CHECK(self.dim() == 1 && other.dim() == 1, "kunlun dot requires 1-D tensors");
    TORCH_CHECK(self.size(0) == other.size(0), "kunlun dot: sizes differ (", self.size(0), " vs ",
                other.size(0), ")");
    return ::torch_kunlun::mm(self.unsqueeze(0), other.unsqueeze(1)).view(at::IntArrayRef{});
}

at::Tensor mv(const at::Tensor& self, const at::Tensor& vec) {
    TORCH_CHECK(self.dim() == 2 && vec.dim() == 1, "kunlun mv requires a matrix and a vector");
    return ::torch_kunlun::mm(self, vec.unsqueeze(1)).view({self.size(0)});
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

// Per-axis convolution parameter: [v] broadcasts, [] takes the default.
std::vector<int64_t> axis_param(at::IntArrayRef v, int64_t k, int64_t dflt, const char* what) {
    if (v.empty()) return std::vector<int64_t>(k, dflt);
    if (v.size() == 1) return std::vector<int64_t>(k, v[0]);
    TORCH_CHECK(static_cast<int64_t>(v.size()) == k, "kunlun conv: ", what, " needs 1 or ", k, " values");
    return v.vec();
}

// Quantised 2-D or 3-D convolution (NCHW / NCDHW, a CHW input is one
// image): one tk_conv3d_q16 call, a 2-D convolution being the 3-D one with
// depth 1.  amax_x / amax_w override the per-tensor scales (device fp32).
at::Tensor conv_impl(const at::Tensor& input, const at::Tensor& weight,
                     const std::optional<at::Tensor>& bias, at::IntArrayRef stride,
                     at::IntArrayRef padding, at::IntArrayRef dilation, int64_t groups,
                     const float* amax_x = nullptr, const float* amax_w = nullptr) {
    check_operand(weight, input, "conv");
    const int64_t k = weight.dim() - 2;
    TORCH_CHECK((k == 2 || k == 3) && (input.dim() == k + 2 || (k == 2 && input.dim() == 3)),
                "kunlun conv requires NCHW (or CHW) input with OIHW weight, or NCDHW with OIDHW");
    const bool batched = input.dim() == k + 2;
    at::Tensor x = (batched ? input : input.unsqueeze(0)).contiguous();
    at::Tensor w = weight.contiguous();
    const auto s = axis_param(stride, k, 1, "stride"), p = axis_param(padding, k, 0, "padding"),
               dl = axis_param(dilation, k, 1, "dilation");
    const int64_t o = k == 3 ? 0 : 1;  // 2-D: the depth axis is absent
    tk_conv3d_desc_t d = {};
    d.dtype = tk_dtype(x.scalar_type());
    d.n = x.size(0);
    d.c = x.size(1);
    d.d = k == 3 ? x.size(2) : 1;
    d.h = x.size(3 - o);
    d.w = x.size(4 - o);
    d.f = w.size(0);
    d.kd = k == 3 ? w.size(2) : 1;
    d.kh = w.size(3 - o);
    d.kw = w.size(4 - o);
    d.stride_d = k == 3 ? s[0] : 1;
    d.stride_h = s[1 - o];
    d.stride_w = s[2 - o];
    d.pad_d = k == 3 ? p[0] : 0;
    d.pad_h = p[1 - o];
    d.pad_w = p[2 - o];
    d.dil_d = k == 3 ? dl[0] : 1;
    d.dil_h = dl[1 - o];
    d.dil_w = dl[2 - o];
    d.groups = groups;
    TORCH_CHECK(groups > 0 && d.c % groups == 0 && w.size(1) == d.c / groups,
                "kunlun conv: weight/input channel mismatch");
    std::vector<int64_t> shape = {d.n, d.f};
    for (int64_t i = 0; i < k; ++i) {
        const int64_t o_i = (x.size(2 + i) + 2 * p[i] - dl[i] * (w.size(2 + i) - 1) - 1) / s[i] + 1;
        TORCH_CHECK(o_i > 0, "kunlun conv produced non-positive output shape");
        shape.push_back(o_i);
    }
    at::Tensor out = at::empty(shape, x.options());
    at::Tensor b;
    if (bias.has_value() && bias->defined()) {
        b = bias->contiguous();
        check_operand(b, x, "conv bias");
        TORCH_CHECK(b.numel() == d.f, "kunlun conv bias size mismatch");
        d.bias = b.data_ptr();
    }
    d.x = x.data_ptr();
    d.weight = w.data_ptr();
    d.out = out.data_ptr();
    d.amax_x = amax_x;
    d.amax_w = amax_w;
    const int dev = x.device().index();
    DeviceScope g(dev);
    if (out.numel() > 0) {
        const size_t ws_bytes = tk_conv3d_workspace_size(&d);
        at::Tensor ws = workspace(ws_bytes, x.device());
        check_tk(tk_conv3d_q16(&d, aligned_base(ws), ws_bytes, current_stream(dev)), "tk_conv3d_q16");
    }
    return batched ? out : out.squeeze(0);
}

at::Tensor conv2d(const at::Tensor& input, const at::Tensor& weight,
                  const std::optional<at::Tensor>& bias, at::IntArrayRef stride,
                  at::IntArrayRef padding, at::IntArrayRef dilation, int64_t groups) {
    TORCH_CHECK(weight.dim() == 4, "kunlun conv2d requires an OIHW weight");
    return conv_impl(input, weight, bias, stride, padding, dilation, groups);
}

// w [A, B, K...] with every spatial axis reversed, as a device strided copy
// that reads the source with negative strides from its last tap.
at::Tensor flip_spatial(const at::Tensor& w_in) {
    at::Tensor w = w_in.contiguous();
    at::Tensor out = at::empty(w.sizes(), w.options());
    if (w.numel() == 0) return out;
    const int64_t nd = w.dim();
    std::vector<int64_t> sizes = w.sizes().vec(), dst = w.strides().vec(), src = dst;
    int64_t last = 0;
    for (int64_t i = 2; i < nd; ++i) {
        src[i] = -dst[i];
        last += (sizes[i] - 1) * dst[i];
    }
    const int dev = w.device().index();
    DeviceScope g(dev);
    const int t = tk_scalar_code(w.scalar_type());
    check_tk(tk_copy_strided(out.data_ptr(), t,
                             static_cast<const char*>(w.data_ptr()) + last * w.element_size(), t,
                             static_cast<int>(nd), sizes.data(), dst.data(), src.data(), current_stream(dev)),
             "tk_copy_strided");
    return out;
}

// Correlation of the zero-inserted (stride), padded g [N, F, O...] with the
// spatially flipped, in/out-swapped weight [F, C/groups, K...]: the input
// gradient of conv(x, weight) for an x of spatial size `in_size`, and equally
// the transposed convolution of g (the reference's conv2d_grad and
// conv2d_transpose, csrc/autograd.cpp:621-682, csrc/ops_nn_extra.cpp:123-159).
// One quantised convolution: inserting zeros changes neither operand's
// max-abs, so every output keeps one exact sum and one rounding.  A padding
// wider than the dilated kernel is a crop of the result.
at::Tensor conv_input_grad(const at::Tensor& g_in, const at::Tensor& weight, const std::vector<int64_t>& in_size,
                           const std::vector<int64_t>& s, const std::vector<int64_t>& p,
                           const std::vector<int64_t>& dl, int64_t groups,
                           const std::optional<at::Tensor>& bias = std::nullopt) {
    const int64_t k = weight.dim() - 2;
    at::Tensor g = g_in.contiguous();
    const int64_t N = g.size(0), F = weight.size(0), Cg = weight.size(1), Fg = F / groups, C = Cg * groups;
    std::vector<int64_t> zsize = {N, F}, pad(k), crop(k), ones(k, 1);
    bool spread = false;
    for (int64_t i = 0; i < k; ++i) {
        const int64_t K = weight.size(2 + i), O = g.size(2 + i);
        const int64_t e = in_size[i] + 2 * p[i] - dl[i] * (K - 1) - 1 - (O - 1) * s[i];
        TORCH_CHECK(e >= 0, "kunlun conv input gradient: inconsistent sizes");
        zsize.push_back((O - 1) * s[i] + 1 + e);
        spread = spread || s[i] > 1 || e > 0;
        const int64_t pi = dl[i] * (K - 1) - p[i];
        pad[i] = std::max<int64_t>(pi, 0);
        crop[i] = std::max<int64_t>(-pi, 0);
    }
    at::Tensor gz = g;
    if (spread) {
        gz = at::zeros(zsize, g.options());
        at::Tensor view = gz;
        for (int64_t i = 0; i < k; ++i) view = view.slice(2 + i, 0, (g.size(2 + i) - 1) * s[i] + 1, s[i]);
        view.copy_(g);
    }
    std::vector<int64_t> wv = {groups, Fg, Cg}, wr = {C, Fg};
    for (int64_t i = 0; i < k; ++i) {
        wv.push_back(weight.size(2 + i));
        wr.push_back(weight.size(2 + i));
    }
    at::Tensor wt = flip_spatial(weight.contiguous().view(wv).transpose(1, 2).reshape(wr));
    at::Tensor r = conv_impl(gz, wt, bias, ones, pad, dl, groups);
    bool cropped = false;
    for (int64_t i = 0; i < k; ++i)
        if (crop[i] > 0) {
            r = r.narrow(2 + i, crop[i], in_size[i]);
            cropped = true;
        }
    return cropped ? r.contiguous() : r;
}

// Gradient of conv(x, weight) with respect to the weight [F, C/groups, K...]:
// one tk_conv3d_wgrad_q16 call (a 2-D convolution being the 3-D one with
// depth 1).  Every gradient element is one exact integer sum over all images
// and output pixels of the quantised grad_output and input, with one scale
// per whole tensor, rounded once -- the weight-gradient half of the
// reference's conv2d_grad (csrc/autograd.cpp:621-682) under the forward's
// contract.
at::Tensor conv_weight_grad(const at::Tensor& x_in, const at::Tensor& g_in, at::IntArrayRef w_size,
                            const std::vector<int64_t>& s, const std::vector<int64_t>& p,
                            const std::vector<int64_t>& dl, int64_t groups) {
    const int64_t k = static_cast<int64_t>(w_size.size()) - 2;
    TORCH_CHECK(k == 2 || k == 3, "kunlun conv weight gradient: 2-D or 3-D convolutions");
    check_operand(g_in, x_in, "conv weight gradient");
    at::Tensor x = x_in.contiguous(), g = g_in.contiguous();
    const int64_t o = k == 3 ? 0 : 1;  // 2-D: the depth axis is absent
    tk_conv3d_wgrad_desc_t d = {};
    d.dtype = tk_dtype(x.scalar_type());
    d.n = x.size(0);
    d.c = x.size(1);
    d.d = k == 3 ? x.size(2) : 1;
    d.h = x.size(3 - o);
    d.w = x.size(4 - o);
    d.f = w_size[0];
    d.kd = k == 3 ? w_size[2] : 1;
    d.kh = w_size[3 - o];
    d.kw = w_size[4 - o];
    d.stride_d = k == 3 ? s[0] : 1;
    d.stride_h = s[1 - o];
    d.stride_w = s[2 - o];
    d.pad_d = k == 3 ? p[0] : 0;
    d.pad_h = p[1 - o];
    d.pad_w = p[2 - o];
    d.dil_d = k == 3 ? dl[0] : 1;
    d.dil_h = dl[1 - o];
    d.dil_w = dl[2 - o];
    d.groups = groups;
    TORCH_CHECK(g.size(0) == d.n && g.size(1) == d.f, "kunlun conv weight gradient: grad_output shape mismatch");
    at::Tensor gw = at::empty(w_size, x.options());
    d.x = x.data_ptr();
    d.grad_out = g.data_ptr();
    d.grad_weight = gw.data_ptr();
    const int dev = x.device().index();
    DeviceScope ds(dev);
    const size_t ws_bytes = tk_conv3d_wgrad_workspace_size(&d);
    TORCH_CHECK(ws_bytes > 0 || d.n == 0, "kunlun conv weight gradient: bad geometry");
    at::Tensor ws = workspace(std::max<size_t>(ws_bytes, 1024), x.device());
    check_tk(tk_conv3d_wgrad_q16(&d, aligned_base(ws), ws_bytes, current_stream(dev)), "tk_conv3d_wgrad_q16");
    return gw;
}

std::vector<int64_t> reduce_dims_for_bias(const at::Tensor& g) {
    std::vector<int64_t> dims = {0};
    for (int64_t i = 2; i < g.dim(); ++i) dims.push_back(i);
    return dims;
}

// aten::convolution_overrideable is where aten::convolution sends backends
// that are not built in: conv1d / conv2d / conv3d and their transposed forms
// on kunlun tensors.  conv1d is conv2d on [N, C, 1, L] as in the reference
// (csrc/ops_nn_extra.cpp:70-86); a transposed convolution is the
// correlation of the zero-inserted input with the flipped weight.
at::Tensor convolution_overrideable(const at::Tensor& input, const at::Tensor& weight,
                                    const std::optional<at::Tensor>& bias, at::IntArrayRef stride,
                                    at::IntArrayRef padding, at::IntArrayRef dilation,
                                    bool transposed, at::IntArrayRef output_padding,
                                    int64_t groups) {
    const int64_t k = weight.dim() - 2;
    TORCH_CHECK(k >= 1 && k <= 3 && input.dim() == weight.dim(),
                "kunlun: convolution needs batched 1-D, 2-D or 3-D operands");
    if (k == 1) {
        const auto s = axis_param(stride, 1, 1, "stride"), p = axis_param(padding, 1, 0, "padding"),
                   dl = axis_param(dilation, 1, 1, "dilation"),
                   op = axis_param(output_padding, 1, 0, "output_padding");
        const int64_t s2[2] = {1, s[0]}, p2[2] = {0, p[0]}, d2[2] = {1, dl[0]}, o2[2] = {0, op[0]};
        return torch_kunlun::convolution_overrideable(input.unsqueeze(2), weight.unsqueeze(2), bias, s2, p2, d2,
                                                      transposed, o2, groups)
            .squeeze(2);
    }
    if (!transposed) return conv_impl(input, weight, bias, stride, padding, dilation, groups);
    const auto s = axis_param(stride, k, 1, "stride"), p = axis_param(padding, k, 0, "padding"),
               dl = axis_param(dilation, k, 1, "dilation"),
               op = axis_param(output_padding, k, 0, "output_padding");
    check_operand(weight, input, "conv_transpose");
    TORCH_CHECK(groups > 0 && input.size(1) == weight.size(0) && weight.size(0) % groups == 0,
                "kunlun conv_transpose: weight/input channel mismatch");
    std::vector<int64_t> out_size(k);
    for (int64_t i = 0; i < k; ++i) {
        TORCH_CHECK(op[i] >= 0 && (op[i] < s[i] || op[i] < dl[i]), "kunlun conv_transpose: bad output_padding");
        out_size[i] = (input.size(2 + i) - 1) * s[i] - 2 * p[i] + dl[i] * (weight.size(2 + i) - 1) + 1 + op[i];
        TORCH_CHECK(out_size[i] > 0, "kunlun conv_transpose produced non-positive output shape");
    }
    return conv_input_grad(input, weight, out_size, s, p, dl, groups, bias);
}

// Gradients of the quantised convolutions (the reference's conv2d_grad,
// csrc/autograd.cpp:621-682, and the conv3d / conv_transpose2d backward of
// csrc/autograd_nn_extra.cpp), each a quantised convolution of the same
// contract with one per-tensor scale per operand; the bias gradient is a sum
// of grad_output over batch and pixels (fp32, one rounding).
//   forward conv:       grad_input  = conv_input_grad(grad_output, weight)
//                       grad_weight = conv_weight_grad(input, grad_output)
//   transposed conv:    grad_input  = conv(grad_output, weight)
//                       grad_weight = conv_weight_grad(grad_output, input)
std::tuple<at::Tensor, at::Tensor, at::Tensor> convolution_backward_overrideable(
    const at::Tensor& grad_output, const at::Tensor& input, const at::Tensor& weight,
    at::IntArrayRef stride, at::IntArrayRef padding, at::IntArrayRef dilation, bool transposed,
    at::IntArrayRef output_padding, int64_t groups, std::array<bool, 3> output_mask) {
    const int64_t k = weight.dim() - 2;
    TORCH_CHECK(k >= 1 && k <= 3 && input.dim() == weight.dim() && grad_output.dim() == weight.dim(),
                "kunlun convolution backward expects batched 1-D, 2-D or 3-D tensors");
    if (k == 1) {
        const auto s = axis_param(stride, 1, 1, "stride"), p = axis_param(padding, 1, 0, "padding"),
                   dl = axis_param(dilation, 1, 1, "dilation"),
                   op = axis_param(output_padding, 1, 0, "output_padding");
        const int64_t s2[2] = {1, s[0]}, p2[2] = {0, p[0]}, d2[2] = {1, dl[0]}, o2[2] = {0, op[0]};
        auto r = torch_kunlun::convolution_backward_overrideable(grad_output.unsqueeze(2), input.unsqueeze(2),
                                                                 weight.unsqueeze(2), s2, p2, d2, transposed, o2,
                                                                 groups, output_mask);
        auto sq = [](const at::Tensor& t) { return t.defined() && t.dim() > 2 ? t.squeeze(2) : t; };
        return std::make_tuple(sq(std::get<0>(r)), sq(std::get<1>(r)), std::get<2>(r));
    }
    const auto s = axis_param(stride, k, 1, "stride"), p = axis_param(padding, k, 0, "padding"),
               dl = axis_param(dilation, k, 1, "dilation");
    at::Tensor gi, gw, gb;
    if (!transposed) {
        if (output_mask[0]) {
            std::vector<int64_t> in_size(input.sizes().begin() + 2, input.sizes().end());
            gi = conv_input_grad(grad_output, weight, in_size, s, p, dl, groups);
        }
        if (output_mask[1]) gw = conv_weight_grad(input, grad_output, weight.sizes(), s, p, dl, groups);
    } else {
        if (output_mask[0]) gi = conv_impl(grad_output.contiguous(), weight, std::nullopt, s, p, dl, groups);
        if (output_mask[1]) gw = conv_weight_grad(grad_output, input, weight.sizes(), s, p, dl, groups);
    }
    if (output_mask[2]) gb = at::sum(grad_output, reduce_dims_for_bias(grad_output));
    return {gi, gw, gb};
}

}  // namespace

// y = act(x @ W^T + b) [+ residual] for x [..., K], W [N, K] in one call.
// amax_x (1-element fp32) replaces x's own max |x| as its scale; amax_out
// (1-element fp32) receives max |y|, the scale of the GEMM that consumes y.
at::Tensor linear_act(const at::Tensor& input, const at::Tensor& weight,
                      const std::optional<at::Tensor>& bias, int64_t act,
                      const std::optional<at::Tensor>& residual,
                      const std::optional<at::Tensor>& amax_x,
                      const std::optional<at::Tensor>& amax_out) {
    TORCH_CHECK(input.dim() >= 1 && weight.dim() == 2, "kunlun linear: bad ranks");
    check_operand(weight, input, "linear");
    const int64_t K = input.size(-1);
    TORCH_CHECK(weight.size(1) == K, "kunlun linear: in_features mismatch (", K, " vs ",
                weight.size(1), ")");
    auto scale_tensor = [&](const std::optional<at::Tensor>& t, const char* what) -> float* {
        if (!t.has_value() || !t->defined()) return nullptr;
        TORCH_CHECK(t->scalar_type() == at::kFloat && t->numel() >= 1 && t->is_contiguous() &&
                        t->device() == input.device(),
                    "kunlun linear: ", what, " must be a 1-element fp32 kunlun tensor");
        return t->data_ptr<float>();
    };
    const float* sx = scale_tensor(amax_x, "amax_x");
    float* so = scale_tensor(amax_out, "amax_out");
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
                  1.0, r3.defined() ? 1.0 : 0.0, static_cast<int>(act), true, sx, nullptr, so);
    } else if (so != nullptr) {
        amax_out->zero_();
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

// Two int8 limb planes [2, rows, round_up(cols, 16)] of a 2-D tensor
// quantised with a given per-tensor scale (1-element fp32 tensor): the form
// in which an operand used by several GEMMs is quantised once.
at::Tensor quantize_limbs(const at::Tensor& x_in, const at::Tensor& amax) {
    TORCH_CHECK(x_in.dim() == 2, "kunlun quantize_limbs: a 2-D tensor");
    TORCH_CHECK(x_in.device().type() == c10::DeviceType::PrivateUse1, "kunlun quantize_limbs: kunlun tensor");
    TORCH_CHECK(amax.scalar_type() == at::kFloat && amax.numel() >= 1 && amax.device() == x_in.device(),
                "kunlun quantize_limbs: the scale must be an fp32 kunlun tensor");
    at::Tensor x = x_in.stride(1) == 1 ? x_in : x_in.contiguous();
    const int64_t rows = x.size(0), cols = x.size(1);
    const int64_t ld = (cols + 15) / 16 * 16;
    at::Tensor out = at::empty({2, rows, ld}, x.options().dtype(at::kChar));
    if (rows * ld == 0) return out;
    const int dev = x.device().index();
    DeviceScope g(dev);
    check_tk(tk_quantize_limbs(tk_dtype(x.scalar_type()), x.data_ptr(), 1, rows, cols, 0, x.stride(0), 1,
                               amax.data_ptr<float>(), 0, out.data_ptr<int8_t>(), current_stream(dev)),
             "tk_quantize_limbs");
    return out;
}

// act(q(a) q(b)^T dequantised + bias) for operands quantised beforehand by
// quantize_limbs with the scales amax_a / amax_b (K <= 32768); out an
// optional row-major [M, N] block of `dtype`.
at::Tensor linear_from_limbs(const at::Tensor& a_limbs, const at::Tensor& b_limbs, int64_t k,
                             const at::Tensor& amax_a, const at::Tensor& amax_b,
                             const std::optional<at::Tensor>& bias, int64_t act,
                             const std::optional<at::Tensor>& out_opt, at::ScalarType dtype,
                             const std::optional<at::Tensor>& gate, const std::optional<at::Tensor>& amax_out) {
    const int64_t ld = (k + 15) / 16 * 16;
    TORCH_CHECK(a_limbs.dim() == 3 && b_limbs.dim() == 3 && a_limbs.size(0) == 2 && b_limbs.size(0) == 2 &&
                    a_limbs.size(2) == ld && b_limbs.size(2) == ld && a_limbs.is_contiguous() &&
                    b_limbs.is_contiguous() && a_limbs.scalar_type() == at::kChar &&
                    b_limbs.scalar_type() == at::kChar,
                "kunlun linear_from_limbs: limbs must be contiguous int8 [2, rows, round_up(k, 16)]");
    TORCH_CHECK(a_limbs.device() == b_limbs.device() && amax_a.device() == a_limbs.device() &&
                    amax_b.device() == a_limbs.device() && amax_a.scalar_type() == at::kFloat &&
                    amax_b.scalar_type() == at::kFloat,
                "kunlun linear_from_limbs: operands and fp32 scales on one kunlun device");
    TORCH_CHECK(dtype == at::kHalf || dtype == at::kFloat, "kunlun linear_from_limbs: fp16 or fp32 output");
    const int64_t M = a_limbs.size(1), N = b_limbs.size(1);
    at::Tensor out;
    if (out_opt.has_value() && out_opt->defined()) {
        out = *out_opt;
        TORCH_CHECK(out.dim() == 2 && out.size(0) == M && out.size(1) == N && out.stride(1) == 1 &&
                        out.scalar_type() == dtype && out.device() == a_limbs.device(),
                    "kunlun linear_from_limbs: out must be a row-major [M, N] block of the output dtype");
    } else {
        out = at::empty({M, N}, a_limbs.options().dtype(dtype));
    }
    if (out.numel() == 0) return out;
    TORCH_CHECK(k > 0, "kunlun linear_from_limbs: K must be positive");
    tk_qgemm_desc_t d = {};
    d.dtype = dtype == at::kHalf ? TK_DTYPE_F16 : TK_DTYPE_F32;
    d.batch = 1;
    d.m = M;
    d.n = N;
    d.k = k;
    d.out = out.data_ptr();
    d.out_sb = M * out.stride(0);
    d.out_sm = out.stride(0);
    at::Tensor b;
    if (bias.has_value() && bias->defined()) {
        b = bias->contiguous();
        TORCH_CHECK(b.numel() == N && b.scalar_type() == dtype && b.device() == out.device(),
                    "kunlun linear_from_limbs: bias [N] of the output dtype");
        d.bias = b.data_ptr();
    }
    d.alpha = 1.0f;
    d.beta = 0.0f;
    d.act = static_cast<tk_act_t>(act);
    d.per_slice_scales = 1;
    at::Tensor gt;
    if (gate.has_value() && gate->defined()) {
        // act TK_ACT_SILU_GATE: y = T(silu(gate)) * (a b^T + bias), gate [M, N] row-major
        gt = *gate;
        TORCH_CHECK(gt.dim() == 2 && gt.size(0) == M && gt.size(1) == N && gt.stride(1) == 1 &&
                        gt.scalar_type() == dtype && gt.device() == out.device(),
                    "kunlun linear_from_limbs: gate must be a row-major [M, N] tensor of the output dtype");
        d.addend = gt.data_ptr();
        d.add_sb = M * gt.stride(0);
        d.add_sm = gt.stride(0);
        d.add_sn = 1;
        d.beta = 1.0f;
    }
    if (amax_out.has_value() && amax_out->defined()) {
        TORCH_CHECK(amax_out->scalar_type() == at::kFloat && amax_out->numel() >= 1 && amax_out->is_contiguous() &&
                        amax_out->device() == out.device(),
                    "kunlun linear_from_limbs: amax_out must be a 1-element fp32 kunlun tensor");
        d.amax_out = amax_out->data_ptr<float>();
    }
    const int dev = out.device().index();
    DeviceScope g(dev);
    check_tk(tk_qgemm_from_limbs(&d, a_limbs.data_ptr<int8_t>(), b_limbs.data_ptr<int8_t>(),
                                 amax_a.data_ptr<float>(), amax_b.data_ptr<float>(), current_stream(dev)),
             "tk_qgemm_from_limbs");
    return out;
}

namespace {

at::Tensor linear_fwd(const at::Tensor& input, const at::Tensor& weight,
                      const std::optional<at::Tensor>& bias) {
    return linear_act(input, weight, bias, TK_ACT_NONE, std::nullopt, std::nullopt, std::nullopt);
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

// conv2d under autograd: with gradients required, route through
// aten::convolution, whose backward is convolution_backward_overrideable.
at::Tensor conv2d_autograd(const at::Tensor& input, const at::Tensor& weight,
                           const std::optional<at::Tensor>& bias, at::IntArrayRef stride,
                           at::IntArrayRef padding, at::IntArrayRef dilation, int64_t groups) {
    const bool needs_grad = at::GradMode::is_enabled() &&
                            (input.requires_grad() || weight.requires_grad() ||
                             (bias.has_value() && bias->defined() && bias->requires_grad()));
    if (needs_grad) {
        const bool batched = input.dim() == 4;
        at::Tensor x = batched ? input : input.unsqueeze(0);
        const int64_t zero[2] = {0, 0};
        at::Tensor out = at::convolution(x, weight, bias, stride, padding, dilation, false, zero, groups);
        return batched ? out : out.squeeze(0);
    }
    at::AutoDispatchBelowADInplaceOrView guard;
    return torch_kunlun::conv2d(input, weight, bias, stride, padding, dilation, groups);
}

}  // namespace
}  // namespace torch_kunlun

TORCH_LIBRARY_IMPL(aten, PrivateUse1, m) {
    m.impl("mm", TORCH_FN(torch_kunlun::mm));
    m.impl("dot", TORCH_FN(torch_kunlun::dot));
    m.impl("mv", TORCH_FN(torch_kunlun::mv));
    m.impl("addmm", TORCH_FN(torch_kunlun::addmm));
    m.impl("bmm", TORCH_FN(torch_kunlun::bmm));
    m.impl("baddbmm", TORCH_FN(torch_kunlun::baddbmm));
    m.impl("linear", TORCH_FN(torch_kunlun::linear_fwd));
    m.impl("conv2d", TORCH_FN(torch_kunlun::conv2d));
    m.impl("convolution_overrideable", TORCH_FN(torch_kunlun::convolution_overrideable));
    m.impl("convolution_backward_overrideable",
           TORCH_FN(torch_kunlun::convolution_backward_overrideable));
}

TORCH_LIBRARY_IMPL(aten, AutogradPrivateUse1, m) {
    m.impl("linear", TORCH_FN(torch_kunlun::linear_autograd));
    m.impl("conv2d", TORCH_FN(torch_kunlun::conv2d_autograd));
}
