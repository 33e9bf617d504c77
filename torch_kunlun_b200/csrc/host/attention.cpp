// attention.cpp -- scaled_dot_product_attention of the kunlun backend.
//
// Follows the reference's composition step for step
// (torch_kunlun/kunlun/attention.py:36-107): per-slice quantised
// bmm(q, k^T), multiply by the scale (rounded to T), add the mask (rounded
// to T; a boolean mask contributes -1e4 where True, a causal mask -1e4 above
// the diagonal), softmax over the keys, per-slice quantised bmm with v.
// Two implementations with the same semantics:
//  * fused (default where supported: head dim <= 128, value dim <= 256,
//    at most 32768 keys): tk_sdpa_q16, which keeps the [L, S] scores on chip;
//    q, k, v and the mask are read through their strides (head-split views
//    of a packed QKV projection need no copies) and the output is allocated
//    as a [B, L, H, Ev] buffer viewed as [B, H, L, Ev], so merging the heads
//    back is a view;
//  * composed: the first three steps are a single tk_qgemm call -- alpha and
//    the addend are applied in the epilogue after the dequantised scores are
//    rounded to T, exactly as the reference's separate bmm, mul.Scalar and
//    add launches round -- then softmax and the second quantised bmm.  K^T
//    is read in place (no host-staged transpose, csrc/ops.cpp:289-350).
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

// Additive mask as a [BHm, L, S] view broadcastable against [B*H, L, S]
// (torch_kunlun/kunlun/attention.py:23-33 reshapes 2/3/4-D masks).
at::Tensor mask_view(const at::Tensor& mask, int64_t batch, int64_t heads, int64_t L, int64_t S) {
    if (mask.dim() == 2) return mask.reshape({1, L, S});
    if (mask.dim() == 3) {
        if (mask.size(0) == batch) {
            // (B, L, S): one mask per batch item, shared by its heads
            return mask.reshape({batch, 1, L, S}).expand({batch, heads, L, S}).reshape({batch * heads, L, S});
        }
        return mask.reshape({batch * heads, L, S});
    }
    TORCH_CHECK(mask.dim() == 4, "unsupported attention mask rank: ", mask.dim());
    return mask.expand({batch, heads, L, S}).reshape({batch * heads, L, S});
}

// [B, H, rows, cols] strides of a 2/3/4-D attention operand (broadcast dims
// get stride 0).
void strides4(const at::Tensor& t, int64_t out[4]) {
    const int d = static_cast<int>(t.dim());
    out[0] = d == 4 ? t.stride(0) : (d == 3 ? t.stride(0) : 0);
    out[1] = d == 4 ? t.stride(1) : 0;
    out[2] = t.stride(d - 2);
    out[3] = t.stride(d - 1);
}

// The user mask as a [B, H, L, S] broadcast view (no copy), following the
// reference's accepted ranks (torch_kunlun/kunlun/attention.py:23-33).
at::Tensor mask4(const at::Tensor& m, int64_t batch, int64_t heads, int64_t L, int64_t S) {
    if (m.dim() == 2) return m.view({1, 1, L, S}).expand({batch, heads, L, S});
    if (m.dim() == 3) {
        if (m.size(0) == batch) return m.unsqueeze(1).expand({batch, heads, L, S});
        return m.reshape({batch, heads, L, S});
    }
    TORCH_CHECK(m.dim() == 4, "unsupported attention mask rank: ", m.dim());
    return m.expand({batch, heads, L, S});
}

bool fused_supported(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v) {
    const auto st = q.scalar_type();
    return (st == at::kHalf || st == at::kFloat) && k.scalar_type() == st &&
           v.scalar_type() == st && q.size(-1) <= 128 && v.size(-1) <= 256 && k.size(-2) <= 32768 &&
           q.dim() == k.dim() && q.dim() == v.dim();
}

at::Tensor sdpa_fused(const at::Tensor& query, const at::Tensor& key, const at::Tensor& value,
                      const at::Tensor& user_mask, bool is_causal, double factor, int64_t batch,
                      int64_t heads, const std::vector<int64_t>& out_shape) {
    const int64_t L = query.size(-2), E = query.size(-1), S = key.size(-2), Ev = value.size(-1);
    const int dev = query.device().index();
    DeviceScope g(dev);
    at::Tensor out;
    if (query.dim() == 4) {
        out = at::empty({batch, L, heads, Ev}, query.options()).transpose(1, 2);
    } else {
        out = at::empty(out_shape, query.options());
    }
    tk_sdpa_desc_t d = {};
    d.dtype = tk_dtype(query.scalar_type());
    d.batch = batch;
    d.heads = heads;
    d.l = L;
    d.s = S;
    d.e = E;
    d.ev = Ev;
    d.q = query.data_ptr();
    d.k = key.data_ptr();
    d.v = value.data_ptr();
    d.out = out.data_ptr();
    strides4(query, d.q_strides);
    strides4(key, d.k_strides);
    strides4(value, d.v_strides);
    strides4(out, d.out_strides);
    at::Tensor mv;
    if (user_mask.defined()) {
        mv = mask4(user_mask, batch, heads, L, S);
        d.mask = mv.data_ptr();
        for (int a = 0; a < 4; ++a) d.mask_strides[a] = mv.stride(a);
    }
    d.causal = is_causal ? 1 : 0;
    d.scale = static_cast<float>(factor);
    const size_t ws_bytes = tk_sdpa_workspace_size(&d);
    TORCH_CHECK(ws_bytes > 0, "kunlun sdpa: ", tk_last_error_string());
    at::Tensor ws = workspace(ws_bytes, query.device());
    check_tk(tk_sdpa_q16(&d, aligned_base(ws), ws_bytes, current_stream(dev)), "tk_sdpa_q16");
    return out;
}

}  // namespace

at::Tensor sdpa(const at::Tensor& query, const at::Tensor& key, const at::Tensor& value,
                const std::optional<at::Tensor>& attn_mask, bool is_causal,
                std::optional<double> scale, bool fused) {
    TORCH_CHECK(query.dim() >= 2 && key.dim() >= 2 && value.dim() >= 2,
                "attention expects tensors with at least 2 dimensions");
    TORCH_CHECK(query.size(-1) == key.size(-1), "query/key head dimensions must match");
    TORCH_CHECK(key.size(-2) == value.size(-2), "key/value sequence lengths must match");
    const int64_t L = query.size(-2), E = query.size(-1), S = key.size(-2), Ev = value.size(-1);
    int64_t batch = 1, heads = 1;
    std::vector<int64_t> out_shape;
    if (query.dim() == 2) {
        out_shape = {L, Ev};
    } else if (query.dim() == 3) {
        batch = query.size(0);
        out_shape = {batch, L, Ev};
    } else {
        TORCH_CHECK(query.dim() == 4, "attention supports 2/3/4-D inputs");
        batch = query.size(0);
        heads = query.size(1);
        out_shape = {batch, heads, L, Ev};
    }
    const int64_t BH = batch * heads;
    const double factor = scale.has_value() ? *scale : 1.0 / std::sqrt(static_cast<double>(E));
    at::Tensor user_mask;
    if (attn_mask.has_value() && attn_mask->defined()) {
        at::Tensor m = attn_mask->to(query.device());
        if (m.scalar_type() == at::kBool) {
            m = m.to(query.scalar_type()) * -1.0e4;
        } else {
            m = m.to(query.scalar_type());
        }
        user_mask = m;
    }
    if (fused && fused_supported(query, key, value) && query.numel() > 0 && key.numel() > 0 &&
        value.numel() > 0)
        return sdpa_fused(query, key, value, user_mask, is_causal, factor, batch, heads, out_shape);

    at::Tensor q3 = query.reshape({BH, L, E});
    at::Tensor k3 = key.reshape({BH, S, E});  // used directly as the [N=S, K=E] operand
    at::Tensor v3 = value.reshape({BH, S, Ev});
    // The reference adds the causal mask and then the user mask as two
    // separately rounded adds; the first goes into the GEMM epilogue.
    at::Tensor causal, user;
    if (is_causal) {
        // -1e4 strictly above the diagonal, built once on the host and copied
        // (torch_kunlun/kunlun/attention.py:89-95).
        at::Tensor c = at::triu(at::ones({L, S}, at::TensorOptions().dtype(query.scalar_type())), 1) *
                       -1.0e4;
        causal = c.to(query.device()).reshape({1, L, S});
    }
    if (user_mask.defined()) user = mask_view(user_mask, batch, heads, L, S);
    at::Tensor additive = causal.defined() ? causal : user;

    // scores = T(T(T(q k^T) * factor) + mask) in one quantised GEMM: baddbmm
    // is beta * addend + alpha * bmm with exactly that rounding order.
    at::Tensor kt = k3.transpose(1, 2);
    at::Tensor scores;
    if (additive.defined()) {
        scores = at::baddbmm(additive.expand({BH, L, S}), q3, kt, 1.0, factor);
    } else if (factor != 1.0) {
        scores = at::baddbmm(at::empty({1, 1, 1}, query.options()), q3, kt, 0.0, factor);
    } else {
        scores = at::bmm(q3, kt);
    }
    if (causal.defined() && user.defined()) scores = scores + user;
    at::Tensor probs = at::_softmax(scores, -1, false);
    at::Tensor out = at::bmm(probs, v3);
    return out.reshape(out_shape);
}

}  // namespace torch_kunlun
