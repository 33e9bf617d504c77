// attention.cpp -- scaled_dot_product_attention of the kunlun backend.
//
// Follows the reference's composition step for step
// (torch_kunlun/kunlun/attention.py:36-107): per-slice quantised
// bmm(q, k^T), multiply by the scale (rounded to T), add the mask (rounded
// to T; a boolean mask contributes -1e4 where True, a causal mask -1e4 above
// the diagonal), softmax over the keys, per-slice quantised bmm with v.
// The first three steps are a single tk_qgemm call -- alpha and the addend are
// applied in the epilogue after the dequantised scores are rounded to T,
// exactly as the reference's separate bmm, mul.Scalar and add launches
// round -- so the [B*H, L, S] score tensor is written once and read once
// by softmax instead of three times; K^T is read in place (no host-staged
// transpose, csrc/ops.cpp:289-350).
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

}  // namespace

at::Tensor sdpa(const at::Tensor& query, const at::Tensor& key, const at::Tensor& value,
                const std::optional<at::Tensor>& attn_mask, bool is_causal,
                std::optional<double> scale) {
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
    at::Tensor q3 = query.reshape({BH, L, E});
    at::Tensor k3 = key.reshape({BH, S, E});  // used directly as the [N=S, K=E] operand
    at::Tensor v3 = value.reshape({BH, S, Ev});
    const double factor = scale.has_value() ? *scale : 1.0 / std::sqrt(static_cast<double>(E));

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
    if (attn_mask.has_value() && attn_mask->defined()) {
        at::Tensor m = attn_mask->to(query.device());
        if (m.scalar_type() == at::kBool) {
            m = m.to(query.scalar_type()) * -1.0e4;
        } else {
            m = m.to(query.scalar_type());
        }
        user = mask_view(m, batch, heads, L, S);
    }
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
