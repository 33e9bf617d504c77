// tk_numerics.cuh -- the numeric contract of the int16-quantised path, shared
// by every kernel of the library so that all paths round identically.
//
//   inv = 32767 / amax (IEEE fp32 division), 0 when amax is 0, NaN or Inf
//   q   = clamp(rint_even(x * inv), -32767, 32767), NaN products give 0
//   s   = fp64(amax_a) * fp64(amax_b) / 32767^2 (one fp64 rounding)
//   r   = T(fp64(acc) * s)  with acc the exact integer dot product
// followed by the reference's separately rounded post-ops.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

#include "../../include/tk_kernels.h"

namespace tk {

__device__ __forceinline__ float quant_inv(float amax) {
    return (amax > 0.0f && amax != __int_as_float(0x7F800000)) ? __fdiv_rn(32767.0f, amax) : 0.0f;
}

// The int16 code of quant_one(v, inv) in the low 16 bits of the result, for
// inv > 0 and |v| <= amax (so |RN(v * inv)| <= 32767.004): RN(v * inv) +
// 1.5 * 2^23, as two binary32 operations the compiler never fuses, rounds
// RN(v * inv) to the nearest integer (ties to even, like __float2int_rn) and
// holds it in two's complement in the low significand bits (magic-number
// rounding) -- no float-to-int conversion on the special-function pipe.
// With inv == 0 and finite v the code is 0 as well.  Only for amax values
// computed from the operand itself; quant_code_bits_clamped takes any v.
__device__ __forceinline__ uint32_t quant_code_bits(float v, float inv) {
    return __float_as_uint(__fadd_rn(__fmul_rn(v, inv), 12582912.0f));
}

// RN(v * inv) limited to the code range [-32767, 32767], NaN mapped to 0:
// quant_one's clamp, for a scaled value that may lie outside the range (an
// amax supplied by the caller below max |x|, or an infinite input).
__device__ __forceinline__ float clamp_code_range(float t) {
    const float c = fminf(fmaxf(t, -32767.0f), 32767.0f);
    return t == t ? c : 0.0f;
}

// quant_code_bits for any v and any inv >= 0: equal to quant_one's code.
__device__ __forceinline__ uint32_t quant_code_bits_clamped(float v, float inv) {
    return __float_as_uint(__fadd_rn(clamp_code_range(__fmul_rn(v, inv)), 12582912.0f));
}

// hi and lo limb bytes of four codes (low 16 bits of r0..r3), code i in byte i.
__device__ __forceinline__ void pack_codes4(uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3,
                                            uint32_t& hi, uint32_t& lo) {
    const uint32_t p01 = __byte_perm(r0, r1, 0x5410), p23 = __byte_perm(r2, r3, 0x5410);
    lo = __byte_perm(p01, p23, 0x6420);
    hi = __byte_perm(p01, p23, 0x7531);
}

__device__ __forceinline__ int quant_one(float v, float inv) {
    const float t = __fmul_rn(v, inv);
    const int q = max(-32767, min(32767, __float2int_rn(t)));
    return t == t ? q : 0;  // a select, so loops over elements stay branch-free
}

__device__ __forceinline__ double dequant_scale(float amax_a, float amax_b) {
    return __ddiv_rn(__dmul_rn(static_cast<double>(amax_a), static_cast<double>(amax_b)),
                     1073676289.0);
}

// The exact integer 65536*hh + 256*mid + ll of three int32 limb accumulators.
__device__ __forceinline__ long long limb_acc_to_i64(uint32_t hh, uint32_t mid, uint32_t ll) {
    return (static_cast<long long>(static_cast<int32_t>(hh)) << 16) +
           (static_cast<long long>(static_cast<int32_t>(mid)) << 8) +
           static_cast<long long>(static_cast<int32_t>(ll));
}

// The same integer as binary64, without a conversion instruction: for
// |acc| < 2^51 the bit pattern of 1.5 * 2^52 plus acc is the binary64 value
// 1.5 * 2^52 + acc.
__device__ __forceinline__ double limb_acc_to_double(uint32_t hh, uint32_t mid, uint32_t ll) {
    const long long acc = limb_acc_to_i64(hh, mid, ll);
    return __longlong_as_double(acc + 0x4338000000000000LL) - 6755399441055744.0;
}

// Round a binary64 value to the output type (0 = fp16, 1 = fp32), returned
// widened to fp32 (exactly).
__device__ __forceinline__ float round_t_from_double(double d, int dtype) {
    if (dtype == 0) return __half2float(__double2half(d));  // one nearest-even rounding
    return __double2float_rn(d);
}

__device__ __forceinline__ float round_t(float v, int dtype) {
    return dtype == 0 ? __half2float(__float2half_rn(v)) : v;
}

__device__ __forceinline__ float load_t(const void* p, int dtype, int64_t i) {
    return dtype == 0 ? __half2float(static_cast<const __half*>(p)[i])
                      : static_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_t(void* p, int dtype, int64_t i, float v) {
    if (dtype == 0)
        static_cast<__half*>(p)[i] = __float2half_rn(v);
    else
        static_cast<float*>(p)[i] = v;
}

__device__ __forceinline__ float gelu_erf(float x) {
    return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}

__device__ __forceinline__ float gelu_tanh(float x) {
    const float k0 = 0.7978845608028654f, k1 = 0.044715f;
    return 0.5f * x * (1.0f + tanhf(k0 * (x + k1 * x * x * x)));
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

// Activation applied to an already T-rounded value; result rounded to T.
__device__ __forceinline__ float apply_act(float r, int act, int dtype) {
    switch (act) {
        case TK_ACT_RELU: return (r > 0.0f || r != r) ? r : 0.0f;
        case TK_ACT_GELU: return round_t(gelu_erf(r), dtype);
        case TK_ACT_GELU_TANH: return round_t(gelu_tanh(r), dtype);
        case TK_ACT_SILU: return round_t(silu_f(r), dtype);
        default: return r;
    }
}

}  // namespace tk
