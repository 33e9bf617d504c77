// eltwise.cu -- device-side data movement and elementwise ops of the
// kunlun backend: strided copy with dtype conversion (replaces the host
// staging of csrc/ops.cpp:289-418), fill (csrc/ops.cpp:162-208 plus the
// host-pattern path), broadcast binary ops (add/sub/mul/div:
// csrc/ops.cpp:117-149, csrc/autograd.cpp:40-100) and activations
// (relu csrc/ops.cpp:151-160, gelu csrc/ops_nn.cpp:132-147, silu
// csrc/ops_extra.cpp:71, scale csrc/autograd.cpp:586-601).
//
// All of these are HBM-bound; arithmetic is fp32 with one rounding to the
// output type, as in the reference's XDNN elementwise calls.
#include <cuda_bf16.h>

#include <algorithm>

#include "tk_internal.h"

namespace tk {
namespace {

constexpr int kMaxDims = 8;
constexpr int kThreads = 256;

struct Strided {
    int ndim;
    int64_t sizes[kMaxDims];
    int64_t s0[kMaxDims];  // strides of operand 0 (destination / a)
    int64_t s1[kMaxDims];  // strides of operand 1 (source / b)
};

__device__ __forceinline__ void offsets(const Strided& d, int64_t i, int64_t& o0, int64_t& o1) {
    o0 = 0;
    o1 = 0;
#pragma unroll 1
    for (int k = d.ndim - 1; k >= 0; --k) {
        const int64_t sz = d.sizes[k];
        const int64_t idx = i % sz;
        i /= sz;
        o0 += idx * d.s0[k];
        o1 += idx * d.s1[k];
    }
}

// ---- scalar type codes (tk_scalar_t in tk_kernels.h) ----
enum : int { T_BOOL = 0, T_U8, T_I8, T_I16, T_I32, T_I64, T_F16, T_BF16, T_F32, T_F64 };

__host__ __device__ inline int scalar_size(int t) {
    switch (t) {
        case T_BOOL: case T_U8: case T_I8: return 1;
        case T_I16: case T_F16: case T_BF16: return 2;
        case T_I32: case T_F32: return 4;
        default: return 8;
    }
}

__device__ __forceinline__ double load_any(const void* p, int t, int64_t i) {
    switch (t) {
        case T_BOOL: return static_cast<const uint8_t*>(p)[i] ? 1.0 : 0.0;
        case T_U8: return static_cast<const uint8_t*>(p)[i];
        case T_I8: return static_cast<const int8_t*>(p)[i];
        case T_I16: return static_cast<const int16_t*>(p)[i];
        case T_I32: return static_cast<const int32_t*>(p)[i];
        case T_I64: return static_cast<double>(static_cast<const long long*>(p)[i]);
        case T_F16: return __half2float(static_cast<const __half*>(p)[i]);
        case T_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
        case T_F32: return static_cast<const float*>(p)[i];
        default: return static_cast<const double*>(p)[i];
    }
}

// binary64 -> binary32 toward zero with the sticky last bit (round to odd),
// so that a following nearest-even rounding to a narrower float is a single
// correct rounding (Boldo & Melquiond, 2005).
__device__ __forceinline__ float d2f_odd(double d) {
    float f = __double2float_rz(d);
    if (static_cast<double>(f) != d) f = __uint_as_float(__float_as_uint(f) | 1u);
    return f;
}

__device__ __forceinline__ void store_any(void* p, int t, int64_t i, double v) {
    switch (t) {
        case T_BOOL: static_cast<uint8_t*>(p)[i] = (v != 0.0) ? 1 : 0; break;
        case T_U8: static_cast<uint8_t*>(p)[i] = static_cast<uint8_t>(static_cast<long long>(v)); break;
        case T_I8: static_cast<int8_t*>(p)[i] = static_cast<int8_t>(static_cast<long long>(v)); break;
        case T_I16: static_cast<int16_t*>(p)[i] = static_cast<int16_t>(static_cast<long long>(v)); break;
        case T_I32: static_cast<int32_t*>(p)[i] = static_cast<int32_t>(static_cast<long long>(v)); break;
        case T_I64: static_cast<long long*>(p)[i] = static_cast<long long>(v); break;
        case T_F16: static_cast<__half*>(p)[i] = __float2half_rn(d2f_odd(v)); break;
        case T_BF16: static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(d2f_odd(v)); break;
        case T_F32: static_cast<float*>(p)[i] = __double2float_rn(v); break;
        default: static_cast<double*>(p)[i] = v; break;
    }
}

// 32-bit index variant for index spaces below 2^31 elements.
template <typename E>
__global__ void copy_same_kernel32(E* __restrict__ dst, const E* __restrict__ src, int n,
                                   Strided d) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        int rem = i;
        long long od = 0, os = 0;
#pragma unroll 1
        for (int k = d.ndim - 1; k >= 0; --k) {
            const int sz = static_cast<int>(d.sizes[k]);
            const int idx = rem % sz;
            rem /= sz;
            od += idx * d.s0[k];
            os += idx * d.s1[k];
        }
        dst[od] = src[os];
    }
}

template <typename E>
__global__ void copy_same_kernel(E* __restrict__ dst, const E* __restrict__ src, int64_t n,
                                 Strided d) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t od, os;
        offsets(d, i, od, os);
        dst[od] = src[os];
    }
}

__global__ void copy_convert_kernel(void* __restrict__ dst, int dt, const void* __restrict__ src,
                                    int st, int64_t n, Strided d) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t od, os;
        offsets(d, i, od, os);
        store_any(dst, dt, od, load_any(src, st, os));
    }
}

// Dense conversions between f16 and f32 (the common .half()/.float()).
__global__ void f32_to_f16_kernel(__half* __restrict__ dst, const float* __restrict__ src, int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        dst[i] = __float2half_rn(src[i]);
}

__global__ void f16_to_f32_kernel(float* __restrict__ dst, const __half* __restrict__ src, int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        dst[i] = __half2float(src[i]);
}

template <typename E>
__global__ void fill_kernel(E* __restrict__ dst, E v, int64_t n, Strided d) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t od, unused;
        offsets(d, i, od, unused);
        dst[od] = v;
    }
}

template <typename E>
__global__ void fill_dense_kernel(E* __restrict__ dst, E v, int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        dst[i] = v;
}

// ---- binary / unary on f16, f32 ----
template <typename T> __device__ __forceinline__ float ld(const T* p, int64_t i);
template <> __device__ __forceinline__ float ld<__half>(const __half* p, int64_t i) { return __half2float(p[i]); }
template <> __device__ __forceinline__ float ld<float>(const float* p, int64_t i) { return p[i]; }
template <typename T> __device__ __forceinline__ void st(T* p, int64_t i, float v);
template <> __device__ __forceinline__ void st<__half>(__half* p, int64_t i, float v) { p[i] = __float2half_rn(v); }
template <> __device__ __forceinline__ void st<float>(float* p, int64_t i, float v) { p[i] = v; }

__device__ __forceinline__ float bin_apply(int op, float a, float b, float alpha) {
    switch (op) {
        case TK_BIN_ADD: return alpha == 1.0f ? __fadd_rn(a, b) : __fadd_rn(a, __fmul_rn(alpha, b));
        case TK_BIN_SUB: return alpha == 1.0f ? __fsub_rn(a, b) : __fsub_rn(a, __fmul_rn(alpha, b));
        case TK_BIN_MUL: return __fmul_rn(a, b);
        case TK_BIN_THRESHOLD_BACKWARD: return b > alpha ? a : 0.0f;
        default: return __fdiv_rn(a, b);
    }
}

template <typename T>
__global__ void binary_kernel(int op, const T* __restrict__ a, const T* __restrict__ b,
                              T* __restrict__ out, int64_t n, float alpha, Strided d) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t oa, ob;
        offsets(d, i, oa, ob);
        st<T>(out, i, bin_apply(op, ld<T>(a, oa), ld<T>(b, ob), alpha));
    }
}

template <typename T>
__global__ void binary_dense_kernel(int op, const T* __restrict__ a, const T* __restrict__ b,
                                    T* __restrict__ out, int64_t n, float alpha) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        st<T>(out, i, bin_apply(op, ld<T>(a, i), ld<T>(b, i), alpha));
}

__device__ __forceinline__ float un_apply(int op, float x, float p0, float p1) {
    switch (op) {
        case TK_UN_RELU: return (x > 0.0f || x != x) ? x : 0.0f;
        case TK_UN_GELU: return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
        case TK_UN_GELU_TANH: {
            const float k0 = 0.7978845608028654f, k1 = 0.044715f;
            return 0.5f * x * (1.0f + tanhf(k0 * (x + k1 * x * x * x)));
        }
        case TK_UN_SILU: return x / (1.0f + expf(-x));
        case TK_UN_SCALE: return __fadd_rn(__fmul_rn(x, p0), p1);
        default: return x;
    }
}

template <typename T>
__global__ void unary_kernel(int op, const T* __restrict__ x, T* __restrict__ y, int64_t n, float p0,
                             float p1) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        st<T>(y, i, un_apply(op, ld<T>(x, i), p0, p1));
}

// silu(gate) * up, each rounded to T like the reference's separate swish and mul.
template <typename T>
__global__ void silu_mul_kernel(const T* __restrict__ g, const T* __restrict__ u, T* __restrict__ y,
                                int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float h = un_apply(TK_UN_SILU, ld<T>(g, i), 0.f, 0.f);
        T hr;  // silu output rounded to T, as the reference stores it
        st<T>(&hr, 0, h);
        st<T>(y, i, __fmul_rn(ld<T>(&hr, 0), ld<T>(u, i)));
    }
}

// The SiLU gate with the per-tensor amax of its output folded in: y as in
// silu_mul_kernel, and the largest |y| (as the bit pattern of a non-negative
// binary32, NaN canonicalised above every number, the order tk_amax uses)
// combined into *amax_bits with one atomicMax per warp.  Eight elements per
// thread with 16-byte accesses when `vec`.
template <typename T> __device__ __forceinline__ void ld8f(const T* p, float (&v)[8]);
template <typename T> __device__ __forceinline__ void st8f(T* p, const float (&v)[8]);

template <typename T>
__device__ __forceinline__ float silu_mul_one(float gv, float uv) {
    T hr;  // silu output rounded to T, as the reference stores it
    st<T>(&hr, 0, un_apply(TK_UN_SILU, gv, 0.f, 0.f));
    T yr;
    st<T>(&yr, 0, __fmul_rn(ld<T>(&hr, 0), uv));
    return ld<T>(&yr, 0);
}

__device__ __forceinline__ unsigned abs_bits(float v) {
    const unsigned b = __float_as_uint(v) & 0x7FFFFFFFu;
    return b > 0x7F800000u ? 0x7FC00000u : b;
}

template <typename T>
__global__ void __launch_bounds__(256)
silu_mul_amax_kernel(const T* __restrict__ g, const T* __restrict__ u, T* __restrict__ y, int64_t n,
                     int vec, unsigned* __restrict__ amax_bits) {
    unsigned m = 0;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t t0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (vec) {
        for (int64_t v = t0; v < n / 8; v += stride) {
            float gv[8], uv[8], out[8];
            ld8f<T>(g + 8 * v, gv);
            ld8f<T>(u + 8 * v, uv);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                out[k] = silu_mul_one<T>(gv[k], uv[k]);
                m = max(m, abs_bits(out[k]));
            }
            st8f<T>(y + 8 * v, out);
        }
    } else {
        for (int64_t i = t0; i < n; i += stride) {
            const float o = silu_mul_one<T>(ld<T>(g, i), ld<T>(u, i));
            st<T>(y, i, o);
            m = max(m, abs_bits(o));
        }
    }
    m = __reduce_max_sync(0xffffffffu, m);
    if ((threadIdx.x & 31) == 0 && m != 0u) atomicMax(amax_bits, m);
}

int grid_for(int64_t n) {
    int64_t g = ceil_div(n, kThreads);
    const int64_t cap = static_cast<int64_t>(sm_count(current_device())) * 16;
    return static_cast<int>(std::max<int64_t>(1, std::min(g, cap)));
}

int fill_strided_desc(Strided& d, int ndim, const int64_t* sizes, const int64_t* s0,
                      const int64_t* s1, int64_t& n) {
    TK_CHECK_ARG(ndim >= 0 && ndim <= kMaxDims, "at most %d dims supported, got %d", kMaxDims, ndim);
    d.ndim = ndim;
    n = 1;
    for (int i = 0; i < ndim; ++i) {
        TK_CHECK_ARG(sizes[i] >= 0, "negative size");
        d.sizes[i] = sizes[i];
        d.s0[i] = s0 ? s0[i] : 0;
        d.s1[i] = s1 ? s1[i] : 0;
        n *= sizes[i];
    }
    if (ndim == 0) {
        d.ndim = 1;
        d.sizes[0] = 1;
        d.s0[0] = d.s1[0] = 0;
    }
    return TK_OK;
}

bool is_dense(int ndim, const int64_t* sizes, const int64_t* strides) {
    int64_t expect = 1;
    for (int i = ndim - 1; i >= 0; --i) {
        if (sizes[i] != 1 && strides[i] != expect) return false;
        expect *= sizes[i];
    }
    return true;
}

// ---- sum over the middle dim of [outer, red, inner] --------------------------

template <typename TI, typename TO>
__device__ __forceinline__ void store_sum(TO* p, int64_t i, float v);
template <> __device__ __forceinline__ void store_sum<__half, __half>(__half* p, int64_t i, float v) { p[i] = __float2half_rn(v); }
template <> __device__ __forceinline__ void store_sum<__half, float>(float* p, int64_t i, float v) { p[i] = v; }
template <> __device__ __forceinline__ void store_sum<float, float>(float* p, int64_t i, float v) { p[i] = v; }

// inner > 1: a 32 x 8 block covers 32 consecutive inner columns of one outer
// index; thread row ty sums red indices ty, ty + 8, ... (coalesced along the
// columns), then the 8 partials are added in a fixed order.
template <typename TI, typename TO>
__global__ void reduce_cols_kernel(const TI* __restrict__ x, TO* __restrict__ out, int64_t red,
                                   int64_t inner) {
    __shared__ float part[8][33];
    const int64_t o = blockIdx.y;
    const int64_t col = static_cast<int64_t>(blockIdx.x) * 32 + threadIdx.x;
    float acc = 0.0f;
    if (col < inner) {
        const TI* xp = x + o * red * inner + col;
        for (int64_t r = threadIdx.y; r < red; r += 8) acc += ld<TI>(xp, r * inner);
    }
    part[threadIdx.y][threadIdx.x] = acc;
    __syncthreads();
    if (threadIdx.y == 0 && col < inner) {
        float s = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; ++k) s += part[k][threadIdx.x];
        store_sum<TI, TO>(out, o * inner + col, s);
    }
}

// outer == 1, red <= 8, inner a multiple of 8 with 16-byte aligned rows (the
// slots of a row-block exchange): 8 consecutive columns per thread, all red
// loads in flight, slots added in index order from 0 -- the same additions and
// rounding as reduce_cols_kernel, at HBM speed.
template <typename T> __device__ __forceinline__ void ld8f(const T* p, float (&v)[8]);
template <> __device__ __forceinline__ void ld8f<__half>(const __half* p, float (&v)[8]) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h[j]);
        v[2 * j] = f.x;
        v[2 * j + 1] = f.y;
    }
}
template <> __device__ __forceinline__ void ld8f<float>(const float* p, float (&v)[8]) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p)), b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <typename T> __device__ __forceinline__ void st8f(T* p, const float (&v)[8]);
template <> __device__ __forceinline__ void st8f<__half>(__half* p, const float (&v)[8]) {
    uint4 u;
    __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) h[j] = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
    *reinterpret_cast<uint4*>(p) = u;
}
template <> __device__ __forceinline__ void st8f<float>(float* p, const float (&v)[8]) {
    reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}

template <typename TI, typename TO>
__global__ void __launch_bounds__(256) sum_slots_kernel(const TI* __restrict__ x, TO* __restrict__ out, int red,
                                                        int64_t inner) {
    const int64_t n8 = inner / 8;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x; i < n8;
         i += static_cast<int64_t>(gridDim.x) * 256) {
        float v[8][8];
#pragma unroll
        for (int r = 0; r < 8; ++r)
            if (r < red) ld8f<TI>(x + r * inner + i * 8, v[r]);
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
#pragma unroll
        for (int r = 0; r < 8; ++r)
            if (r < red) {
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[j] += v[r][j];
            }
        st8f<TO>(out + i * 8, acc);
    }
}

// inner == 1: one warp per row, lane-strided partials, shuffle tree.
template <typename TI, typename TO>
__global__ void reduce_rows_kernel(const TI* __restrict__ x, TO* __restrict__ out, int64_t rows,
                                   int64_t red) {
    const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + threadIdx.y;
    if (row >= rows) return;
    const TI* xp = x + row * red;
    float acc = 0.0f;
    for (int64_t r = threadIdx.x; r < red; r += 32) acc += ld<TI>(xp, r);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (threadIdx.x == 0) store_sum<TI, TO>(out, row, acc);
}

template <typename TI, typename TO>
int reduce_launch(const void* x, int64_t outer, int64_t red, int64_t inner, void* out,
                  cudaStream_t stream) {
    const dim3 block(32, 8);
    if (outer == 1 && red >= 1 && red <= 8 && inner % 8 == 0 &&
        reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
        (inner * static_cast<int64_t>(sizeof(TI))) % 16 == 0) {
        const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>(ceil_div(inner / 8, 256),
                                                                      8LL * sm_count(current_device())));
        sum_slots_kernel<TI, TO><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
            static_cast<const TI*>(x), static_cast<TO*>(out), static_cast<int>(red), inner);
        return launch_status("reduce_sum");
    }
    if (inner == 1) {
        const int64_t blocks = ceil_div(outer, 8);
        TK_CHECK_ARG(blocks < (1LL << 31), "tk_reduce_sum: too many rows");
        reduce_rows_kernel<TI, TO><<<static_cast<unsigned>(blocks), block, 0, stream>>>(
            static_cast<const TI*>(x), static_cast<TO*>(out), outer, red);
    } else {
        TK_CHECK_ARG(ceil_div(inner, 32) < (1LL << 31), "tk_reduce_sum: inner extent too large");
        for (int64_t o0 = 0; o0 < outer; o0 += 65535) {  // grid.y is limited to 65535
            const int64_t no = std::min<int64_t>(65535, outer - o0);
            const dim3 grid(static_cast<unsigned>(ceil_div(inner, 32)), static_cast<unsigned>(no));
            reduce_cols_kernel<TI, TO><<<grid, block, 0, stream>>>(
                static_cast<const TI*>(x) + o0 * red * inner, static_cast<TO*>(out) + o0 * inner, red,
                inner);
        }
    }
    return launch_status("reduce_sum");
}

// Merge adjacent dims that are contiguous in both operands, drop size-1 dims.
void collapse(Strided& d) {
    Strided o;
    o.ndim = 0;
    for (int k = 0; k < d.ndim; ++k) {
        if (d.sizes[k] == 1) continue;
        if (o.ndim > 0) {
            const int j = o.ndim - 1;
            if (o.s0[j] == d.sizes[k] * d.s0[k] && o.s1[j] == d.sizes[k] * d.s1[k]) {
                o.sizes[j] *= d.sizes[k];
                o.s0[j] = d.s0[k];
                o.s1[j] = d.s1[k];
                continue;
            }
        }
        o.sizes[o.ndim] = d.sizes[k];
        o.s0[o.ndim] = d.s0[k];
        o.s1[o.ndim] = d.s1[k];
        ++o.ndim;
    }
    if (o.ndim == 0) {
        o.ndim = 1;
        o.sizes[0] = 1;
        o.s0[0] = o.s1[0] = 0;
    }
    d = o;
}

// Same-dtype strided copy: collapsed dims, 16-byte vectors along a shared
// contiguous innermost dim when alignment allows, 32-bit indexing when the
// index space fits.
int copy_same_fast(void* dst, const void* src, int es, Strided d, cudaStream_t stream) {
    collapse(d);
    const int last = d.ndim - 1;
    const int vec = 16 / es;
    bool v16 = d.s0[last] == 1 && d.s1[last] == 1 && d.sizes[last] % vec == 0 &&
               reinterpret_cast<uintptr_t>(dst) % 16 == 0 && reinterpret_cast<uintptr_t>(src) % 16 == 0;
    for (int k = 0; k < last && v16; ++k) v16 = d.s0[k] % vec == 0 && d.s1[k] % vec == 0;
    int e = es;
    if (v16) {
        d.sizes[last] /= vec;
        for (int k = 0; k < last; ++k) {
            d.s0[k] /= vec;
            d.s1[k] /= vec;
        }
        e = 16;
    }
    int64_t n = 1;
    for (int k = 0; k < d.ndim; ++k) n *= d.sizes[k];
    const int grid = grid_for(n);
    const bool small = n < (1LL << 31);
    auto go = [&](auto tag) {
        using E = decltype(tag);
        if (small)
            copy_same_kernel32<E><<<grid, kThreads, 0, stream>>>(
                static_cast<E*>(dst), static_cast<const E*>(src), static_cast<int>(n), d);
        else
            copy_same_kernel<E><<<grid, kThreads, 0, stream>>>(static_cast<E*>(dst),
                                                                static_cast<const E*>(src), n, d);
    };
    switch (e) {
        case 1: go(uint8_t{}); break;
        case 2: go(uint16_t{}); break;
        case 4: go(uint32_t{}); break;
        case 8: go(static_cast<unsigned long long>(0)); break;
        default: go(uint4{}); break;
    }
    return launch_status("copy_strided");
}

}  // namespace
}  // namespace tk

extern "C" {

int tk_copy_strided(void* dst, int dst_type, const void* src, int src_type, int ndim,
                    const int64_t* sizes, const int64_t* dst_strides, const int64_t* src_strides,
                    void* stream_) {
    using namespace tk;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    TK_CHECK_ARG(dst_type >= 0 && dst_type <= T_F64 && src_type >= 0 && src_type <= T_F64,
                 "tk_copy_strided: bad scalar type");
    Strided d;
    int64_t n = 0;
    int rc = fill_strided_desc(d, ndim, sizes, dst_strides, src_strides, n);
    if (rc) return rc;
    if (n == 0) return TK_OK;
    TK_CHECK_ARG(dst && src, "tk_copy_strided: NULL pointer");
    const bool dd = is_dense(ndim, sizes, dst_strides), sd = is_dense(ndim, sizes, src_strides);
    if (dst_type == src_type && dd && sd) {
        TK_CUDA_TRY(cudaMemcpyAsync(dst, src, static_cast<size_t>(n) * scalar_size(dst_type),
                                    cudaMemcpyDeviceToDevice, stream));
        return TK_OK;
    }
    const int grid = grid_for(n);
    if (dd && sd && dst_type == T_F16 && src_type == T_F32) {
        f32_to_f16_kernel<<<grid, kThreads, 0, stream>>>(static_cast<__half*>(dst),
                                                         static_cast<const float*>(src), n);
        return launch_status("copy f32->f16");
    }
    if (dd && sd && dst_type == T_F32 && src_type == T_F16) {
        f16_to_f32_kernel<<<grid, kThreads, 0, stream>>>(static_cast<float*>(dst),
                                                         static_cast<const __half*>(src), n);
        return launch_status("copy f16->f32");
    }
    if (dst_type == src_type) return copy_same_fast(dst, src, scalar_size(dst_type), d, stream);
    copy_convert_kernel<<<grid, kThreads, 0, stream>>>(dst, dst_type, src, src_type, n, d);
    return launch_status("copy_convert");
}

int tk_fill_strided(void* dst, int type, double value, int64_t ivalue, int ndim,
                    const int64_t* sizes, const int64_t* strides, void* stream_) {
    using namespace tk;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    Strided d;
    int64_t n = 0;
    int rc = fill_strided_desc(d, ndim, sizes, strides, nullptr, n);
    if (rc) return rc;
    if (n == 0) return TK_OK;
    TK_CHECK_ARG(dst != nullptr, "tk_fill_strided: NULL pointer");
    const bool dense = is_dense(ndim, sizes, strides);
    const int grid = grid_for(n);
    auto launch = [&](auto v) {
        using E = decltype(v);
        if (dense)
            fill_dense_kernel<E><<<grid, kThreads, 0, stream>>>(static_cast<E*>(dst), v, n);
        else
            fill_kernel<E><<<grid, kThreads, 0, stream>>>(static_cast<E*>(dst), v, n, d);
    };
    switch (type) {
        case T_BOOL: launch(static_cast<uint8_t>(ivalue != 0)); break;
        case T_U8: launch(static_cast<uint8_t>(ivalue)); break;
        case T_I8: launch(static_cast<int8_t>(ivalue)); break;
        case T_I16: launch(static_cast<int16_t>(ivalue)); break;
        case T_I32: launch(static_cast<int32_t>(ivalue)); break;
        case T_I64: launch(static_cast<long long>(ivalue)); break;
        case T_F16: { __half h = __float2half_rn(static_cast<float>(value));
                      launch(*reinterpret_cast<uint16_t*>(&h)); break; }
        case T_BF16: { __nv_bfloat16 h = __float2bfloat16_rn(static_cast<float>(value));
                       launch(*reinterpret_cast<uint16_t*>(&h)); break; }
        case T_F32: launch(static_cast<float>(value)); break;
        case T_F64: launch(value); break;
        default: TK_FAIL(TK_ERR_INVALID_ARG, "tk_fill_strided: bad scalar type %d", type);
    }
    return launch_status("fill");
}

int tk_binary(int op, tk_dtype_t dt, const void* a, const int64_t* a_strides, const void* b,
              const int64_t* b_strides, void* out, int ndim, const int64_t* sizes, float alpha,
              void* stream_) {
    using namespace tk;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    TK_CHECK_ARG(op >= TK_BIN_ADD && op <= TK_BIN_THRESHOLD_BACKWARD, "tk_binary: bad op %d", op);
    TK_CHECK_ARG(dt == TK_DTYPE_F16 || dt == TK_DTYPE_F32, "tk_binary: bad dtype");
    Strided d;
    int64_t n = 0;
    int rc = fill_strided_desc(d, ndim, sizes, a_strides, b_strides, n);
    if (rc) return rc;
    if (n == 0) return TK_OK;
    TK_CHECK_ARG(a && b && out, "tk_binary: NULL pointer");
    const bool dense = is_dense(ndim, sizes, a_strides) && is_dense(ndim, sizes, b_strides);
    const int grid = grid_for(n);
    if (dt == TK_DTYPE_F16) {
        if (dense)
            binary_dense_kernel<__half><<<grid, kThreads, 0, stream>>>(
                op, static_cast<const __half*>(a), static_cast<const __half*>(b),
                static_cast<__half*>(out), n, alpha);
        else
            binary_kernel<__half><<<grid, kThreads, 0, stream>>>(
                op, static_cast<const __half*>(a), static_cast<const __half*>(b),
                static_cast<__half*>(out), n, alpha, d);
    } else {
        if (dense)
            binary_dense_kernel<float><<<grid, kThreads, 0, stream>>>(
                op, static_cast<const float*>(a), static_cast<const float*>(b),
                static_cast<float*>(out), n, alpha);
        else
            binary_kernel<float><<<grid, kThreads, 0, stream>>>(
                op, static_cast<const float*>(a), static_cast<const float*>(b),
                static_cast<float*>(out), n, alpha, d);
    }
    return launch_status("binary");
}

int tk_reduce_sum(tk_dtype_t in_dtype, tk_dtype_t out_dtype, const void* x, int64_t outer,
                  int64_t red, int64_t inner, void* out, void* stream_) {
    using namespace tk;
    TK_CHECK_ARG(outer >= 0 && red >= 0 && inner >= 0, "tk_reduce_sum: negative size");
    if (outer == 0 || inner == 0) return TK_OK;
    TK_CHECK_ARG(x && out, "tk_reduce_sum: NULL pointer");
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    if (in_dtype == TK_DTYPE_F16 && out_dtype == TK_DTYPE_F16)
        return reduce_launch<__half, __half>(x, outer, red, inner, out, stream);
    if (in_dtype == TK_DTYPE_F16 && out_dtype == TK_DTYPE_F32)
        return reduce_launch<__half, float>(x, outer, red, inner, out, stream);
    if (in_dtype == TK_DTYPE_F32 && out_dtype == TK_DTYPE_F32)
        return reduce_launch<float, float>(x, outer, red, inner, out, stream);
    TK_FAIL(TK_ERR_UNSUPPORTED, "tk_reduce_sum: unsupported dtype combination");
}

int tk_unary(int op, tk_dtype_t dt, const void* x, void* y, int64_t n, float p0, float p1,
             void* stream_) {
    using namespace tk;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    TK_CHECK_ARG(op >= TK_UN_RELU && op <= TK_UN_SCALE, "tk_unary: bad op %d", op);
    TK_CHECK_ARG(n >= 0, "tk_unary: negative size");
    if (n == 0) return TK_OK;
    TK_CHECK_ARG(x && y, "tk_unary: NULL pointer");
    const int grid = grid_for(n);
    if (dt == TK_DTYPE_F16)
        unary_kernel<__half><<<grid, kThreads, 0, stream>>>(op, static_cast<const __half*>(x),
                                                             static_cast<__half*>(y), n, p0, p1);
    else
        unary_kernel<float><<<grid, kThreads, 0, stream>>>(op, static_cast<const float*>(x),
                                                            static_cast<float*>(y), n, p0, p1);
    return launch_status("unary");
}

int tk_silu_mul_amax(tk_dtype_t dt, const void* gate, const void* up, void* y, int64_t n, float* amax_out,
                     void* stream_) {
    using namespace tk;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    TK_CHECK_ARG(n >= 0, "tk_silu_mul_amax: negative size");
    TK_CHECK_ARG(amax_out != nullptr, "tk_silu_mul_amax: amax_out is NULL");
    TK_CHECK_ARG(dt == TK_DTYPE_F16 || dt == TK_DTYPE_F32, "tk_silu_mul_amax: bad dtype");
    TK_CUDA_TRY(cudaMemsetAsync(amax_out, 0, sizeof(float), stream));
    if (n == 0) return TK_OK;
    TK_CHECK_ARG(gate && up && y, "tk_silu_mul_amax: NULL pointer");
    const bool vec = n % 8 == 0 && reinterpret_cast<uintptr_t>(gate) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(up) % 16 == 0 && reinterpret_cast<uintptr_t>(y) % 16 == 0;
    const int grid = grid_for(vec ? n / 8 : n);
    unsigned* bits = reinterpret_cast<unsigned*>(amax_out);
    if (dt == TK_DTYPE_F16)
        silu_mul_amax_kernel<__half><<<grid, kThreads, 0, stream>>>(
            static_cast<const __half*>(gate), static_cast<const __half*>(up), static_cast<__half*>(y), n,
            vec ? 1 : 0, bits);
    else
        silu_mul_amax_kernel<float><<<grid, kThreads, 0, stream>>>(
            static_cast<const float*>(gate), static_cast<const float*>(up), static_cast<float*>(y), n,
            vec ? 1 : 0, bits);
    return launch_status("silu_mul_amax");
}

int tk_silu_mul(tk_dtype_t dt, const void* gate, const void* up, void* y, int64_t n, void* stream_) {
    using namespace tk;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    TK_CHECK_ARG(n >= 0, "tk_silu_mul: negative size");
    if (n == 0) return TK_OK;
    TK_CHECK_ARG(gate && up && y, "tk_silu_mul: NULL pointer");
    const int grid = grid_for(n);
    if (dt == TK_DTYPE_F16)
        silu_mul_kernel<__half><<<grid, kThreads, 0, stream>>>(
            static_cast<const __half*>(gate), static_cast<const __half*>(up),
            static_cast<__half*>(y), n);
    else
        silu_mul_kernel<float><<<grid, kThreads, 0, stream>>>(
            static_cast<const float*>(gate), static_cast<const float*>(up),
            static_cast<float*>(y), n);
    return launch_status("silu_mul");
}

}  // extern "C"
