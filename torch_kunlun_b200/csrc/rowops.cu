// rowops.cu -- softmax and layer_norm over the last dimension.
//
// Replace xdnn::softmax (csrc/ops_nn.cpp:73-83) and xdnn::layer_norm
// (csrc/ops_nn.cpp:85-130).  Both are HBM-bound row kernels: a row of up to
// kRegCols elements is held in registers by one warp (128-bit loads), reduced
// with warp shuffles in a fixed order (so results are deterministic), and
// written back once.  Longer rows use a block per row with a shared-memory
// reduction.  Arithmetic is fp32; outputs are rounded once to the row dtype.
#include <algorithm>
#include <mutex>

#include "tk_internal.h"

namespace tk {
namespace {

constexpr int kRegCols = 2048;  // per-warp path: 64 values per lane max

template <typename T> __device__ __forceinline__ float ldf(const T* p, int64_t i);
template <> __device__ __forceinline__ float ldf<__half>(const __half* p, int64_t i) { return __half2float(p[i]); }
template <> __device__ __forceinline__ float ldf<float>(const float* p, int64_t i) { return p[i]; }
template <typename T> __device__ __forceinline__ void stf(T* p, int64_t i, float v);
template <> __device__ __forceinline__ void stf<__half>(__half* p, int64_t i, float v) { p[i] = __float2half_rn(v); }
template <> __device__ __forceinline__ void stf<float>(float* p, int64_t i, float v) { p[i] = v; }

// N consecutive elements (N * sizeof(T) a multiple of 16 bytes, p 16-byte
// aligned) loaded / stored with 128-bit accesses.
template <int N>
__device__ __forceinline__ void ldv(const __half* p, float (&o)[N]) {
#pragma unroll
    for (int c = 0; c < N / 8; ++c) {
        const uint4 u = *reinterpret_cast<const uint4*>(p + 8 * c);
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const float2 f = __half22float2(h[t]);
            o[8 * c + 2 * t] = f.x;
            o[8 * c + 2 * t + 1] = f.y;
        }
    }
}
template <int N>
__device__ __forceinline__ void ldv(const float* p, float (&o)[N]) {
#pragma unroll
    for (int c = 0; c < N / 4; ++c) {
        const float4 f = *reinterpret_cast<const float4*>(p + 4 * c);
        o[4 * c] = f.x;
        o[4 * c + 1] = f.y;
        o[4 * c + 2] = f.z;
        o[4 * c + 3] = f.w;
    }
}
template <int N>
__device__ __forceinline__ void stv(__half* p, const float (&v)[N]) {
#pragma unroll
    for (int c = 0; c < N / 8; ++c) {
        uint4 u;
        __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
        for (int t = 0; t < 4; ++t) h[t] = __floats2half2_rn(v[8 * c + 2 * t], v[8 * c + 2 * t + 1]);
        *reinterpret_cast<uint4*>(p + 8 * c) = u;
    }
}
template <int N>
__device__ __forceinline__ void stv(float* p, const float (&v)[N]) {
#pragma unroll
    for (int c = 0; c < N / 4; ++c)
        *reinterpret_cast<float4*>(p + 4 * c) = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
}

// exp(x) as 2^(x log2 e) on the special-function unit (relative error of a
// few binary32 ulps, inside the bound the softmax parity tests state).
__device__ __forceinline__ float exp_sfu(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x * 1.4426950408889634f));
    return y;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// One warp per row; each lane holds PER columns: lane l owns columns
// l*VEC + j*32*VEC + t (t < VEC), loaded and stored as 128-bit vectors.
template <typename TI, typename TO, int PER>
__global__ void softmax_warp_kernel(const TI* __restrict__ x, TO* __restrict__ y, int64_t rows,
                                    int cols) {
    constexpr int VEC = 16 / sizeof(TI);
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const TI* xr = x + row * cols;
    float v[PER];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < PER / VEC; ++j) {
        const int c0 = (j * 32 + lane) * VEC;
        float t[VEC];
        if (c0 < cols) {  // cols is a multiple of VEC on this path
            ldv<VEC>(xr + c0, t);
        } else {
#pragma unroll
            for (int i = 0; i < VEC; ++i) t[i] = -INFINITY;
        }
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
            v[j * VEC + i] = t[i];
            m = fmaxf(m, t[i]);
        }
    }
    m = warp_max(m);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        v[i] = (v[i] == -INFINITY) ? 0.f : exp_sfu(v[i] - m);
        s += v[i];
    }
    s = warp_sum(s);
    const float inv = 1.0f / s;
    TO* yr = y + row * cols;
#pragma unroll
    for (int j = 0; j < PER / VEC; ++j) {
        const int c0 = (j * 32 + lane) * VEC;
        if (c0 < cols) {
            float o[VEC];
#pragma unroll
            for (int i = 0; i < VEC; ++i) o[i] = v[j * VEC + i] * inv;
            stv<VEC>(yr + c0, o);
        }
    }
}

// Block per row for long rows (three passes over the row, reads cached in L2).
template <typename TI, typename TO>
__global__ void softmax_block_kernel(const TI* __restrict__ x, TO* __restrict__ y, int cols) {
    __shared__ float red[32];
    const int64_t row = blockIdx.x;
    const TI* xr = x + row * cols;
    TO* yr = y + row * cols;
    float m = -INFINITY;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) m = fmaxf(m, ldf<TI>(xr, c));
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : -INFINITY;
        t = warp_max(t);
        if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    m = red[0];
    __syncthreads();
    float s = 0.f;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) s += exp_sfu(ldf<TI>(xr, c) - m);
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    const float inv = 1.0f / red[0];
    for (int c = threadIdx.x; c < cols; c += blockDim.x) stf<TO>(yr, c, exp_sfu(ldf<TI>(xr, c) - m) * inv);
}

template <typename T, typename TW, int PER>
__global__ void layer_norm_warp_kernel(const T* __restrict__ x, const TW* __restrict__ gamma,
                                       const TW* __restrict__ beta, T* __restrict__ y,
                                       float* __restrict__ mean_out, float* __restrict__ rstd_out,
                                       int64_t rows, int cols, float eps) {
    constexpr int VEC = 16 / sizeof(T);
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const T* xr = x + row * cols;
    float v[PER];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < PER / VEC; ++j) {
        const int c0 = (j * 32 + lane) * VEC;
        float t[VEC];
        if (c0 < cols) {  // cols is a multiple of VEC on this path
            ldv<VEC>(xr + c0, t);
        } else {
#pragma unroll
            for (int i = 0; i < VEC; ++i) t[i] = 0.f;
        }
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
            v[j * VEC + i] = t[i];
            s += t[i];
        }
    }
    const float mean = warp_sum(s) / cols;
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < PER / VEC; ++j) {
        const int c0 = (j * 32 + lane) * VEC;
#pragma unroll
        for (int t = 0; t < VEC; ++t) {
            const float d = (c0 < cols) ? v[j * VEC + t] - mean : 0.f;
            q += d * d;
        }
    }
    const float var = warp_sum(q) / cols;
    const float rstd = rsqrtf(var + eps);
    T* yr = y + row * cols;
#pragma unroll
    for (int j = 0; j < PER / VEC; ++j) {
        const int c0 = (j * 32 + lane) * VEC;
        if (c0 < cols) {
            float o[VEC], g[VEC], b[VEC];
#pragma unroll
            for (int t = 0; t < VEC; ++t) o[t] = (v[j * VEC + t] - mean) * rstd;
            if (gamma) {
                ldv<VEC>(gamma + c0, g);
#pragma unroll
                for (int t = 0; t < VEC; ++t) o[t] = o[t] * g[t];
            }
            if (beta) {
                ldv<VEC>(beta + c0, b);
#pragma unroll
                for (int t = 0; t < VEC; ++t) o[t] = o[t] + b[t];
            }
            stv<VEC>(yr + c0, o);
        }
    }
    if (lane == 0) {
        if (mean_out) mean_out[row] = mean;
        if (rstd_out) rstd_out[row] = rstd;
    }
}

template <typename T, typename TW>
__global__ void layer_norm_block_kernel(const T* __restrict__ x, const TW* __restrict__ gamma,
                                        const TW* __restrict__ beta, T* __restrict__ y,
                                        float* __restrict__ mean_out, float* __restrict__ rstd_out,
                                        int cols, float eps) {
    __shared__ float red[32];
    const int64_t row = blockIdx.x;
    const T* xr = x + row * cols;
    auto block_sum = [&](float v) {
        v = warp_sum(v);
        __syncthreads();
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
        __syncthreads();
        float t = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x & 31] : 0.f;
        if (threadIdx.x < 32) t = warp_sum(t);
        if (threadIdx.x == 0) red[0] = t;
        __syncthreads();
        return red[0];
    };
    float s = 0.f;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) s += ldf<T>(xr, c);
    const float mean = block_sum(s) / cols;
    float q = 0.f;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
        const float d = ldf<T>(xr, c) - mean;
        q += d * d;
    }
    const float rstd = rsqrtf(block_sum(q) / cols + eps);
    T* yr = y + row * cols;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
        float o = (ldf<T>(xr, c) - mean) * rstd;
        if (gamma) o = o * ldf<TW>(gamma, c);
        if (beta) o = o + ldf<TW>(beta, c);
        stf<T>(yr, c, o);
    }
    if (threadIdx.x == 0) {
        if (mean_out) mean_out[row] = mean;
        if (rstd_out) rstd_out[row] = rstd;
    }
}

// ---- persistent row kernels: the next row's loads in flight ----------------
//
// One warp per row as above (lane l owns the 16-byte vectors l, l + 32, ...
// of the row, so the per-lane partial sums and the butterfly reduction run in
// the same order), but a warp walks rows with a grid stride and issues the
// next row's loads before it reduces the current one: the HBM latency of a
// row overlaps the arithmetic of the previous one, and a grid of a few waves
// of warps replaces one warp per row.
template <typename T, int NV>
__device__ __forceinline__ void load_row_vecs(const T* row, int cols, int lane, uint4 (&v)[NV]) {
    constexpr int VEC = 16 / sizeof(T);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        const int c0 = (j * 32 + lane) * VEC;
        v[j] = c0 < cols ? __ldg(reinterpret_cast<const uint4*>(row + c0)) : make_uint4(0, 0, 0, 0);
    }
}

template <typename T>
__device__ __forceinline__ void unpack_vec(const uint4& u, float* o) {
    if constexpr (sizeof(T) == 2) {
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const float2 f = __half22float2(h[t]);
            o[2 * t] = f.x;
            o[2 * t + 1] = f.y;
        }
    } else {
        o[0] = __uint_as_float(u.x); o[1] = __uint_as_float(u.y);
        o[2] = __uint_as_float(u.z); o[3] = __uint_as_float(u.w);
    }
}

// Up to 3 vectors per lane: four resident blocks per SM (64 registers), so
// more rows are in flight (64x512x512 fp16: 19.0 -> 17.1 us).
template <typename TI, typename TO, int NV>
__global__ void __launch_bounds__(256, NV <= 3 ? 4 : 2) softmax_rows_kernel(const TI* __restrict__ x, TO* __restrict__ y,
                                                           int64_t rows, int cols) {
    constexpr int VEC = 16 / sizeof(TI);
    const int lane = threadIdx.x & 31;
    const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
    int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
    uint4 cur[NV];
    if (row < rows) load_row_vecs<TI, NV>(x + row * cols, cols, lane, cur);
    for (; row < rows; row += nw) {
        uint4 nxt[NV];
        if (row + nw < rows) load_row_vecs<TI, NV>(x + (row + nw) * cols, cols, lane, nxt);
        float v[NV * VEC];
        float m = -INFINITY;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int c0 = (j * 32 + lane) * VEC;
            unpack_vec<TI>(cur[j], v + j * VEC);
#pragma unroll
            for (int i = 0; i < VEC; ++i) {
                if (c0 >= cols) v[j * VEC + i] = -INFINITY;
                m = fmaxf(m, v[j * VEC + i]);
            }
        }
        m = warp_max(m);
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < NV * VEC; ++i) {
            v[i] = (v[i] == -INFINITY) ? 0.f : exp_sfu(v[i] - m);
            s += v[i];
        }
        s = warp_sum(s);
        const float inv = 1.0f / s;
        TO* yr = y + row * cols;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int c0 = (j * 32 + lane) * VEC;
            if (c0 < cols) {
                float o[VEC];
#pragma unroll
                for (int i = 0; i < VEC; ++i) o[i] = v[j * VEC + i] * inv;
                stv<VEC>(yr + c0, o);
            }
        }
#pragma unroll
        for (int j = 0; j < NV; ++j) cur[j] = nxt[j];
    }
}

template <typename T, typename TW, int NV>
__global__ void __launch_bounds__(256)
layer_norm_rows_kernel(const T* __restrict__ x, const TW* __restrict__ gamma, const TW* __restrict__ beta,
                       T* __restrict__ y, float* __restrict__ mean_out, float* __restrict__ rstd_out,
                       int64_t rows, int cols, float eps) {
    constexpr int VEC = 16 / sizeof(T);
    const int lane = threadIdx.x & 31;
    const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
    int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
    uint4 cur[NV];
    if (row < rows) load_row_vecs<T, NV>(x + row * cols, cols, lane, cur);
    for (; row < rows; row += nw) {
        uint4 nxt[NV];
        if (row + nw < rows) load_row_vecs<T, NV>(x + (row + nw) * cols, cols, lane, nxt);
        float v[NV * VEC];
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            unpack_vec<T>(cur[j], v + j * VEC);  // columns past the row load as 0
#pragma unroll
            for (int i = 0; i < VEC; ++i) s += v[j * VEC + i];
        }
        const float mean = warp_sum(s) / cols;
        float q = 0.f;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int c0 = (j * 32 + lane) * VEC;
#pragma unroll
            for (int t = 0; t < VEC; ++t) {
                const float d = (c0 < cols) ? v[j * VEC + t] - mean : 0.f;
                q += d * d;
            }
        }
        const float var = warp_sum(q) / cols;
        const float rstd = rsqrtf(var + eps);
        T* yr = y + row * cols;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int c0 = (j * 32 + lane) * VEC;
            if (c0 < cols) {
                // gamma / beta: the same columns for every row, L1-resident
                float o[VEC], g[VEC], b[VEC];
                if (gamma) ldv<VEC>(gamma + c0, g);
                if (beta) ldv<VEC>(beta + c0, b);
#pragma unroll
                for (int t = 0; t < VEC; ++t) {
                    o[t] = (v[j * VEC + t] - mean) * rstd;
                    if (gamma) o[t] = o[t] * g[t];
                    if (beta) o[t] = o[t] + b[t];
                }
                stv<VEC>(yr + c0, o);
            }
        }
        if (lane == 0) {
            if (mean_out) mean_out[row] = mean;
            if (rstd_out) rstd_out[row] = rstd;
        }
#pragma unroll
        for (int j = 0; j < NV; ++j) cur[j] = nxt[j];
    }
}

// Blocks of a persistent row kernel: every block resident at once (the
// occupancy of the instantiation times the SM count), or fewer when there
// are fewer rows than warps.
template <auto Kernel>
int64_t row_grid(int64_t rows) {
    static std::once_flag once;
    static int per_sm = 1;
    std::call_once(once, [] {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, Kernel, 256, 0) == cudaSuccess && n > 0) per_sm = n;
    });
    const int64_t resident = static_cast<int64_t>(per_sm) * sm_count(current_device());
    return std::max<int64_t>(1, std::min<int64_t>(resident, ceil_div(rows, 8)));
}

template <typename TI, typename TO>
int softmax_launch(const void* x, void* y, int64_t rows, int64_t cols, cudaStream_t st) {
    const TI* xp = static_cast<const TI*>(x);
    TO* yp = static_cast<TO*>(y);
    constexpr int VEC = 16 / sizeof(TI);
    if (cols <= kRegCols && (cols % VEC) == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
        reinterpret_cast<uintptr_t>(y) % 16 == 0 && (cols * sizeof(TO)) % 16 == 0) {
        const int nv = static_cast<int>(ceil_div(cols, 32 * VEC));
#define TK_SOFTMAX_ROWS(NV)                                                                          \
    if (nv == NV) {                                                                                   \
        const unsigned rgrid = static_cast<unsigned>(row_grid<softmax_rows_kernel<TI, TO, NV>>(rows)); \
        softmax_rows_kernel<TI, TO, NV><<<rgrid, 256, 0, st>>>(xp, yp, rows, (int)cols);             \
        return launch_status("softmax");                                                              \
    }
        TK_SOFTMAX_ROWS(1) TK_SOFTMAX_ROWS(2) TK_SOFTMAX_ROWS(3) TK_SOFTMAX_ROWS(4)
#undef TK_SOFTMAX_ROWS
        const int warps = 8;
        const unsigned grid = static_cast<unsigned>(ceil_div(rows, warps));
        const int per = static_cast<int>(round_up(static_cast<size_t>(ceil_div(cols, 32)), VEC));
#define TK_SOFTMAX_CASE(P)                                                                   \
    if (per <= P) {                                                                          \
        softmax_warp_kernel<TI, TO, P><<<grid, warps * 32, 0, st>>>(xp, yp, rows, (int)cols); \
        return launch_status("softmax");                                                      \
    }
        TK_SOFTMAX_CASE(8) TK_SOFTMAX_CASE(16) TK_SOFTMAX_CASE(32) TK_SOFTMAX_CASE(64)
#undef TK_SOFTMAX_CASE
    }
    TK_CHECK_ARG(rows <= 0x7FFFFFFF, "softmax: too many rows");
    softmax_block_kernel<TI, TO><<<static_cast<unsigned>(rows), 512, 0, st>>>(xp, yp, (int)cols);
    return launch_status("softmax");
}

template <typename T, typename TW>
int layer_norm_launch(const void* x, const void* g, const void* b, void* y, float* mean,
                      float* rstd, int64_t rows, int64_t cols, float eps, cudaStream_t st) {
    const T* xp = static_cast<const T*>(x);
    T* yp = static_cast<T*>(y);
    const TW* gp = static_cast<const TW*>(g);
    const TW* bp = static_cast<const TW*>(b);
    constexpr int VEC = 16 / sizeof(T);
    if (cols <= kRegCols && (cols % VEC) == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
        reinterpret_cast<uintptr_t>(y) % 16 == 0 && reinterpret_cast<uintptr_t>(g) % 16 == 0 &&
        reinterpret_cast<uintptr_t>(b) % 16 == 0) {
        const int nv = static_cast<int>(ceil_div(cols, 32 * VEC));
#define TK_LN_ROWS(NV)                                                                                \
    if (nv == NV) {                                                                                   \
        const unsigned rgrid = static_cast<unsigned>(row_grid<layer_norm_rows_kernel<T, TW, NV>>(rows)); \
        layer_norm_rows_kernel<T, TW, NV><<<rgrid, 256, 0, st>>>(xp, gp, bp, yp, mean, rstd, rows,  \
                                                                 (int)cols, eps);                    \
        return launch_status("layer_norm");                                                           \
    }
        TK_LN_ROWS(1) TK_LN_ROWS(2) TK_LN_ROWS(3) TK_LN_ROWS(4)
#undef TK_LN_ROWS
        const int warps = 8;
        const unsigned grid = static_cast<unsigned>(ceil_div(rows, warps));
        const int per = static_cast<int>(round_up(static_cast<size_t>(ceil_div(cols, 32)), VEC));
#define TK_LN_CASE(P)                                                                             \
    if (per <= P) {                                                                               \
        layer_norm_warp_kernel<T, TW, P><<<grid, warps * 32, 0, st>>>(xp, gp, bp, yp, mean, rstd, \
                                                                      rows, (int)cols, eps);      \
        return launch_status("layer_norm");                                                       \
    }
        TK_LN_CASE(8) TK_LN_CASE(16) TK_LN_CASE(32) TK_LN_CASE(64)
#undef TK_LN_CASE
    }
    TK_CHECK_ARG(rows <= 0x7FFFFFFF, "layer_norm: too many rows");
    layer_norm_block_kernel<T, TW><<<static_cast<unsigned>(rows), 512, 0, st>>>(
        xp, gp, bp, yp, mean, rstd, (int)cols, eps);
    return launch_status("layer_norm");
}

}  // namespace
}  // namespace tk

extern "C" {

int tk_softmax(tk_dtype_t in_dtype, tk_dtype_t out_dtype, const void* x, void* y, int64_t rows,
               int64_t cols, void* stream) {
    using namespace tk;
    TK_CHECK_ARG(rows >= 0 && cols >= 0, "tk_softmax: negative size");
    if (rows == 0 || cols == 0) return TK_OK;
    TK_CHECK_ARG(x && y, "tk_softmax: NULL pointer");
    TK_CHECK_ARG(cols < (1LL << 31), "tk_softmax: row too long");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (in_dtype == TK_DTYPE_F16 && out_dtype == TK_DTYPE_F16)
        return softmax_launch<__half, __half>(x, y, rows, cols, st);
    if (in_dtype == TK_DTYPE_F16 && out_dtype == TK_DTYPE_F32)
        return softmax_launch<__half, float>(x, y, rows, cols, st);
    if (in_dtype == TK_DTYPE_F32 && out_dtype == TK_DTYPE_F32)
        return softmax_launch<float, float>(x, y, rows, cols, st);
    TK_FAIL(TK_ERR_UNSUPPORTED, "tk_softmax: unsupported dtype combination");
}

int tk_layer_norm(tk_dtype_t dtype, tk_dtype_t wdtype, const void* x, const void* gamma,
                  const void* beta, void* y, float* mean, float* rstd, int64_t rows, int64_t cols,
                  float eps, void* stream) {
    using namespace tk;
    TK_CHECK_ARG(rows >= 0 && cols > 0, "tk_layer_norm: bad size");
    if (rows == 0) return TK_OK;
    TK_CHECK_ARG(x && y, "tk_layer_norm: NULL pointer");
    TK_CHECK_ARG(cols < (1LL << 31), "tk_layer_norm: row too long");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (dtype == TK_DTYPE_F16 && wdtype == TK_DTYPE_F16)
        return layer_norm_launch<__half, __half>(x, gamma, beta, y, mean, rstd, rows, cols, eps, st);
    if (dtype == TK_DTYPE_F16 && wdtype == TK_DTYPE_F32)
        return layer_norm_launch<__half, float>(x, gamma, beta, y, mean, rstd, rows, cols, eps, st);
    if (dtype == TK_DTYPE_F32 && wdtype == TK_DTYPE_F32)
        return layer_norm_launch<float, float>(x, gamma, beta, y, mean, rstd, rows, cols, eps, st);
    TK_FAIL(TK_ERR_UNSUPPORTED, "tk_layer_norm: unsupported dtype combination");
}

}  // extern "C"
