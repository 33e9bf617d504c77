// quant.cu -- per-tensor (or per-slice) max-abs reduction and int16
// quantisation into signed-high / unsigned-low int8 limb planes.
//
// These replace the max-find and quantise steps that XDNN runs inside
// fc/conv2d when called with null max pointers (csrc/ops.cpp:224-227,
// csrc/ops.cpp:264-268, csrc/ops_nn.cpp:214-218).  Both kernels are
// HBM-bound: amax reads 2 B (fp16) per element with 128-bit loads and a
// packed-halves max; quantisation reads 2 B and writes 2 B (two limbs) per
// element through a 64x64 shared-memory tile so that either operand layout
// (K-contiguous or transposed) is read and written coalesced.
#include <mutex>

#include "tk_internal.h"
#include "tk_numerics.cuh"
#include "tk_ptx.cuh"

namespace tk {
namespace {

constexpr int kAmaxThreads = 256;

__device__ __forceinline__ float load_f(const __half* p) { return __half2float(*p); }
__device__ __forceinline__ float load_f(const float* p) { return *p; }

// Block-wide max of an unsigned value; result valid in thread 0.
__device__ __forceinline__ unsigned block_max_u32(unsigned v) {
    __shared__ unsigned red[kAmaxThreads / 32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x < 32) {
        v = threadIdx.x < (kAmaxThreads / 32) ? red[threadIdx.x] : 0u;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    }
    return v;
}

__global__ void amax_f32_kernel(const float* __restrict__ x, int64_t slice_stride,
                                int64_t slice_len, int64_t chunk, bool vec,
                                unsigned* __restrict__ out_bits) {
    const int64_t s = blockIdx.y;
    const unsigned* base = reinterpret_cast<const unsigned*>(x + s * slice_stride);
    const int64_t start = static_cast<int64_t>(blockIdx.x) * chunk;
    const int64_t end = min(start + chunk, slice_len);
    unsigned m = 0;
    int64_t i = start;
    if (vec) {
        const int64_t nv = (end - start) / 4;
        const uint4* pv = reinterpret_cast<const uint4*>(base + start);
        for (int64_t j = threadIdx.x; j < nv; j += blockDim.x) {
            uint4 w = __ldg(pv + j);
            m = max(m, w.x & 0x7FFFFFFFu);
            m = max(m, w.y & 0x7FFFFFFFu);
            m = max(m, w.z & 0x7FFFFFFFu);
            m = max(m, w.w & 0x7FFFFFFFu);
        }
        i = start + nv * 4;
    }
    for (int64_t j = i + threadIdx.x; j < end; j += blockDim.x) {
        m = max(m, base[j] & 0x7FFFFFFFu);
    }
    m = block_max_u32(m);
    if (threadIdx.x == 0 && m != 0u) atomicMax(out_bits + s, m);
}

constexpr int kQT = 64;        // quantise tile: 64 rows x 64 columns
constexpr int kQThreads = 256;

// One 64x64 tile of one batch slice: load (coalesced along the source's
// contiguous axis), quantise into shared memory, then write both limb planes
// coalesced along the column (K) axis.
template <typename T, bool kColContig>
__global__ void __launch_bounds__(kQThreads)
quant_limbs_kernel(const T* __restrict__ x, int64_t rows, int64_t cols, int64_t ld, int64_t sb,
                   int64_t sr, int64_t sc, const float* __restrict__ amax, int64_t amax_stride,
                   int8_t* __restrict__ limbs) {
    __shared__ short tile[kQT][kQT + 2];
    const int64_t b = blockIdx.z;
    const int64_t r0 = static_cast<int64_t>(blockIdx.y) * kQT;
    const int64_t c0 = static_cast<int64_t>(blockIdx.x) * kQT;
    const float inv = quant_inv(amax[b * amax_stride]);
    const T* xb = x + b * sb;
    const int t = threadIdx.x;
#pragma unroll 4
    for (int p = 0; p < (kQT * kQT) / kQThreads; ++p) {
        int r, c;
        if (kColContig) {
            c = t % kQT;
            r = p * (kQThreads / kQT) + t / kQT;
        } else {
            r = t % kQT;
            c = p * (kQThreads / kQT) + t / kQT;
        }
        const int64_t gr = r0 + r, gc = c0 + c;
        int q = 0;
        if (gr < rows && gc < cols) q = quant_one(load_f(xb + gr * sr + gc * sc), inv);
        tile[r][c] = static_cast<short>(q);
    }
    __syncthreads();
    const int64_t plane = rows * ld;
    int8_t* hi_plane = limbs + (b * 2) * plane;
    int8_t* lo_plane = hi_plane + plane;
#pragma unroll
    for (int p = 0; p < (kQT * kQT) / (kQThreads * 4); ++p) {
        const int r = p * (kQThreads / 16) + t / 16;
        const int c = (t % 16) * 4;
        const int64_t gr = r0 + r, gc = c0 + c;
        if (gr < rows && gc < ld) {
            unsigned hi = 0, lo = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int q = tile[r][c + j];
                hi |= (static_cast<unsigned>(q >> 8) & 0xFFu) << (8 * j);
                lo |= (static_cast<unsigned>(q) & 0xFFu) << (8 * j);
            }
            *reinterpret_cast<unsigned*>(hi_plane + gr * ld + gc) = hi;
            *reinterpret_cast<unsigned*>(lo_plane + gr * ld + gc) = lo;
        }
    }
}


// ---- fused multi-operand paths used by the GEMM ------------------------------

// One amax descriptor: nslices dense ranges of slice_len elements.
struct AmaxDesc {
    const void* x;
    int64_t nslices, slice_stride, slice_len, chunk, chunks;  // chunks per slice
    unsigned* out;
    bool vec;
};

__device__ __forceinline__ uint4 ldg_nc_v4(const uint4* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// max(m, |a|) over the four fp16 pairs of w, as 16-bit magnitudes.
__device__ __forceinline__ unsigned fold_abs_max_h2x4(unsigned m, const uint4& w) {
    asm volatile(
        "{\n\t.reg .b32 t;\n\t"
        "and.b32 t, %1, 0x7FFF7FFF;\n\tmax.u16x2 %0, %0, t;\n\t"
        "and.b32 t, %2, 0x7FFF7FFF;\n\tmax.u16x2 %0, %0, t;\n\t"
        "and.b32 t, %3, 0x7FFF7FFF;\n\tmax.u16x2 %0, %0, t;\n\t"
        "and.b32 t, %4, 0x7FFF7FFF;\n\tmax.u16x2 %0, %0, t;\n\t}"
        : "+r"(m)
        : "r"(w.x), "r"(w.y), "r"(w.z), "r"(w.w));
    return m;
}

template <typename T>
__device__ __forceinline__ unsigned amax_range(const T* base, int64_t start, int64_t end, bool vec);

template <>
__device__ __forceinline__ unsigned amax_range<__half>(const __half* xh, int64_t start, int64_t end,
                                                       bool vec) {
    const unsigned short* base = reinterpret_cast<const unsigned short*>(xh);
    unsigned m2 = 0;
    int64_t i = start;
    if (vec) {
        const int64_t nv = (end - start) / 8;
        const uint4* pv = reinterpret_cast<const uint4*>(base + start);
        int64_t j = threadIdx.x;
        for (; j + 7 * static_cast<int64_t>(blockDim.x) < nv; j += 8 * blockDim.x) {
            uint4 w[8];
            // loads and folds are volatile, so the eight 128-bit loads are
            // all issued (in flight together) before the first fold
#pragma unroll
            for (int u = 0; u < 8; ++u) w[u] = ldg_nc_v4(pv + j + u * blockDim.x);
#pragma unroll
            for (int u = 0; u < 8; ++u) m2 = fold_abs_max_h2x4(m2, w[u]);
        }
        for (; j < nv; j += blockDim.x) {
            const uint4 w = __ldg(pv + j);
            m2 = __vmaxu2(m2, w.x & 0x7FFF7FFFu);
            m2 = __vmaxu2(m2, w.y & 0x7FFF7FFFu);
            m2 = __vmaxu2(m2, w.z & 0x7FFF7FFFu);
            m2 = __vmaxu2(m2, w.w & 0x7FFF7FFFu);
        }
        i = start + nv * 8;
    }
    for (int64_t j = i + threadIdx.x; j < end; j += blockDim.x)
        m2 = __vmaxu2(m2, static_cast<unsigned>(base[j] & 0x7FFFu));
    const unsigned h = max(m2 & 0xFFFFu, m2 >> 16);
    // widen the fp16 magnitude bits to the fp32 magnitude bits (NaN -> canonical)
    if ((h & 0x7C00u) == 0x7C00u && (h & 0x3FFu) != 0u) return 0x7FC00000u;
    return __float_as_uint(__half2float(__ushort_as_half(static_cast<unsigned short>(h)))) & 0x7FFFFFFFu;
}

template <>
__device__ __forceinline__ unsigned amax_range<float>(const float* xf, int64_t start, int64_t end,
                                                      bool vec) {
    const unsigned* base = reinterpret_cast<const unsigned*>(xf);
    unsigned m = 0;
    int64_t i = start;
    if (vec) {
        const int64_t nv = (end - start) / 4;
        const uint4* pv = reinterpret_cast<const uint4*>(base + start);
        for (int64_t j = threadIdx.x; j < nv; j += blockDim.x) {
            const uint4 w = __ldg(pv + j);
            m = max(m, max(max(w.x & 0x7FFFFFFFu, w.y & 0x7FFFFFFFu),
                           max(w.z & 0x7FFFFFFFu, w.w & 0x7FFFFFFFu)));
        }
        i = start + nv * 4;
    }
    for (int64_t j = i + threadIdx.x; j < end; j += blockDim.x) m = max(m, base[j] & 0x7FFFFFFFu);
    return m;
}

// Blocks [0, blocks0) reduce descriptor d0, the rest d1.  Each block takes one
// chunk of one slice and folds its maximum into out[slice] with atomicMax on
// the fp32 magnitude bits (the order of non-negative floats, NaN on top).
template <typename T>
__global__ void __launch_bounds__(kAmaxThreads)
amax_multi_kernel(AmaxDesc d0, AmaxDesc d1, int64_t blocks0) {
    pdl_trigger();  // a quantise kernel launched next may be placed now (it waits for this grid)
    int64_t b = blockIdx.x;
    const AmaxDesc& d = b < blocks0 ? d0 : d1;
    if (b >= blocks0) b -= blocks0;
    const int64_t slice = b / d.chunks;
    const int64_t c = b - slice * d.chunks;
    const int64_t start = c * d.chunk;
    const int64_t end = min(start + d.chunk, d.slice_len);
    const T* base = static_cast<const T*>(d.x) + slice * d.slice_stride;
    unsigned m = amax_range<T>(base, start, end, d.vec);
    m = block_max_u32(m);
    if (threadIdx.x == 0 && m != 0u) atomicMax(d.out + slice, m);
}

// Row-contiguous operand quantised 8 columns per thread: one 128-bit load
// (two for fp32) and two 64-bit limb stores per step.
__device__ __forceinline__ int64_t ceil_div_dev(int64_t a, int64_t b) { return (a + b - 1) / b; }

struct QVecDesc {
    const void* x;
    int64_t rows, cols, ld, sb, sr;
    int64_t groups;  // ld / 8
    int64_t items;   // batch * rows * groups
    const float* amax;
    int64_t amax_stride;
    int8_t* limbs;
};

template <typename T>
__device__ __forceinline__ void load8(const T* p, int64_t n, float (&v)[8]);

template <>
__device__ __forceinline__ void load8<__half>(const __half* p, int64_t n, float (&v)[8]) {
    if (n >= 8) {
        const uint4 w = __ldg(reinterpret_cast<const uint4*>(p));
        const __half2* h = reinterpret_cast<const __half2*>(&w);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = __half22float2(h[j]);
            v[2 * j] = f.x;
            v[2 * j + 1] = f.y;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = j < n ? __half2float(p[j]) : 0.0f;
    }
}

template <>
__device__ __forceinline__ void load8<float>(const float* p, int64_t n, float (&v)[8]) {
    if (n >= 8) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(p));
        const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = j < n ? p[j] : 0.0f;
    }
}

// Codes of 8 values by magic-number rounding (the classic float-to-int
// conversion by adding 1.5 * 2^23): for |t| < 2^22 the binary32 sum
// t + 1.5 * 2^23 rounds t to the nearest integer, ties to even (the rounding
// of every binary32 add), and holds that integer in two's complement in the
// low bits of its significand; the low 16 bits of the sum's bit pattern are
// the int16 code.  t = RN(v * inv) is the same binary32 product quant_one
// rounds, so the codes are identical -- provided the product is rounded
// before the add: a fused multiply-add would round v * inv + 1.5 * 2^23
// once and break ties of RN(v * inv) (e.g. v = amax / 2 gives
// RN(v * inv) = 16383.5, code 16384, while the exact product lies just below
// the tie).  The products run two lanes per instruction; each is then
// clamped to [-32767, 32767] with NaN mapped to 0 (quant_one's clamp: a
// caller may supply an amax below max |x|, and an infinite input scales to
// infinity), and the adds are __fadd_rn, which the compiler never contracts
// into a multiply-add.  The inv == 0 case is handled by the caller: every
// code is 0.
__device__ __forceinline__ uint64_t f32x2_mul_add_magic(uint64_t v2, uint64_t inv2) {
    constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
    uint64_t t;
    asm volatile("mul.rn.f32x2 %0, %1, %2;" : "=l"(t) : "l"(v2), "l"(inv2));
    const float lo = __fadd_rn(clamp_code_range(__uint_as_float(static_cast<unsigned>(t))), kMagic);
    const float hi = __fadd_rn(clamp_code_range(__uint_as_float(static_cast<unsigned>(t >> 32))), kMagic);
    return static_cast<uint64_t>(__float_as_uint(lo)) | (static_cast<uint64_t>(__float_as_uint(hi)) << 32);
}

__device__ __forceinline__ uint64_t pack_f32x2(float a, float b) {
    return static_cast<uint64_t>(__float_as_uint(a)) | (static_cast<uint64_t>(__float_as_uint(b)) << 32);
}

// r[j]: bit patterns whose low 16 bits are the codes -> hi / lo limb words.
__device__ __forceinline__ void pack_codes8(const uint64_t (&r)[4], uint2& hi, uint2& lo) {
    unsigned p[4];  // two codes per word: code_2i | code_2i+1 << 16
#pragma unroll
    for (int j = 0; j < 4; ++j)
        p[j] = __byte_perm(static_cast<unsigned>(r[j]), static_cast<unsigned>(r[j] >> 32), 0x5410);
    lo.x = __byte_perm(p[0], p[1], 0x6420);
    hi.x = __byte_perm(p[0], p[1], 0x7531);
    lo.y = __byte_perm(p[2], p[3], 0x6420);
    hi.y = __byte_perm(p[2], p[3], 0x7531);
}

__device__ __forceinline__ void quant8_magic(const float (&v)[8], float inv, uint2& hi, uint2& lo) {
    const uint64_t inv2 = pack_f32x2(inv, inv);
    uint64_t r[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) r[j] = f32x2_mul_add_magic(pack_f32x2(v[2 * j], v[2 * j + 1]), inv2);
    pack_codes8(r, hi, lo);
}

__device__ __forceinline__ void quant8_magic_h(const uint4& w, float inv, uint2& hi, uint2& lo) {
    const uint64_t inv2 = pack_f32x2(inv, inv);
    const __half2* h = reinterpret_cast<const __half2*>(&w);
    uint64_t r[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h[j]);
        r[j] = f32x2_mul_add_magic(pack_f32x2(f.x, f.y), inv2);
    }
    pack_codes8(r, hi, lo);
}

// One warp quantises one segment of kSegGroups 8-column groups of a row:
// each lane issues its four 128-bit loads before using any of them, and the
// small segments give a fine-grained, balanced grid.
constexpr int kSegGroups = 128;

template <typename T>
__device__ __forceinline__ void quant_vec_segment(const QVecDesc& d, int64_t row, int64_t seg, int lane) {
    const int64_t b = row / d.rows;
    const int64_t r = row - b * d.rows;
    const float inv = quant_inv(d.amax[b * d.amax_stride]);
    const T* src = static_cast<const T*>(d.x) + b * d.sb + r * d.sr;
    const int64_t plane = d.rows * d.ld;
    int8_t* dst = d.limbs + (b * 2) * plane + r * d.ld;
    const int64_t g0 = seg * kSegGroups + lane;
    if (inv == 0.0f) {  // amax 0 or not finite: every code is 0
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t g = g0 + 32 * u;
            if (g < d.groups) {
                *reinterpret_cast<uint2*>(dst + g * 8) = make_uint2(0, 0);
                *reinterpret_cast<uint2*>(dst + plane + g * 8) = make_uint2(0, 0);
            }
        }
        return;
    }
    if constexpr (sizeof(T) == 2) {
        // keep the four loads as raw 128-bit words (16 registers) until used
        uint4 w[4];
        bool part[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t c0 = (g0 + 32 * u) * 8;
            const int64_t n = d.cols - c0;
            part[u] = n > 0 && n < 8;
            w[u] = (g0 + 32 * u < d.groups && n >= 8) ? __ldg(reinterpret_cast<const uint4*>(src + c0))
                                                      : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t g = g0 + 32 * u;
            if (g < d.groups) {
                const int64_t c0 = g * 8;
                uint2 hi, lo;
                if (part[u]) {
                    float v[8];
                    load8<T>(src + c0, d.cols - c0, v);
                    quant8_magic(v, inv, hi, lo);
                } else {
                    quant8_magic_h(w[u], inv, hi, lo);
                }
                *reinterpret_cast<uint2*>(dst + c0) = hi;
                *reinterpret_cast<uint2*>(dst + plane + c0) = lo;
            }
        }
    } else {
        float v[4][8];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t g = g0 + 32 * u;
            const int64_t c0 = g * 8;
            const int64_t n = d.cols - c0;
            if (g < d.groups && n > 0) {
                load8<T>(src + c0, n, v[u]);
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) v[u][j] = 0.0f;
            }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t g = g0 + 32 * u;
            if (g < d.groups) {
                uint2 hi, lo;
                quant8_magic(v[u], inv, hi, lo);
                const int64_t c0 = g * 8;
                *reinterpret_cast<uint2*>(dst + c0) = hi;
                *reinterpret_cast<uint2*>(dst + plane + c0) = lo;
            }
        }
    }
}

// Warp items [0, items0) are (row, segment) pairs of d0, the rest of d1.
template <typename T>
__global__ void __launch_bounds__(256) quant_vec_kernel(QVecDesc d0, QVecDesc d1, int64_t items0,
                                                        int64_t items_total) {
    pdl_trigger();  // the GEMM that consumes the limbs may begin its prologue
    pdl_wait();     // the amax (and whatever wrote x) has completed
    const int64_t item = static_cast<int64_t>(blockIdx.x) * 8 + threadIdx.y;
    if (item >= items_total) return;
    const bool first = item < items0;
    const QVecDesc& d = first ? d0 : d1;
    const int64_t it = first ? item : item - items0;
    const int64_t segs = ceil_div_dev(d.groups, kSegGroups);
    quant_vec_segment<T>(d, it / segs, it - (it / segs) * segs, threadIdx.x);
}

}  // namespace

int amax_wave_blocks(tk_dtype_t dtype, int dev);

int amax_launch(tk_dtype_t dtype, const void* x, int64_t nslices, int64_t slice_stride,
                int64_t slice_len, float* amax_out, cudaStream_t stream) {
    TK_CHECK_ARG(nslices >= 0 && slice_len >= 0, "tk_amax: negative size");
    TK_CHECK_ARG(nslices <= 65535, "tk_amax: at most 65535 slices per call, got %lld",
                 (long long)nslices);
    if (nslices == 0) return TK_OK;
    TK_CHECK_ARG(amax_out != nullptr, "tk_amax: amax_out is NULL");
    TK_CUDA_TRY(cudaMemsetAsync(amax_out, 0, sizeof(float) * nslices, stream));
    if (slice_len == 0) return TK_OK;
    TK_CHECK_ARG(x != nullptr, "tk_amax: x is NULL");
    const size_t es = dtype_size(dtype);
    const int dev = current_device();
    if (dtype == TK_DTYPE_F16) {
        // One resident wave of amax_multi_kernel blocks (eight 128-bit loads
        // per thread in flight), shared evenly by the slices.
        AmaxDesc d = {};
        d.x = x;
        d.nslices = nslices;
        d.slice_stride = slice_stride;
        d.slice_len = slice_len;
        const int64_t per_slice = std::max<int64_t>(1, (amax_wave_blocks(dtype, dev) - 2) / nslices);
        d.chunk = std::max<int64_t>(static_cast<int64_t>(kAmaxThreads) * 64, ceil_div(slice_len, per_slice));
        d.chunk = (d.chunk + 7) / 8 * 8;
        d.chunks = ceil_div(slice_len, d.chunk);
        d.out = reinterpret_cast<unsigned*>(amax_out);
        d.vec = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && ((slice_stride * static_cast<int64_t>(es)) % 16 == 0);
        const int64_t total = d.chunks * nslices;
        TK_CHECK_ARG(total < (1LL << 31), "tk_amax: too many blocks");
        amax_multi_kernel<__half><<<static_cast<unsigned>(total), kAmaxThreads, 0, stream>>>(d, d, total);
        return launch_status("amax");
    }
    const int64_t per_block = static_cast<int64_t>(kAmaxThreads) * 32;  // elements
    int64_t blocks = ceil_div(slice_len, per_block);
    const int64_t want = std::max<int64_t>(1, (4LL * sm_count(dev)) / nslices);
    blocks = std::min(blocks, std::max<int64_t>(want, 1));
    blocks = std::max<int64_t>(blocks, 1);
    int64_t chunk = ceil_div(slice_len, blocks);
    chunk = (chunk + 7) / 8 * 8;
    blocks = ceil_div(slice_len, chunk);
    const bool vec = (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                     ((slice_stride * static_cast<int64_t>(es)) % 16 == 0);
    dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(nslices));
    unsigned* ob = reinterpret_cast<unsigned*>(amax_out);
    amax_f32_kernel<<<grid, kAmaxThreads, 0, stream>>>(static_cast<const float*>(x), slice_stride, slice_len,
                                                       chunk, vec, ob);
    return launch_status("amax");
}

// Blocks of amax_multi_kernel that are resident at once on the device: the
// amax passes size their chunks so that all blocks run in one wave (a second,
// partial wave left most SMs idle at the end).
int amax_wave_blocks(tk_dtype_t dtype, int dev) {
    static std::once_flag once[2];
    static int per_sm[2] = {0, 0};
    const int t = dtype == TK_DTYPE_F16 ? 0 : 1;
    std::call_once(once[t], [&] {
        int n = 0;
        const cudaError_t e = t == 0
            ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, amax_multi_kernel<__half>, kAmaxThreads, 0)
            : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, amax_multi_kernel<float>, kAmaxThreads, 0);
        per_sm[t] = (e == cudaSuccess && n > 0) ? n : 4;
    });
    return per_sm[t] * sm_count(dev);
}

// max |x| of two whole tensors in one launch (out[0] for x, out[1] for w):
// one memset of both slots, one amax_multi_kernel with a chunk size shared by
// both operands.
int amax_pair_launch(tk_dtype_t dtype, const void* x, int64_t nx, const void* w, int64_t nw, float* out,
                     cudaStream_t stream) {
    TK_CHECK_ARG(nx >= 0 && nw >= 0 && out != nullptr, "amax_pair: bad arguments");
    TK_CUDA_TRY(cudaMemsetAsync(out, 0, 2 * sizeof(float), stream));
    const int dev = current_device();
    const int64_t chunk_goal = std::max<int64_t>(static_cast<int64_t>(kAmaxThreads) * 64,
                                                 ceil_div(nx + nw, amax_wave_blocks(dtype, dev) - 2));
    AmaxDesc ad[2] = {};
    int64_t blocks[2] = {0, 0};
    const void* src[2] = {x, w};
    const int64_t len[2] = {nx, nw};
    for (int i = 0; i < 2; ++i) {
        if (len[i] == 0) continue;
        TK_CHECK_ARG(src[i] != nullptr, "amax_pair: NULL operand");
        AmaxDesc& d = ad[i];
        d.x = src[i];
        d.out = reinterpret_cast<unsigned*>(out + i);
        d.nslices = 1;
        d.slice_stride = 0;
        d.slice_len = len[i];
        const int64_t chunks = std::max<int64_t>(1, ceil_div(len[i], chunk_goal));
        d.chunk = (ceil_div(len[i], chunks) + 7) / 8 * 8;
        d.chunks = ceil_div(len[i], d.chunk);
        d.vec = reinterpret_cast<uintptr_t>(src[i]) % 16 == 0;
        blocks[i] = d.chunks;
    }
    const int64_t total = blocks[0] + blocks[1];
    if (total == 0) return TK_OK;
    TK_CHECK_ARG(total < (1LL << 31), "amax_pair: too many blocks");
    const AmaxDesc& first = blocks[0] ? ad[0] : ad[1];
    const AmaxDesc& second = blocks[0] ? ad[1] : ad[0];
    const int64_t b0 = blocks[0] ? blocks[0] : blocks[1];
    if (dtype == TK_DTYPE_F16)
        amax_multi_kernel<__half><<<static_cast<unsigned>(total), kAmaxThreads, 0, stream>>>(first, second, b0);
    else
        amax_multi_kernel<float><<<static_cast<unsigned>(total), kAmaxThreads, 0, stream>>>(first, second, b0);
    return launch_status("amax");
}

// One launch of quant_vec_kernel over up to two row-contiguous operands.
int launch_quant_vec(tk_dtype_t dt, const QVecDesc* vd, int nvec, cudaStream_t stream) {
    auto warp_items = [](const QVecDesc& d) {
        return d.items / d.groups * ceil_div(d.groups, kSegGroups);  // rows x segments
    };
    const int64_t items0 = warp_items(vd[0]);
    const int64_t items1 = nvec > 1 ? warp_items(vd[1]) : 0;
    const int64_t blocks = ceil_div(items0 + items1, 8);
    TK_CHECK_ARG(blocks < (1LL << 31), "quantise: too many rows");
    const QVecDesc second = nvec > 1 ? vd[1] : vd[0];
    const int64_t total = items0 + items1;
    const dim3 grid(static_cast<unsigned>(blocks)), block(32, 8);  // 8 warps, one item (row segment) each
    if (dt == TK_DTYPE_F16)
        TK_CUDA_TRY(launch_pdl(quant_vec_kernel<__half>, grid, block, 0, stream, vd[0], second, items0, total));
    else
        TK_CUDA_TRY(launch_pdl(quant_vec_kernel<float>, grid, block, 0, stream, vd[0], second, items0, total));
    return launch_status("quantise");
}

bool quant_vec_ok(tk_dtype_t dt, const QuantOperand& o);

int quantize_limbs_launch(tk_dtype_t dtype, const void* x, int64_t batch, int64_t rows,
                          int64_t cols, int64_t sb, int64_t sr, int64_t sc, const float* amax,
                          int64_t amax_stride, int8_t* limbs, cudaStream_t stream) {
    TK_CHECK_ARG(batch >= 0 && rows >= 0 && cols >= 0, "tk_quantize_limbs: negative size");
    if (batch == 0 || rows == 0) return TK_OK;
    TK_CHECK_ARG(batch <= 65535, "tk_quantize_limbs: at most 65535 slices per call");
    TK_CHECK_ARG(limbs != nullptr && amax != nullptr, "tk_quantize_limbs: NULL pointer");
    TK_CHECK_ARG(reinterpret_cast<uintptr_t>(limbs) % 16 == 0,
                 "tk_quantize_limbs: limbs must be 16-byte aligned");
    const int64_t ld = static_cast<int64_t>(round_up(static_cast<size_t>(cols), 16));
    if (ld == 0) return TK_OK;
    TK_CHECK_ARG(cols == 0 || x != nullptr, "tk_quantize_limbs: x is NULL");
    {
        // row-contiguous views: the vectorised kernel (16-byte loads, one
        // warp per 1024-column row segment)
        const QuantOperand o = {x, batch, rows, cols, sb, sr, sc, amax_stride != 0, amax, nullptr, limbs};
        if (cols > 0 && quant_vec_ok(dtype, o)) {
            QVecDesc d = {};
            d.x = x;
            d.rows = rows;
            d.cols = cols;
            d.ld = ld;
            d.sb = sb;
            d.sr = sr;
            d.groups = ld / 8;
            d.items = batch * rows * d.groups;
            d.amax = amax;
            d.amax_stride = amax_stride;
            d.limbs = limbs;
            return launch_quant_vec(dtype, &d, 1, stream);
        }
    }
    dim3 grid(static_cast<unsigned>(ceil_div(ld, kQT)), static_cast<unsigned>(ceil_div(rows, kQT)),
              static_cast<unsigned>(batch));
    TK_CHECK_ARG(grid.y <= 65535, "tk_quantize_limbs: too many rows (%lld)", (long long)rows);
    const bool col_contig = (sc == 1) || (sr != 1);
    if (dtype == TK_DTYPE_F16) {
        auto* xp = static_cast<const __half*>(x);
        if (col_contig)
            quant_limbs_kernel<__half, true><<<grid, kQThreads, 0, stream>>>(
                xp, rows, cols, ld, sb, sr, sc, amax, amax_stride, limbs);
        else
            quant_limbs_kernel<__half, false><<<grid, kQThreads, 0, stream>>>(
                xp, rows, cols, ld, sb, sr, sc, amax, amax_stride, limbs);
    } else {
        auto* xp = static_cast<const float*>(x);
        if (col_contig)
            quant_limbs_kernel<float, true><<<grid, kQThreads, 0, stream>>>(
                xp, rows, cols, ld, sb, sr, sc, amax, amax_stride, limbs);
        else
            quant_limbs_kernel<float, false><<<grid, kQThreads, 0, stream>>>(
                xp, rows, cols, ld, sb, sr, sc, amax, amax_stride, limbs);
    }
    return launch_status("quantize_limbs");
}


bool quant_vec_ok(tk_dtype_t dt, const QuantOperand& o) {
    const int64_t es = static_cast<int64_t>(dtype_size(dt));
    if (o.sc != 1 && o.cols > 1) return false;
    if (reinterpret_cast<uintptr_t>(o.x) % 16 != 0) return false;
    if ((o.sr * es) % 16 != 0 && o.rows > 1) return false;
    if ((o.sb * es) % 16 != 0 && o.batch > 1) return false;
    return true;
}

// Quantise up to two operands for one GEMM: one launch computes every amax
// that is not given, one launch quantises every row-contiguous operand, and
// any transposed operand goes through the shared-memory tile kernel.  The
// caller has zeroed the amax slots.
int quantise_operands(tk_dtype_t dt, const QuantOperand* ops, int nops, cudaStream_t stream) {
    TK_CHECK_ARG(nops >= 1 && nops <= 2, "quantise_operands: 1 or 2 operands");
    const int dev = current_device();
    AmaxDesc ad[2] = {};
    int64_t ablocks[2] = {0, 0};
    // one chunk size for every operand, all blocks in one resident wave, so
    // the larger operand gets proportionally more blocks (each operand's last
    // chunk may be short: two blocks of slack)
    int64_t amax_elems = 0;
    for (int i = 0; i < nops; ++i)
        if (ops[i].given_amax == nullptr) amax_elems += ops[i].batch * ops[i].rows * ops[i].cols;
    const int64_t chunk_goal = std::max<int64_t>(static_cast<int64_t>(kAmaxThreads) * 64,
                                                 ceil_div(amax_elems, amax_wave_blocks(dt, dev) - 2));
    for (int i = 0; i < nops; ++i) {
        const QuantOperand& o = ops[i];
        if (o.given_amax != nullptr || o.batch * o.rows * o.cols == 0) continue;
        AmaxDesc& d = ad[i];
        d.x = o.x;
        d.out = reinterpret_cast<unsigned*>(o.amax_out);
        if (o.per_slice) {
            d.nslices = o.batch;
            d.slice_stride = o.sb;
            d.slice_len = o.rows * o.cols;
        } else {
            d.nslices = 1;
            d.slice_stride = 0;
            d.slice_len = o.batch * o.rows * o.cols;
        }
        const int64_t chunks = std::max<int64_t>(1, ceil_div(d.slice_len, chunk_goal));
        d.chunk = (ceil_div(d.slice_len, chunks) + 7) / 8 * 8;
        d.chunks = ceil_div(d.slice_len, d.chunk);
        const size_t es = dtype_size(dt);
        d.vec = reinterpret_cast<uintptr_t>(o.x) % 16 == 0 &&
                ((d.slice_stride * static_cast<int64_t>(es)) % 16 == 0);
        ablocks[i] = d.nslices * d.chunks;
    }
    if (ablocks[0] + ablocks[1] > 0) {
        const AmaxDesc& first = ablocks[0] ? ad[0] : ad[1];
        const AmaxDesc& second = ablocks[0] ? ad[1] : ad[0];
        const int64_t b0 = ablocks[0] ? ablocks[0] : ablocks[1];
        const int64_t total = ablocks[0] + ablocks[1];
        TK_CHECK_ARG(total < (1LL << 31), "quantise: too many amax blocks");
        if (dt == TK_DTYPE_F16)
            amax_multi_kernel<__half><<<static_cast<unsigned>(total), kAmaxThreads, 0, stream>>>(
                first, second, b0);
        else
            amax_multi_kernel<float><<<static_cast<unsigned>(total), kAmaxThreads, 0, stream>>>(
                first, second, b0);
        int rc = launch_status("amax");
        if (rc) return rc;
    }
    QVecDesc vd[2] = {};
    int nvec = 0;
    for (int i = 0; i < nops; ++i) {
        const QuantOperand& o = ops[i];
        const float* amax = o.given_amax ? o.given_amax : o.amax_out;
        if (o.batch * o.rows == 0) continue;
        const int64_t ld = static_cast<int64_t>(round_up(static_cast<size_t>(o.cols), 16));
        if (quant_vec_ok(dt, o)) {
            QVecDesc& d = vd[nvec++];
            d.x = o.x;
            d.rows = o.rows;
            d.cols = o.cols;
            d.ld = ld;
            d.sb = o.sb;
            d.sr = o.sr;
            d.groups = ld / 8;
            d.items = o.batch * o.rows * d.groups;
            d.amax = amax;
            d.amax_stride = o.per_slice ? 1 : 0;
            d.limbs = o.limbs;
        } else {
            int rc = quantize_limbs_launch(dt, o.x, o.batch, o.rows, o.cols, o.sb, o.sr, o.sc, amax,
                                           o.per_slice ? 1 : 0, o.limbs, stream);
            if (rc) return rc;
        }
    }
    if (nvec > 0) return launch_quant_vec(dt, vd, nvec, stream);
    return TK_OK;
}

}  // namespace tk

extern "C" {

int tk_amax(tk_dtype_t dtype, const void* x, int64_t nslices, int64_t slice_stride,
            int64_t slice_len, float* amax_out, void* stream) {
    return tk::amax_launch(dtype, x, nslices, slice_stride, slice_len, amax_out,
                           static_cast<cudaStream_t>(stream));
}

int tk_quantize_limbs(tk_dtype_t dtype, const void* x, int64_t batch, int64_t rows,
                      int64_t cols, int64_t sb, int64_t sr, int64_t sc, const float* amax,
                      int64_t amax_stride, int8_t* limbs, void* stream) {
    return tk::quantize_limbs_launch(dtype, x, batch, rows, cols, sb, sr, sc, amax, amax_stride,
                                     limbs, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
