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
#include "tk_internal.h"
#include "tk_numerics.cuh"

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

// |x| of an fp16 pair as two 16-bit magnitudes; the unsigned order of the
// magnitudes is the float order, with every NaN above +Inf.
__global__ void amax_f16_kernel(const __half* __restrict__ x, int64_t slice_stride,
                                int64_t slice_len, int64_t chunk, bool vec,
                                unsigned* __restrict__ out_bits) {
    const int64_t s = blockIdx.y;
    const unsigned short* base = reinterpret_cast<const unsigned short*>(x + s * slice_stride);
    const int64_t start = static_cast<int64_t>(blockIdx.x) * chunk;
    const int64_t end = min(start + chunk, slice_len);
    unsigned m2 = 0;  // two packed 16-bit maxima
    int64_t i = start;
    if (vec) {
        const int64_t nv = (end - start) / 8;
        const uint4* pv = reinterpret_cast<const uint4*>(base + start);
        for (int64_t j = threadIdx.x; j < nv; j += blockDim.x) {
            uint4 w = __ldg(pv + j);
            m2 = __vmaxu2(m2, w.x & 0x7FFF7FFFu);
            m2 = __vmaxu2(m2, w.y & 0x7FFF7FFFu);
            m2 = __vmaxu2(m2, w.z & 0x7FFF7FFFu);
            m2 = __vmaxu2(m2, w.w & 0x7FFF7FFFu);
        }
        i = start + nv * 8;
    }
    for (int64_t j = i + threadIdx.x; j < end; j += blockDim.x) {
        m2 = __vmaxu2(m2, static_cast<unsigned>(base[j] & 0x7FFFu));
    }
    unsigned h = max(m2 & 0xFFFFu, m2 >> 16);
    h = block_max_u32(h);
    if (threadIdx.x == 0 && h != 0u) {
        float f = __half2float(__ushort_as_half(static_cast<unsigned short>(h)));
        unsigned bits = __float_as_uint(f) & 0x7FFFFFFFu;
        if ((h & 0x7C00u) == 0x7C00u && (h & 0x3FFu) != 0u) bits = 0x7FC00000u;  // NaN
        atomicMax(out_bits + s, bits);
    }
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

}  // namespace

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
    if (dtype == TK_DTYPE_F16) {
        amax_f16_kernel<<<grid, kAmaxThreads, 0, stream>>>(static_cast<const __half*>(x),
                                                           slice_stride, slice_len, chunk, vec, ob);
    } else {
        amax_f32_kernel<<<grid, kAmaxThreads, 0, stream>>>(static_cast<const float*>(x),
                                                           slice_stride, slice_len, chunk, vec, ob);
    }
    return launch_status("amax");
}

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
