// conv.cu -- int16-quantised conv2d and conv3d (NC[D]HW input, OI[D]HW
// weight, bias, stride, padding, dilation, groups).
//
// Replaces baidu::xpu::api::conv2d<T,T,T,TGEMM> and the bias broadcast_add
// that follows it (csrc/ops.cpp:237-285), and xdnn conv3d + add
// (csrc/ops_nn_extra.cpp:88-121).  Per the reference, the whole input and the
// whole weight are each quantised with one per-tensor scale.  A 2-D
// convolution is handled as the 3-D one with D = KD = 1.
//
// Paths:
//   * 2-D, groups == C == F/mult (depthwise): CUDA-core kernels with exact
//     integer sums of the KHxKW taps.  Multiplier 1, unit stride and
//     dilation: the amax-partials kernel and depthwise_scaled_kernel,
//     which starts loading its planes while the partials form (programmatic
//     dependent launch) and quantises from shared memory, when its grid fits
//     in one wave; else the amax launch and the row kernel; other depthwise
//     shapes use the plane, flat or per-output kernels.
//   * groups == 1, stride 1: implicit GEMM on the tensor cores (conv_tc.cu),
//     no patch matrix in HBM.
//   * otherwise a GEMM per (image, group) on the tensor-core limb kernel:
//     A = the image's input patches [OD*OH*OW, C/g*KD*KH*KW] quantised
//     straight into limb planes (1x1 stride-1 convolutions read NCHW
//     directly as a transposed operand; larger kernels gather patches in the
//     same pass), B = the group's weights [F/g, C/g*KD*KH*KW] (shared by all
//     images), and the epilogue writes the pixels x channels tile into NCHW.
#include "tk_internal.h"
#include "tk_numerics.cuh"
#include "tk_ptx.cuh"

namespace tk {

int amax_launch(tk_dtype_t dtype, const void* x, int64_t nslices, int64_t slice_stride,
                int64_t slice_len, float* amax_out, cudaStream_t stream);
int amax_pair_launch(tk_dtype_t dtype, const void* x, int64_t nx, const void* w, int64_t nw, float* out,
                     cudaStream_t stream);
int quantize_limbs_launch(tk_dtype_t dtype, const void* x, int64_t batch, int64_t rows,
                          int64_t cols, int64_t sb, int64_t sr, int64_t sc, const float* amax,
                          int64_t amax_stride, int8_t* limbs, cudaStream_t stream);
int qgemm_limbs_ex(const tk_qgemm_desc_t& d, const int8_t* la, const int8_t* lb,
                   const float* amax_a, const float* amax_b, int b_mod, int64_t out_sn,
                   int64_t bias_mod, cudaStream_t stream);
int qgemm_limbs_acc64(const tk_qgemm_desc_t& d, const int8_t* la, const int8_t* lb,
                      unsigned long long* acc64, int acc_mod, cudaStream_t stream);
int qgemm_acc64_finish(const tk_qgemm_desc_t& d, const long long* acc64, int64_t slices,
                       const float* amax_a, const float* amax_b, int64_t out_sn, cudaStream_t stream);
size_t conv_tc_workspace(int64_t N, int64_t C, int64_t D, int64_t H, int64_t W, int64_t F, int64_t KD,
                         int64_t KH, int64_t KW, int64_t ph, int64_t pw);
int conv_tc(tk_dtype_t dtype, const void* x, const void* w, const void* bias, void* out, int64_t N,
            int64_t C, int64_t D, int64_t H, int64_t W, int64_t F, int64_t KD, int64_t KH, int64_t KW,
            int64_t pd, int64_t ph, int64_t pw, int64_t dd, int64_t dh, int64_t dw, int64_t OD, int64_t OH,
            int64_t OW, const float* amax_x, const float* amax_w, uint8_t* ws, cudaStream_t stream,
            bool x_scale_own = false);

namespace {

struct ConvGeom {
    int64_t N, C, H, W, F, KH, KW, sh, sw, ph, pw, dh, dw, groups, OH, OW;
    int64_t D, KD, sd, pd, dd, OD;  // depth (1, 1, 1, 0, 1, 1 for 2-D)
};

template <typename T>
__device__ __forceinline__ float ldx(const T* p, int64_t i);
template <> __device__ __forceinline__ float ldx<__half>(const __half* p, int64_t i) { return __half2float(p[i]); }
template <> __device__ __forceinline__ float ldx<float>(const float* p, int64_t i) { return p[i]; }

// Patch gather + quantisation.  Slice b = n*groups + g, row
// p = (od*OH + oh)*OW + ow, column k = ((c*KD + t)*KH + r)*KW + s over the
// group's channels; 4 columns per thread so that both limb planes are written
// with 32-bit stores.
template <typename T>
__global__ void im2col_quant_kernel(const T* __restrict__ x, ConvGeom g, int64_t K, int64_t ld,
                                    const float* __restrict__ amax, int8_t* __restrict__ limbs) {
    const int64_t P = g.OD * g.OH * g.OW;
    const int64_t k4n = ld / 4;
    const int64_t total = g.N * g.groups * P * k4n;
    const float inv = quant_inv(amax[0]);
    const int64_t cg = g.C / g.groups;
    const int64_t khw = g.KH * g.KW;
    const int64_t kdhw = g.KD * khw;
    for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t k4 = idx % k4n;
        const int64_t rest = idx / k4n;
        const int64_t p = rest % P;
        const int64_t b = rest / P;
        const int64_t n = b / g.groups, grp = b % g.groups;
        const int64_t ow = p % g.OW, oh = (p / g.OW) % g.OH, od = p / (g.OW * g.OH);
        unsigned hi = 0, lo = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t k = k4 * 4 + j;
            int q = 0;
            if (k < K) {
                const int64_t c = k / kdhw;
                const int64_t trs = k - c * kdhw;
                const int64_t t = trs / khw, rs = trs - t * khw;
                const int64_t r = rs / g.KW, s = rs - r * g.KW;
                const int64_t id = od * g.sd - g.pd + t * g.dd;
                const int64_t ih = oh * g.sh - g.ph + r * g.dh;
                const int64_t iw = ow * g.sw - g.pw + s * g.dw;
                if (id >= 0 && id < g.D && ih >= 0 && ih < g.H && iw >= 0 && iw < g.W) {
                    const int64_t ci = grp * cg + c;
                    q = quant_one(ldx<T>(x, (((n * g.C + ci) * g.D + id) * g.H + ih) * g.W + iw), inv);
                }
            }
            hi |= (static_cast<unsigned>(q >> 8) & 0xFFu) << (8 * j);
            lo |= (static_cast<unsigned>(q) & 0xFFu) << (8 * j);
        }
        const int64_t plane = P * ld;
        int8_t* base = limbs + (b * 2) * plane + p * ld + k4 * 4;
        *reinterpret_cast<unsigned*>(base) = hi;
        *reinterpret_cast<unsigned*>(base + plane) = lo;
    }
}

// Transposed patch gather + quantisation for the weight gradient.  Slice
// b = (n - n0)*groups + g of images [n0, n0 + nimg), row
// m = ((c*KD + t)*KH + r)*KW + s over the group's channels, column
// p = (od*OH + oh)*OW + ow (the reduction axis): x at the input position
// that output pixel p reads through tap (t, r, s), zero in the padding.
// 8 columns per thread, written as one 8-byte word per limb plane; columns
// [P, ld) are zero.
template <typename T>
__global__ void im2col_t_quant_kernel(const T* __restrict__ x, ConvGeom g, int64_t n0, int64_t nimg,
                                      int64_t M, int64_t ld, const float* __restrict__ amax,
                                      int8_t* __restrict__ limbs) {
    const int64_t P = g.OD * g.OH * g.OW;
    const int64_t p8n = ld / 8;
    const int64_t total = nimg * g.groups * M * p8n;
    const float inv = quant_inv(amax[0]);
    const int64_t cg = g.C / g.groups;
    const int64_t khw = g.KH * g.KW;
    const int64_t kdhw = g.KD * khw;
    for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t p8 = idx % p8n;
        const int64_t rest = idx / p8n;
        const int64_t m = rest % M;
        const int64_t b = rest / M;
        const int64_t n = n0 + b / g.groups, grp = b % g.groups;
        const int64_t c = m / kdhw;
        const int64_t trs = m - c * kdhw;
        const int64_t t = trs / khw, rs = trs - t * khw;
        const int64_t r = rs / g.KW, sx = rs - r * g.KW;
        const T* xc = x + (n * g.C + grp * cg + c) * g.D * g.H * g.W;
        unsigned hi[2] = {0u, 0u}, lo[2] = {0u, 0u};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int64_t p = p8 * 8 + j;
            int q = 0;
            if (p < P) {
                const int64_t ow = p % g.OW, oh = (p / g.OW) % g.OH, od = p / (g.OW * g.OH);
                const int64_t id = od * g.sd - g.pd + t * g.dd;
                const int64_t ih = oh * g.sh - g.ph + r * g.dh;
                const int64_t iw = ow * g.sw - g.pw + sx * g.dw;
                if (id >= 0 && id < g.D && ih >= 0 && ih < g.H && iw >= 0 && iw < g.W)
                    q = quant_one(ldx<T>(xc, (id * g.H + ih) * g.W + iw), inv);
            }
            hi[j >> 2] |= (static_cast<unsigned>(q >> 8) & 0xFFu) << (8 * (j & 3));
            lo[j >> 2] |= (static_cast<unsigned>(q) & 0xFFu) << (8 * (j & 3));
        }
        const int64_t plane = M * ld;
        int8_t* base = limbs + (b * 2) * plane + m * ld + p8 * 8;
        *reinterpret_cast<uint2*>(base) = make_uint2(hi[0], hi[1]);
        *reinterpret_cast<uint2*>(base + plane) = make_uint2(lo[0], lo[1]);
    }
}

// Depthwise (one input channel per group): output channel f reads input
// channel f / mult.  Exact int64 accumulation, then the shared epilogue
// (dequantise + round, then bias added after rounding).
template <typename T, int DT>
__global__ void depthwise_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                 const T* __restrict__ bias, T* __restrict__ out, ConvGeom g,
                                 const float* __restrict__ amax_x, const float* __restrict__ amax_w) {
    const int64_t total = g.N * g.F * g.OH * g.OW;
    const float ax = amax_x[0], aw = amax_w[0];
    const float invx = quant_inv(ax), invw = quant_inv(aw);
    const double s = dequant_scale(ax, aw);
    const int64_t mult = g.F / g.C;
    for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t ow = idx % g.OW;
        int64_t t = idx / g.OW;
        const int64_t oh = t % g.OH;
        t /= g.OH;
        const int64_t f = t % g.F;
        const int64_t n = t / g.F;
        const int64_t c = f / mult;
        const T* xc = x + (n * g.C + c) * g.H * g.W;
        const T* wf = w + f * g.KH * g.KW;
        long long acc = 0;
        for (int64_t r = 0; r < g.KH; ++r) {
            const int64_t ih = oh * g.sh - g.ph + r * g.dh;
            if (ih < 0 || ih >= g.H) continue;
            for (int64_t sx = 0; sx < g.KW; ++sx) {
                const int64_t iw = ow * g.sw - g.pw + sx * g.dw;
                if (iw < 0 || iw >= g.W) continue;
                acc += static_cast<long long>(quant_one(ldx<T>(xc, ih * g.W + iw), invx)) *
                       static_cast<long long>(quant_one(ldx<T>(wf, r * g.KW + sx), invw));
            }
        }
        float v = round_t_from_double(__dmul_rn(static_cast<double>(acc), s), DT);
        if (bias != nullptr) v = round_t(__fadd_rn(v, ldx<T>(bias, f)), DT);
        store_t(out, DT, idx, v);
    }
}

// Depthwise on small planes: one warp per output plane (n, f).  The warp
// quantises its input plane (channel f / mult) into shared memory with
// coalesced loads, then each lane produces outputs along the row with exact
// int64 accumulation of the taps; stores are coalesced along ow.
constexpr int kDwPlaneMax = 1024;  // input elements per plane held in shared memory
constexpr int kDwWarps = 8;

template <typename T, int DT>
__global__ void __launch_bounds__(32 * kDwWarps)
depthwise_plane_kernel(const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ bias,
                       T* __restrict__ out, ConvGeom g, const float* __restrict__ amax_x,
                       const float* __restrict__ amax_w) {
    __shared__ int16_t plane[kDwWarps][kDwPlaneMax];
    __shared__ int wq[kDwWarps][64];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t pl = static_cast<int64_t>(blockIdx.x) * kDwWarps + warp;  // n * F + f
    if (pl >= g.N * g.F) return;
    const int64_t f = pl % g.F, n = pl / g.F;
    const int64_t c = f / (g.F / g.C);
    const float ax = __ldg(amax_x), aw = __ldg(amax_w);
    const float invx = quant_inv(ax), invw = quant_inv(aw);
    const double s = dequant_scale(ax, aw);
    const int HW = static_cast<int>(g.H * g.W);
    const T* xp = x + (n * g.C + c) * HW;
    for (int i = lane; i < HW; i += 32) plane[warp][i] = static_cast<int16_t>(quant_one(ldx<T>(xp, i), invx));
    const int taps = static_cast<int>(g.KH * g.KW);
    for (int i = lane; i < taps; i += 32) wq[warp][i] = quant_one(ldx<T>(w, f * taps + i), invw);
    __syncwarp();
    float bv = 0.0f;
    if (bias != nullptr) bv = ldx<T>(bias, f);
    const int OHW = static_cast<int>(g.OH * g.OW);
    T* op = out + pl * OHW;
    for (int o = lane; o < OHW; o += 32) {
        const int oh = o / static_cast<int>(g.OW), ow = o - oh * static_cast<int>(g.OW);
        long long acc = 0;
        for (int r = 0; r < g.KH; ++r) {
            const int ih = oh * static_cast<int>(g.sh) - static_cast<int>(g.ph) + r * static_cast<int>(g.dh);
            if (ih < 0 || ih >= g.H) continue;
            for (int q = 0; q < g.KW; ++q) {
                const int iw = ow * static_cast<int>(g.sw) - static_cast<int>(g.pw) + q * static_cast<int>(g.dw);
                if (iw < 0 || iw >= g.W) continue;
                acc += static_cast<long long>(plane[warp][ih * g.W + iw]) * wq[warp][r * g.KW + q];
            }
        }
        float v = round_t_from_double(__dmul_rn(static_cast<double>(acc), s), DT);
        if (bias != nullptr) v = round_t(__fadd_rn(v, bv), DT);
        store_t(op, DT, o, v);
    }
}

// Depthwise with one output channel per input channel (multiplier 1) on
// small planes: a block takes a run of whole planes, which is one contiguous
// span of the NCHW input and of the output.  It quantises the span into
// shared memory with coalesced loads, then threads produce consecutive
// outputs (coalesced stores), each with exact int64 accumulation of the taps.
constexpr int kDwFlatElems = 4096;  // input elements per block in shared memory

template <typename T, int DT>
__global__ void __launch_bounds__(256)
depthwise_flat_kernel(const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ bias,
                      T* __restrict__ out, ConvGeom g, int planes_per_block,
                      const float* __restrict__ amax_x, const float* __restrict__ amax_w) {
    __shared__ int16_t xs[kDwFlatElems];
    __shared__ int wsq[kDwFlatElems / 4];
    const int HW = static_cast<int>(g.H * g.W), OHW = static_cast<int>(g.OH * g.OW);
    const int taps = static_cast<int>(g.KH * g.KW);
    const int64_t planes = g.N * g.C;
    const int64_t pl0 = static_cast<int64_t>(blockIdx.x) * planes_per_block;
    const int np = static_cast<int>(min(static_cast<int64_t>(planes_per_block), planes - pl0));
    const float ax = __ldg(amax_x), aw = __ldg(amax_w);
    const float invx = quant_inv(ax), invw = quant_inv(aw);
    const double s = dequant_scale(ax, aw);
    const T* xb = x + pl0 * HW;
    for (int i = threadIdx.x; i < np * HW; i += blockDim.x)
        xs[i] = static_cast<int16_t>(quant_one(ldx<T>(xb, i), invx));
    for (int i = threadIdx.x; i < np * taps; i += blockDim.x) {
        const int pp = i / taps, tp = i - (i / taps) * taps;
        const int64_t c = (pl0 + pp) % g.C;
        wsq[i] = quant_one(ldx<T>(w, c * taps + tp), invw);
    }
    __syncthreads();
    T* ob = out + pl0 * OHW;
    const int OW = static_cast<int>(g.OW);
    for (int o = threadIdx.x; o < np * OHW; o += blockDim.x) {
        const int pp = o / OHW, rem = o - (o / OHW) * OHW;
        const int oh = rem / OW, ow = rem - (rem / OW) * OW;
        const int16_t* xp = xs + pp * HW;
        const int* wp = wsq + pp * taps;
        long long acc = 0;
        for (int r = 0; r < g.KH; ++r) {
            const int ih = oh * static_cast<int>(g.sh) - static_cast<int>(g.ph) + r * static_cast<int>(g.dh);
            if (ih < 0 || ih >= g.H) continue;
            for (int q = 0; q < g.KW; ++q) {
                const int iw = ow * static_cast<int>(g.sw) - static_cast<int>(g.pw) + q * static_cast<int>(g.dw);
                if (iw < 0 || iw >= g.W) continue;
                acc += static_cast<long long>(xp[ih * g.W + iw]) * wp[r * g.KW + q];
            }
        }
        float v = round_t_from_double(__dmul_rn(static_cast<double>(acc), s), DT);
        if (bias != nullptr) v = round_t(__fadd_rn(v, ldx<T>(bias, (pl0 + pp) % g.C)), DT);
        store_t(ob, DT, o, v);
    }
}

// Depthwise with multiplier 1, unit stride and unit dilation (the depthwise
// layers of the benchmark networks): a block takes a run of whole planes --
// one contiguous span of the NCHW input and of the output -- quantises it
// into zero-padded planes in shared memory (so the tap loops need no bounds
// checks), and each thread produces a whole output row: kDwRowOut outputs at
// a time from a sliding window of KW + kDwRowOut - 1 inputs per filter row,
// int32 products (|q| <= 32767, so each product is below 2^30) summed exactly
// in int64, then the shared epilogue.  HBM-bound: every input and output
// element crosses HBM once.
constexpr int kDwRowThreads = 256;
constexpr int kDwRowSpan = 8192;  // padded input elements per block
constexpr int kDwRowTaps = 1024;  // weight taps per block (planes x KH x KW)
constexpr int kDwRowOut = 8;      // outputs per window along a row

template <typename T, int DT, int KW>
__global__ void __launch_bounds__(kDwRowThreads)
depthwise_rows_kernel(const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ bias,
                      T* __restrict__ out, ConvGeom g, int ppb, const float* __restrict__ amax_x,
                      const float* __restrict__ amax_w) {
    // slack after the last plane: the last window of a row reads up to
    // kDwRowOut + KW - 2 elements past the row's last output column
    __shared__ int16_t xs[kDwRowSpan + kDwRowOut + KW];
    __shared__ int wsq[kDwRowTaps];
    const int H = static_cast<int>(g.H), W = static_cast<int>(g.W);
    const int ph = static_cast<int>(g.ph), pw = static_cast<int>(g.pw);
    const int Hp = H + 2 * ph, Wp = W + 2 * pw;
    const int KH = static_cast<int>(g.KH);
    const int OH = static_cast<int>(g.OH), OW = static_cast<int>(g.OW);
    const int HW = H * W, PHW = Hp * Wp, taps = KH * KW;
    const int64_t planes = g.N * g.C;
    const int64_t pl0 = static_cast<int64_t>(blockIdx.x) * ppb;
    const int np = static_cast<int>(min(static_cast<int64_t>(ppb), planes - pl0));
    const float ax = __ldg(amax_x), aw = __ldg(amax_w);
    const float invx = quant_inv(ax), invw = quant_inv(aw);
    const double s = dequant_scale(ax, aw);
    const int span = np * PHW;
    for (int i = threadIdx.x; i < span + kDwRowOut + KW; i += blockDim.x) xs[i] = 0;
    __syncthreads();
    const int C = static_cast<int>(g.C);
    const int c0 = static_cast<int>(pl0 % g.C);  // channel of the block's first plane
    // the span's elements [0, n): a scalar head up to the first 16-byte
    // boundary, 16-byte vectors, a scalar tail (all loads in flight at once)
    const T* xb = x + pl0 * HW;
    const int n = np * HW;
    constexpr int VEC = 16 / sizeof(T);
    auto put = [&](int i, float v) {
        const int pp = i / HW, r = i - pp * HW;
        const int ih = r / W, iw = r - ih * W;
        xs[pp * PHW + (ih + ph) * Wp + iw + pw] = static_cast<int16_t>(quant_one(v, invx));
    };
    const bool aligned = reinterpret_cast<uintptr_t>(x) % 16 == 0;
    const int head = aligned ? min(n, static_cast<int>((VEC - (pl0 * HW) % VEC) % VEC)) : n;
    const int nv = (n - head) / VEC;
    for (int i = threadIdx.x; i < head; i += blockDim.x) put(i, ldx<T>(xb, i));
    for (int v = threadIdx.x; v < nv; v += blockDim.x) {
        const int i0 = head + v * VEC;
        float f[VEC];
        if constexpr (sizeof(T) == 2) {
            const uint4 u = __ldg(reinterpret_cast<const uint4*>(xb + i0));
            const __half2* h2 = reinterpret_cast<const __half2*>(&u);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 t = __half22float2(h2[e]);
                f[2 * e] = t.x;
                f[2 * e + 1] = t.y;
            }
        } else {
            const float4 t = __ldg(reinterpret_cast<const float4*>(xb + i0));
            f[0] = t.x; f[1] = t.y; f[2] = t.z; f[3] = t.w;
        }
#pragma unroll
        for (int e = 0; e < VEC; ++e) put(i0 + e, f[e]);
    }
    for (int i = head + nv * VEC + threadIdx.x; i < n; i += blockDim.x) put(i, ldx<T>(xb, i));
    for (int i = threadIdx.x; i < np * taps; i += blockDim.x) {
        const int pp = i / taps, t = i - pp * taps;
        int c = c0 + pp;
        while (c >= C) c -= C;
        wsq[i] = quant_one(ldx<T>(w, static_cast<int64_t>(c) * taps + t), invw);
    }
    __syncthreads();
    T* ob = out + pl0 * OH * OW;
    for (int row = threadIdx.x; row < np * OH; row += blockDim.x) {
        const int pp = row / OH, oh = row - pp * OH;
        const int16_t* xr = xs + pp * PHW + oh * Wp;
        const int* wp = wsq + pp * taps;
        int c = c0 + pp;
        while (c >= C) c -= C;
        const float bv = bias != nullptr ? ldx<T>(bias, c) : 0.0f;
        T* orow = ob + static_cast<int64_t>(row) * OW;
        for (int ow0 = 0; ow0 < OW; ow0 += kDwRowOut) {
            long long acc[kDwRowOut];
#pragma unroll
            for (int j = 0; j < kDwRowOut; ++j) acc[j] = 0;
            for (int r = 0; r < KH; ++r) {
                int xv[kDwRowOut + KW - 1];
#pragma unroll
                for (int j = 0; j < kDwRowOut + KW - 1; ++j) xv[j] = xr[r * Wp + ow0 + j];
#pragma unroll
                for (int k = 0; k < KW; ++k) {
                    const int wv = wp[r * KW + k];
#pragma unroll
                    for (int j = 0; j < kDwRowOut; ++j) acc[j] += xv[j + k] * wv;
                }
            }
#pragma unroll
            for (int j = 0; j < kDwRowOut; ++j) {
                if (ow0 + j < OW) {
                    float v = round_t_from_double(__dmul_rn(static_cast<double>(acc[j]), s), DT);
                    if (bias != nullptr) v = round_t(__fadd_rn(v, bv), DT);
                    store_t(orow, DT, ow0 + j, v);
                }
            }
        }
    }
}

// The same depthwise convolution as two launches that overlap through
// programmatic dependent launch.  depthwise_amax_kernel folds the fp32
// magnitude bits (NaN above everything, as the amax kernels) of one chunk of
// the input and one chunk of the filters per block into its own partial
// word -- plain stores, so no memset is needed -- and first of all lets the
// dependent launch start.  depthwise_scaled_kernel, launched with
// programmatic stream serialisation, loads its block's planes and filters
// into shared memory while the partials are still being formed, waits
// (griddepcontrol.wait: the first grid has completed and its stores are
// visible) and folds the partials; then it quantises from shared memory,
// convolves and stores the block's contiguous span of the output with
// 16-byte vectors.  No grid barrier and no co-residency requirement.
constexpr int kDwMaxThreads = 512;
constexpr int kDwAmaxThreads = 256;
constexpr int kDwAmaxMaxBlocks = 512;  // partial words per operand in the workspace

struct DwMagic {
    uint32_t hw, w, taps, ohw, ow, h, oh;  // floor(2^32 / d) + 1 for i / d with i, d < 2^16
};

__device__ __forceinline__ int round_up_dev(int v, int a) { return (v + a - 1) / a * a; }

__device__ __forceinline__ int div_magic(int i, uint32_t m) {
    return static_cast<int>(__umulhi(static_cast<uint32_t>(i), m));
}

template <typename T>
__device__ __forceinline__ unsigned mag_bits(T v);
template <>
__device__ __forceinline__ unsigned mag_bits<__half>(__half v) {
    const unsigned h = __half_as_ushort(v) & 0x7FFFu;
    if ((h & 0x7C00u) == 0x7C00u && (h & 0x3FFu) != 0u) return 0x7FC00000u;  // NaN, canonical
    return __float_as_uint(__half2float(__ushort_as_half(static_cast<unsigned short>(h))));
}
template <>
__device__ __forceinline__ unsigned mag_bits<float>(float v) {
    return __float_as_uint(v) & 0x7FFFFFFFu;
}

__device__ __forceinline__ unsigned block_max_bits(unsigned v, unsigned* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    v = 0u;
    for (int k = 0; k < static_cast<int>(blockDim.x >> 5); ++k) v = max(v, red[k]);
    return v;
}

// Magnitude bits (mag_bits) of p[b0, b1): 16-byte loads when `vec` (p
// 16-byte aligned and b0 a multiple of the vector width).
template <typename T>
__device__ __forceinline__ unsigned span_max_bits(const T* __restrict__ p, int64_t b0, int64_t b1, bool vec) {
    constexpr int VEC = 16 / sizeof(T);
    unsigned m = 0u;
    if (vec) {
        const int64_t nv = (b1 - b0) / VEC;
        const uint4* pv = reinterpret_cast<const uint4*>(p + b0);
        for (int64_t j = threadIdx.x; j < nv; j += blockDim.x) {
            const uint4 u = __ldg(pv + j);
            const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
            for (int k = 0; k < VEC; ++k) m = max(m, mag_bits<T>(e[k]));
        }
        b0 += nv * VEC;
    }
    for (int64_t i = b0 + threadIdx.x; i < b1; i += blockDim.x) m = max(m, mag_bits<T>(p[i]));
    return m;
}

// Block b: part[b] = magnitude bits of max |x| over x[b*cx, (b+1)*cx),
// part[gridDim.x + b] the same of w over w[b*cw, (b+1)*cw).
template <typename T>
__global__ void __launch_bounds__(kDwAmaxThreads)
depthwise_amax_kernel(const T* __restrict__ x, int64_t nx, int64_t cx, int vx, const T* __restrict__ w,
                      int64_t nw, int64_t cw, int vw, unsigned* __restrict__ part) {
    __shared__ unsigned red[kDwAmaxThreads / 32];
    // the convolution kernel may be scheduled now: it only loads its inputs
    // until it waits for this grid
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int64_t b = blockIdx.x;
    unsigned mx = span_max_bits<T>(x, min(nx, b * cx), min(nx, (b + 1) * cx), vx != 0);
    unsigned mw = span_max_bits<T>(w, min(nw, b * cw), min(nw, (b + 1) * cw), vw != 0);
    mx = block_max_bits(mx, red);
    __syncthreads();
    mw = block_max_bits(mw, red);
    if (threadIdx.x == 0) {
        part[b] = mx;
        part[gridDim.x + b] = mw;
    }
}

template <typename T, int DT, int KW>
__global__ void __launch_bounds__(kDwMaxThreads)
depthwise_scaled_kernel(const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ bias,
                        T* __restrict__ out, ConvGeom g, int ppb, DwMagic mg, const unsigned* part, int nparts) {
    extern __shared__ __align__(16) uint8_t dsm[];
    const int H = static_cast<int>(g.H), W = static_cast<int>(g.W);
    const int ph = static_cast<int>(g.ph), pw = static_cast<int>(g.pw);
    const int Hp = H + 2 * ph, Wp = W + 2 * pw;
    const int KH = static_cast<int>(g.KH);
    const int OH = static_cast<int>(g.OH), OW = static_cast<int>(g.OW);
    const int HW = H * W, PHW = Hp * Wp, taps = KH * KW;
    const int64_t planes = g.N * g.C;
    const int64_t pl0 = static_cast<int64_t>(blockIdx.x) * ppb;
    const int np = static_cast<int>(min(static_cast<int64_t>(ppb), planes - pl0));
    const int C = static_cast<int>(g.C);
    const int c0 = static_cast<int>(pl0 % g.C);
    // shared memory: raw span (reused for the output span), padded codes,
    // filter values then codes, reduction scratch
    const int raw_elems = ppb * max(HW, OH * OW);
    T* raw = reinterpret_cast<T*>(dsm);
    int16_t* xs = reinterpret_cast<int16_t*>(dsm + round_up_dev(raw_elems * static_cast<int>(sizeof(T)), 16));
    float* wf = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(xs) +
                                         round_up_dev((ppb * PHW + kDwRowOut + KW) * 2, 16));
    int* wsq = reinterpret_cast<int*>(wf);
    unsigned* red = reinterpret_cast<unsigned*>(wf + ppb * taps);

    // ---- phase 1: the block's input span and filters (neither is written
    // by the amax grid, so they load before the wait)
    const T* xb = x + pl0 * HW;
    const int n = np * HW;
    constexpr int VEC = 16 / sizeof(T);
    const bool aligned = reinterpret_cast<uintptr_t>(x) % 16 == 0;
    const int head = aligned ? min(n, static_cast<int>((VEC - (pl0 * HW) % VEC) % VEC)) : n;
    const int nv = (n - head) / VEC;
    for (int i = threadIdx.x; i < head; i += blockDim.x) raw[i] = xb[i];
    for (int v = threadIdx.x; v < nv; v += blockDim.x) {
        const int i0 = head + v * VEC;  // 16-byte aligned in global memory, not in the span
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(xb + i0));
        const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
        for (int k = 0; k < VEC; ++k) raw[i0 + k] = e[k];
    }
    for (int i = head + nv * VEC + threadIdx.x; i < n; i += blockDim.x) raw[i] = xb[i];
    for (int i = threadIdx.x; i < np * taps; i += blockDim.x) {
        const int pp = div_magic(i, mg.taps), t = i - pp * taps;
        int c = c0 + pp;
        while (c >= C) c -= C;
        wf[i] = static_cast<float>(w[static_cast<int64_t>(c) * taps + t]);
    }
    // ---- the scales: wait for the amax grid, fold its partials (plain
    // loads of words that grid stored)
    asm volatile("griddepcontrol.wait;" ::: "memory");
    unsigned mx = 0u, mw = 0u;
    for (int i = threadIdx.x; i < nparts; i += blockDim.x) {
        mx = max(mx, part[i]);
        mw = max(mw, part[nparts + i]);
    }
    mx = block_max_bits(mx, red);
    __syncthreads();
    mw = block_max_bits(mw, red);
    __syncthreads();
    const float ax = __uint_as_float(mx), aw = __uint_as_float(mw);
    const float invx = quant_inv(ax), invw = quant_inv(aw);
    const double s = dequant_scale(ax, aw);

    // ---- phase 2: codes into zero-padded planes, filter codes.  The scales
    // are the operands' own max-abs, so every |v * inv| <= 32767.004 and the
    // magic-number codes need no clamp; a non-finite scale (a NaN or an
    // infinity in an operand) turns every output into NaN below, whatever
    // the codes of the non-finite values were.
    // One thread per input row writes the whole padded row (left and right
    // padding included); the rows next to the top and bottom padding also
    // zero those padding rows; thread 0 zeroes the slack after the last plane.
    for (int rr = threadIdx.x; rr < np * H; rr += blockDim.x) {
        const int pp = div_magic(rr, mg.h), ih = rr - pp * H;
        const T* src = raw + pp * HW + ih * W;
        int16_t* plane = xs + pp * PHW;
        int16_t* dst = plane + (ih + ph) * Wp;
        for (int k = 0; k < pw; ++k) {
            dst[k] = 0;
            dst[pw + W + k] = 0;
        }
        for (int iw = 0; iw < W; ++iw)
            dst[pw + iw] = static_cast<int16_t>(quant_code_bits(ldx<T>(src, iw), invx) & 0xFFFFu);
        if (ih == 0)
            for (int k = 0; k < ph * Wp; ++k) plane[k] = 0;
        if (ih == H - 1)
            for (int k = 0; k < ph * Wp; ++k) plane[(ph + H) * Wp + k] = 0;
    }
    if (threadIdx.x == 0)
        for (int k = 0; k < kDwRowOut + KW; ++k) xs[np * PHW + k] = 0;
    // filter codes split as 256 * hi + lo (hi in [-128, 127], lo in [0, 255])
    // so both partial sums below stay int32: |x| * 128 and |x| * 255 over at
    // most 49 taps are below 2^29
    for (int i = threadIdx.x; i < np * taps; i += blockDim.x) {
        const int q = static_cast<int16_t>(quant_code_bits(wf[i], invw) & 0xFFFFu);
        wsq[i] = (q >> 8) * 65536 + (q & 255);  // hi in the upper half, lo in the lower
    }
    const bool s_finite = s <= 1.7976931348623157e308;
    __syncthreads();
    // ---- each thread a whole output row, into the staged output span
    for (int row = threadIdx.x; row < np * OH; row += blockDim.x) {
        const int pp = div_magic(row, mg.oh), oh = row - pp * OH;
        const int16_t* xr = xs + pp * PHW + oh * Wp;
        const int* wp = wsq + pp * taps;
        int c = c0 + pp;
        while (c >= C) c -= C;
        const float bv = bias != nullptr ? ldx<T>(bias, c) : 0.0f;
        T* orow = raw + row * OW;
        for (int ow0 = 0; ow0 < OW; ow0 += kDwRowOut) {
            int acc_hi[kDwRowOut], acc_lo[kDwRowOut];
#pragma unroll
            for (int j = 0; j < kDwRowOut; ++j) acc_hi[j] = acc_lo[j] = 0;
            for (int r = 0; r < KH; ++r) {
                int xv[kDwRowOut + KW - 1];
#pragma unroll
                for (int j = 0; j < kDwRowOut + KW - 1; ++j) xv[j] = xr[r * Wp + ow0 + j];
#pragma unroll
                for (int k = 0; k < KW; ++k) {
                    const int wv = wp[r * KW + k];
                    const int wh = wv >> 16, wl = wv & 0xFFFF;
#pragma unroll
                    for (int j = 0; j < kDwRowOut; ++j) {
                        acc_hi[j] += xv[j + k] * wh;
                        acc_lo[j] += xv[j + k] * wl;
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < kDwRowOut; ++j) {
                if (ow0 + j < OW) {
                    // the exact sum 256 * hi + lo as binary64: both int32 through
                    // their bit patterns, joined by one exact multiply-add
                    const double dh = __hiloint2double(0x43300000, acc_hi[j] ^ static_cast<int>(0x80000000u)) -
                                      4503601774854144.0;
                    const double dl = __hiloint2double(0x43300000, acc_lo[j] ^ static_cast<int>(0x80000000u)) -
                                      4503601774854144.0;
                    float v = round_t_from_double(__dmul_rn(__fma_rn(dh, 256.0, dl), s), DT);
                    v = s_finite ? v : __int_as_float(0x7FC00000);
                    if (bias != nullptr) v = round_t(__fadd_rn(v, bv), DT);
                    store_t(orow, DT, ow0 + j, v);
                }
            }
        }
    }
    __syncthreads();
    // ---- the block's output span, 16-byte vectors where aligned
    const int no = np * OH * OW;
    T* obase = out + pl0 * OH * OW;
    const bool oal = reinterpret_cast<uintptr_t>(out) % 16 == 0;
    const int ohead = oal ? min(no, static_cast<int>((VEC - (pl0 * OH * OW) % VEC) % VEC)) : no;
    const int onv = (no - ohead) / VEC;
    for (int i = threadIdx.x; i < ohead; i += blockDim.x) obase[i] = raw[i];
    for (int v = threadIdx.x; v < onv; v += blockDim.x) {
        const int i0 = ohead + v * VEC;
        uint4 u;
        T* e = reinterpret_cast<T*>(&u);
#pragma unroll
        for (int k = 0; k < VEC; ++k) e[k] = raw[i0 + k];
        *reinterpret_cast<uint4*>(obase + i0) = u;
    }
    for (int i = ohead + onv * VEC + threadIdx.x; i < no; i += blockDim.x) obase[i] = raw[i];
}

// Shared-memory bytes of depthwise_scaled_kernel for `ppb` planes.
size_t depthwise_scaled_smem(const ConvGeom& g, int ppb, size_t esize) {
    const int64_t hw = g.H * g.W, ohw = g.OH * g.OW;
    const int64_t phw = (g.H + 2 * g.ph) * (g.W + 2 * g.pw);
    size_t b = round_up(static_cast<size_t>(ppb * std::max(hw, ohw)) * esize, 16);
    b += round_up(static_cast<size_t>(ppb * phw + kDwRowOut + g.KW) * 2, 16);
    b += static_cast<size_t>(ppb * g.KH * g.KW) * 4;
    b += 32 * sizeof(unsigned);
    return b;
}

// Planes per block of depthwise_rows_kernel for this geometry (0: the
// kernel does not apply): at most one output row per thread, within the
// shared-memory spans.
int depthwise_rows_ppb(const ConvGeom& g) {
    if (!(g.D == 1 && g.KD == 1 && g.groups == g.C && g.groups > 1 && g.F == g.C)) return 0;
    if (g.sh != 1 || g.sw != 1 || g.dh != 1 || g.dw != 1) return 0;
    if (g.KW != 3 && g.KW != 5 && g.KW != 7) return 0;
    const int64_t phw = (g.H + 2 * g.ph) * (g.W + 2 * g.pw);
    const int64_t taps = g.KH * g.KW;
    if (phw > kDwRowSpan || taps > kDwRowTaps || g.OW > 4096) return 0;
    // whole planes whose output rows fit one round of the block's threads
    int64_t ppb = std::max<int64_t>(1, kDwRowThreads / g.OH);
    ppb = std::min(ppb, kDwRowSpan / phw);
    ppb = std::min(ppb, kDwRowTaps / taps);
    return static_cast<int>(std::max<int64_t>(ppb, 1));
}

uint32_t magic_div(int64_t d) { return static_cast<uint32_t>((1ULL << 32) / static_cast<uint64_t>(d) + 1); }

// The depthwise convolution with its scales from the amax grid and the
// convolution grid overlapping (programmatic dependent launch), when the row
// kernel's geometry applies and the grid fits the device in one wave;
// TK_ERR_UNSUPPORTED otherwise (the caller takes the two-pass path).
// `part` holds 2 * kDwAmaxMaxBlocks words.
int depthwise_scaled_launch(const tk_conv3d_desc_t& d, const ConvGeom& g, unsigned* part, cudaStream_t stream) {
    int ppb = depthwise_rows_ppb(g);
    // the kernel's int32 partial sums hold up to 64 taps
    if (ppb == 0 || g.KH * g.KW > 64) return TK_ERR_UNSUPPORTED;
    const int64_t planes = g.N * g.C;
    const int64_t hw = g.H * g.W, ohw = g.OH * g.OW;
    const int64_t taps = g.KH * g.KW;
    const size_t esize = d.dtype == TK_DTYPE_F16 ? 2 : 4;
    const int dev = current_device();
    const void* fn = nullptr;
    if (d.dtype == TK_DTYPE_F16) {
        fn = g.KW == 3 ? reinterpret_cast<const void*>(depthwise_scaled_kernel<__half, 0, 3>)
           : g.KW == 5 ? reinterpret_cast<const void*>(depthwise_scaled_kernel<__half, 0, 5>)
                       : reinterpret_cast<const void*>(depthwise_scaled_kernel<__half, 0, 7>);
    } else {
        fn = g.KW == 3 ? reinterpret_cast<const void*>(depthwise_scaled_kernel<float, 1, 3>)
           : g.KW == 5 ? reinterpret_cast<const void*>(depthwise_scaled_kernel<float, 1, 5>)
                       : reinterpret_cast<const void*>(depthwise_scaled_kernel<float, 1, 7>);
    }
    TK_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024));
    // One resident wave (its blocks start loading while the partials form).
    // Preferred: a balanced grid, the
    // same number k of blocks on every SM (planes per block = planes / (k x
    // SMs), rounded up) with enough threads that each block's input and
    // output rows take two rounds of its threads.  Else the planes per block
    // fill whole rounds of kDwRowThreads threads, for the fewest rounds r
    // whose grid fits.  Both within the shared-memory spans.
    const int sms = sm_count(dev);
    const int64_t rows_pp = std::max(g.H, g.OH);
    // the kernel's magic-number divisions hold for indices below 2^16; its
    // spans are all in dynamic shared memory
    auto spans_ok = [&](int64_t cand) {
        return cand * std::max(hw, ohw) < 65536 && cand * taps < 65536 &&
               depthwise_scaled_smem(g, static_cast<int>(cand), esize) <= 96 * 1024;
    };
    int64_t blocks = 0;
    size_t smem = 0;
    int threads = kDwRowThreads;
    bool fits = false;
    for (int k = 2; k <= 4 && !fits; ++k) {
        const int64_t cand = ceil_div(planes, static_cast<int64_t>(k) * sms);
        const int64_t t = static_cast<int64_t>(round_up(static_cast<size_t>(ceil_div(cand * rows_pp, 2)), 32));
        if (t > kDwMaxThreads || !spans_ok(cand)) continue;
        smem = depthwise_scaled_smem(g, static_cast<int>(cand), esize);
        int per_sm = 0;
        TK_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, static_cast<int>(t), smem));
        ppb = static_cast<int>(cand);
        threads = static_cast<int>(t);
        blocks = ceil_div(planes, cand);
        fits = per_sm > 0 && blocks <= static_cast<int64_t>(per_sm) * sms;
    }
    for (int r = 1; r <= 8 && !fits; ++r) {
        const int64_t cand = std::max<int64_t>(1, (static_cast<int64_t>(r) * kDwRowThreads) / g.OH);
        if (!spans_ok(cand)) break;
        smem = depthwise_scaled_smem(g, static_cast<int>(cand), esize);
        int per_sm = 0;
        TK_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kDwRowThreads, smem));
        ppb = static_cast<int>(cand);
        threads = kDwRowThreads;
        blocks = ceil_div(planes, cand);
        fits = per_sm > 0 && blocks <= static_cast<int64_t>(per_sm) * sms;
    }
    if (!fits) return TK_ERR_UNSUPPORTED;
    // the partials: chunks of about 4 KB of the input per block (one or two
    // 16-byte loads per thread), in whole 16-byte vectors
    const int64_t nx = planes * hw, nw = g.C * taps;
    const int64_t vecw = static_cast<int64_t>(16 / esize);
    const int64_t nparts = std::max<int64_t>(
        1, std::min<int64_t>(kDwAmaxMaxBlocks, ceil_div(nx * static_cast<int64_t>(esize), 4 * 1024)));
    const int64_t cx = round_up(static_cast<size_t>(ceil_div(nx, nparts)), static_cast<size_t>(vecw));
    const int64_t cw = round_up(static_cast<size_t>(ceil_div(nw, nparts)), static_cast<size_t>(vecw));
    const int vx = reinterpret_cast<uintptr_t>(d.x) % 16 == 0 ? 1 : 0;
    const int vw = reinterpret_cast<uintptr_t>(d.weight) % 16 == 0 ? 1 : 0;
    if (d.dtype == TK_DTYPE_F16)
        depthwise_amax_kernel<__half><<<static_cast<unsigned>(nparts), kDwAmaxThreads, 0, stream>>>(
            static_cast<const __half*>(d.x), nx, cx, vx, static_cast<const __half*>(d.weight), nw, cw, vw, part);
    else
        depthwise_amax_kernel<float><<<static_cast<unsigned>(nparts), kDwAmaxThreads, 0, stream>>>(
            static_cast<const float*>(d.x), nx, cx, vx, static_cast<const float*>(d.weight), nw, cw, vw, part);
    int rc = launch_status("conv2d depthwise (amax partials)");
    if (rc) return rc;
    ConvGeom gg = g;
    int ppb_arg = ppb;
    DwMagic mg;
    mg.hw = magic_div(hw);
    mg.w = magic_div(g.W);
    mg.taps = magic_div(g.KH * g.KW);
    mg.ohw = magic_div(ohw);
    mg.ow = magic_div(g.OW);
    mg.h = magic_div(g.H);
    mg.oh = magic_div(g.OH);
    const void* xp = d.x;
    const void* wp = d.weight;
    const void* bp = d.bias;
    void* op = d.out;
    const unsigned* pp = part;
    int np_arg = static_cast<int>(nparts);
    void* args[] = {const_cast<void**>(&xp), const_cast<void**>(&wp), const_cast<void**>(&bp), &op, &gg, &ppb_arg,
                    &mg, &pp, &np_arg};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(blocks));
    cfg.blockDim = dim3(static_cast<unsigned>(threads));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    TK_CUDA_TRY(cudaLaunchKernelExC(&cfg, fn, args));
    return launch_status("conv2d depthwise (scaled)");
}

int grid_1d(int64_t n, int threads) {
    const int64_t g = ceil_div(n, threads);
    const int64_t cap = static_cast<int64_t>(sm_count(current_device())) * 32;
    return static_cast<int>(std::max<int64_t>(1, std::min(g, cap)));
}

int geometry(const tk_conv3d_desc_t& d, ConvGeom& g) {
    TK_CHECK_ARG(d.dtype == TK_DTYPE_F16 || d.dtype == TK_DTYPE_F32, "conv: bad dtype");
    TK_CHECK_ARG(d.n >= 0 && d.c > 0 && d.d > 0 && d.h > 0 && d.w > 0 && d.f > 0 && d.kd > 0 &&
                     d.kh > 0 && d.kw > 0,
                 "conv: bad shape");
    TK_CHECK_ARG(d.stride_d > 0 && d.stride_h > 0 && d.stride_w > 0 && d.dil_d > 0 && d.dil_h > 0 &&
                     d.dil_w > 0 && d.pad_d >= 0 && d.pad_h >= 0 && d.pad_w >= 0,
                 "conv: bad stride/padding/dilation");
    TK_CHECK_ARG(d.groups > 0 && d.c % d.groups == 0 && d.f % d.groups == 0,
                 "conv: channels must be divisible by groups");
    g = {d.n, d.c, d.h, d.w, d.f, d.kh, d.kw, d.stride_h, d.stride_w, d.pad_h, d.pad_w,
         d.dil_h, d.dil_w, d.groups, 0, 0, d.d, d.kd, d.stride_d, d.pad_d, d.dil_d, 0};
    g.OD = (d.d + 2 * d.pad_d - d.dil_d * (d.kd - 1) - 1) / d.stride_d + 1;
    g.OH = (d.h + 2 * d.pad_h - d.dil_h * (d.kh - 1) - 1) / d.stride_h + 1;
    g.OW = (d.w + 2 * d.pad_w - d.dil_w * (d.kw - 1) - 1) / d.stride_w + 1;
    TK_CHECK_ARG(g.OD > 0 && g.OH > 0 && g.OW > 0, "conv: non-positive output size");
    return TK_OK;
}

tk_conv3d_desc_t as_3d(const tk_conv2d_desc_t& d) {
    tk_conv3d_desc_t e = {};
    e.dtype = d.dtype;
    e.n = d.n; e.c = d.c; e.d = 1; e.h = d.h; e.w = d.w;
    e.f = d.f; e.kd = 1; e.kh = d.kh; e.kw = d.kw;
    e.stride_d = 1; e.stride_h = d.stride_h; e.stride_w = d.stride_w;
    e.pad_d = 0; e.pad_h = d.pad_h; e.pad_w = d.pad_w;
    e.dil_d = 1; e.dil_h = d.dil_h; e.dil_w = d.dil_w;
    e.groups = d.groups;
    e.x = d.x; e.weight = d.weight; e.bias = d.bias; e.out = d.out;
    e.amax_x = d.amax_x; e.amax_w = d.amax_w;
    return e;
}

bool is_2d(const ConvGeom& g) { return g.D == 1 && g.KD == 1 && g.pd == 0; }
bool is_depthwise(const ConvGeom& g) { return is_2d(g) && g.groups == g.C && g.groups > 1; }
// Implicit GEMM on the tensor cores: one group, unit stride (any padding and
// dilation), and per-tap channel depth within the exact-accumulation limit.
bool is_implicit(const ConvGeom& g) {
    return g.groups == 1 && g.sd == 1 && g.sh == 1 && g.sw == 1 &&
           round_up(g.C, 64) * g.KD * g.KH * g.KW <= 32768 && g.N * g.D * g.H < (1LL << 31);
}
bool is_pointwise(const ConvGeom& g) {
    return g.KD == 1 && g.KH == 1 && g.KW == 1 && g.sd == 1 && g.sh == 1 && g.sw == 1 && g.pd == 0 &&
           g.ph == 0 && g.pw == 0 && g.groups == 1;
}

struct ConvLayout {
    int64_t K, ld;
    size_t off_amax, off_la, off_lb, total;
};

ConvLayout conv_layout(const ConvGeom& g) {
    ConvLayout L;
    L.K = (g.C / g.groups) * g.KD * g.KH * g.KW;
    L.ld = static_cast<int64_t>(round_up(static_cast<size_t>(L.K), 16));
    const int64_t P = g.OD * g.OH * g.OW;
    L.off_amax = 0;
    L.off_la = 1024;
    if (is_depthwise(g)) {
        // the partial maxima of depthwise_scaled_launch follow the amax slots
        L.off_lb = L.off_la;
        L.total = L.off_la + 2 * kDwAmaxMaxBlocks * sizeof(unsigned);
        return L;
    }
    if (is_implicit(g)) {
        L.off_lb = L.off_la;
        L.total = L.off_la + conv_tc_workspace(g.N, g.C, g.D, g.H, g.W, g.F, g.KD, g.KH, g.KW, g.ph, g.pw);
        return L;
    }
    L.off_lb = round_up(L.off_la + static_cast<size_t>(g.N * g.groups * 2 * P * L.ld), 1024);
    L.total = round_up(L.off_lb + static_cast<size_t>(g.groups * 2 * (g.F / g.groups) * L.ld), 1024);
    return L;
}

// ---- weight gradient ----------------------------------------------------------

// Geometry of a weight-gradient descriptor (the forward convolution's).
int wgrad_geometry(const tk_conv3d_wgrad_desc_t& d, ConvGeom& g) {
    tk_conv3d_desc_t f = {};
    f.dtype = d.dtype;
    f.n = d.n; f.c = d.c; f.d = d.d; f.h = d.h; f.w = d.w;
    f.f = d.f; f.kd = d.kd; f.kh = d.kh; f.kw = d.kw;
    f.stride_d = d.stride_d; f.stride_h = d.stride_h; f.stride_w = d.stride_w;
    f.pad_d = d.pad_d; f.pad_h = d.pad_h; f.pad_w = d.pad_w;
    f.dil_d = d.dil_d; f.dil_h = d.dil_h; f.dil_w = d.dil_w;
    f.groups = d.groups;
    return geometry(f, g);
}

constexpr size_t kWgradPatchBudget = 512ull << 20;  // bytes of patch limbs per GEMM launch

struct WgradLayout {
    int64_t M, P, ld, nchunk;
    size_t off_amax, off_acc, off_lb, off_la, total;
};

// [amax x, amax g] | acc64 [groups][M][F/g] | dy limbs [N*groups][2][F/g][ld]
// | patch limbs of nchunk images [nchunk*groups][2][M][ld]
WgradLayout wgrad_layout(const ConvGeom& g) {
    WgradLayout L;
    L.M = (g.C / g.groups) * g.KD * g.KH * g.KW;
    L.P = g.OD * g.OH * g.OW;
    L.ld = static_cast<int64_t>(round_up(static_cast<size_t>(L.P), 16));
    const int64_t fg = g.F / g.groups;
    const int64_t per_image = g.groups * 2 * L.M * L.ld;
    L.nchunk = std::max<int64_t>(1, std::min<int64_t>(g.N, static_cast<int64_t>(kWgradPatchBudget) / per_image));
    L.nchunk = std::max<int64_t>(1, std::min<int64_t>(L.nchunk, 65535 / g.groups));
    L.off_amax = 0;
    L.off_acc = 1024;
    L.off_lb = round_up(L.off_acc + sizeof(int64_t) * static_cast<size_t>(g.groups * L.M * fg), 1024);
    L.off_la = round_up(L.off_lb + static_cast<size_t>(g.N * g.groups * 2 * fg * L.ld), 1024);
    L.total = round_up(L.off_la + static_cast<size_t>(L.nchunk * per_image), 1024);
    return L;
}

}  // namespace
}  // namespace tk

extern "C" {

size_t tk_conv3d_wgrad_workspace_size(const tk_conv3d_wgrad_desc_t* desc) {
    using namespace tk;
    if (desc == nullptr) return 0;
    ConvGeom g;
    if (wgrad_geometry(*desc, g) != TK_OK || g.N == 0) return 0;
    return wgrad_layout(g).total;
}

int tk_conv3d_wgrad_q16(const tk_conv3d_wgrad_desc_t* desc, void* workspace, size_t workspace_bytes,
                        void* stream_) {
    using namespace tk;
    TK_CHECK_ARG(desc != nullptr, "conv wgrad: desc is NULL");
    const tk_conv3d_wgrad_desc_t& d = *desc;
    ConvGeom g;
    int rc = wgrad_geometry(d, g);
    if (rc) return rc;
    TK_CHECK_ARG(d.grad_weight != nullptr, "conv wgrad: grad_weight is NULL");
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    const int64_t fg = g.F / g.groups, cg = g.C / g.groups;
    const int64_t wnum = g.F * cg * g.KD * g.KH * g.KW;
    if (g.N == 0) {  // empty reduction: every gradient is T(0 * scale) = 0
        TK_CUDA_TRY(cudaMemsetAsync(d.grad_weight, 0, wnum * dtype_size(d.dtype), stream));
        return TK_OK;
    }
    TK_CHECK_ARG(d.x != nullptr && d.grad_out != nullptr, "conv wgrad: NULL pointer");
    const WgradLayout L = wgrad_layout(g);
    TK_CHECK_ARG(workspace != nullptr && workspace_bytes >= L.total &&
                     reinterpret_cast<uintptr_t>(workspace) % 1024 == 0,
                 "conv wgrad: workspace must be >= %zu bytes and 1024-byte aligned", L.total);
    TK_CHECK_ARG(g.N * g.groups <= 65535, "conv wgrad: n * groups must be <= 65535");
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    float* amax = reinterpret_cast<float*>(ws + L.off_amax);
    const int64_t xnum = g.N * g.C * g.D * g.H * g.W, gnum = g.N * g.F * L.P;
    const float* ax = d.amax_x;
    const float* ag = d.amax_g;
    if (ax == nullptr && ag == nullptr) {
        rc = amax_pair_launch(d.dtype, d.x, xnum, d.grad_out, gnum, amax, stream);
        if (rc) return rc;
        ax = amax;
        ag = amax + 1;
    }
    if (ax == nullptr) {
        rc = amax_launch(d.dtype, d.x, 1, 0, xnum, amax, stream);
        if (rc) return rc;
        ax = amax;
    }
    if (ag == nullptr) {
        rc = amax_launch(d.dtype, d.grad_out, 1, 0, gnum, amax + 1, stream);
        if (rc) return rc;
        ag = amax + 1;
    }
    auto* acc64 = reinterpret_cast<unsigned long long*>(ws + L.off_acc);
    int8_t* lb = reinterpret_cast<int8_t*>(ws + L.off_lb);
    int8_t* la = reinterpret_cast<int8_t*>(ws + L.off_la);
    TK_CUDA_TRY(cudaMemsetAsync(acc64, 0, sizeof(int64_t) * static_cast<size_t>(g.groups * L.M * fg), stream));
    // B: grad_out as N*groups slices [F/g, P] (row-contiguous), one scale
    rc = quantize_limbs_launch(d.dtype, d.grad_out, g.N * g.groups, fg, L.P, fg * L.P, L.P, 1, ag, 0, lb,
                               stream);
    if (rc) return rc;
    tk_qgemm_desc_t q = {};
    q.dtype = d.dtype;
    q.m = L.M;
    q.n = fg;
    q.k = L.P;
    q.out = d.grad_weight;
    q.alpha = 1.0f;
    q.act = TK_ACT_NONE;
    q.per_slice_scales = 0;
    for (int64_t n0 = 0; n0 < g.N; n0 += L.nchunk) {
        const int64_t nimg = std::min(L.nchunk, g.N - n0);
        const int64_t total = nimg * g.groups * L.M * (L.ld / 8);
        const int grid = grid_1d(total, 256);
        if (d.dtype == TK_DTYPE_F16)
            im2col_t_quant_kernel<__half><<<grid, 256, 0, stream>>>(static_cast<const __half*>(d.x), g, n0, nimg,
                                                                    L.M, L.ld, ax, la);
        else
            im2col_t_quant_kernel<float><<<grid, 256, 0, stream>>>(static_cast<const float*>(d.x), g, n0, nimg,
                                                                   L.M, L.ld, ax, la);
        rc = launch_status("conv wgrad patches");
        if (rc) return rc;
        q.batch = nimg * g.groups;
        rc = qgemm_limbs_acc64(q, la, lb + n0 * g.groups * 2 * fg * L.ld, acc64, static_cast<int>(g.groups),
                               stream);
        if (rc) return rc;
    }
    // grad_weight[grp*F/g + f][c][t][r][s] = epilogue(acc64[grp][(c,t,r,s)][f])
    q.batch = g.groups;
    q.out_sb = fg * L.M;
    q.out_sm = 1;
    return qgemm_acc64_finish(q, reinterpret_cast<const long long*>(acc64), g.groups, ax, ag, /*out_sn=*/L.M,
                              stream);
}

size_t tk_conv3d_workspace_size(const tk_conv3d_desc_t* desc) {
    using namespace tk;
    if (desc == nullptr) return 0;
    ConvGeom g;
    if (geometry(*desc, g) != TK_OK) return 0;
    return conv_layout(g).total;
}

size_t tk_conv2d_workspace_size(const tk_conv2d_desc_t* desc) {
    if (desc == nullptr) return 0;
    const tk_conv3d_desc_t e = tk::as_3d(*desc);
    return tk_conv3d_workspace_size(&e);
}

int tk_conv2d_q16(const tk_conv2d_desc_t* desc, void* workspace, size_t workspace_bytes,
                  void* stream) {
    using namespace tk;
    TK_CHECK_ARG(desc != nullptr, "conv2d: desc is NULL");
    const tk_conv3d_desc_t e = as_3d(*desc);
    return tk_conv3d_q16(&e, workspace, workspace_bytes, stream);
}

int tk_conv3d_q16(const tk_conv3d_desc_t* desc, void* workspace, size_t workspace_bytes,
                  void* stream_) {
    using namespace tk;
    TK_CHECK_ARG(desc != nullptr, "conv: desc is NULL");
    const tk_conv3d_desc_t& d = *desc;
    ConvGeom g;
    int rc = geometry(d, g);
    if (rc) return rc;
    if (g.N == 0) return TK_OK;
    TK_CHECK_ARG(d.x && d.weight && d.out, "conv: NULL pointer");
    const ConvLayout L = conv_layout(g);
    TK_CHECK_ARG(workspace != nullptr && workspace_bytes >= L.total &&
                     reinterpret_cast<uintptr_t>(workspace) % 1024 == 0,
                 "conv: workspace must be >= %zu bytes and 1024-byte aligned", L.total);
    TK_CHECK_ARG(L.K <= 32768, "conv: C/groups*KD*KH*KW = %lld exceeds 32768", (long long)L.K);
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    float* amax = reinterpret_cast<float*>(ws + L.off_amax);  // [0] input, [1] weight
    const float* ax = d.amax_x;
    const float* aw = d.amax_w;
    if (ax == nullptr && aw == nullptr) {
        rc = depthwise_scaled_launch(d, g, reinterpret_cast<unsigned*>(ws + L.off_la), stream);
        if (rc != TK_ERR_UNSUPPORTED) return rc;
    }
    if (ax == nullptr && aw == nullptr) {  // both scales in one launch
        rc = amax_pair_launch(d.dtype, d.x, g.N * g.C * g.D * g.H * g.W, d.weight,
                              g.F * (g.C / g.groups) * g.KD * g.KH * g.KW, amax, stream);
        if (rc) return rc;
        ax = amax;
        aw = amax + 1;
    }
    if (ax == nullptr) {
        rc = amax_launch(d.dtype, d.x, 1, 0, g.N * g.C * g.D * g.H * g.W, amax, stream);
        if (rc) return rc;
        ax = amax;
    }
    if (aw == nullptr) {
        rc = amax_launch(d.dtype, d.weight, 1, 0, g.F * (g.C / g.groups) * g.KD * g.KH * g.KW, amax + 1,
                         stream);
        if (rc) return rc;
        aw = amax + 1;
    }
    const int64_t P = g.OD * g.OH * g.OW;
    if (const int ppb = depthwise_rows_ppb(g)) {
        const int64_t blocks = ceil_div(g.N * g.C, ppb);
        TK_CHECK_ARG(blocks < (1LL << 31), "conv2d: too many planes");
        const unsigned grid = static_cast<unsigned>(blocks);
#define TK_DW_ROWS(KWV)                                                                                  \
    if (d.dtype == TK_DTYPE_F16)                                                                         \
        depthwise_rows_kernel<__half, 0, KWV><<<grid, kDwRowThreads, 0, stream>>>(                      \
            static_cast<const __half*>(d.x), static_cast<const __half*>(d.weight),                      \
            static_cast<const __half*>(d.bias), static_cast<__half*>(d.out), g, ppb, ax, aw);           \
    else                                                                                                 \
        depthwise_rows_kernel<float, 1, KWV><<<grid, kDwRowThreads, 0, stream>>>(                       \
            static_cast<const float*>(d.x), static_cast<const float*>(d.weight),                        \
            static_cast<const float*>(d.bias), static_cast<float*>(d.out), g, ppb, ax, aw);
        if (g.KW == 3) {
            TK_DW_ROWS(3)
        } else if (g.KW == 5) {
            TK_DW_ROWS(5)
        } else {
            TK_DW_ROWS(7)
        }
#undef TK_DW_ROWS
        return launch_status("conv2d depthwise");
    }
    if (is_depthwise(g) && g.F == g.C && g.H * g.W <= kDwFlatElems / 2 &&
        g.KH * g.KW * (kDwFlatElems / (g.H * g.W)) <= kDwFlatElems / 4) {
        const int ppb = static_cast<int>(kDwFlatElems / (g.H * g.W));
        const int64_t blocks = ceil_div(g.N * g.C, ppb);
        TK_CHECK_ARG(blocks < (1LL << 31), "conv2d: too many planes");
        if (d.dtype == TK_DTYPE_F16)
            depthwise_flat_kernel<__half, 0><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
                static_cast<const __half*>(d.x), static_cast<const __half*>(d.weight),
                static_cast<const __half*>(d.bias), static_cast<__half*>(d.out), g, ppb, ax, aw);
        else
            depthwise_flat_kernel<float, 1><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
                static_cast<const float*>(d.x), static_cast<const float*>(d.weight),
                static_cast<const float*>(d.bias), static_cast<float*>(d.out), g, ppb, ax, aw);
        return launch_status("conv2d depthwise");
    }
    if (is_depthwise(g) && g.H * g.W <= kDwPlaneMax && g.KH * g.KW <= 64) {
        const int64_t planes = g.N * g.F;
        TK_CHECK_ARG(ceil_div(planes, kDwWarps) < (1LL << 31), "conv2d: too many planes");
        const unsigned grid = static_cast<unsigned>(ceil_div(planes, kDwWarps));
        if (d.dtype == TK_DTYPE_F16)
            depthwise_plane_kernel<__half, 0><<<grid, 32 * kDwWarps, 0, stream>>>(
                static_cast<const __half*>(d.x), static_cast<const __half*>(d.weight),
                static_cast<const __half*>(d.bias), static_cast<__half*>(d.out), g, ax, aw);
        else
            depthwise_plane_kernel<float, 1><<<grid, 32 * kDwWarps, 0, stream>>>(
                static_cast<const float*>(d.x), static_cast<const float*>(d.weight),
                static_cast<const float*>(d.bias), static_cast<float*>(d.out), g, ax, aw);
        return launch_status("conv2d depthwise");
    }
    if (is_depthwise(g)) {
        const int64_t total = g.N * g.F * P;
        const int grid = grid_1d(total, 256);
        if (d.dtype == TK_DTYPE_F16)
            depthwise_kernel<__half, 0><<<grid, 256, 0, stream>>>(
                static_cast<const __half*>(d.x), static_cast<const __half*>(d.weight),
                static_cast<const __half*>(d.bias), static_cast<__half*>(d.out), g, ax, aw);
        else
            depthwise_kernel<float, 1><<<grid, 256, 0, stream>>>(
                static_cast<const float*>(d.x), static_cast<const float*>(d.weight),
                static_cast<const float*>(d.bias), static_cast<float*>(d.out), g, ax, aw);
        return launch_status("conv2d depthwise");
    }
    if (is_implicit(g))
        return conv_tc(d.dtype, d.x, d.weight, d.bias, d.out, g.N, g.C, g.D, g.H, g.W, g.F, g.KD, g.KH,
                       g.KW, g.pd, g.ph, g.pw, g.dd, g.dh, g.dw, g.OD, g.OH, g.OW, ax, aw, ws + L.off_la,
                       stream, d.amax_x == nullptr);
    int8_t* la = reinterpret_cast<int8_t*>(ws + L.off_la);  // patches [N*groups][2][P][ld]
    int8_t* lb = reinterpret_cast<int8_t*>(ws + L.off_lb);  // weights [groups][2][F/g][ld]
    const int64_t fg = g.F / g.groups;
    // weights: contiguous OI[D]HW, one [F/g, K] slice per group
    rc = quantize_limbs_launch(d.dtype, d.weight, g.groups, fg, L.K, fg * L.K, L.K, 1, aw, 0, lb,
                               stream);
    if (rc) return rc;
    if (is_pointwise(g)) {
        // A[n] = x[n] viewed as [P, C] with strides (1, P): a transposed read.
        rc = quantize_limbs_launch(d.dtype, d.x, g.N, P, g.C, g.C * P, 1, P, ax, 0, la, stream);
        if (rc) return rc;
    } else {
        const int64_t total = g.N * g.groups * P * (L.ld / 4);
        const int grid = grid_1d(total, 256);
        if (d.dtype == TK_DTYPE_F16)
            im2col_quant_kernel<__half><<<grid, 256, 0, stream>>>(
                static_cast<const __half*>(d.x), g, L.K, L.ld, ax, la);
        else
            im2col_quant_kernel<float><<<grid, 256, 0, stream>>>(
                static_cast<const float*>(d.x), g, L.K, L.ld, ax, la);
        rc = launch_status("conv2d im2col");
        if (rc) return rc;
    }
    tk_qgemm_desc_t q = {};
    q.dtype = d.dtype;
    q.batch = g.N * g.groups;
    q.m = P;
    q.n = fg;
    q.k = L.K;
    q.out = d.out;
    q.out_sb = fg * P;  // slice (n, grp) starts at out[n][grp*fg][0][0]
    q.out_sm = 1;       // pixels are contiguous in NCHW
    q.bias = d.bias;
    q.alpha = 1.0f;
    q.beta = 0.0f;
    q.act = TK_ACT_NONE;
    q.per_slice_scales = 0;
    return qgemm_limbs_ex(q, la, lb, ax, aw, static_cast<int>(g.groups), /*out_sn=*/P,
                          /*bias_mod=*/g.groups > 1 ? g.groups : 0, stream);
}

}  // extern "C"
