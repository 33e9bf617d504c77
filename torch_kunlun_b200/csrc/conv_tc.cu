// conv_tc.cu -- implicit-GEMM int16-quantised conv2d / conv3d on sm_100a
// tensor cores.
//
// Replaces baidu::xpu::api::conv2d<T,T,T,TGEMM> plus the bias broadcast_add
// of conv2d_impl (csrc/ops.cpp:237-285), and xdnn conv3d of conv3d
// (csrc/ops_nn_extra.cpp:88-121), for groups == 1, stride 1 (any padding and
// dilation).  A 2-D convolution is the 3-D one with D = KD = 1.  Semantics are those of the explicit path in
// conv.cu: one max-abs scale for the whole input and one for the whole
// weight, exact integer MAC, T(acc * s), then the bias added and rounded.
//
// Data flow (no patch matrix in HBM):
//   conv_prep_kernel one launch whose blocks do three disjoint jobs:
//     x_limbs_block  NC(D)HW input -> quantised N(D)HWC limb rows: per pixel, per
//                    group of 64 channels, 128 bytes [hi of the 64 | lo of
//                    the 64] (hi = q >> 8 signed, lo = q & 255 unsigned);
//     w_limbs_block  OI(D)HW weight -> [F][KD][KH][KW][channel groups] limb rows of
//                    the same 128-byte form (w_stack_blocks: the stacked
//                    tiles of the stacked-limb kernel);
//     zero_ring_blocks the zero ring of the padded planes (window kernels);
//   conv_tc_kernel   one CTA per SM, persistent over output tiles of
//                    TH x TW pixels of one (image, output depth) x BN
//                    filters.  Each K step is one (tap, 64-channel group):
//                    a 5-D TMA box {128 B, TW, TH, 1, 1} at (group,
//                    ow0 + kw*dw - pw, oh0 + kh*dh - ph, od + kd*dd - pd, n)
//                    gathers the shifted input window
//                    (out-of-range rows and columns -- the padding -- load as
//                    zero), a 2-D box brings the BN filters' rows, and four
//                    tcgen05 kind::i8 MMAs per 32-byte sub-block build the
//                    HH / MID / LL accumulators in TMEM.  Sixteen epilogue
//                    warps recombine exactly, dequantise, add the bias and
//                    store NCHW: lanes are consecutive pixels, so every
//                    store instruction is coalesced along the output row.
// The 128-row MMA covers TH*TW <= 128 pixels (TW = min(OW, 128)); rows past
// TH*TW hold stale shared memory and are never stored.  With BN = 64 the
// accumulators are double-buffered so the epilogue of one tile overlaps the
// MMAs of the next.
//   conv_win_kernel  the same MMA and epilogue for up to 64 filters and
//                    filters larger than 1x1: the input is stored
//                    zero-padded and each 128-position tile loads one halo
//                    window per channel group that every tap reads at its
//                    own row offset; when the filter block fits (<= 96 KB)
//                    it stays resident in shared memory.
//   conv_stk_kernel  the window kernel with both weight limbs stacked along
//                    N (two N = 144 MMAs per sub-block instead of four).
//   conv1x1_q_kernel 1x1 filters (fp16, <= 64 filters, <= 256 channels):
//                    no limb pass -- the input is read as fp16 NCHW boxes
//                    and quantised into the limb tiles inside the kernel.
// Every wait is bounded; no TMA multicast is used.
#include <cuda.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>
#include <utility>

#include "tk_internal.h"
#include "tk_numerics.cuh"
#include "tk_ptx.cuh"

namespace tk {
namespace {

constexpr int BM = 128;
constexpr int KB = 128;  // bytes per K step: one 64-channel group, both limbs
constexpr int NUM_EPI_WARPS = 16;  // four per TMEM lane quarter
constexpr int NUM_THREADS = 64 + 32 * NUM_EPI_WARPS;
constexpr uint32_t TMEM_COLS = 512;
constexpr int A_BYTES = BM * KB;

// K steps are small (one 64-channel group, 8 MMAs), so the ring is deep to
// keep enough TMA bytes in flight to cover L2 latency.
template <int BN_, int NBUF_, int STAGES_>
struct ConvCfg {
    static constexpr int BN = BN_;
    static constexpr int NBUF = NBUF_;
    static constexpr int STAGES = STAGES_;
    static constexpr int B_BYTES = BN * KB;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int BUF_COLS = NBUF == 1 ? 3 * BN : 256;
    static constexpr int OFF_BAR = STAGES * STAGE_BYTES;
    static constexpr int SMEM = OFF_BAR + 256 + 1024;
    static constexpr uint32_t IDESC_SS = idesc_i8(BM, BN, true, true);
    static constexpr uint32_t IDESC_SU = idesc_i8(BM, BN, true, false);
    static constexpr uint32_t IDESC_US = idesc_i8(BM, BN, false, true);
    static constexpr uint32_t IDESC_UU = idesc_i8(BM, BN, false, false);
    static_assert(NBUF * BUF_COLS <= TMEM_COLS && 3 * BN <= BUF_COLS, "TMEM budget");
};
using ConvNarrow = ConvCfg<64, 2, 8>;
using ConvWide = ConvCfg<128, 1, 6>;

struct ConvTcParams {
    int N, F, OD, OH, OW, KD, KH, KW, pd, ph, pw, dd, dh, dw, Cg;
    int TH, TW, tiles_h, tiles_w, tiles_f, tiles;
    int num_kb;
    const float* amax_x;
    const float* amax_w;
    const void* bias;
    void* out;
    unsigned* err;
};

__device__ __forceinline__ void decode(const ConvTcParams& p, int t, int& n, int& od, int& oh0, int& ow0,
                                       int& fb) {
    fb = t % p.tiles_f;
    int r = t / p.tiles_f;
    const int tw = r % p.tiles_w;
    r /= p.tiles_w;
    const int th = r % p.tiles_h;
    r /= p.tiles_h;
    od = r % p.OD;
    n = r / p.OD;
    oh0 = th * p.TH;
    ow0 = tw * p.TW;
}

template <class C, int DT>
__global__ void __launch_bounds__(NUM_THREADS, 1)
conv_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
               const ConvTcParams p) {
    constexpr int BN = C::BN;
    constexpr int NBUF = C::NBUF;
    constexpr int STAGES = C::STAGES;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* full_bar = bars;
    uint64_t* empty_bar = bars + STAGES;
    uint64_t* acc_full = bars + 2 * STAGES;
    uint64_t* acc_empty = acc_full + NBUF;
    uint64_t* drain_bar = acc_empty + NBUF;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(full_bar + s), 1);
            mbar_init(smem_u32(empty_bar + s), 1);
        }
        for (int b = 0; b < NBUF; ++b) {
            mbar_init(smem_u32(acc_full + b), 1);
            mbar_init(smem_u32(acc_empty + b), NUM_EPI_WARPS);
        }
        mbar_init(smem_u32(drain_bar), 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmX);
        tma_prefetch_desc(&tmW);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();  // prologue done; the limbs (or fp16 input), weights and scales are read after this
    const uint32_t a_bytes = static_cast<uint32_t>(p.TH * p.TW * KB);

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        int stage = 0;
        uint32_t phase = 0;
        uint32_t last_phase[STAGES];
        bool used[STAGES];
        for (int s = 0; s < STAGES; ++s) { used[s] = false; last_phase[s] = 0; }
        bool ok = true;
        for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x) {
            int n, od, oh0, ow0, fb;
            decode(p, t, n, od, oh0, ow0, fb);
            int cg = 0, kw = 0, kh = 0, kd = 0;
            for (int kb = 0; kb < p.num_kb; ++kb) {
                if (!mbar_wait_bounded(smem_u32(empty_bar + stage), phase ^ 1u, abort_flag, p.err,
                                       kDevErrWaitEmpty)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    const uint32_t fbar = smem_u32(full_bar + stage);
                    uint8_t* sb = smem + stage * C::STAGE_BYTES;
                    mbar_arrive_expect_tx(fbar, a_bytes + C::B_BYTES);
                    tma_load_5d(smem_u32(sb), &tmX, fbar, cg * KB, ow0 + kw * p.dw - p.pw,
                                oh0 + kh * p.dh - p.ph, od + kd * p.dd - p.pd, n);
                    tma_load_3d(smem_u32(sb + A_BYTES), &tmW, fbar, kb * KB, fb * BN, 0);
                }
                __syncwarp();
                used[stage] = true;
                last_phase[stage] = phase;
                if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                if (++cg == p.Cg) {
                    cg = 0;
                    if (++kw == p.KW) {
                        kw = 0;
                        if (++kh == p.KH) { kh = 0; ++kd; }
                    }
                }
            }
        }
        volatile int no_abort = 0;
        for (int s = 0; s < STAGES; ++s)
            if (used[s])
                mbar_wait_bounded(smem_u32(full_bar + s), last_phase[s], &no_abort, p.err, kDevErrWaitDrain);
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        int local = 0;
        for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x, ++local) {
            const int buf = local % NBUF;
            const uint32_t acc_phase = static_cast<uint32_t>(local / NBUF) & 1u;
            if (!mbar_wait_bounded(smem_u32(acc_empty + buf), acc_phase ^ 1u, abort_flag, p.err,
                                   kDevErrWaitAccEmpty))
                break;
            tc_fence_after();
            const uint32_t acc_hh = tmem_base + buf * C::BUF_COLS;
            const uint32_t acc_mid = acc_hh + BN;
            const uint32_t acc_ll = acc_hh + 2 * BN;
            for (int kb = 0; kb < p.num_kb; ++kb) {
                if (!mbar_wait_bounded(smem_u32(full_bar + stage), phase, abort_flag, p.err,
                                       kDevErrWaitFull)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t sb = smem_u32(smem + stage * C::STAGE_BYTES);
                    const uint64_t a0 = smem_desc_kmajor_sw128(sb);
                    const uint64_t b0 = smem_desc_kmajor_sw128(sb + A_BYTES);
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const uint64_t hi = static_cast<uint64_t>((u * 32) >> 4);
                        const uint64_t lo = static_cast<uint64_t>((64 + u * 32) >> 4);
                        const uint32_t acc = (kb > 0 || u > 0) ? 1u : 0u;
                        tc_mma_i8(acc_hh, a0 + hi, b0 + hi, C::IDESC_SS, acc);
                        tc_mma_i8(acc_mid, a0 + hi, b0 + lo, C::IDESC_SU, acc);
                        tc_mma_i8(acc_mid, a0 + lo, b0 + hi, C::IDESC_US, 1u);
                        tc_mma_i8(acc_ll, a0 + lo, b0 + lo, C::IDESC_UU, acc);
                    }
                    tc_commit(smem_u32(empty_bar + stage));
                }
                __syncwarp();
                if (++stage == STAGES) { stage = 0; phase ^= 1u; }
            }
            if (!ok) break;
            if (lane == 0) tc_commit(smem_u32(acc_full + buf));
            __syncwarp();
        }
        if (lane == 0) tc_commit(smem_u32(drain_bar));
        __syncwarp();
        volatile int no_abort = 0;
        mbar_wait_bounded(smem_u32(drain_bar), 0, &no_abort, p.err, kDevErrWaitDrain);
    } else {
        // ---------------- epilogue (warps 2..9) ----------------
        const int quarter = warp & 3;
        const int sub = (warp - 2) >> 2;  // which quarter of the BN columns
        const int row = quarter * 32 + lane;
        const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
        const double s = dequant_scale(__ldg(p.amax_x), __ldg(p.amax_w));
        const int64_t plane = static_cast<int64_t>(p.OD) * p.OH * p.OW;
        const int th = row / p.TW, tw = row - (row / p.TW) * p.TW;
        constexpr int ES = DT == 0 ? 2 : 4;
        int local = 0;
        for (int t = blockIdx.x; t < p.tiles; t += gridDim.x, ++local) {
            int n, od, oh0, ow0, fb;
            decode(p, t, n, od, oh0, ow0, fb);
            const int buf = local % NBUF;
            const uint32_t acc_phase = static_cast<uint32_t>(local / NBUF) & 1u;
            if (!mbar_wait_bounded(smem_u32(acc_full + buf), acc_phase, abort_flag, p.err,
                                   kDevErrWaitAccFull))
                break;
            tc_fence_after();
            const uint32_t t_buf = t_row + buf * C::BUF_COLS;
            const int oh = oh0 + th, ow = ow0 + tw;
            const bool pix_ok = row < p.TH * p.TW && oh < p.OH && ow < p.OW;
            const int64_t pix = (static_cast<int64_t>(od) * p.OH + oh) * p.OW + ow;
#pragma unroll 1
            for (int c = sub * (BN / 64); c < (sub + 1) * (BN / 64); ++c) {  // 16-column blocks
                uint32_t hh[16], mid[16], ll[16];
                tmem_ld_32x32b_x16(t_buf + c * 16, hh);
                tmem_ld_32x32b_x16(t_buf + BN + c * 16, mid);
                tmem_ld_32x32b_x16(t_buf + 2 * BN + c * 16, ll);
                tc_wait_ld();
                const int f0 = fb * BN + c * 16;
                if (!pix_ok || f0 >= p.F) continue;
                // column f of this pixel sits plane elements after column f - 1
                char* o = static_cast<char*>(p.out) + ((static_cast<int64_t>(n) * p.F + f0) * plane + pix) * ES;
                const int64_t step = plane * ES;
                const int nf = min(16, p.F - f0);
                if constexpr (DT == 0) {
                    // T(acc * s) rounds once from binary64 to binary16; the bias
                    // add in binary16 equals the binary32 add rounded to binary16
                    // (binary32 carries more than 2*11 + 2 significand bits).
                    __half bv[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) bv[j] = __ushort_as_half(0);
                    if (p.bias != nullptr) {
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            if (j < nf) bv[j] = static_cast<const __half*>(p.bias)[f0 + j];
                    }
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        __half h = __double2half(__dmul_rn(limb_acc_to_double(hh[j], mid[j], ll[j]), s));
                        if (p.bias != nullptr) h = __hadd(h, bv[j]);
                        if (j < nf) *reinterpret_cast<__half*>(o + j * step) = h;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        if (j < nf) {
                            float v = __double2float_rn(__dmul_rn(limb_acc_to_double(hh[j], mid[j], ll[j]), s));
                            if (p.bias != nullptr) v = __fadd_rn(v, static_cast<const float*>(p.bias)[f0 + j]);
                            *reinterpret_cast<float*>(o + j * step) = v;
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(acc_empty + buf));
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// ---- window variant: one halo window per channel group for all taps ----------
//
// With the input stored zero-padded ([N][H+2ph][W+2pw] limb rows) the output
// pixel (oh, ow) maps to the linear position r = oh*Wp + ow of the padded
// plane, and tap (kh, kw) reads the input row r + kh*dh*Wp + kw*dw.  A tile
// of 128 consecutive positions therefore needs, per channel group, one window
// of 128 + max_tap_offset rows; the MMA for each tap reads 128 rows of it
// starting at that tap's offset.  The window buffer is 1024-byte aligned and
// the 128B swizzle is a function of the shared-memory address, so a plain
// descriptor at any 128-byte row reads the rows TMA wrote there (no matrix
// base offset).  Positions with ow >= OW are computed and not stored.
// The input crosses L2 once per channel group instead of once per tap.

constexpr int WIN_ROWS = 256;           // window buffer rows (TMA box limit)
constexpr int WIN_BYTES = WIN_ROWS * KB;
constexpr int kMaxTaps = 32;

// RES: the whole weight block of the (single) filter tile stays in shared
// memory for the CTA's lifetime -- loaded once, no per-tap weight loads.
constexpr int kResWeightBytes = 96 * 1024;

template <int BN_, int NBUF_, int SB_, bool RES_>
struct WinCfg {
    static constexpr int BN = BN_;
    static constexpr int NBUF = NBUF_;
    static constexpr int SB = SB_;  // weight-tile ring depth
    static constexpr bool RES = RES_;
    static constexpr int B_BYTES = BN * KB;
    static constexpr int BUF_COLS = NBUF == 1 ? 3 * BN : 256;
    static constexpr int OFF_B = 2 * WIN_BYTES;
    static constexpr int OFF_BAR = OFF_B + (RES ? kResWeightBytes : SB * B_BYTES);
    static constexpr int SMEM = OFF_BAR + 512 + 1024;
    static constexpr uint32_t IDESC_SS = idesc_i8(BM, BN, true, true);
    static constexpr uint32_t IDESC_SU = idesc_i8(BM, BN, true, false);
    static constexpr uint32_t IDESC_US = idesc_i8(BM, BN, false, true);
    static constexpr uint32_t IDESC_UU = idesc_i8(BM, BN, false, false);
    static_assert(NBUF * BUF_COLS <= TMEM_COLS && 3 * BN <= BUF_COLS, "TMEM budget");
};
using WinNarrow = WinCfg<64, 2, 8, false>;
using WinResident = WinCfg<64, 2, 1, true>;

struct ConvWinParams {
    int N, F, OH, OW, Hp, Wp, Cg, taps;
    int win_rows;            // rows loaded per window (<= WIN_ROWS)
    int pos_tiles, tiles_f, tiles;
    int tap_off[kMaxTaps];   // row offset of each tap inside the window
    const float* amax_x;
    const float* amax_w;
    const void* bias;
    void* out;
    unsigned* err;
    int clamp_x;             // conv1x1_q_kernel: the input scale was supplied, clamp the codes
    const __half* w;         // conv1x1_q_kernel: fp16 weights [F][C], stacked in the kernel
    int C;                   // conv1x1_q_kernel: input channels
    int w_vec;               // conv1x1_q_kernel: 16-byte weight loads (C % 8 == 0, aligned)
};

template <class C, int DT>
__global__ void __launch_bounds__(NUM_THREADS, 1)
conv_win_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                const ConvWinParams p) {
    constexpr int BN = C::BN;
    constexpr int NBUF = C::NBUF;
    constexpr int SB = C::SB;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* a_full = bars;             // [2]
    uint64_t* a_empty = bars + 2;        // [2]
    uint64_t* b_full = bars + 4;         // [SB]
    uint64_t* b_empty = b_full + SB;     // [SB]
    uint64_t* acc_full = b_empty + SB;   // [NBUF]
    uint64_t* acc_empty = acc_full + NBUF;
    uint64_t* drain_bar = acc_empty + NBUF;
    uint64_t* w_full = drain_bar + 1;    // resident weights landed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(w_full + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    constexpr bool RES = C::RES;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(w_full), 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(smem_u32(a_full + i), 1);
            mbar_init(smem_u32(a_empty + i), 1);
        }
        for (int i = 0; i < SB; ++i) {
            mbar_init(smem_u32(b_full + i), 1);
            mbar_init(smem_u32(b_empty + i), 1);
        }
        for (int i = 0; i < NBUF; ++i) {
            mbar_init(smem_u32(acc_full + i), 1);
            mbar_init(smem_u32(acc_empty + i), NUM_EPI_WARPS);
        }
        mbar_init(smem_u32(drain_bar), 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmX);
        tma_prefetch_desc(&tmW);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();  // prologue done; the limbs (or fp16 input), weights and scales are read after this
    const int64_t plane = static_cast<int64_t>(p.Hp) * p.Wp;

    if (warp == 0) {
        // ---------------- TMA producer: window per channel group, weights per tap ----------------
        int ab = 0, bs = 0;
        uint32_t aph = 0, bph = 0;
        uint32_t a_last[2] = {0, 0}, b_last[SB];
        bool a_used[2] = {false, false}, b_used[SB];
        for (int i = 0; i < SB; ++i) { b_used[i] = false; b_last[i] = 0; }
        bool ok = true;
        if (RES) {
            // every (tap, group) weight tile of filter tile 0, once
            if (lane == 0) {
                const uint32_t fbar = smem_u32(w_full);
                mbar_arrive_expect_tx(fbar, static_cast<uint32_t>(p.taps * p.Cg * C::B_BYTES));
                for (int kb = 0; kb < p.taps * p.Cg; ++kb)
                    tma_load_3d(smem_u32(smem + C::OFF_B + kb * C::B_BYTES), &tmW, fbar, kb * KB, 0, 0);
            }
            __syncwarp();
        }
        for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x) {
            const int fb = t % p.tiles_f;
            const int pt = (t / p.tiles_f) % p.pos_tiles;
            const int n = t / (p.tiles_f * p.pos_tiles);
            const int row0 = static_cast<int>(n * plane) + pt * BM;
            for (int g = 0; g < p.Cg && ok; ++g) {
                if (!mbar_wait_bounded(smem_u32(a_empty + ab), aph ^ 1u, abort_flag, p.err, kDevErrWaitEmpty)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    const uint32_t fbar = smem_u32(a_full + ab);
                    mbar_arrive_expect_tx(fbar, static_cast<uint32_t>(p.win_rows * KB));
                    tma_load_3d(smem_u32(smem + ab * WIN_BYTES), &tmX, fbar, g * KB, row0, 0);
                }
                __syncwarp();
                a_used[ab] = true;
                a_last[ab] = aph;
                if (++ab == 2) { ab = 0; aph ^= 1u; }
                for (int tap = 0; tap < p.taps && !RES; ++tap) {
                    if (!mbar_wait_bounded(smem_u32(b_empty + bs), bph ^ 1u, abort_flag, p.err, kDevErrWaitEmpty)) {
                        ok = false;
                        break;
                    }
                    if (lane == 0) {
                        const uint32_t fbar = smem_u32(b_full + bs);
                        mbar_arrive_expect_tx(fbar, C::B_BYTES);
                        tma_load_3d(smem_u32(smem + C::OFF_B + bs * C::B_BYTES), &tmW, fbar,
                                    (tap * p.Cg + g) * KB, fb * BN, 0);
                    }
                    __syncwarp();
                    b_used[bs] = true;
                    b_last[bs] = bph;
                    if (++bs == SB) { bs = 0; bph ^= 1u; }
                }
            }
        }
        volatile int no_abort = 0;
        if (RES) mbar_wait_bounded(smem_u32(w_full), 0, &no_abort, p.err, kDevErrWaitDrain);
        for (int i = 0; i < 2; ++i)
            if (a_used[i]) mbar_wait_bounded(smem_u32(a_full + i), a_last[i], &no_abort, p.err, kDevErrWaitDrain);
        for (int i = 0; i < SB; ++i)
            if (b_used[i]) mbar_wait_bounded(smem_u32(b_full + i), b_last[i], &no_abort, p.err, kDevErrWaitDrain);
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        int ab = 0, bs = 0;
        uint32_t aph = 0, bph = 0;
        bool ok = true;
        int local = 0;
        if (RES && !mbar_wait_bounded(smem_u32(w_full), 0, abort_flag, p.err, kDevErrWaitFull)) ok = false;
        for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x, ++local) {
            const int buf = local % NBUF;
            const uint32_t acc_phase = static_cast<uint32_t>(local / NBUF) & 1u;
            if (!mbar_wait_bounded(smem_u32(acc_empty + buf), acc_phase ^ 1u, abort_flag, p.err,
                                   kDevErrWaitAccEmpty))
                break;
            tc_fence_after();
            const uint32_t acc_hh = tmem_base + buf * C::BUF_COLS;
            const uint32_t acc_mid = acc_hh + BN;
            const uint32_t acc_ll = acc_hh + 2 * BN;
            for (int g = 0; g < p.Cg && ok; ++g) {
                if (!mbar_wait_bounded(smem_u32(a_full + ab), aph, abort_flag, p.err, kDevErrWaitFull)) {
                    ok = false;
                    break;
                }
                const uint32_t win = smem_u32(smem + ab * WIN_BYTES);
                for (int tap = 0; tap < p.taps; ++tap) {
                    if (!RES && !mbar_wait_bounded(smem_u32(b_full + bs), bph, abort_flag, p.err, kDevErrWaitFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (lane == 0) {
                        const uint32_t a_row = win + static_cast<uint32_t>(p.tap_off[tap]) * KB;
                        const uint32_t b_tile = smem_u32(
                            smem + C::OFF_B + (RES ? (tap * p.Cg + g) : bs) * C::B_BYTES);
#pragma unroll
                        for (int u = 0; u < 2; ++u) {
                            const uint64_t a_hi = smem_desc_kmajor_sw128(a_row + u * 32);
                            const uint64_t a_lo = smem_desc_kmajor_sw128(a_row + 64 + u * 32);
                            const uint64_t b_hi = smem_desc_kmajor_sw128(b_tile + u * 32);
                            const uint64_t b_lo = smem_desc_kmajor_sw128(b_tile + 64 + u * 32);
                            const uint32_t acc = (g > 0 || tap > 0 || u > 0) ? 1u : 0u;
                            tc_mma_i8(acc_hh, a_hi, b_hi, C::IDESC_SS, acc);
                            tc_mma_i8(acc_mid, a_hi, b_lo, C::IDESC_SU, acc);
                            tc_mma_i8(acc_mid, a_lo, b_hi, C::IDESC_US, 1u);
                            tc_mma_i8(acc_ll, a_lo, b_lo, C::IDESC_UU, acc);
                        }
                        if (!RES) tc_commit(smem_u32(b_empty + bs));
                    }
                    __syncwarp();
                    if (!RES && ++bs == SB) { bs = 0; bph ^= 1u; }
                }
                if (!ok) break;
                if (lane == 0) tc_commit(smem_u32(a_empty + ab));
                __syncwarp();
                if (++ab == 2) { ab = 0; aph ^= 1u; }
            }
            if (!ok) break;
            if (lane == 0) tc_commit(smem_u32(acc_full + buf));
            __syncwarp();
        }
        if (lane == 0) tc_commit(smem_u32(drain_bar));
        __syncwarp();
        volatile int no_abort = 0;
        mbar_wait_bounded(smem_u32(drain_bar), 0, &no_abort, p.err, kDevErrWaitDrain);
    } else {
        // ---------------- epilogue (warps 2..17) ----------------
        const int quarter = warp & 3;
        const int sub = (warp - 2) >> 2;
        const int row = quarter * 32 + lane;
        const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
        const double s = dequant_scale(__ldg(p.amax_x), __ldg(p.amax_w));
        const int64_t oplane = static_cast<int64_t>(p.OH) * p.OW;
        constexpr int ES = DT == 0 ? 2 : 4;
        int local = 0;
        for (int t = blockIdx.x; t < p.tiles; t += gridDim.x, ++local) {
            const int fb = t % p.tiles_f;
            const int pt = (t / p.tiles_f) % p.pos_tiles;
            const int n = t / (p.tiles_f * p.pos_tiles);
            const int buf = local % NBUF;
            const uint32_t acc_phase = static_cast<uint32_t>(local / NBUF) & 1u;
            if (!mbar_wait_bounded(smem_u32(acc_full + buf), acc_phase, abort_flag, p.err, kDevErrWaitAccFull))
                break;
            tc_fence_after();
            const uint32_t t_buf = t_row + buf * C::BUF_COLS;
            const int pos = pt * BM + row;
            const int oh = pos / p.Wp, ow = pos - (pos / p.Wp) * p.Wp;
            const bool pix_ok = oh < p.OH && ow < p.OW;
            const int64_t pix = static_cast<int64_t>(oh) * p.OW + ow;
#pragma unroll 1
            for (int c = sub * (BN / 64); c < (sub + 1) * (BN / 64); ++c) {
                uint32_t hh[16], mid[16], ll[16];
                tmem_ld_32x32b_x16(t_buf + c * 16, hh);
                tmem_ld_32x32b_x16(t_buf + BN + c * 16, mid);
                tmem_ld_32x32b_x16(t_buf + 2 * BN + c * 16, ll);
                tc_wait_ld();
                const int f0 = fb * BN + c * 16;
                if (!pix_ok || f0 >= p.F) continue;
                char* o = static_cast<char*>(p.out) + ((static_cast<int64_t>(n) * p.F + f0) * oplane + pix) * ES;
                const int64_t step = oplane * ES;
                const int nf = min(16, p.F - f0);
                if constexpr (DT == 0) {
                    __half bv[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) bv[j] = __ushort_as_half(0);
                    if (p.bias != nullptr) {
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            if (j < nf) bv[j] = static_cast<const __half*>(p.bias)[f0 + j];
                    }
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        __half h = __double2half(__dmul_rn(limb_acc_to_double(hh[j], mid[j], ll[j]), s));
                        if (p.bias != nullptr) h = __hadd(h, bv[j]);
                        if (j < nf) *reinterpret_cast<__half*>(o + j * step) = h;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        if (j < nf) {
                            float v = __double2float_rn(__dmul_rn(limb_acc_to_double(hh[j], mid[j], ll[j]), s));
                            if (p.bias != nullptr) v = __fadd_rn(v, static_cast<const float*>(p.bias)[f0 + j]);
                            *reinterpret_cast<float*>(o + j * step) = v;
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(acc_empty + buf));
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// ---- stacked-limb window variant: two wide MMAs per K sub-block -------------
//
// For up to 64 filters the four limb products per 32-channel sub-block
// (hi*hi, hi*lo, lo*hi, lo*lo) are four N = 64 MMAs that each re-read their
// 4 KB A tile for 262K MACs.  Here both weight limbs are stacked along N in
// one unsigned operand -- rows 0-63 the hi limbs offset to u8 (b_hi + 128),
// rows 64-127 the lo limbs, rows 128-143 all ones -- so each sub-block is two
// N = 144 MMAs: acc1 = a_hi x stack, acc2 = a_lo x stack.  With
// S_hi = sum a_hi and S_lo = sum a_lo (the ones columns):
//   HH  = acc1[f] - 128 S_hi
//   MID = acc1[64 + f] + acc2[f] - 128 S_lo
//   LL  = acc2[64 + f]
// all exact in 32-bit two's complement (every true value fits; |acc2| <=
// 255 * 255 * 32768 < 2^31).  Two K steps (tap, group) share one 128-byte
// weight row: step 2p + h sits at byte 64 h of pair p's 144-row tile.  The
// whole stacked filter block stays resident; the epilogue copies the
// accumulators out of TMEM and releases them before its arithmetic, so the
// single accumulator buffer (288 of 512 columns) overlaps the next tile.
// Four input windows are in flight, so 1x1 convolutions with several channel
// groups (one 16 KB window each) keep enough TMA bytes outstanding.

constexpr int STK_N = 144;
constexpr int STK_TILE = STK_N * KB;             // bytes per pair of K steps
constexpr int STK_MAX_PAIRS = kResWeightBytes / STK_TILE;
constexpr int STK_NWIN = 4;                     // input windows in flight
constexpr int STK_OFF_B = STK_NWIN * WIN_BYTES;
constexpr int STK_OFF_BAR = STK_OFF_B + STK_MAX_PAIRS * STK_TILE;
constexpr int STK_SMEM = STK_OFF_BAR + 256 + 1024;
constexpr uint32_t STK_IDESC_SU = idesc_i8(BM, STK_N, true, false);
constexpr uint32_t STK_IDESC_UU = idesc_i8(BM, STK_N, false, false);
static_assert(STK_TILE % 1024 == 0, "stacked tiles keep the 1024-byte swizzle alignment");
static_assert(STK_SMEM <= 227 * 1024, "stacked kernel fits the shared-memory limit of one CTA");

template <int DT>
__global__ void __launch_bounds__(NUM_THREADS, 1)
conv_stk_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                const ConvWinParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STK_OFF_BAR);
    uint64_t* a_full = bars;
    uint64_t* a_empty = bars + STK_NWIN;
    uint64_t* acc_full = bars + 2 * STK_NWIN;
    uint64_t* acc_empty = acc_full + 1;
    uint64_t* drain_bar = acc_full + 2;
    uint64_t* w_full = acc_full + 3;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 4);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int nkb = p.taps * p.Cg;
    const int npairs = (nkb + 1) / 2;
    if (threadIdx.x == 0) {
        for (int i = 0; i < STK_NWIN; ++i) {
            mbar_init(smem_u32(a_full + i), 1);
            mbar_init(smem_u32(a_empty + i), 1);
        }
        mbar_init(smem_u32(acc_full), 1);
        mbar_init(smem_u32(acc_empty), NUM_EPI_WARPS);
        mbar_init(smem_u32(drain_bar), 1);
        mbar_init(smem_u32(w_full), 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmX);
        tma_prefetch_desc(&tmW);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();  // prologue done; the limbs (or fp16 input), weights and scales are read after this
    const int64_t plane = static_cast<int64_t>(p.Hp) * p.Wp;

    if (warp == 0) {
        // ---------------- TMA producer: stacked weights once, a window per channel group ----------------
        int ab = 0;
        uint32_t aph = 0;
        uint32_t a_last[STK_NWIN];
        bool a_used[STK_NWIN];
        for (int i = 0; i < STK_NWIN; ++i) { a_last[i] = 0; a_used[i] = false; }
        bool ok = true;
        if (lane == 0) {
            const uint32_t fbar = smem_u32(w_full);
            mbar_arrive_expect_tx(fbar, static_cast<uint32_t>(npairs * STK_TILE));
            for (int q = 0; q < npairs; ++q)
                tma_load_3d(smem_u32(smem + STK_OFF_B + q * STK_TILE), &tmW, fbar, 0, q * STK_N, 0);
        }
        __syncwarp();
        for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x) {
            const int pt = t % p.pos_tiles;
            const int n = t / p.pos_tiles;
            const int row0 = static_cast<int>(n * plane) + pt * BM;
            for (int g = 0; g < p.Cg && ok; ++g) {
                if (!mbar_wait_bounded(smem_u32(a_empty + ab), aph ^ 1u, abort_flag, p.err, kDevErrWaitEmpty)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    const uint32_t fbar = smem_u32(a_full + ab);
                    mbar_arrive_expect_tx(fbar, static_cast<uint32_t>(p.win_rows * KB));
                    tma_load_3d(smem_u32(smem + ab * WIN_BYTES), &tmX, fbar, g * KB, row0, 0);
                }
                __syncwarp();
                a_used[ab] = true;
                a_last[ab] = aph;
                if (++ab == STK_NWIN) { ab = 0; aph ^= 1u; }
            }
        }
        volatile int no_abort = 0;
        mbar_wait_bounded(smem_u32(w_full), 0, &no_abort, p.err, kDevErrWaitDrain);
        for (int i = 0; i < STK_NWIN; ++i)
            if (a_used[i]) mbar_wait_bounded(smem_u32(a_full + i), a_last[i], &no_abort, p.err, kDevErrWaitDrain);
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        int ab = 0;
        uint32_t aph = 0;
        bool ok = mbar_wait_bounded(smem_u32(w_full), 0, abort_flag, p.err, kDevErrWaitFull);
        int local = 0;
        const uint32_t acc1 = tmem_base, acc2 = tmem_base + STK_N;
        for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x, ++local) {
            if (!mbar_wait_bounded(smem_u32(acc_empty), (static_cast<uint32_t>(local) & 1u) ^ 1u, abort_flag,
                                   p.err, kDevErrWaitAccEmpty))
                break;
            tc_fence_after();
            for (int g = 0; g < p.Cg && ok; ++g) {
                if (!mbar_wait_bounded(smem_u32(a_full + ab), aph, abort_flag, p.err, kDevErrWaitFull)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t win = smem_u32(smem + ab * WIN_BYTES);
                if (lane == 0) {
                    for (int tap = 0; tap < p.taps; ++tap) {
                        const int kb = tap * p.Cg + g;
                        const uint32_t a_row = win + static_cast<uint32_t>(p.tap_off[tap]) * KB;
                        const uint32_t b_row = smem_u32(smem + STK_OFF_B + (kb >> 1) * STK_TILE) + (kb & 1) * 64;
#pragma unroll
                        for (int u = 0; u < 2; ++u) {
                            const uint64_t a_hi = smem_desc_kmajor_sw128(a_row + u * 32);
                            const uint64_t a_lo = smem_desc_kmajor_sw128(a_row + 64 + u * 32);
                            const uint64_t b = smem_desc_kmajor_sw128(b_row + u * 32);
                            const uint32_t acc = (g > 0 || tap > 0 || u > 0) ? 1u : 0u;
                            tc_mma_i8(acc1, a_hi, b, STK_IDESC_SU, acc);
                            tc_mma_i8(acc2, a_lo, b, STK_IDESC_UU, acc);
                        }
                    }
                    tc_commit(smem_u32(a_empty + ab));
                }
                __syncwarp();
                if (++ab == STK_NWIN) { ab = 0; aph ^= 1u; }
            }
            if (!ok) break;
            if (lane == 0) tc_commit(smem_u32(acc_full));
            __syncwarp();
        }
        if (lane == 0) tc_commit(smem_u32(drain_bar));
        __syncwarp();
        volatile int no_abort = 0;
        mbar_wait_bounded(smem_u32(drain_bar), 0, &no_abort, p.err, kDevErrWaitDrain);
    } else {
        // ---------------- epilogue (warps 2..17): 16 filters of 32 positions each ----------------
        const int quarter = warp & 3;
        const int sub = (warp - 2) >> 2;
        const int row = quarter * 32 + lane;
        const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
        const double s = dequant_scale(__ldg(p.amax_x), __ldg(p.amax_w));
        const int64_t oplane = static_cast<int64_t>(p.OH) * p.OW;
        constexpr int ES = DT == 0 ? 2 : 4;
        const int f0 = sub * 16;
        int local = 0;
        for (int t = blockIdx.x; t < p.tiles; t += gridDim.x, ++local) {
            const int pt = t % p.pos_tiles;
            const int n = t / p.pos_tiles;
            if (!mbar_wait_bounded(smem_u32(acc_full), static_cast<uint32_t>(local) & 1u, abort_flag, p.err,
                                   kDevErrWaitAccFull))
                break;
            tc_fence_after();
            uint32_t h1[16], m1[16], m2[16], l2[16], s_hi, s_lo;
            tmem_ld_32x32b_x16(t_row + f0, h1);
            tmem_ld_32x32b_x16(t_row + 64 + f0, m1);
            tmem_ld_32x32b_x16(t_row + STK_N + f0, m2);
            tmem_ld_32x32b_x16(t_row + STK_N + 64 + f0, l2);
            tmem_ld_32x32b_x1(t_row + 128, s_hi);
            tmem_ld_32x32b_x1(t_row + STK_N + 128, s_lo);
            tc_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(acc_empty));  // TMEM free for the next tile
            const int pos = pt * BM + row;
            const int oh = pos / p.Wp, ow = pos - (pos / p.Wp) * p.Wp;
            if (oh >= p.OH || ow >= p.OW || f0 >= p.F) continue;
            const int64_t pix = static_cast<int64_t>(oh) * p.OW + ow;
            char* o = static_cast<char*>(p.out) + ((static_cast<int64_t>(n) * p.F + f0) * oplane + pix) * ES;
            const int64_t step = oplane * ES;
            const int nf = min(16, p.F - f0);
            const uint32_t c_hi = 128u * s_hi, c_lo = 128u * s_lo;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const uint32_t hh = h1[j] - c_hi;
                const uint32_t mid = m1[j] + m2[j] - c_lo;
                const double v = __dmul_rn(limb_acc_to_double(hh, mid, l2[j]), s);
                if constexpr (DT == 0) {
                    __half h = __double2half(v);
                    if (p.bias != nullptr) h = __hadd(h, static_cast<const __half*>(p.bias)[f0 + j < p.F ? f0 + j : 0]);
                    if (j < nf) *reinterpret_cast<__half*>(o + j * step) = h;
                } else {
                    float r = __double2float_rn(v);
                    if (p.bias != nullptr) r = __fadd_rn(r, static_cast<const float*>(p.bias)[f0 + j < p.F ? f0 + j : 0]);
                    if (j < nf) *reinterpret_cast<float*>(o + j * step) = r;
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// ---- 1x1 convolution with the input quantised inside the kernel -------------
//
// For a 1x1 filter (stride 1, no padding, groups 1, at most 64 filters, fp16
// input with a plane of 8k pixels) the implicit GEMM needs no halo, so the
// input limbs need not be staged in HBM: the TMA warp loads fp16 boxes of
// 64 channels x 128 consecutive pixels straight from the NCHW input, the 16
// worker warps quantise them (the library's codes, magic-number rounding)
// into the swizzled K-major limb tile the MMAs read, and the stacked-limb
// MMAs of conv_stk_kernel accumulate the tile.  The same workers run the
// epilogue of the previous tile while the MMA warp works on the next, so
// the input crosses HBM once after its amax pass (the limb pass read it and
// wrote and re-read 2 bytes per element).
constexpr int Q1_NRAW = 4;                         // fp16 input boxes in flight
constexpr int Q1_NA = 4;                           // limb tiles in flight
constexpr int Q1_RAW_BYTES = 64 * BM * 2;          // 64 channels x 128 pixels fp16
// A tile's channel groups must all fit the limb-tile ring (the workers
// dequantise the previous tile only after quantising the current one, so the
// MMAs of the current tile cannot free limb tiles before its last group is
// in), and its stacked filter block must stay resident: C <= 256.
constexpr int Q1_MAX_PAIRS = 2;
static_assert(2 * Q1_MAX_PAIRS <= Q1_NA, "every channel group of a tile fits the limb-tile ring");
constexpr int Q1_OFF_A = Q1_NRAW * Q1_RAW_BYTES;
constexpr int Q1_OFF_B = Q1_OFF_A + Q1_NA * A_BYTES;
constexpr int Q1_OFF_BAR = Q1_OFF_B + Q1_MAX_PAIRS * STK_TILE;
constexpr int Q1_SMEM = Q1_OFF_BAR + 256 + 1024;
static_assert(Q1_OFF_A % 1024 == 0 && Q1_OFF_B % 1024 == 0, "swizzled tiles on 1024-byte boundaries");
static_assert(Q1_SMEM <= 227 * 1024, "fits one CTA's shared memory");
static_assert(NUM_EPI_WARPS == 16, "four worker warps per lane quarter");

// The stacked filter block of conv1x1_q_kernel (the layout of
// w_stack_blocks, swizzled as the MMAs read it) written by the 512 worker
// threads into `stk`: 16-byte piece `pc8` of row n of pair `pair`, one piece
// per thread at a time.  Out of line, so its temporaries do not crowd the
// registers of the quantise / epilogue loop.
__device__ __noinline__ void stack_weights_1x1(uint8_t* stk, const __half* w, const float* amax_w, int F, int C,
                                               bool w_vec, int npairs, int Cg, int wt) {
    const float inv_w = quant_inv(__ldg(amax_w));
    const int pieces = npairs * STK_N * 8;
    for (int it = wt; it < pieces; it += NUM_EPI_WARPS * 32) {
        const int pc8 = it & 7, r = it >> 3;
        const int n = r % STK_N, pair = r / STK_N;
        const int kb = 2 * pair + (pc8 >> 2);  // the channel group
        const int c0 = kb * 64 + (pc8 & 3) * 16;
        uint32_t word[4];
        if (n >= 128) {
#pragma unroll
            for (int j = 0; j < 4; ++j) word[j] = 0x01010101u;
        } else {
            const int f = n & 63;
            const bool live = kb < Cg && f < F;
            const __half* wrow = w + static_cast<int64_t>(f) * C + c0;
            uint4 u0 = make_uint4(0, 0, 0, 0), u1 = make_uint4(0, 0, 0, 0);
            const bool vec = live && w_vec && c0 + 16 <= C;
            if (vec) {
                u0 = __ldg(reinterpret_cast<const uint4*>(wrow));
                u1 = __ldg(reinterpret_cast<const uint4*>(wrow) + 1);
            }
            const uint32_t wd[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t b = 0;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int c = 4 * j + e;
                    int v = 0;
                    if (vec)
                        v = quant_one(__half2float(__ushort_as_half(
                                          static_cast<unsigned short>(wd[c >> 1] >> (16 * (c & 1))))),
                                      inv_w);
                    else if (live && c0 + c < C) v = quant_one(__half2float(__ldg(wrow + c)), inv_w);
                    const uint32_t byte = n < 64 ? static_cast<uint32_t>(((v >> 8) + 128) & 0xFF)
                                                 : static_cast<uint32_t>(v & 0xFF);
                    b |= byte << (8 * e);
                }
                word[j] = b;
            }
        }
        *reinterpret_cast<uint4*>(stk + pair * STK_TILE + n * KB + ((pc8 ^ (n & 7)) << 4)) =
            make_uint4(word[0], word[1], word[2], word[3]);
    }
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
conv1x1_q_kernel(const __grid_constant__ CUtensorMap tmX, const ConvWinParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Q1_OFF_BAR);
    uint64_t* raw_full = bars;
    uint64_t* raw_empty = raw_full + Q1_NRAW;
    uint64_t* a_full = raw_empty + Q1_NRAW;
    uint64_t* a_empty = a_full + Q1_NA;
    uint64_t* acc_full = a_empty + Q1_NA;
    uint64_t* acc_empty = acc_full + 1;
    uint64_t* drain_bar = acc_full + 2;
    uint64_t* w_full = acc_full + 3;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 4);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int Cg = p.Cg;
    const int npairs = (Cg + 1) / 2;
    if (threadIdx.x == 0) {
        for (int i = 0; i < Q1_NRAW; ++i) {
            mbar_init(smem_u32(raw_full + i), 1);
            mbar_init(smem_u32(raw_empty + i), NUM_EPI_WARPS);
        }
        for (int i = 0; i < Q1_NA; ++i) {
            mbar_init(smem_u32(a_full + i), NUM_EPI_WARPS);
            mbar_init(smem_u32(a_empty + i), 1);
        }
        mbar_init(smem_u32(acc_full), 1);
        mbar_init(smem_u32(acc_empty), NUM_EPI_WARPS);
        mbar_init(smem_u32(drain_bar), 1);
        mbar_init(smem_u32(w_full), NUM_EPI_WARPS);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmX);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();  // prologue done; the limbs (or fp16 input), weights and scales are read after this

    if (warp == 0) {
        // ---------------- TMA: fp16 input boxes ----------------
        int rb = 0;
        uint32_t rph = 0;
        uint32_t r_last[Q1_NRAW];
        bool r_used[Q1_NRAW];
        for (int i = 0; i < Q1_NRAW; ++i) { r_last[i] = 0; r_used[i] = false; }
        bool ok = true;
        for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x) {
            const int pt = t % p.pos_tiles;
            const int n = t / p.pos_tiles;
            for (int g = 0; g < Cg; ++g) {
                if (!mbar_wait_bounded(smem_u32(raw_empty + rb), rph ^ 1u, abort_flag, p.err, kDevErrWaitEmpty)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    const uint32_t fbar = smem_u32(raw_full + rb);
                    mbar_arrive_expect_tx(fbar, Q1_RAW_BYTES);
                    tma_load_3d(smem_u32(smem + rb * Q1_RAW_BYTES), &tmX, fbar, pt * BM, g * 64, n);
                }
                __syncwarp();
                r_used[rb] = true;
                r_last[rb] = rph;
                if (++rb == Q1_NRAW) { rb = 0; rph ^= 1u; }
            }
        }
        volatile int no_abort = 0;
        for (int i = 0; i < Q1_NRAW; ++i)
            if (r_used[i]) mbar_wait_bounded(smem_u32(raw_full + i), r_last[i], &no_abort, p.err, kDevErrWaitDrain);
    } else if (warp == 1) {
        // ---------------- MMA issuer: two stacked MMAs per 32 channels ----------------
        int ab = 0;
        uint32_t aph = 0;
        bool ok = mbar_wait_bounded(smem_u32(w_full), 0, abort_flag, p.err, kDevErrWaitFull);
        int local = 0;
        const uint32_t acc1 = tmem_base, acc2 = tmem_base + STK_N;
        for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x, ++local) {
            if (!mbar_wait_bounded(smem_u32(acc_empty), (static_cast<uint32_t>(local) & 1u) ^ 1u, abort_flag,
                                   p.err, kDevErrWaitAccEmpty))
                break;
            tc_fence_after();
            for (int g = 0; g < Cg && ok; ++g) {
                if (!mbar_wait_bounded(smem_u32(a_full + ab), aph, abort_flag, p.err, kDevErrWaitFull)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t a_row = smem_u32(smem + Q1_OFF_A + ab * A_BYTES);
                    const uint32_t b_row = smem_u32(smem + Q1_OFF_B + (g >> 1) * STK_TILE) + (g & 1) * 64;
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const uint64_t a_hi = smem_desc_kmajor_sw128(a_row + u * 32);
                        const uint64_t a_lo = smem_desc_kmajor_sw128(a_row + 64 + u * 32);
                        const uint64_t b = smem_desc_kmajor_sw128(b_row + u * 32);
                        const uint32_t acc = (g > 0 || u > 0) ? 1u : 0u;
                        tc_mma_i8(acc1, a_hi, b, STK_IDESC_SU, acc);
                        tc_mma_i8(acc2, a_lo, b, STK_IDESC_UU, acc);
                    }
                    tc_commit(smem_u32(a_empty + ab));
                }
                __syncwarp();
                if (++ab == Q1_NA) { ab = 0; aph ^= 1u; }
            }
            if (!ok) break;
            if (lane == 0) tc_commit(smem_u32(acc_full));
            __syncwarp();
        }
        if (lane == 0) tc_commit(smem_u32(drain_bar));
        __syncwarp();
        volatile int no_abort = 0;
        mbar_wait_bounded(smem_u32(drain_bar), 0, &no_abort, p.err, kDevErrWaitDrain);
    } else {
        // ---------------- workers (warps 2..17): quantise the input boxes, then the epilogue ----------------
        const int wt = threadIdx.x - 64;
        const int px = wt & (BM - 1);          // the pixel (limb-tile row) this thread quantises
        const int cq = wt >> 7;                // its 16 channels: 16 cq .. 16 cq + 15
        const int sw = px & 7;
        const float inv_x = quant_inv(__ldg(p.amax_x));
        const int quarter = warp & 3;
        const int sub = (warp - 2) >> 2;
        const int row = quarter * 32 + lane;
        const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
        const double s = dequant_scale(__ldg(p.amax_x), __ldg(p.amax_w));
        const bool s_finite = s <= 1.7976931348623157e308;
        const int64_t plane = static_cast<int64_t>(p.OH) * p.OW;
        const int f0 = sub * 16;
        int rb = 0, ab = 0;
        uint32_t rph = 0, aph = 0;
        bool ok = true;
        // dequantise the accumulators of tile t (the local-th of this CTA)
        auto epilogue = [&](int t, int local) {
            const int pt = t % p.pos_tiles;
            const int n = t / p.pos_tiles;
            if (!mbar_wait_bounded(smem_u32(acc_full), static_cast<uint32_t>(local) & 1u, abort_flag, p.err,
                                   kDevErrWaitAccFull)) {
                ok = false;
                return;
            }
            tc_fence_after();
            uint32_t h1[16], m1[16], m2[16], l2[16], s_hi, s_lo;
            tmem_ld_32x32b_x16(t_row + f0, h1);
            tmem_ld_32x32b_x16(t_row + 64 + f0, m1);
            tmem_ld_32x32b_x16(t_row + STK_N + f0, m2);
            tmem_ld_32x32b_x16(t_row + STK_N + 64 + f0, l2);
            tmem_ld_32x32b_x1(t_row + 128, s_hi);
            tmem_ld_32x32b_x1(t_row + STK_N + 128, s_lo);
            tc_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(acc_empty));  // TMEM free for the next tile
            const int64_t pix = static_cast<int64_t>(pt) * BM + row;
            if (pix >= plane || f0 >= p.F) return;
            __half* o = static_cast<__half*>(p.out) + (static_cast<int64_t>(n) * p.F + f0) * plane + pix;
            const int nf = min(16, p.F - f0);
            const uint32_t c_hi = 128u * s_hi, c_lo = 128u * s_lo;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const uint32_t hh = h1[j] - c_hi;
                const uint32_t mid = m1[j] + m2[j] - c_lo;
                __half h = __double2half(__dmul_rn(limb_acc_to_double(hh, mid, l2[j]), s));
                // a non-finite scale (a NaN or an infinity in an operand) gives NaN
                // everywhere, whatever the codes of the non-finite inputs were
                h = s_finite ? h : __ushort_as_half(0x7E00);
                if (p.bias != nullptr) h = __hadd(h, static_cast<const __half*>(p.bias)[f0 + j < p.F ? f0 + j : 0]);
                if (j < nf) o[j * plane] = h;
            }
        };
        // the stacked filter block, while the TMA warp brings the first input boxes
        stack_weights_1x1(smem + Q1_OFF_B, p.w, p.amax_w, p.F, p.C, p.w_vec != 0, npairs, Cg, wt);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(w_full));
        // Half the warps of each SMSP (odd `sub`) run the previous tile's
        // epilogue before quantising this tile, the other half after it, so
        // the two latency-bound phases interleave on every SMSP.  Either
        // order only waits for work the other warps finished in their
        // previous iteration.
        const bool epi_first = (sub & 1) != 0;
        int local = 0, prev_t = -1;
        for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x, ++local) {
            if (epi_first && prev_t >= 0) {
                epilogue(prev_t, local - 1);
                if (!ok) break;
            }
            for (int g = 0; g < Cg; ++g) {
                if (!mbar_wait_bounded(smem_u32(raw_full + rb), rph, abort_flag, p.err, kDevErrWaitFull) ||
                    !mbar_wait_bounded(smem_u32(a_empty + ab), aph ^ 1u, abort_flag, p.err, kDevErrWaitEmpty)) {
                    ok = false;
                    break;
                }
                // channels 16 cq .. 16 cq + 15 of this pixel: codes, then the
                // hi limbs into 16-byte chunk cq and the lo limbs into chunk
                // 4 + cq of the pixel's 128-byte row (swizzled by row & 7)
                const __half* src = reinterpret_cast<const __half*>(smem + rb * Q1_RAW_BYTES) + (16 * cq) * BM + px;
                uint32_t hw[4], lw[4];
                if (p.clamp_x) {
#pragma unroll
                    for (int w4 = 0; w4 < 4; ++w4) {
                        uint32_t r[4];
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            r[k] = quant_code_bits_clamped(__half2float(src[(4 * w4 + k) * BM]), inv_x);
                        pack_codes4(r[0], r[1], r[2], r[3], hw[w4], lw[w4]);
                    }
                } else {
                    // the scale is this input's own max-abs: |v * inv| <= 32767.004,
                    // and a non-finite input makes every output NaN whatever its codes
#pragma unroll
                    for (int w4 = 0; w4 < 4; ++w4) {
                        uint32_t r[4];
#pragma unroll
                        for (int k = 0; k < 4; ++k) r[k] = quant_code_bits(__half2float(src[(4 * w4 + k) * BM]), inv_x);
                        pack_codes4(r[0], r[1], r[2], r[3], hw[w4], lw[w4]);
                    }
                }
                uint8_t* arow = smem + Q1_OFF_A + ab * A_BYTES + px * KB;
                *reinterpret_cast<uint4*>(arow + ((cq ^ sw) << 4)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                *reinterpret_cast<uint4*>(arow + (((4 + cq) ^ sw) << 4)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(smem_u32(raw_empty + rb));
                    mbar_arrive(smem_u32(a_full + ab));
                }
                if (++rb == Q1_NRAW) { rb = 0; rph ^= 1u; }
                if (++ab == Q1_NA) { ab = 0; aph ^= 1u; }
            }
            if (!ok) break;
            // the previous tile's epilogue runs while the MMAs of this one do
            if (!epi_first && prev_t >= 0) epilogue(prev_t, local - 1);
            prev_t = t;
        }
        if (ok && prev_t >= 0) epilogue(prev_t, local - 1);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// ---- operand quantisation into 128-byte limb rows ---------------------------

constexpr int XQ_W = 128;   // pixels per block pass
constexpr int XQ_THREADS = 256;

__device__ __forceinline__ int64_t ceil_div_dev(int64_t a, int64_t b) { return (a + b - 1) / b; }

template <typename T> __device__ __forceinline__ float ldt(const T* p, int64_t i);
template <> __device__ __forceinline__ float ldt<__half>(const __half* p, int64_t i) { return __half2float(__ldg(p + i)); }
template <> __device__ __forceinline__ float ldt<float>(const float* p, int64_t i) { return __ldg(p + i); }

__device__ __forceinline__ void pack16(const int16_t* q, int stride, uint4& hi, uint4& lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        h[w] = 0;
        l[w] = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int v = q[(4 * w + k) * stride];
            h[w] |= static_cast<uint32_t>((v >> 8) & 0xFF) << (8 * k);
            l[w] |= static_cast<uint32_t>(v & 0xFF) << (8 * k);
        }
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// One block per (image, 128-pixel run of the flattened D*H*W volume, 64-channel
// group).  Thread (cc4, pg) reads 4 channels x 8 consecutive pixels (16-byte
// vectors along the pixels when aligned) and forms their codes by
// magic-number rounding: RN(v * inv) + 1.5 * 2^23 as two unfused binary32
// operations holds RN(v * inv) rounded to the nearest integer (ties to even)
// in its low significand bits, so the low 16 bits are the int16 code that
// quant_one gives (the scaled value is clamped to the code range first, as
// the amax may be supplied by the caller; inv == 0 makes every code 0).  Byte permutes turn 4 channels' codes of one pixel
// into a hi word and a lo word, stored into the pixel's 128-byte shared row
// [hi of 64 channels | lo of 64 channels] -- the output row itself -- which
// phase 2 copies out with 16-byte stores.  A warp covers 8 pixel groups x 4
// channel quads (coalesced 128-byte loads per channel); the row's eight
// 16-byte chunks are XOR-swizzled by the pixel group, so each of its stores
// hits 32 different banks.
template <typename T>
__device__ __forceinline__ void x_limbs_block(const T* __restrict__ x, int C, int64_t HW, int W, int ph, int pw,
                                              int Hp, int Wp, int Cg, int vec, const float* __restrict__ amax,
                                              uint8_t* __restrict__ xl, int64_t bid) {
    static_assert(XQ_THREADS == 256 && XQ_W == 128, "16 channel quads x 16 pixel groups of 8");
    __shared__ __align__(16) uint32_t rows[XQ_W][32];
    const int64_t runs = ceil_div_dev(HW, XQ_W);
    const int g = static_cast<int>(bid % Cg);
    const int64_t r = bid / Cg;
    const int64_t p0 = (r % runs) * XQ_W;
    const int64_t n = r / runs;
    const int pn = static_cast<int>(HW - p0 < XQ_W ? HW - p0 : XQ_W);
    const float inv = quant_inv(__ldg(amax));
    const T* xs = x + (n * C + g * 64) * HW + p0;
    const int pg = (threadIdx.x & 7) + 8 * (threadIdx.x >> 7);
    const int cc4 = (threadIdx.x >> 3) & 15;
    const int pbase = pg * 8;
    uint32_t code[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int cl = cc4 * 4 + i;
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = 0.0f;
        if (g * 64 + cl < C && pbase < pn && inv != 0.0f) {
            const T* src = xs + static_cast<int64_t>(cl) * HW + pbase;
            if (vec && pbase + 8 <= pn) {
                if constexpr (sizeof(T) == 2) {
                    const uint4 u = __ldg(reinterpret_cast<const uint4*>(src));
                    const __half2* h2 = reinterpret_cast<const __half2*>(&u);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 f = __half22float2(h2[e]);
                        v[2 * e] = f.x;
                        v[2 * e + 1] = f.y;
                    }
                } else {
                    const float4 f0 = __ldg(reinterpret_cast<const float4*>(src));
                    const float4 f1 = __ldg(reinterpret_cast<const float4*>(src) + 1);
                    v[0] = f0.x; v[1] = f0.y; v[2] = f0.z; v[3] = f0.w;
                    v[4] = f1.x; v[5] = f1.y; v[6] = f1.z; v[7] = f1.w;
                }
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e)
                    if (pbase + e < pn) v[e] = ldt<T>(src, e);
            }
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) code[i][e] = quant_code_bits_clamped(v[e], inv);
    }
    const int swz = pg & 7;  // chunk swizzle of this pixel group's rows
    const int hi_w = 4 * ((cc4 >> 2) ^ swz) + (cc4 & 3);
    const int lo_w = 4 * ((4 + (cc4 >> 2)) ^ swz) + (cc4 & 3);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const uint32_t p01 = __byte_perm(code[0][e], code[1][e], 0x5410);
        const uint32_t p23 = __byte_perm(code[2][e], code[3][e], 0x5410);
        rows[pbase + e][hi_w] = __byte_perm(p01, p23, 0x7531);
        rows[pbase + e][lo_w] = __byte_perm(p01, p23, 0x6420);
    }
    __syncthreads();
    // pixel (h, w) of the plane is row (h + ph) * Wp + (w + pw) of the image's padded plane
    uint8_t* out = xl + (n * Hp * Wp * Cg + g) * static_cast<int64_t>(128);
    for (int it = threadIdx.x; it < pn * 8; it += XQ_THREADS) {
        const int pp = it >> 3, ch = it & 7;
        const int pix = static_cast<int>(p0) + pp;  // HW < 2^31
        int64_t prow = pix;
        if (ph | pw) {
            const int h = pix / W, w = pix - (pix / W) * W;
            prow = static_cast<int64_t>(h + ph) * Wp + (w + pw);
        }
        *reinterpret_cast<uint4*>(out + prow * (Cg * 128) + ch * 16) =
            *reinterpret_cast<const uint4*>(&rows[pp][4 * (ch ^ ((pp >> 3) & 7))]);
    }
}

// Zero the padding ring of the zero-padded limb planes [N][Hp][Wp][Cg*128]
// (x_limbs_block writes the interior): thread per 16-byte piece of a ring
// position; the ring of one image is ph full rows at the top and bottom and
// pw columns at both ends of the H rows between.
__device__ __forceinline__ void zero_ring_blocks(uint8_t* __restrict__ xl, int64_t N, int H, int W, int ph, int pw,
                                                 int Cg, int64_t bid, int64_t nblocks) {
    const int Hp = H + 2 * ph, Wp = W + 2 * pw;
    const int64_t ring = static_cast<int64_t>(Hp) * Wp - static_cast<int64_t>(H) * W;
    const int pieces = Cg * 8;
    const int64_t total = N * ring * pieces;
    for (int64_t it = bid * blockDim.x + threadIdx.x; it < total; it += nblocks * blockDim.x) {
        const int piece = static_cast<int>(it % pieces);
        const int64_t r = it / pieces;
        const int64_t n = r / ring;
        int64_t i = r - n * ring;
        int hp, wp;
        const int64_t band = static_cast<int64_t>(ph) * Wp;
        if (i < band) {
            hp = static_cast<int>(i / Wp);
            wp = static_cast<int>(i % Wp);
        } else if (i < 2 * band) {
            i -= band;
            hp = H + ph + static_cast<int>(i / Wp);
            wp = static_cast<int>(i % Wp);
        } else {
            i -= 2 * band;
            const int k = static_cast<int>(i % (2 * pw));
            hp = ph + static_cast<int>(i / (2 * pw));
            wp = k < pw ? k : W + k;
        }
        uint8_t* dst = xl + ((n * Hp + hp) * Wp + wp) * static_cast<int64_t>(Cg) * 128 + piece * 16;
        *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    }
}

// Stacked weight tiles for conv_stk_kernel: [pairs][144 rows][128 B]; byte
// 64 h + c of row n in pair p belongs to K step kb = 2p + h (tap kb / Cg,
// channel group kb % Cg, channel c of the group): rows 0-63 hold
// (q >> 8) + 128 of filter n, rows 64-127 q & 255 of filter n - 64, rows
// 128-143 ones.  Thread per 16-byte piece.
template <typename T>
__device__ __forceinline__ void w_stack_blocks(const T* __restrict__ w, int F, int C, int taps, int Cg, int npairs,
                                               const float* __restrict__ amax, uint8_t* __restrict__ ws,
                                               int64_t bid, int64_t nblocks) {
    const int64_t total = static_cast<int64_t>(npairs) * STK_N * 8;
    const float inv = quant_inv(__ldg(amax));
    const int nkb = taps * Cg;
    for (int64_t it = bid * blockDim.x + threadIdx.x; it < total; it += nblocks * blockDim.x) {
        const int piece = static_cast<int>(it & 7);  // 16-byte piece of the 128-byte row
        const int64_t r = it >> 3;
        const int n = static_cast<int>(r % STK_N);
        const int pair = static_cast<int>(r / STK_N);
        const int h = piece >> 2, pc = piece & 3;
        const int kb = 2 * pair + h;
        // the 16 bytes as four little-endian words, built in registers
        uint32_t b4[4] = {0x01010101u, 0x01010101u, 0x01010101u, 0x01010101u};
        if (n < 128) {
            const int f = n & 63;
            const int tap = kb / Cg, g = kb - (kb / Cg) * Cg;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int c = g * 64 + pc * 16 + j;
                int q = 0;
                if (kb < nkb && f < F && c < C)
                    q = quant_one(ldt<T>(w, (static_cast<int64_t>(f) * C + c) * taps + tap), inv);
                const uint32_t byte = static_cast<uint32_t>(n < 64 ? ((q >> 8) + 128) & 0xFF : q & 0xFF);
                if ((j & 3) == 0) b4[j >> 2] = 0u;
                b4[j >> 2] |= byte << (8 * (j & 3));
            }
        }
        *reinterpret_cast<uint4*>(ws + r * KB + piece * 16) = make_uint4(b4[0], b4[1], b4[2], b4[3]);
    }
}

// Weight limb rows [F][taps][Cg][128 B].  One block per (filter, 64-channel
// group, run of WQ_TAPS taps): the 64 x WQ_TAPS codes are read with the taps
// contiguous (OI[D]HW order), quantised into shared memory, and each thread
// packs the 16-channel hi and lo pieces of one tap's row.
constexpr int WQ_TAPS = 32;

template <typename T>
__device__ __forceinline__ void w_limbs_block(const T* __restrict__ w, int F, int C, int taps, int Cg,
                                              const float* __restrict__ amax, uint8_t* __restrict__ wl,
                                              int bid) {
    __shared__ int16_t q[64][WQ_TAPS + 2];
    const int runs = (taps + WQ_TAPS - 1) / WQ_TAPS;
    const int run = bid % runs;
    const int g = (bid / runs) % Cg;
    const int f = bid / (runs * Cg);
    const int t0 = run * WQ_TAPS;
    const int nt = min(WQ_TAPS, taps - t0);
    const float inv = quant_inv(__ldg(amax));
    // only the run's nt taps (columns t >= nt of q are never packed); for one
    // run the 64 x nt values are one contiguous span of w
    for (int it = threadIdx.x; it < 64 * nt; it += blockDim.x) {
        const int cc = it / nt, t = it - (it / nt) * nt;
        const int c = g * 64 + cc;
        int v = 0;
        if (c < C) v = quant_one(ldt<T>(w, (static_cast<int64_t>(f) * C + c) * taps + t0 + t), inv);
        q[cc][t] = static_cast<int16_t>(v);
    }
    __syncthreads();
    for (int it = threadIdx.x; it < nt * 4; it += blockDim.x) {
        const int t = it >> 2, pc = it & 3;
        uint4 hi, lo;
        pack16(&q[pc * 16][t], WQ_TAPS + 2, hi, lo);
        uint8_t* dst = wl + ((static_cast<int64_t>(f) * taps + t0 + t) * Cg + g) * 128 + pc * 16;
        *reinterpret_cast<uint4*>(dst) = hi;
        *reinterpret_cast<uint4*>(dst + 64) = lo;
    }
}

// Everything the implicit-GEMM kernels read, prepared by one launch of
// 256-thread blocks split by block index into three independent parts: the
// weight's limb rows (stacked tiles or per-filter rows), the zero ring of the
// padded input planes, and the input's limb rows.  The parts write disjoint
// bytes.  The weight blocks come first, so their short, latency-bound work
// starts at once and overlaps the input blocks instead of following them as
// separate launches.
template <typename T>
struct ConvPrepArgs {
    const T* x;
    const T* w;
    const float* amax_x;
    const float* amax_w;
    uint8_t* xl;
    uint8_t* wl;
    int64_t N, DHW;
    int C, F, H, W, ph, pw, sh, sw, Cg, taps, npairs, xvec;
    int stk;          // stacked weight tiles (w_stack) instead of per-filter rows (w_limbs)
    unsigned wgrid;   // blocks of the weight part
    unsigned zgrid;   // blocks of the ring part (0 without padding)
};

template <typename T>
__global__ void __launch_bounds__(XQ_THREADS) conv_prep_kernel(ConvPrepArgs<T> a) {
    pdl_trigger();  // the convolution kernel may begin its prologue
    pdl_wait();     // the amax pass has completed
    unsigned b = blockIdx.x;
    if (b < a.wgrid) {
        if (a.stk)
            w_stack_blocks<T>(a.w, a.F, a.C, a.taps, a.Cg, a.npairs, a.amax_w, a.wl, b, a.wgrid);
        else
            w_limbs_block<T>(a.w, a.F, a.C, a.taps, a.Cg, a.amax_w, a.wl, static_cast<int>(b));
        return;
    }
    b -= a.wgrid;
    if (b < a.zgrid) {
        zero_ring_blocks(a.xl, a.N, a.H, a.W, a.ph, a.pw, a.Cg, b, a.zgrid);
        return;
    }
    b -= a.zgrid;
    x_limbs_block<T>(a.x, a.C, a.DHW, a.W, a.ph, a.pw, a.sh, a.sw, a.Cg, a.xvec, a.amax_x, a.xl,
                     static_cast<int64_t>(b));
}

template <class C, int DT>
int launch_conv(const CUtensorMap& tx, const CUtensorMap& tw, const ConvTcParams& p, int dev,
                cudaStream_t stream) {
    static std::once_flag once[64];
    static cudaError_t err[64];
    const int slot = std::min(dev, 63);
    std::call_once(once[slot], [&] {
        err[slot] = cudaFuncSetAttribute(conv_tc_kernel<C, DT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::SMEM);
    });
    if (err[slot] != cudaSuccess) TK_FAIL(TK_ERR_CUDA, "conv smem attribute: %s", cudaGetErrorString(err[slot]));
    const int grid = std::min(p.tiles, sm_count(dev));
    TK_CUDA_TRY(launch_pdl(conv_tc_kernel<C, DT>, grid, NUM_THREADS, C::SMEM, stream, tx, tw, p));
    return launch_status("conv2d implicit GEMM");
}

template <class C, int DT>
int launch_win(const CUtensorMap& tx, const CUtensorMap& tw, const ConvWinParams& p, int dev,
               cudaStream_t stream) {
    static std::once_flag once[64];
    static cudaError_t err[64];
    const int slot = std::min(dev, 63);
    std::call_once(once[slot], [&] {
        err[slot] = cudaFuncSetAttribute(conv_win_kernel<C, DT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::SMEM);
    });
    if (err[slot] != cudaSuccess) TK_FAIL(TK_ERR_CUDA, "conv smem attribute: %s", cudaGetErrorString(err[slot]));
    const int grid = std::min(p.tiles, sm_count(dev));
    TK_CUDA_TRY(launch_pdl(conv_win_kernel<C, DT>, grid, NUM_THREADS, C::SMEM, stream, tx, tw, p));
    return launch_status("conv2d window implicit GEMM");
}

template <int DT>
int launch_stk(const CUtensorMap& tx, const CUtensorMap& tw, const ConvWinParams& p, int dev, cudaStream_t stream) {
    static std::once_flag once[64];
    static cudaError_t err[64];
    const int slot = std::min(dev, 63);
    std::call_once(once[slot], [&] {
        err[slot] = cudaFuncSetAttribute(conv_stk_kernel<DT>, cudaFuncAttributeMaxDynamicSharedMemorySize, STK_SMEM);
    });
    if (err[slot] != cudaSuccess) TK_FAIL(TK_ERR_CUDA, "conv smem attribute: %s", cudaGetErrorString(err[slot]));
    TK_CHECK_ARG(p.tiles_f == 1, "conv stacked kernel: at most 64 filters");
    const int grid = std::min(p.tiles, sm_count(dev));
    TK_CUDA_TRY(launch_pdl(conv_stk_kernel<DT>, grid, NUM_THREADS, STK_SMEM, stream, tx, tw, p));
    return launch_status("conv2d stacked window implicit GEMM");
}

// 1x1, stride 1, no padding, groups 1, at most 64 filters and 256 channels,
// fp16: the input
// is quantised inside conv1x1_q_kernel (no limb pass); weights stacked as
// for conv_stk_kernel into `ws`.
int conv1x1_q(const void* x, const void* w, const void* bias, void* out, int64_t N, int64_t C, int64_t HW,
              int64_t F, const float* amax_x, const float* amax_w, uint8_t* ws, int dev, cudaStream_t stream,
              bool x_scale_own) {
    const int64_t Cg = ceil_div(C, 64);
    EncodeTiledFn enc = tensor_map_encoder();
    if (enc == nullptr) TK_FAIL(TK_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    CUtensorMap tx;
    {
        // NCHW fp16 as [N][C][HW]: boxes of 128 pixels x 64 channels; pixels
        // past the plane and channels past C read as zero
        cuuint64_t dims[3] = {static_cast<cuuint64_t>(HW), static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(N)};
        cuuint64_t strides[2] = {static_cast<cuuint64_t>(HW * 2), static_cast<cuuint64_t>(C * HW * 2)};
        cuuint32_t box[3] = {static_cast<cuuint32_t>(BM), 64, 1};
        cuuint32_t estr[3] = {1, 1, 1};
        CUresult r = enc(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(x), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) TK_FAIL(TK_ERR_CUDA, "conv2d 1x1 input tensor map failed (%d)", (int)r);
    }
    ConvWinParams p = {};
    p.N = static_cast<int>(N);
    p.F = static_cast<int>(F);
    p.OH = 1;
    p.OW = static_cast<int>(HW);
    p.Hp = 1;
    p.Wp = static_cast<int>(HW);
    p.Cg = static_cast<int>(Cg);
    p.taps = 1;
    p.win_rows = BM;
    p.pos_tiles = static_cast<int>(ceil_div(HW, BM));
    p.tiles_f = 1;
    p.tiles = static_cast<int>(N * p.pos_tiles);
    p.amax_x = amax_x;
    p.amax_w = amax_w;
    p.bias = bias;
    p.out = out;
    p.err = device_error_word(dev);
    p.clamp_x = x_scale_own ? 0 : 1;
    p.w = static_cast<const __half*>(w);
    p.C = static_cast<int>(C);
    p.w_vec = C % 8 == 0 && reinterpret_cast<uintptr_t>(w) % 16 == 0;
    static std::once_flag once[64];
    static cudaError_t err[64];
    const int slot = std::min(dev, 63);
    std::call_once(once[slot], [&] {
        err[slot] = cudaFuncSetAttribute(conv1x1_q_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Q1_SMEM);
    });
    if (err[slot] != cudaSuccess) TK_FAIL(TK_ERR_CUDA, "conv smem attribute: %s", cudaGetErrorString(err[slot]));
    const int grid = std::min(p.tiles, sm_count(dev));
    TK_CUDA_TRY(launch_pdl(conv1x1_q_kernel, grid, NUM_THREADS, Q1_SMEM, stream, tx, p));
    return launch_status("conv2d 1x1 implicit GEMM (input quantised in the kernel)");
}

// The window variant applies when one window of 128 + max tap offset rows
// fits a TMA box.
bool window_fits(int64_t KH, int64_t KW, int64_t dh, int64_t dw, int64_t Wp) {
    return KH * KW <= kMaxTaps && BM + (KH - 1) * dh * Wp + (KW - 1) * dw <= WIN_ROWS;
}

}  // namespace

// Workspace bytes of the implicit-GEMM path (limb rows of the zero-padded x
// and of w).
size_t conv_tc_workspace(int64_t N, int64_t C, int64_t D, int64_t H, int64_t W, int64_t F, int64_t KD,
                         int64_t KH, int64_t KW, int64_t ph, int64_t pw) {
    const int64_t Cg = ceil_div(C, 64);
    const int64_t nkb = KD * KH * KW * Cg;
    const int64_t w_bytes = std::max<int64_t>(F * nkb * 128, ceil_div(nkb, 2) * STK_TILE);
    return round_up(static_cast<size_t>(N * D * (H + 2 * ph) * (W + 2 * pw) * Cg * 128), 1024) +
           round_up(static_cast<size_t>(w_bytes), 1024);
}

// Implicit-GEMM conv (2-D with D = KD = 1, or 3-D) for groups == 1 and
// stride 1; `ws` is 1024-aligned with conv_tc_workspace(...) bytes;
// amax_x / amax_w are device scalars.
int conv_tc(tk_dtype_t dtype, const void* x, const void* w, const void* bias, void* out, int64_t N,
            int64_t C, int64_t D, int64_t H, int64_t W, int64_t F, int64_t KD, int64_t KH, int64_t KW,
            int64_t pd, int64_t ph, int64_t pw, int64_t dd, int64_t dh, int64_t dw, int64_t OD, int64_t OH,
            int64_t OW, const float* amax_x, const float* amax_w, uint8_t* ws, cudaStream_t stream,
            bool x_scale_own) {
    const int dev = current_device();
    const int64_t Cg = ceil_div(C, 64);
    const int64_t Hp = H + 2 * ph, Wp = W + 2 * pw;
    if (dtype == TK_DTYPE_F16 && D == 1 && KD == 1 && KH == 1 && KW == 1 && ph == 0 && pw == 0 && F <= 64 &&
        Cg <= 2 * Q1_MAX_PAIRS && (H * W) % 8 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
        N * ceil_div(H * W, BM) < (1LL << 31) && N * C * H * W < (1LL << 40))
        return conv1x1_q(x, w, bias, out, N, C, H * W, F, amax_x, amax_w, ws, dev, stream, x_scale_own);
    // Window variant (input stored zero-padded, one window per channel group)
    // for up to 64 filters.  With 128-filter tiles the per-tap ring measured
    // faster (3x3 256->256 @14, batch 64: 77 vs 83 us).  A 1x1 filter has no
    // halo: it takes the window path only with the stacked-limb MMAs, which
    // halve its MMA count; the four-MMA window kernel was slower than the
    // per-tap kernel there.
    const int64_t npairs = ceil_div(KD * KH * KW * Cg, 2);
    const bool stk_fits = npairs <= STK_MAX_PAIRS;
    const bool win = D == 1 && KD == 1 && F <= 64 && (KH * KW > 1 || stk_fits) &&
                     window_fits(KH, KW, dh, dw, Wp) && N * Hp * Wp < (1LL << 31);
    // stored rows per image: the padded plane (window variant, D == 1) or the
    // unpadded volume D*H*W (as D*H rows of W pixels)
    const int64_t sh = win ? Hp : D * H, sw = win ? Wp : W;
    const size_t x_bytes = static_cast<size_t>(N * sh * sw * Cg * 128);
    uint8_t* xl = ws;
    uint8_t* wl = ws + round_up(x_bytes, 1024);
    int64_t zblocks = 0;
    if (win && (ph > 0 || pw > 0)) {
        const int64_t ring = Hp * Wp - H * W;
        const int64_t total = N * ring * Cg * 8;
        zblocks = std::max<int64_t>(1, std::min<int64_t>(ceil_div(total, 256), 8LL * sm_count(dev)));
    }
    const int64_t DHW = D * H * W;  // the image's flattened volume (rows of limbs)
    const int64_t runs = ceil_div(DHW, XQ_W);
    TK_CHECK_ARG(N * runs * Cg < (1LL << 31) && DHW < (1LL << 31), "conv: input too large");
    const int64_t xblocks = N * runs * Cg;
    const size_t es = dtype_size(dtype);
    const int xvec = (DHW % static_cast<int64_t>(16 / es) == 0 &&
                      reinterpret_cast<uintptr_t>(x) % 16 == 0) ? 1 : 0;
    const int64_t taps = KD * KH * KW;
    // stacked-limb window kernel when the stacked filter block stays resident
    // (the four-MMA window kernel otherwise)
    const bool stk = win && stk_fits;
    const int64_t wblocks = stk ? ceil_div(npairs * STK_N * 8, 256) : F * Cg * ceil_div(taps, WQ_TAPS);
    TK_CHECK_ARG(wblocks + zblocks + xblocks < (1LL << 31), "conv: weight or input too large");
    auto prep = [&](auto* tag) {
        using T = std::remove_pointer_t<decltype(tag)>;
        ConvPrepArgs<T> a;
        a.x = static_cast<const T*>(x);
        a.w = static_cast<const T*>(w);
        a.amax_x = amax_x;
        a.amax_w = amax_w;
        a.xl = xl;
        a.wl = wl;
        a.N = N;
        a.DHW = DHW;
        a.C = (int)C; a.F = (int)F; a.H = (int)H; a.W = (int)W;
        a.ph = win ? (int)ph : 0;  // the stored planes are padded only for the window kernels
        a.pw = win ? (int)pw : 0;
        a.sh = (int)sh; a.sw = (int)sw; a.Cg = (int)Cg; a.taps = (int)taps; a.npairs = (int)npairs;
        a.xvec = xvec;
        a.stk = stk ? 1 : 0;
        a.wgrid = static_cast<unsigned>(wblocks);
        a.zgrid = static_cast<unsigned>(zblocks);
        const unsigned grid = static_cast<unsigned>(wblocks + zblocks + xblocks);
        return launch_pdl(conv_prep_kernel<T>, grid, XQ_THREADS, 0, stream, a);
    };
    const cudaError_t le = dtype == TK_DTYPE_F16 ? prep(static_cast<__half*>(nullptr))
                                                 : prep(static_cast<float*>(nullptr));
    if (le != cudaSuccess) TK_FAIL(TK_ERR_CUDA, "conv2d limbs launch: %s", cudaGetErrorString(le));
    int rc = launch_status("conv2d limbs");
    if (rc) return rc;

    EncodeTiledFn enc = tensor_map_encoder();
    if (enc == nullptr) TK_FAIL(TK_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    const bool narrow = F <= 64;
    const int BN = narrow ? ConvNarrow::BN : ConvWide::BN;
    CUtensorMap tx, tw;
    if (stk) {
        // [pairs * 144 rows][128 B], one 144-row box per pair of K steps
        const uint64_t rows = static_cast<uint64_t>(npairs * STK_N);
        cuuint64_t dims[3] = {128, rows, 1};
        cuuint64_t strides[2] = {128, 128 * rows};
        cuuint32_t box[3] = {128, static_cast<cuuint32_t>(STK_N), 1};
        cuuint32_t estr[3] = {1, 1, 1};
        CUresult r = enc(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, wl, dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) TK_FAIL(TK_ERR_CUDA, "conv2d stacked weight tensor map failed (%d)", (int)r);
    } else {
        const uint64_t row = static_cast<uint64_t>(taps * Cg) * 128;
        cuuint64_t dims[3] = {row, static_cast<cuuint64_t>(F), 1};
        cuuint64_t strides[2] = {row, row * F};
        cuuint32_t box[3] = {128, static_cast<cuuint32_t>(BN), 1};
        cuuint32_t estr[3] = {1, 1, 1};
        CUresult r = enc(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, wl, dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) TK_FAIL(TK_ERR_CUDA, "conv2d weight tensor map failed (%d)", (int)r);
    }
    const int64_t tiles_f = ceil_div(F, BN);

    if (win) {
        ConvWinParams q;
        q.N = (int)N; q.F = (int)F; q.OH = (int)OH; q.OW = (int)OW; q.Hp = (int)Hp; q.Wp = (int)Wp;
        q.Cg = (int)Cg; q.taps = (int)(KH * KW);
        int max_off = 0;
        for (int64_t kh = 0; kh < KH; ++kh)
            for (int64_t kw = 0; kw < KW; ++kw) {
                const int off = static_cast<int>(kh * dh * Wp + kw * dw);
                q.tap_off[kh * KW + kw] = off;
                max_off = std::max(max_off, off);
            }
        q.win_rows = BM + max_off;
        q.pos_tiles = static_cast<int>(ceil_div((OH - 1) * Wp + OW, BM));
        q.tiles_f = static_cast<int>(tiles_f);
        const int64_t tiles = N * q.pos_tiles * tiles_f;
        TK_CHECK_ARG(tiles < (1LL << 31), "conv2d: too many tiles");
        q.tiles = static_cast<int>(tiles);
        q.amax_x = amax_x;
        q.amax_w = amax_w;
        q.bias = bias;
        q.out = out;
        q.err = device_error_word(dev);
        const uint64_t row = static_cast<uint64_t>(Cg) * 128;
        const uint64_t rows = static_cast<uint64_t>(N * Hp * Wp);
        cuuint64_t dims[3] = {row, rows, 1};
        cuuint64_t strides[2] = {row, row * rows};
        cuuint32_t box[3] = {128, static_cast<cuuint32_t>(q.win_rows), 1};
        cuuint32_t estr[3] = {1, 1, 1};
        CUresult r = enc(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, xl, dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) TK_FAIL(TK_ERR_CUDA, "conv2d window tensor map failed (%d)", (int)r);
        if (stk) return dtype == TK_DTYPE_F16 ? launch_stk<0>(tx, tw, q, dev, stream)
                                              : launch_stk<1>(tx, tw, q, dev, stream);
        if (KH * KW * Cg * WinResident::B_BYTES <= kResWeightBytes)
            return dtype == TK_DTYPE_F16 ? launch_win<WinResident, 0>(tx, tw, q, dev, stream)
                                         : launch_win<WinResident, 1>(tx, tw, q, dev, stream);
        return dtype == TK_DTYPE_F16 ? launch_win<WinNarrow, 0>(tx, tw, q, dev, stream)
                                     : launch_win<WinNarrow, 1>(tx, tw, q, dev, stream);
    }

    ConvTcParams p;
    p.N = (int)N; p.F = (int)F; p.OD = (int)OD; p.OH = (int)OH; p.OW = (int)OW;
    p.KD = (int)KD; p.KH = (int)KH; p.KW = (int)KW;
    p.pd = (int)pd; p.ph = (int)ph; p.pw = (int)pw; p.dd = (int)dd; p.dh = (int)dh; p.dw = (int)dw;
    p.Cg = (int)Cg;
    p.TW = static_cast<int>(std::min<int64_t>(OW, BM));
    p.TH = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(BM / p.TW, OH)));
    p.tiles_h = static_cast<int>(ceil_div(OH, p.TH));
    p.tiles_w = static_cast<int>(ceil_div(OW, p.TW));
    p.tiles_f = static_cast<int>(tiles_f);
    const int64_t tiles = N * OD * p.tiles_h * p.tiles_w * p.tiles_f;
    TK_CHECK_ARG(tiles < (1LL << 31), "conv: too many tiles");
    p.tiles = static_cast<int>(tiles);
    p.num_kb = static_cast<int>(taps * Cg);
    p.amax_x = amax_x;
    p.amax_w = amax_w;
    p.bias = bias;
    p.out = out;
    p.err = device_error_word(dev);
    {
        const uint64_t row = static_cast<uint64_t>(Cg) * 128;
        cuuint64_t dims[5] = {row, static_cast<cuuint64_t>(W), static_cast<cuuint64_t>(H),
                              static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(N)};
        cuuint64_t strides[4] = {row, row * W, row * W * H, row * W * H * D};
        cuuint32_t box[5] = {128, static_cast<cuuint32_t>(p.TW), static_cast<cuuint32_t>(p.TH), 1, 1};
        cuuint32_t estr[5] = {1, 1, 1, 1, 1};
        CUresult r = enc(&tx, CU_TENSOR_MAP_DATA_TYPE_UINT8, 5, xl, dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) TK_FAIL(TK_ERR_CUDA, "conv2d input tensor map failed (%d)", (int)r);
    }
    if (narrow)
        return dtype == TK_DTYPE_F16 ? launch_conv<ConvNarrow, 0>(tx, tw, p, dev, stream)
                                     : launch_conv<ConvNarrow, 1>(tx, tw, p, dev, stream);
    return dtype == TK_DTYPE_F16 ? launch_conv<ConvWide, 0>(tx, tw, p, dev, stream)
                                 : launch_conv<ConvWide, 1>(tx, tw, p, dev, stream);
}

}  // namespace tk
