// qgemm.cu -- int16-quantised GEMM on sm_100a tensor cores.
//
// Replaces baidu::xpu::api::fc<T,T,T,TGEMM> (called from csrc/ops.cpp:224 for
// mm/linear and per batch slice from csrc/ops_nn.cpp:214 for bmm) together
// with the bias/scale/add launches that follow it in the reference.
//
// Numerics: each int16 operand q is stored as two int8 limb planes,
// q = 256*hi + lo with hi signed in [-128,127] and lo unsigned in [0,255].
// Four tcgen05 kind::i8 MMAs per K-step produce three int32 TMEM accumulators
//   HH = sum hi_a*hi_b,  MID = sum hi_a*lo_b + lo_a*hi_b,  LL = sum lo_a*lo_b
// which are exact for K <= 32768 (|MID| <= K*65280 < 2^31).  The epilogue
// rebuilds acc = 65536*HH + 256*MID + LL exactly in binary64 (every partial
// result is an integer below 2^53), multiplies by the dequant scale
// amax_a*amax_b/32767^2 and rounds once to fp16/fp32, then applies the
// reference's post-GEMM ops in its order (alpha, bias, beta*addend, act).
//
// Longer reductions (the reference's fc takes any K) are split: each output
// tile's K range is cut into chunks of at most 32768 (kb_per_split blocks),
// every chunk is its own work unit, and the epilogue adds the chunk's exact
// int64 sum into an int64 workspace with integer atomics (order-independent,
// so the result is deterministic).  A finishing kernel then converts each
// int64 sum to binary64 (round to nearest, as the oracle's conversion),
// dequantises with the single rounding and applies the post-GEMM ops.  The
// same mode splits long-K problems with too few output tiles to fill the
// GPU, and sums over batch slices (acc_mod) for reductions that span them
// (the weight gradient of a convolution).
//
// Kernel structure (one persistent CTA per SM, 320 threads):
//   warp 0      TMA producer: 4 boxes per stage (A hi/lo, B hi/lo), 128 rows
//               x 128 bytes each, 128-byte swizzle, 3-stage ring;
//   warp 1      TMEM owner + MMA issuer (one thread), 16 MMAs per stage;
//   warps 2..9  epilogue, two per TMEM lane quarter taking alternate
//               16-column chunks: tcgen05.ld of the three accumulators of
//               its 32 TMEM lanes, binary64 recombine, dequant, fused ops,
//               vector stores.
// Tiles are 128x128 (K < 2048) or 128x160; the three accumulators fill 384
// or 480 of the 512 TMEM columns, so the MMA warp waits for the epilogue to
// drain them before the next tile (the 128x64 / 128x80 overlap variants
// double-buffer them instead).
// No TMA multicast is used anywhere.
#include <cuda.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <mutex>
#include <string>

#include "tk_internal.h"
#include "tk_numerics.cuh"
#include "tk_ptx.cuh"

namespace tk {

int amax_launch(tk_dtype_t dtype, const void* x, int64_t nslices, int64_t slice_stride,
                int64_t slice_len, float* amax_out, cudaStream_t stream);
int quantize_limbs_launch(tk_dtype_t dtype, const void* x, int64_t batch, int64_t rows,
                          int64_t cols, int64_t sb, int64_t sr, int64_t sc, const float* amax,
                          int64_t amax_stride, int8_t* limbs, cudaStream_t stream);

namespace {

constexpr int BM = 128;
constexpr int BK = 128;  // bytes (int8 elements) per stage along K
constexpr int UMMA_K = 32;
constexpr int NUM_EPI_WARPS = 8;  // two warps per TMEM lane quarter
constexpr int NUM_THREADS = 64 + 32 * NUM_EPI_WARPS;
constexpr int TMEM_COLS = 512;
constexpr int kMaxK = 32768;

// Tile configuration: BN columns per tile, a STAGES-deep TMA ring and NBUF
// accumulator buffers in TMEM (each buffer holds HH, MID and LL, 3*BN
// columns).  With NBUF = 2 the epilogue of one tile overlaps the MMAs of the
// next; 2*3*BN <= 512 limits that to BN <= 80.
template <int BN_, int STAGES_, int NBUF_>
struct TileCfg {
    static constexpr int BN = BN_;
    static constexpr int STAGES = STAGES_;
    static constexpr int NBUF = NBUF_;
    static constexpr int A_BYTES = BM * BK;   // one limb plane of the A tile
    static constexpr int B_BYTES = BN * BK;   // one limb plane of the B tile
    static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
    static constexpr int BUF_COLS = NBUF == 1 ? 3 * BN : 256;
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align slack*/ + 256 /*barriers*/;
    static constexpr uint32_t IDESC_SS = idesc_i8(BM, BN, true, true);
    static constexpr uint32_t IDESC_SU = idesc_i8(BM, BN, true, false);
    static constexpr uint32_t IDESC_US = idesc_i8(BM, BN, false, true);
    static constexpr uint32_t IDESC_UU = idesc_i8(BM, BN, false, false);
    static_assert(B_BYTES % 1024 == 0, "B tile must be a whole number of swizzle atoms");
    static_assert(NBUF * BUF_COLS <= TMEM_COLS && 3 * BN <= BUF_COLS, "TMEM budget");
    static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M=128");
    static_assert(SMEM <= 232448, "shared memory budget");
};
// Measured on B200 (int16-quantised GEMMs, K-major limb operands): 128x160
// tiles are 5-14% faster than 128x128 once K >= 2048 (less operand traffic
// per MMA, fewer waves for N = 4096) and slower for short K, where the
// non-overlapped epilogue dominates.  A double-buffered 128x80 variant
// (epilogue overlapped with the next tile's MMAs) was 30% slower at 4096^3:
// operand delivery, not the epilogue, limits these tiles.
using CfgWide = TileCfg<128, 3, 1>;   // 128x128 tiles, accumulators single-buffered
using CfgWider = TileCfg<160, 3, 1>;  // 128x160 tiles (480 TMEM columns), single-buffered
using CfgOverlap64 = TileCfg<64, 4, 2>;  // 128x64 tiles, epilogue overlapped with the next tile
using CfgOverlap80 = TileCfg<80, 4, 2>;  // 128x80 tiles, epilogue overlapped with the next tile

constexpr int kMaxRowDests = 8;

struct EpiParams {
    int dtype;  // 0 fp16, 1 fp32
    int64_t M, N;
    void* out;
    int64_t out_sb, out_sm, out_sn;  // out_sn == 1 except for transposed (NCHW) stores
    const void* bias;
    int64_t bias_mod;  // 0: bias[n]; else bias[(b % bias_mod) * N + n] (grouped conv)
    const void* addend;
    int64_t add_sb, add_sm, add_sn;
    float alpha, beta;
    int act;
    const float* amax_a;
    const float* amax_b;
    int64_t scale_stride;  // 1: per-slice amax; 0: one amax for all slices
    bool vec_store;
    bool bias_vec;  // bias is 16-byte aligned: vector loads per 16-column chunk
    bool add_vec;   // addend rows contiguous and 16-byte aligned: vector loads
    int32_t* dbg;  // [3][M][N] raw accumulators of slice 0, or null
    unsigned* amax_out;  // fp32 magnitude bits of max |out| (atomicMax), or null; fast path only
    // Row scatter (batch 1): rows [q*R, (q+1)*R) go to row_dest[q] at local
    // row m - q*R (row stride out_sm) instead of out; R = row_dest_rows > 0.
    // The destinations may be other GPUs' memory (CUDA IPC over NVLink).
    void* row_dest[kMaxRowDests];
    int64_t row_dest_rows;
    int row_dest_n;
};

// Destination buffer and element offset of row m's first column.
__device__ __forceinline__ void* row_out(const EpiParams& p, int64_t b, int64_t m, int64_t& row_off) {
    if (p.row_dest_rows > 0) {
        const int64_t q = min(m / p.row_dest_rows, static_cast<int64_t>(p.row_dest_n - 1));
        row_off = (m - q * p.row_dest_rows) * p.out_sm;
        return p.row_dest[q];
    }
    row_off = b * p.out_sb + m * p.out_sm;
    return p.out;
}

struct TileParams {
    int batch, tiles_m, tiles_n, num_tiles, num_kb;
    int b_mod;  // 0: B slice b; else B slice (b % b_mod) (operand shared across images)
    // K split: every (slice, tile) is ksplit work units of kb_per_split K
    // blocks each; with acc64 set the epilogue adds exact int64 sums into
    // acc64[(slice * M + m) * N + n], slice = acc_mod ? b % acc_mod : b.
    int ksplit, kb_per_split;
    unsigned long long* acc64;
    int acc_mod;
    unsigned* err;
};

// ---- numerics (device): tk_numerics.cuh holds the shared contract ----------

__device__ __forceinline__ double epi_scale(const EpiParams& p, int64_t b) {
    return ::tk::dequant_scale(p.amax_a[b * p.scale_stride], p.amax_b[b * p.scale_stride]);
}

template <int ACT>
__device__ __forceinline__ float act_t(float r, int dtype) {
    if constexpr (ACT == TK_ACT_NONE) {
        return r;
    } else if constexpr (ACT == TK_ACT_RELU) {
        return (r > 0.0f || r != r) ? r : 0.0f;
    } else {
        return apply_act(r, ACT, dtype);
    }
}



// The reference's post-GEMM sequence on one element (see file header).
__device__ __forceinline__ float epilogue_one(const EpiParams& p, double s, double acc, int64_t b,
                                              int64_t m, int64_t n) {
    float r = round_t_from_double(__dmul_rn(acc, s), p.dtype);
    if (p.alpha != 1.0f) r = round_t(__fmul_rn(r, p.alpha), p.dtype);
    if (p.bias != nullptr) r = round_t(__fadd_rn(r, load_t(p.bias, p.dtype, n)), p.dtype);
    if (p.addend != nullptr && p.beta != 0.0f) {
        float a = load_t(p.addend, p.dtype, b * p.add_sb + m * p.add_sm + n * p.add_sn);
        if (p.beta != 1.0f) a = round_t(__fmul_rn(a, p.beta), p.dtype);
        r = round_t(__fadd_rn(r, a), p.dtype);
    }
    return apply_act(r, p.act, p.dtype);
}


// Work unit t -> (K chunk ks, slice b, M tile mt, N tile nt).  The K chunk
// varies slowest, so the units running together share K ranges and reuse
// operand tiles through L2 as the unsplit GEMM does.
__device__ __forceinline__ void decode_tile(const TileParams& tp, int t, int& b, int& mt, int& nt,
                                            int& ks) {
    const int per_batch = tp.tiles_m * tp.tiles_n;
    const int per_split = per_batch * tp.batch;
    ks = t / per_split;
    t -= ks * per_split;
    b = t / per_batch;
    const int id = t - b * per_batch;
    constexpr int GROUP = 8;  // M-tiles per raster group (keeps B tiles hot in L2)
    const int width = GROUP * tp.tiles_n;
    const int g = id / width;
    const int first_m = g * GROUP;
    const int gsize = min(tp.tiles_m - first_m, GROUP);
    const int r = id - g * width;
    mt = first_m + r % gsize;
    nt = r / gsize;
}

// ---- tensor-core kernel --------------------------------------------------------

// EW: epilogue warps.  FO: the fast-only epilogue, for fp16 outputs on the
// fast path for the whole problem (no alpha, vector bias / addend / stores,
// no split reduction, N a multiple of 16), compiled without the general
// path.  It reads each of its chunks out of TMEM into binary16 values (the
// one rounding of the dequantised product), releases the accumulator buffer,
// and only then adds bias / addend, applies the activation and stores, so
// the next tile's MMAs overlap that work.  128x128 tiles run it on 16 warps
// (four per TMEM lane quarter; 96 registers), 128x160 tiles on 8.  Measured:
// BERT FFN1 16384x3072x768 + GELU 249 -> 208 us, the TP MLP's K = 8192
// GEMMs +2.5 %, 2048x4096x4096 and 4096^3 -3 % step time.
template <class C, int DT, int ACT, int EW = NUM_EPI_WARPS, bool FO = false>
__global__ void __launch_bounds__(64 + 32 * EW, 1)
qgemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const TileParams tp, const EpiParams ep) {
    constexpr bool FAST_ONLY = FO;
    static_assert(!FAST_ONLY || DT == 0, "the fast-only epilogue is the fp16 fast path");
    static_assert(!FAST_ONLY || (C::BN / 16) % (EW / 4) == 0, "every warp takes the same number of chunks");
    constexpr int STAGES = C::STAGES;
    constexpr int STAGE_BYTES = C::STAGE_BYTES;
    constexpr int BN = C::BN;
    constexpr int NBUF = C::NBUF;
    constexpr int OFF_ALO = C::A_BYTES;
    constexpr int OFF_BHI = 2 * C::A_BYTES;
    constexpr int OFF_BLO = 2 * C::A_BYTES + C::B_BYTES;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
    uint64_t* full_bar = bars;                 // [STAGES] TMA -> MMA
    uint64_t* empty_bar = bars + STAGES;       // [STAGES] MMA -> TMA
    uint64_t* acc_full = bars + 2 * STAGES;    // [NBUF] MMA -> epilogue
    uint64_t* acc_empty = acc_full + NBUF;     // [NBUF] epilogue -> MMA (one arrival per epilogue warp)
    uint64_t* drain_bar = acc_empty + NBUF;    // MMA teardown
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(full_bar + s), 1);
            mbar_init(smem_u32(empty_bar + s), 1);
        }
        for (int i = 0; i < NBUF; ++i) {
            mbar_init(smem_u32(acc_full + i), 1);
            mbar_init(smem_u32(acc_empty + i), EW);
        }
        mbar_init(smem_u32(drain_bar), 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // launched with programmatic stream serialisation: the prologue above
    // touched only shared memory, TMEM and the kernel's parameters; the
    // limbs, amax values, bias and residual are read after this
    pdl_wait();

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        int stage = 0;
        uint32_t phase = 0;
        uint32_t last_phase[STAGES];
        bool used[STAGES];
        for (int s = 0; s < STAGES; ++s) { used[s] = false; last_phase[s] = 0; }
        bool ok = true;
        for (int t = blockIdx.x; t < tp.num_tiles && ok; t += gridDim.x) {
            int b, mt, nt, ks;
            decode_tile(tp, t, b, mt, nt, ks);
            const int kb0 = ks * tp.kb_per_split;
            const int kb1 = min(tp.num_kb, kb0 + tp.kb_per_split);
            for (int kb = kb0; kb < kb1; ++kb) {
                if (!mbar_wait_bounded(smem_u32(empty_bar + stage), phase ^ 1u, abort_flag,
                                       tp.err, kDevErrWaitEmpty)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    const uint32_t fb = smem_u32(full_bar + stage);
                    mbar_arrive_expect_tx(fb, STAGE_BYTES);
                    uint8_t* sbase = smem + stage * STAGE_BYTES;
                    const int kx = kb * BK;
                    tma_load_3d(smem_u32(sbase), &tmA, fb, kx, mt * BM, 2 * b + 0);
                    tma_load_3d(smem_u32(sbase + OFF_ALO), &tmA, fb, kx, mt * BM, 2 * b + 1);
                    const int bb = tp.b_mod ? b % tp.b_mod : b;
                    tma_load_3d(smem_u32(sbase + OFF_BHI), &tmB, fb, kx, nt * BN, 2 * bb + 0);
                    tma_load_3d(smem_u32(sbase + OFF_BLO), &tmB, fb, kx, nt * BN, 2 * bb + 1);
                }
                __syncwarp();
                used[stage] = true;
                last_phase[stage] = phase;
                if (++stage == STAGES) { stage = 0; phase ^= 1u; }
            }
        }
        // Drain: every box this warp issued must have landed before exit.
        for (int s = 0; s < STAGES; ++s) {
            if (used[s]) {
                volatile int no_abort = 0;
                mbar_wait_bounded(smem_u32(full_bar + s), last_phase[s], &no_abort, tp.err,
                                  kDevErrWaitDrain);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        int local = 0;  // tiles processed by this CTA
        for (int t = blockIdx.x; t < tp.num_tiles && ok; t += gridDim.x, ++local) {
            const int buf = local % NBUF;
            const uint32_t acc_phase = static_cast<uint32_t>(local / NBUF) & 1u;
            if (!mbar_wait_bounded(smem_u32(acc_empty + buf), acc_phase ^ 1u, abort_flag, tp.err,
                                   kDevErrWaitAccEmpty)) {
                break;
            }
            tc_fence_after();
            const uint32_t acc_hh = tmem_base + buf * C::BUF_COLS;
            const uint32_t acc_mid = acc_hh + BN;
            const uint32_t acc_ll = acc_hh + 2 * BN;
            int b, mt, nt, ks;
            decode_tile(tp, t, b, mt, nt, ks);
            const int kb0 = ks * tp.kb_per_split;
            const int kb1 = min(tp.num_kb, kb0 + tp.kb_per_split);
            for (int kb = kb0; kb < kb1; ++kb) {
                if (!mbar_wait_bounded(smem_u32(full_bar + stage), phase, abort_flag, tp.err,
                                       kDevErrWaitFull)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t sb = smem_u32(smem + stage * STAGE_BYTES);
                    const uint64_t a_hi = smem_desc_kmajor_sw128(sb);
                    const uint64_t a_lo = smem_desc_kmajor_sw128(sb + OFF_ALO);
                    const uint64_t b_hi = smem_desc_kmajor_sw128(sb + OFF_BHI);
                    const uint64_t b_lo = smem_desc_kmajor_sw128(sb + OFF_BLO);
#pragma unroll
                    for (int kk = 0; kk < BK / UMMA_K; ++kk) {
                        // K advance inside the 128-byte swizzle row: start address
                        // moves by kk*32 bytes (encoded >> 4).
                        const uint64_t off = static_cast<uint64_t>((kk * UMMA_K) >> 4);
                        const uint32_t acc = (kb > kb0 || kk > 0) ? 1u : 0u;
                        tc_mma_i8(acc_hh, a_hi + off, b_hi + off, C::IDESC_SS, acc);
                        tc_mma_i8(acc_mid, a_hi + off, b_lo + off, C::IDESC_SU, acc);
                        tc_mma_i8(acc_mid, a_lo + off, b_hi + off, C::IDESC_US, 1u);
                        tc_mma_i8(acc_ll, a_lo + off, b_lo + off, C::IDESC_UU, acc);
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
        // Drain: all MMAs issued by this thread complete before TMEM is freed.
        if (lane == 0) tc_commit(smem_u32(drain_bar));
        __syncwarp();
        volatile int no_abort = 0;
        mbar_wait_bounded(smem_u32(drain_bar), 0, &no_abort, tp.err, kDevErrWaitDrain);
    } else {
        // ---------------- epilogue (warps 2..9) ----------------
        // Warp w reads TMEM lane quarter (w % 4) -- the hardware restricts a
        // warp to lanes [32*(w%4), 32*(w%4)+32) -- and columns
        // [64*half, 64*half + 64) of each accumulator.
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;
        const int row = quarter * 32 + lane;
        const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
        const bool has_bias = ep.bias != nullptr;
        const bool has_add = ep.addend != nullptr && ep.beta != 0.0f;
        const bool has_alpha = ep.alpha != 1.0f;
        const bool fast_ok = ep.vec_store && !has_alpha && ep.dbg == nullptr &&
                             (!has_bias || (ep.bias_vec && ep.bias_mod == 0)) &&
                             (!has_add || (ep.add_vec && ep.beta == 1.0f));
        const void* bias_base = ep.bias;
        uint32_t out_mag2 = 0;  // max |out| of this thread's fast-path outputs, two 16-bit lanes
        int local = 0;
        for (int t = blockIdx.x; t < tp.num_tiles; t += gridDim.x, ++local) {
            int b, mt, nt, ks;
            decode_tile(tp, t, b, mt, nt, ks);
            const int buf = local % NBUF;
            const uint32_t acc_phase = static_cast<uint32_t>(local / NBUF) & 1u;
            if (!mbar_wait_bounded(smem_u32(acc_full + buf), acc_phase, abort_flag, tp.err,
                                   kDevErrWaitAccFull)) {
                break;
            }
            tc_fence_after();
            const uint32_t t_buf = t_row + buf * C::BUF_COLS;
            const int64_t m = static_cast<int64_t>(mt) * BM + row;
            // a split reduction's chunks only add integer sums: no scale (the
            // scale pointers may be unset until the finishing pass)
            const double s = tp.acc64 != nullptr ? 0.0 : epi_scale(ep, b);
            const bool row_ok = m < ep.M;
            int64_t out_row;
            void* const obase = row_out(ep, b, m, out_row);
            if constexpr (FAST_ONLY) {
                // Two phases: the accumulators of this warp's chunks become
                // their binary16 values (the one rounding of the dequantised
                // product) and the TMEM buffer is released at once, so the
                // next tile's MMAs run during the bias / addend / activation
                // arithmetic and the stores.
                constexpr int NCH = (BN / 16) / (EW / 4);
                __half2 hv[NCH][8];
#pragma unroll
                for (int i = 0; i < NCH; ++i) {
                    const int c = half + i * (EW / 4);
                    uint32_t hh[16], mid[16], ll[16];
                    tmem_ld_32x32b_x16(t_buf + c * 16, hh);
                    tmem_ld_32x32b_x16(t_buf + BN + c * 16, mid);
                    tmem_ld_32x32b_x16(t_buf + 2 * BN + c * 16, ll);
                    tc_wait_ld();
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        hv[i][j] = __halves2half2(
                            __double2half(__dmul_rn(limb_acc_to_double(hh[2 * j], mid[2 * j], ll[2 * j]), s)),
                            __double2half(__dmul_rn(limb_acc_to_double(hh[2 * j + 1], mid[2 * j + 1], ll[2 * j + 1]), s)));
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(acc_empty + buf));
                if (!row_ok) continue;
#pragma unroll
                for (int i = 0; i < NCH; ++i) {
                    const int64_t n0 = static_cast<int64_t>(nt) * BN + (half + i * (EW / 4)) * 16;
                    if (n0 >= ep.N) continue;
                    // the fast path's order: bias, then addend, then activation,
                    // each a binary16 operation rounded once
                    if (has_bias) {
                        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const __half*>(bias_base) + n0);
                        const uint4 q0 = __ldg(src), q1 = __ldg(src + 1);
                        const __half2* b0 = reinterpret_cast<const __half2*>(&q0);
                        const __half2* b1 = reinterpret_cast<const __half2*>(&q1);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            hv[i][j] = __hadd2(hv[i][j], b0[j]);
                            hv[i][4 + j] = __hadd2(hv[i][4 + j], b1[j]);
                        }
                    }
                    if (has_add) {
                        const uint4* src = reinterpret_cast<const uint4*>(
                            static_cast<const __half*>(ep.addend) + b * ep.add_sb + m * ep.add_sm + n0);
                        const uint4 q0 = __ldg(src), q1 = __ldg(src + 1);
                        const __half2* a0 = reinterpret_cast<const __half2*>(&q0);
                        const __half2* a1 = reinterpret_cast<const __half2*>(&q1);
                        if constexpr (ACT == TK_ACT_SILU_GATE) {
                            // y = T(T(silu(gate)) * up): the product of two binary16
                            // values is exact in binary32, so the packed multiply
                            // rounds it once, as the separate swish + mul
#pragma unroll
                            for (int j = 0; j < 8; ++j) {
                                const float2 g = __half22float2(j < 4 ? a0[j] : a1[j - 4]);
                                hv[i][j] = __hmul2(hv[i][j], __floats2half2_rn(silu_f(g.x), silu_f(g.y)));
                            }
                        } else {
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                hv[i][j] = __hadd2(hv[i][j], a0[j]);
                                hv[i][4 + j] = __hadd2(hv[i][4 + j], a1[j]);
                            }
                        }
                    }
                    if constexpr (ACT != TK_ACT_NONE && ACT != TK_ACT_SILU_GATE) {
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const float2 f = __half22float2(hv[i][j]);
                            hv[i][j] = __floats2half2_rn(act_t<ACT>(f.x, DT), act_t<ACT>(f.y, DT));
                        }
                    }
                    if (ep.amax_out != nullptr) {
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            out_mag2 = __vmaxu2(out_mag2, *reinterpret_cast<const uint32_t*>(&hv[i][j]) & 0x7FFF7FFFu);
                    }
                    uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(obase) + out_row + n0);
                    const uint4* w = reinterpret_cast<const uint4*>(hv[i]);
                    dst[0] = w[0];
                    dst[1] = w[1];
                }
            } else {
#pragma unroll 1
                for (int c = half; c < BN / 16; c += EW / 4) {  // 16-column chunks, the quarter's warps alternating
                    const int64_t n0 = static_cast<int64_t>(nt) * BN + c * 16;
                    const bool full = n0 + 16 <= ep.N;
                    // fp16 fast path: whole chunk, no alpha, vector bias / addend / store
                    const bool fast = FAST_ONLY || (DT == 0 && fast_ok && row_ok && full);
                    uint4 add_q[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
                    if (fast && has_add) {  // issued before the TMEM loads to hide its latency
                        const uint4* src = reinterpret_cast<const uint4*>(
                            static_cast<const __half*>(ep.addend) + b * ep.add_sb + m * ep.add_sm + n0);
                        add_q[0] = __ldg(src);
                        add_q[1] = __ldg(src + 1);
                    }
                    uint32_t hh[16], mid[16], ll[16];
                    tmem_ld_32x32b_x16(t_buf + c * 16, hh);
                    tmem_ld_32x32b_x16(t_buf + BN + c * 16, mid);
                    tmem_ld_32x32b_x16(t_buf + 2 * BN + c * 16, ll);
                    tc_wait_ld();
                    if (!row_ok || n0 >= ep.N) continue;
                    if (!FAST_ONLY && tp.acc64 != nullptr) {
                        // K chunk of a split reduction: add its exact int64 sums
                        const int64_t slice = tp.acc_mod ? b % tp.acc_mod : b;
                        unsigned long long* dst = tp.acc64 + (slice * ep.M + m) * ep.N + n0;
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            if (full || n0 + j < ep.N)
                                atomicAdd(dst + j, static_cast<unsigned long long>(
                                                       limb_acc_to_i64(hh[j], mid[j], ll[j])));
                        continue;
                    }
                    if constexpr (DT == 0) {
                        if (fast) {
                            // One binary64 -> binary16 rounding, then the bias and
                            // addend in binary16: each add of two binary16 values
                            // rounded once equals the binary32 add rounded to
                            // binary16 (binary32 has more than 2*11 + 2 bits).
                            __half2 hv[8];
#pragma unroll
                            for (int j = 0; j < 8; ++j)
                                hv[j] = __halves2half2(
                                    __double2half(__dmul_rn(limb_acc_to_double(hh[2 * j], mid[2 * j], ll[2 * j]), s)),
                                    __double2half(__dmul_rn(limb_acc_to_double(hh[2 * j + 1], mid[2 * j + 1], ll[2 * j + 1]), s)));
                            if (has_bias) {
                                const uint4* src = reinterpret_cast<const uint4*>(static_cast<const __half*>(bias_base) + n0);
                                const uint4 q0 = __ldg(src), q1 = __ldg(src + 1);
                                const __half2* b0 = reinterpret_cast<const __half2*>(&q0);
                                const __half2* b1 = reinterpret_cast<const __half2*>(&q1);
#pragma unroll
                                for (int j = 0; j < 4; ++j) {
                                    hv[j] = __hadd2(hv[j], b0[j]);
                                    hv[4 + j] = __hadd2(hv[4 + j], b1[j]);
                                }
                            }
                            if (has_add) {
                                const __half2* a2 = reinterpret_cast<const __half2*>(add_q);
#pragma unroll
                                for (int j = 0; j < 8; ++j) hv[j] = __hadd2(hv[j], a2[j]);
                            }
                            if constexpr (ACT != TK_ACT_NONE) {
#pragma unroll
                                for (int j = 0; j < 8; ++j) {
                                    const float2 f = __half22float2(hv[j]);
                                    hv[j] = __floats2half2_rn(act_t<ACT>(f.x, DT), act_t<ACT>(f.y, DT));
                                }
                            }
                            if (ep.amax_out != nullptr) {
                                // magnitudes as 16-bit patterns: NaN > Inf > finite
#pragma unroll
                                for (int j = 0; j < 8; ++j)
                                    out_mag2 = __vmaxu2(out_mag2, *reinterpret_cast<const uint32_t*>(&hv[j]) & 0x7FFF7FFFu);
                            }
                            uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(obase) + out_row + n0);
                            const uint4* w = reinterpret_cast<const uint4*>(hv);
                            dst[0] = w[0];
                            dst[1] = w[1];
                            continue;
                        }
                    }
                    if constexpr (!FAST_ONLY) {
                    float v[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        v[j] = round_t_from_double(__dmul_rn(limb_acc_to_double(hh[j], mid[j], ll[j]), s), DT);
                    if (has_alpha) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[j] = round_t(__fmul_rn(v[j], ep.alpha), DT);
                    }
                    if (has_bias) {
                        float bv[16];
                        const void* bias_base = ep.bias_mod
                            ? static_cast<const void*>(static_cast<const char*>(ep.bias) +
                                  (b % ep.bias_mod) * ep.N * (DT == 0 ? 2 : 4))
                            : ep.bias;
                        if (full && ep.bias_vec) {
                            // 16 consecutive bias values with 128-bit loads (the
                            // same addresses for the whole warp: one broadcast).
                            if constexpr (DT == 0) {
                                const uint4* src = reinterpret_cast<const uint4*>(
                                    static_cast<const __half*>(bias_base) + n0);
                                uint4 q[2] = {__ldg(src), __ldg(src + 1)};
                                const __half2* h2 = reinterpret_cast<const __half2*>(q);
#pragma unroll
                                for (int j = 0; j < 8; ++j) {
                                    const float2 f = __half22float2(h2[j]);
                                    bv[2 * j] = f.x;
                                    bv[2 * j + 1] = f.y;
                                }
                            } else {
                                const float4* src = reinterpret_cast<const float4*>(
                                    static_cast<const float*>(bias_base) + n0);
#pragma unroll
                                for (int j = 0; j < 4; ++j) {
                                    const float4 f = __ldg(src + j);
                                    bv[4 * j] = f.x; bv[4 * j + 1] = f.y;
                                    bv[4 * j + 2] = f.z; bv[4 * j + 3] = f.w;
                                }
                            }
                        } else {
#pragma unroll
                            for (int j = 0; j < 16; ++j)
                                bv[j] = (n0 + j < ep.N) ? load_t(bias_base, DT, n0 + j) : 0.0f;
                        }
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[j] = round_t(__fadd_rn(v[j], bv[j]), DT);
                    }
                    if (has_add) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            if (!full && n0 + j >= ep.N) continue;
                            float a = load_t(ep.addend, DT, b * ep.add_sb + m * ep.add_sm + (n0 + j) * ep.add_sn);
                            if (ep.beta != 1.0f) a = round_t(__fmul_rn(a, ep.beta), DT);
                            v[j] = round_t(__fadd_rn(v[j], a), DT);
                        }
                    }
                    if constexpr (ACT != TK_ACT_NONE) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[j] = act_t<ACT>(v[j], DT);
                    }
                    if (ep.dbg != nullptr && b == 0) {
                        for (int j = 0; j < 16 && n0 + j < ep.N; ++j) {
                            ep.dbg[(0 * ep.M + m) * ep.N + n0 + j] = static_cast<int32_t>(hh[j]);
                            ep.dbg[(1 * ep.M + m) * ep.N + n0 + j] = static_cast<int32_t>(mid[j]);
                            ep.dbg[(2 * ep.M + m) * ep.N + n0 + j] = static_cast<int32_t>(ll[j]);
                        }
                    }
                    if (ep.vec_store && full) {
                        if constexpr (DT == 0) {
                            uint32_t w[8];
#pragma unroll
                            for (int j = 0; j < 8; ++j) {
                                __half2 h2 = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
                                w[j] = *reinterpret_cast<uint32_t*>(&h2);
                            }
                            uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(obase) + out_row + n0);
                            dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
                            dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
                        } else {
                            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(obase) + out_row + n0);
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            if (full || n0 + j < ep.N) store_t(obase, ep.dtype, out_row + (n0 + j) * ep.out_sn, v[j]);
                    }
                    }  // !FAST_ONLY
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(acc_empty + buf));
            }
        }
        if (ep.amax_out != nullptr) {
            unsigned hmag = max(out_mag2 & 0xFFFFu, out_mag2 >> 16);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) hmag = max(hmag, __shfl_xor_sync(0xffffffffu, hmag, o));
            if (lane == 0 && hmag != 0u) {
                // widened to the fp32 magnitude bits (NaN canonical), as the amax kernels
                const unsigned bits = ((hmag & 0x7C00u) == 0x7C00u && (hmag & 0x3FFu) != 0u)
                                          ? 0x7FC00000u
                                          : (__float_as_uint(__half2float(__ushort_as_half(
                                                 static_cast<unsigned short>(hmag)))) & 0x7FFFFFFFu);
                atomicMax(ep.amax_out, bits);
            }
        }
        // stores into other GPUs' memory are ordered before anything this
        // GPU does after the kernel
        if (ep.row_dest_rows > 0) __threadfence_system();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// ---- CUDA-core cross-check kernel ------------------------------------------------

__global__ void qgemm_simt_kernel(const int8_t* __restrict__ la, const int8_t* __restrict__ lb,
                                  int64_t batch, int64_t K, int64_t ld, EpiParams ep) {
    const int64_t n = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t m = blockIdx.y;
    const int64_t b = blockIdx.z;
    if (n >= ep.N) return;
    const int64_t pa = ep.M * ld, pb = ep.N * ld;
    const int8_t* ahi = la + (2 * b) * pa + m * ld;
    const int8_t* alo = ahi + pa;
    const int8_t* bhi = lb + (2 * b) * pb + n * ld;
    const int8_t* blo = bhi + pb;
    int64_t acc = 0;
    for (int64_t k = 0; k < K; ++k) {
        const int64_t qa = 256 * static_cast<int64_t>(ahi[k]) +
                           static_cast<int64_t>(static_cast<uint8_t>(alo[k]));
        const int64_t qb = 256 * static_cast<int64_t>(bhi[k]) +
                           static_cast<int64_t>(static_cast<uint8_t>(blo[k]));
        acc += qa * qb;
    }
    const double s = epi_scale(ep, b);
    const float v = epilogue_one(ep, s, static_cast<double>(acc), b, m, n);
    int64_t row_off;
    void* base = row_out(ep, b, m, row_off);
    store_t(base, ep.dtype, row_off + n * ep.out_sn, v);
}

// The epilogue of a split reduction: acc64 [slices][M][N] holds the exact
// int64 sums; each is converted to binary64 with one round-to-nearest (exact
// below 2^53) and goes through the same post-GEMM sequence as the fused
// epilogue.
__global__ void qgemm_acc64_finish_kernel(const long long* __restrict__ acc, int64_t slices,
                                          EpiParams ep) {
    const int64_t mn = ep.M * ep.N;
    const int64_t total = slices * mn;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t b = i / mn;
        const int64_t r = i - b * mn;
        const int64_t m = r / ep.N;
        const int64_t n = r - m * ep.N;
        const double s = epi_scale(ep, b);
        const float v = epilogue_one(ep, s, __ll2double_rn(acc[i]), b, m, n);
        int64_t row_off;
        void* base = row_out(ep, b, m, row_off);
        store_t(base, ep.dtype, row_off + n * ep.out_sn, v);
    }
}

// ---- host side --------------------------------------------------------------------

EncodeTiledFn get_encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<EncodeTiledFn>(p);
        }
    });
    return fn;
}

// Tensor map over limb planes [planes][rows][ld] (uint8), box 128 x 128 x 1.
int make_limb_map(CUtensorMap* map, const int8_t* base, int64_t planes, int64_t rows, int64_t ld,
                  int box_rows) {
    EncodeTiledFn enc = get_encode_fn();
    if (enc == nullptr) TK_FAIL(TK_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(ld), static_cast<cuuint64_t>(rows),
                          static_cast<cuuint64_t>(planes)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld), static_cast<cuuint64_t>(rows * ld)};
    cuuint32_t box[3] = {BK, static_cast<cuuint32_t>(box_rows), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t*>(base), dims,
                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) TK_FAIL(TK_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return TK_OK;
}

// N-tile width of the tile configuration choose_tiles picks (below).
int tile_bn(int64_t k) { return k >= 2048 ? CfgWider::BN : CfgWide::BN; }

// Split reductions (see the file header): always for K > 32768, and for
// K >= 4096 when the problem has at most 64 output tiles (a weight-gradient
// shape: a small output over a long reduction), which would otherwise leave
// most SMs idle.  The decision depends on the descriptor alone, so the
// workspace size is known without a device.
bool split_k(const tk_qgemm_desc_t& d) {
    if (d.k > kMaxK) return true;
    const int64_t tiles = d.batch * ceil_div(d.m, BM) * ceil_div(d.n, tile_bn(d.k));
    return d.k >= 4096 && tiles <= 64;
}

struct Layout {
    int64_t ld;        // padded K (bytes per limb row)
    size_t off_amax_a, off_amax_b, off_la, off_lb, off_acc, total;
    bool split;        // acc64 [batch][m][n] int64 sums at off_acc
};

Layout workspace_layout(const tk_qgemm_desc_t& d) {
    Layout L;
    L.ld = static_cast<int64_t>(round_up(static_cast<size_t>(std::max<int64_t>(d.k, 1)), 16));
    const int64_t nscale = d.per_slice_scales ? d.batch : 1;
    L.off_amax_a = 0;
    L.off_amax_b = round_up(sizeof(float) * nscale, 256);
    L.off_la = round_up(L.off_amax_b + sizeof(float) * nscale, 1024);
    L.off_lb = round_up(L.off_la + static_cast<size_t>(d.batch * 2 * d.m * L.ld), 1024);
    L.off_acc = round_up(L.off_lb + static_cast<size_t>(d.batch * 2 * d.n * L.ld), 1024);
    L.split = split_k(d);
    L.total = L.off_acc;
    if (L.split) L.total = round_up(L.off_acc + sizeof(int64_t) * static_cast<size_t>(d.batch * d.m * d.n), 1024);
    return L;
}

int validate(const tk_qgemm_desc_t& d) {
    TK_CHECK_ARG(d.dtype == TK_DTYPE_F16 || d.dtype == TK_DTYPE_F32, "qgemm: bad dtype %d",
                 (int)d.dtype);
    TK_CHECK_ARG(d.batch >= 0 && d.m >= 0 && d.n >= 0 && d.k >= 0, "qgemm: negative size");
    TK_CHECK_ARG(d.batch <= 65535 && d.m < (1LL << 31) && d.n < (1LL << 31) && d.k < (1LL << 31),
                 "qgemm: size out of range");
    TK_CHECK_ARG(d.act >= TK_ACT_NONE && d.act <= TK_ACT_SILU_GATE, "qgemm: bad act %d", (int)d.act);
    if (d.act == TK_ACT_SILU_GATE)
        TK_CHECK_ARG(d.dtype == TK_DTYPE_F16 && d.addend != nullptr && d.beta == 1.0f,
                     "qgemm: TK_ACT_SILU_GATE needs fp16, the gate as addend and beta == 1");
    if (d.batch * d.m * d.n > 0) TK_CHECK_ARG(d.out != nullptr, "qgemm: out is NULL");
    return TK_OK;
}

bool slice_dense(int64_t rows, int64_t cols, int64_t sr, int64_t sc) {
    if (rows <= 1 || cols <= 1) return true;
    return (sr == cols && sc == 1) || (sr == 1 && sc == rows);
}

// An operand whose amax is computed by the call must be laid out densely:
// every slice a row- or column-major block and, for one shared scale, the
// slices one contiguous block.
int check_dense(const void* x, int64_t batch, int64_t rows, int64_t cols, int64_t sb, int64_t sr,
                int64_t sc, bool per_slice, const float* given_amax, const char* name) {
    if (given_amax != nullptr || rows * cols == 0) return TK_OK;
    TK_CHECK_ARG(x != nullptr, "qgemm: operand %s is NULL", name);
    if (!slice_dense(rows, cols, sr, sc))
        TK_FAIL(TK_ERR_UNSUPPORTED, "qgemm: operand %s slices must be dense (row- or column-major)",
                name);
    if (!per_slice && batch > 1 && sb != rows * cols)
        TK_FAIL(TK_ERR_UNSUPPORTED, "qgemm: operand %s must be one dense block for a shared scale",
                name);
    return TK_OK;
}

EpiParams make_epi(const tk_qgemm_desc_t& d, const float* amax_a, const float* amax_b,
                   int32_t* dbg) {
    EpiParams ep;
    ep.dtype = d.dtype == TK_DTYPE_F16 ? 0 : 1;
    ep.M = d.m;
    ep.N = d.n;
    ep.out = d.out;
    ep.out_sb = d.out_sb;
    ep.out_sm = d.out_sm;
    ep.out_sn = 1;
    ep.bias = d.bias;
    ep.bias_mod = 0;
    ep.addend = d.addend;
    ep.add_sb = d.add_sb;
    ep.add_sm = d.add_sm;
    ep.add_sn = d.add_sn;
    ep.alpha = d.alpha;
    ep.beta = d.beta;
    ep.act = d.act;
    ep.amax_a = amax_a;
    ep.amax_b = amax_b;
    ep.scale_stride = d.per_slice_scales ? 1 : 0;
    const size_t es = dtype_size(d.dtype);
    ep.vec_store = (reinterpret_cast<uintptr_t>(d.out) % 16 == 0) &&
                   ((d.out_sm * static_cast<int64_t>(es)) % 16 == 0) &&
                   (d.batch <= 1 || (d.out_sb * static_cast<int64_t>(es)) % 16 == 0);
    ep.bias_vec = d.bias != nullptr && reinterpret_cast<uintptr_t>(d.bias) % 16 == 0 &&
                  (ep.bias_mod == 0 || (d.n * static_cast<int64_t>(es)) % 16 == 0);
    ep.add_vec = d.addend != nullptr && reinterpret_cast<uintptr_t>(d.addend) % 16 == 0 &&
                 d.add_sn == 1 && (d.add_sm * static_cast<int64_t>(es)) % 16 == 0 &&
                 (d.add_sb * static_cast<int64_t>(es)) % 16 == 0;
    ep.dbg = dbg;
    ep.amax_out = nullptr;
    for (int i = 0; i < kMaxRowDests; ++i) ep.row_dest[i] = nullptr;
    ep.row_dest_rows = 0;
    ep.row_dest_n = 0;
    return ep;
}

// Rows scattered over destination buffers (tk_qgemm_scatter_rows).
struct RowScatter {
    void* const* dest;
    int n;
    int64_t rows;
};

enum class Path { TensorCore, Simt };

template <class C, int DT, int ACT, int EW, bool FO>
int launch_one(int dev, int grid, const CUtensorMap& tmA, const CUtensorMap& tmB,
               const TileParams& tp, const EpiParams& ep, cudaStream_t stream) {
    static std::once_flag attr_once[64];
    if (dev >= 0 && dev < 64) {
        std::call_once(attr_once[dev], [] {
            cudaFuncSetAttribute(qgemm_tc_kernel<C, DT, ACT, EW, FO>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        });
    }
    // programmatic stream serialisation: the CTAs may be placed and run
    // their prologue while the quantise kernel before them drains
    TK_CUDA_TRY(launch_pdl(qgemm_tc_kernel<C, DT, ACT, EW, FO>, static_cast<unsigned>(grid), 64 + 32 * EW,
                           C::SMEM, stream, tmA, tmB, tp, ep));
    return TK_OK;
}

template <class C, int DT, int EW, bool FO>
int dispatch_act_ew(int act, int dev, int grid, const CUtensorMap& tmA, const CUtensorMap& tmB,
                    const TileParams& tp, const EpiParams& ep, cudaStream_t stream) {
    switch (act) {
        case TK_ACT_NONE: return launch_one<C, DT, TK_ACT_NONE, EW, FO>(dev, grid, tmA, tmB, tp, ep, stream);
        case TK_ACT_RELU: return launch_one<C, DT, TK_ACT_RELU, EW, FO>(dev, grid, tmA, tmB, tp, ep, stream);
        case TK_ACT_GELU: return launch_one<C, DT, TK_ACT_GELU, EW, FO>(dev, grid, tmA, tmB, tp, ep, stream);
        case TK_ACT_GELU_TANH:
            return launch_one<C, DT, TK_ACT_GELU_TANH, EW, FO>(dev, grid, tmA, tmB, tp, ep, stream);
        case TK_ACT_SILU: return launch_one<C, DT, TK_ACT_SILU, EW, FO>(dev, grid, tmA, tmB, tp, ep, stream);
        case TK_ACT_SILU_GATE:
            if constexpr (FO) {
                return launch_one<C, DT, TK_ACT_SILU_GATE, EW, FO>(dev, grid, tmA, tmB, tp, ep, stream);
            } else {
                TK_FAIL(TK_ERR_UNSUPPORTED, "qgemm: TK_ACT_SILU_GATE runs on the fp16 vector epilogue only");
            }
        default: TK_FAIL(TK_ERR_INVALID_ARG, "qgemm: bad act %d", act);
    }
}

// Whether the whole problem takes the fp16 fast epilogue (every chunk full,
// no alpha, vector bias / addend / stores, no split reduction): then the
// 16-warp epilogue runs.
bool fast_epilogue_ep(const EpiParams& ep) {
    return ep.dtype == 0 && ep.vec_store && ep.alpha == 1.0f && ep.dbg == nullptr &&
           (ep.bias == nullptr || (ep.bias_vec && ep.bias_mod == 0)) &&
           (ep.addend == nullptr || ep.beta == 0.0f || (ep.add_vec && ep.beta == 1.0f)) && ep.N % 16 == 0;
}

bool fast_epilogue(const TileParams& tp, const EpiParams& ep) {
    return tp.acc64 == nullptr && fast_epilogue_ep(ep);
}

template <class C, int DT>
int dispatch_act(int act, int dev, int grid, const CUtensorMap& tmA, const CUtensorMap& tmB,
                 const TileParams& tp, const EpiParams& ep, cudaStream_t stream) {
    // The fast-only epilogue (fp16 fast path for the whole problem) frees the
    // accumulators as soon as they are binary16 values.  Short reductions
    // (128x128 tiles, K < 2048), where the epilogue outweighs the tile's
    // MMAs, run it on sixteen warps; with K >= 2048 sixteen warps measured no
    // faster (2048x4096x4096) or slower (the TP MLP's K = 8192 GEMMs, 3 %),
    // so the 128x160 tiles keep eight.
    if constexpr (DT == 0 && (C::BN == 128 || C::BN == 160)) {
        if (fast_epilogue(tp, ep)) {
            constexpr int EWF = C::BN == 128 ? 2 * NUM_EPI_WARPS : NUM_EPI_WARPS;
            return dispatch_act_ew<C, DT, EWF, true>(act, dev, grid, tmA, tmB, tp, ep, stream);
        }
    }
    return dispatch_act_ew<C, DT, NUM_EPI_WARPS, false>(act, dev, grid, tmA, tmB, tp, ep, stream);
}

// Tile configuration for a problem: 128x160 tiles for K >= 2048, else
// 128x128.  The double-buffered 128x64 / 128x80 configurations
// (CfgOverlap64 / CfgOverlap80) measured slower on every benchmark shape and
// are not selected.
enum class TileChoice { Wide, Wider };

TileChoice choose_tiles(const tk_qgemm_desc_t& d) {
    return tile_bn(d.k) == CfgWider::BN ? TileChoice::Wider : TileChoice::Wide;
}

// Where a split reduction adds its int64 sums (acc64 == nullptr: no split).
struct SplitAcc {
    unsigned long long* acc64 = nullptr;
    int acc_mod = 0;
};

template <class C>
int launch_cfg(const tk_qgemm_desc_t& d, const int8_t* la, const int8_t* lb, int64_t ld,
               const EpiParams& ep, cudaStream_t stream, int b_mod, const SplitAcc& sa) {
    CUtensorMap tmA, tmB;
    int rc = make_limb_map(&tmA, la, 2 * d.batch, d.m, ld, BM);
    if (rc) return rc;
    rc = make_limb_map(&tmB, lb, 2 * (b_mod ? b_mod : d.batch), d.n, ld, C::BN);
    if (rc) return rc;
    TileParams tp;
    tp.b_mod = b_mod;
    tp.batch = static_cast<int>(d.batch);
    tp.tiles_m = static_cast<int>(ceil_div(d.m, BM));
    tp.tiles_n = static_cast<int>(ceil_div(d.n, C::BN));
    const int64_t tiles = static_cast<int64_t>(tp.tiles_m) * tp.tiles_n * d.batch;
    tp.num_kb = static_cast<int>(ceil_div(d.k, BK));
    const int dev = current_device();
    // K chunks: at most kMaxK / BK blocks each (exact int32 limb sums); with
    // few tiles, enough chunks of at least 16 blocks to occupy the SMs
    int ksplit = 1;
    if (sa.acc64 != nullptr) {
        ksplit = static_cast<int>(ceil_div(tp.num_kb, kMaxK / BK));
        const int64_t fill = std::min<int64_t>(ceil_div(sm_count(dev), tiles), tp.num_kb / 16);
        ksplit = static_cast<int>(std::max<int64_t>(ksplit, fill));
        ksplit = std::max(ksplit, 1);
    }
    tp.kb_per_split = static_cast<int>(ceil_div(tp.num_kb, ksplit));
    tp.ksplit = static_cast<int>(ceil_div(tp.num_kb, tp.kb_per_split));
    tp.acc64 = sa.acc64;
    tp.acc_mod = sa.acc_mod;
    const int64_t nt = tiles * tp.ksplit;
    TK_CHECK_ARG(nt < (1LL << 31), "qgemm: too many tiles");
    tp.num_tiles = static_cast<int>(nt);
    tp.err = device_error_word(dev);
    const int grid = static_cast<int>(std::min<int64_t>(nt, sm_count(dev)));
    rc = d.dtype == TK_DTYPE_F16
             ? dispatch_act<C, 0>(static_cast<int>(d.act), dev, grid, tmA, tmB, tp, ep, stream)
             : dispatch_act<C, 1>(static_cast<int>(d.act), dev, grid, tmA, tmB, tp, ep, stream);
    if (rc) return rc;
    return launch_status("qgemm_tc");
}

int launch_tc(const tk_qgemm_desc_t& d, const int8_t* la, const int8_t* lb, int64_t ld,
              const EpiParams& ep, cudaStream_t stream, int b_mod = 0, const SplitAcc& sa = SplitAcc{}) {
    if (sa.acc64 == nullptr)
        TK_CHECK_ARG(d.k <= kMaxK, "qgemm: K=%lld exceeds %d on a path without a split workspace",
                     (long long)d.k, kMaxK);
    switch (choose_tiles(d)) {
        case TileChoice::Wider: return launch_cfg<CfgWider>(d, la, lb, ld, ep, stream, b_mod, sa);
        default: return launch_cfg<CfgWide>(d, la, lb, ld, ep, stream, b_mod, sa);
    }
}

// The finishing pass of a split reduction over acc64 [slices][M][N].
int launch_finish(const long long* acc64, int64_t slices, const EpiParams& ep, cudaStream_t stream) {
    const int64_t total = slices * ep.M * ep.N;
    if (total == 0) return TK_OK;
    const int dev = current_device();
    const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>(ceil_div(total, 256), 8LL * sm_count(dev)));
    qgemm_acc64_finish_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(acc64, slices, ep);
    return launch_status("qgemm_finish");
}

int run(const tk_qgemm_desc_t* desc, void* ws, size_t ws_bytes, cudaStream_t stream, Path path,
        int32_t* dbg, const RowScatter* scatter = nullptr) {
    TK_CHECK_ARG(desc != nullptr, "qgemm: desc is NULL");
    const tk_qgemm_desc_t& d = *desc;
    int rc = scatter ? TK_OK : validate(d);
    if (scatter) {
        tk_qgemm_desc_t v = d;
        v.out = scatter->n > 0 ? scatter->dest[0] : nullptr;  // validated below per destination
        rc = validate(v);
    }
    if (rc) return rc;
    if (d.batch == 0 || d.m == 0 || d.n == 0) return TK_OK;
    const Layout L = workspace_layout(d);
    TK_CHECK_ARG(ws != nullptr && ws_bytes >= L.total,
                 "qgemm: workspace too small (%zu < %zu bytes)", ws_bytes, L.total);
    TK_CHECK_ARG(reinterpret_cast<uintptr_t>(ws) % 1024 == 0,
                 "qgemm: workspace must be 1024-byte aligned");
    uint8_t* w = static_cast<uint8_t*>(ws);
    float* amax_a = reinterpret_cast<float*>(w + L.off_amax_a);
    float* amax_b = reinterpret_cast<float*>(w + L.off_amax_b);
    int8_t* la = reinterpret_cast<int8_t*>(w + L.off_la);
    int8_t* lb = reinterpret_cast<int8_t*>(w + L.off_lb);
    const bool per = d.per_slice_scales != 0;
    // Both amax slots are cleared with one memset (they are adjacent), then one
    // launch reduces every amax that was not given and one quantises both
    // row-contiguous operands.
    TK_CUDA_TRY(cudaMemsetAsync(amax_a, 0, L.off_la, stream));
    if (d.k > 0) {
        rc = check_dense(d.a, d.batch, d.m, d.k, d.a_sb, d.a_sm, d.a_sk, per, d.amax_a, "A");
        if (rc) return rc;
        rc = check_dense(d.b, d.batch, d.n, d.k, d.b_sb, d.b_sn, d.b_sk, per, d.amax_b, "B");
        if (rc) return rc;
        QuantOperand ops[2] = {
            {d.a, d.batch, d.m, d.k, d.a_sb, d.a_sm, d.a_sk, per, d.amax_a, amax_a, la},
            {d.b, d.batch, d.n, d.k, d.b_sb, d.b_sn, d.b_sk, per, d.amax_b, amax_b, lb}};
        rc = quantise_operands(d.dtype, ops, 2, stream);
        if (rc) return rc;
    }
    const float* sa = (d.k > 0 && d.amax_a) ? d.amax_a : amax_a;
    const float* sb = (d.k > 0 && d.amax_b) ? d.amax_b : amax_b;
    EpiParams ep = make_epi(d, sa, sb, dbg);
    if (scatter) {
        const size_t es = dtype_size(d.dtype);
        bool vec = (d.out_sm * static_cast<int64_t>(es)) % 16 == 0;
        for (int i = 0; i < scatter->n; ++i) {
            ep.row_dest[i] = scatter->dest[i];
            vec = vec && reinterpret_cast<uintptr_t>(scatter->dest[i]) % 16 == 0;
        }
        ep.row_dest_rows = scatter->rows;
        ep.row_dest_n = scatter->n;
        ep.out = nullptr;
        ep.vec_store = vec;
    }

    // max |out| for the caller: folded into the fp16 vector epilogue, or one
    // pass over the finished output
    bool amax_folded = false;
    if (d.amax_out != nullptr) {
        TK_CHECK_ARG(scatter == nullptr, "qgemm: amax_out with scattered rows is not supported");
        amax_folded = path == Path::TensorCore && d.k > 0 && !(L.split && dbg == nullptr) && fast_epilogue_ep(ep);
        if (amax_folded) {
            TK_CUDA_TRY(cudaMemsetAsync(d.amax_out, 0, sizeof(float), stream));
            ep.amax_out = reinterpret_cast<unsigned*>(d.amax_out);
        } else {
            TK_CHECK_ARG(d.out_sm == d.n && (d.batch <= 1 || d.out_sb == d.m * d.n),
                         "qgemm: amax_out needs a contiguous output on this path");
        }
    }
    auto out_amax_pass = [&]() -> int {
        if (d.amax_out == nullptr || amax_folded) return TK_OK;
        return amax_launch(d.dtype, d.out, 1, 0, d.batch * d.m * d.n, d.amax_out, stream);
    };

    if (path == Path::Simt || d.k == 0) {
        if (d.act == TK_ACT_SILU_GATE) TK_FAIL(TK_ERR_UNSUPPORTED, "qgemm: TK_ACT_SILU_GATE needs K > 0 on the tensor-core path");
        dim3 grid(static_cast<unsigned>(ceil_div(d.n, 128)), static_cast<unsigned>(d.m),
                  static_cast<unsigned>(d.batch));
        TK_CHECK_ARG(d.m <= 65535 || path == Path::TensorCore,
                     "qgemm_simt: m must be <= 65535");
        if (d.m > 65535) TK_FAIL(TK_ERR_UNSUPPORTED, "qgemm: K=0 with m > 65535");
        qgemm_simt_kernel<<<grid, 128, 0, stream>>>(la, lb, d.batch, d.k, L.ld, ep);
        rc = launch_status("qgemm_simt");
        return rc ? rc : out_amax_pass();
    }

    if (L.split && dbg == nullptr && scatter == nullptr) {
        SplitAcc sa;
        sa.acc64 = reinterpret_cast<unsigned long long*>(w + L.off_acc);
        TK_CUDA_TRY(cudaMemsetAsync(sa.acc64, 0, sizeof(int64_t) * static_cast<size_t>(d.batch * d.m * d.n),
                                    stream));
        rc = launch_tc(d, la, lb, L.ld, ep, stream, 0, sa);
        if (rc) return rc;
        rc = launch_finish(reinterpret_cast<const long long*>(sa.acc64), d.batch, ep, stream);
        return rc ? rc : out_amax_pass();
    }
    rc = launch_tc(d, la, lb, L.ld, ep, stream);
    return rc ? rc : out_amax_pass();
}

}  // namespace

EncodeTiledFn tensor_map_encoder() { return get_encode_fn(); }

int qgemm_validate(const tk_qgemm_desc_t& d) { return validate(d); }

// Split-reduction GEMM on prepared limbs that only adds its exact int64 sums
// into acc64 (slice b % acc_mod, or b when acc_mod is 0); the caller zeroes
// acc64 once and runs qgemm_acc64_finish after the last contribution.  Used
// by the convolution weight gradient, whose reduction runs over images and
// pixels.
int qgemm_limbs_acc64(const tk_qgemm_desc_t& d, const int8_t* la, const int8_t* lb,
                      unsigned long long* acc64, int acc_mod, cudaStream_t stream) {
    int rc = validate(d);
    if (rc) return rc;
    if (d.batch == 0 || d.m == 0 || d.n == 0 || d.k == 0) return TK_OK;
    TK_CHECK_ARG(acc64 != nullptr && la != nullptr && lb != nullptr, "qgemm_acc64: NULL pointer");
    TK_CHECK_ARG(d.amax_out == nullptr, "qgemm_acc64: amax_out is not supported");
    const int64_t ld = static_cast<int64_t>(round_up(static_cast<size_t>(d.k), 16));
    EpiParams ep = make_epi(d, nullptr, nullptr, nullptr);
    SplitAcc sa;
    sa.acc64 = acc64;
    sa.acc_mod = acc_mod;
    return launch_tc(d, la, lb, ld, ep, stream, 0, sa);
}

// The epilogue of d (dequantise with amax_a / amax_b per tensor, alpha,
// bias, addend, activation) over acc64 [slices][m][n], output element
// (b, m, n) at out[b*out_sb + m*out_sm + n*out_sn].
int qgemm_acc64_finish(const tk_qgemm_desc_t& d, const long long* acc64, int64_t slices,
                       const float* amax_a, const float* amax_b, int64_t out_sn, cudaStream_t stream) {
    int rc = validate(d);
    if (rc) return rc;
    TK_CHECK_ARG(d.amax_out == nullptr, "qgemm_acc64_finish: amax_out is not supported");
    EpiParams ep = make_epi(d, amax_a, amax_b, nullptr);
    ep.out_sn = out_sn;
    ep.scale_stride = 0;
    return launch_finish(acc64, slices, ep, stream);
}

// Internal entry used by the conv path: GEMM on prepared limbs where the B
// operand (weights) has b_mod slices shared across the batch, the output is
// written with column stride out_sn (NCHW from a pixels x channels tile) and
// the bias is indexed per group.
int qgemm_limbs_ex(const tk_qgemm_desc_t& d, const int8_t* la, const int8_t* lb,
                   const float* amax_a, const float* amax_b, int b_mod, int64_t out_sn,
                   int64_t bias_mod, cudaStream_t stream) {
    int rc = validate(d);
    if (rc) return rc;
    if (d.batch == 0 || d.m == 0 || d.n == 0) return TK_OK;
    TK_CHECK_ARG(d.k > 0, "qgemm: K must be positive");
    TK_CHECK_ARG(d.amax_out == nullptr, "qgemm_limbs_ex: amax_out is not supported");
    const int64_t ld = static_cast<int64_t>(round_up(static_cast<size_t>(d.k), 16));
    EpiParams ep = make_epi(d, amax_a, amax_b, nullptr);
    ep.out_sn = out_sn;
    ep.bias_mod = bias_mod;
    if (out_sn != 1) ep.vec_store = false;
    const size_t es = dtype_size(d.dtype);
    ep.bias_vec = d.bias != nullptr && reinterpret_cast<uintptr_t>(d.bias) % 16 == 0 &&
                  (bias_mod == 0 || (d.n * static_cast<int64_t>(es)) % 16 == 0);
    return launch_tc(d, la, lb, ld, ep, stream, b_mod);
}

}  // namespace tk

extern "C" {

size_t tk_qgemm_workspace_size(const tk_qgemm_desc_t* desc) {
    if (desc == nullptr) return 0;
    return tk::workspace_layout(*desc).total;
}

int tk_qgemm(const tk_qgemm_desc_t* desc, void* workspace, size_t workspace_bytes, void* stream) {
    return tk::run(desc, workspace, workspace_bytes, static_cast<cudaStream_t>(stream),
                   tk::Path::TensorCore, nullptr);
}

int tk_qgemm_simt(const tk_qgemm_desc_t* desc, void* workspace, size_t workspace_bytes,
                  void* stream) {
    return tk::run(desc, workspace, workspace_bytes, static_cast<cudaStream_t>(stream),
                   tk::Path::Simt, nullptr);
}

int tk_qgemm_from_limbs(const tk_qgemm_desc_t* desc, const int8_t* a_limbs, const int8_t* b_limbs,
                        const float* amax_a, const float* amax_b, void* stream) {
    using namespace tk;
    TK_CHECK_ARG(desc != nullptr, "qgemm_from_limbs: desc is NULL");
    const tk_qgemm_desc_t& d = *desc;
    int rc = validate(d);
    if (rc) return rc;
    if (d.batch == 0 || d.m == 0 || d.n == 0) return TK_OK;
    TK_CHECK_ARG(d.k > 0, "qgemm_from_limbs: K must be positive");
    TK_CHECK_ARG(a_limbs && b_limbs && amax_a && amax_b, "qgemm_from_limbs: NULL pointer");
    TK_CHECK_ARG(reinterpret_cast<uintptr_t>(a_limbs) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(b_limbs) % 16 == 0,
                 "qgemm_from_limbs: limb planes must be 16-byte aligned");
    const int64_t ld = static_cast<int64_t>(round_up(static_cast<size_t>(d.k), 16));
    EpiParams ep = make_epi(d, amax_a, amax_b, nullptr);
    if (d.amax_out != nullptr) {
        // folded into the fp16 vector epilogue, which every output takes
        TK_CHECK_ARG(fast_epilogue_ep(ep), "qgemm_from_limbs: amax_out needs the fp16 vector epilogue");
        TK_CUDA_TRY(cudaMemsetAsync(d.amax_out, 0, sizeof(float), static_cast<cudaStream_t>(stream)));
        ep.amax_out = reinterpret_cast<unsigned*>(d.amax_out);
    }
    return launch_tc(d, a_limbs, b_limbs, ld, ep, static_cast<cudaStream_t>(stream));
}

int tk_qgemm_debug(const tk_qgemm_desc_t* desc, void* workspace, size_t workspace_bytes,
                   int32_t* acc3, void* stream) {
    return tk::run(desc, workspace, workspace_bytes, static_cast<cudaStream_t>(stream),
                   tk::Path::TensorCore, acc3);
}

int tk_qgemm_scatter_rows(const tk_qgemm_desc_t* desc, void* const* row_dest, int ndest,
                          int64_t rows_per_dest, void* workspace, size_t workspace_bytes, void* stream) {
    using namespace tk;
    TK_CHECK_ARG(desc != nullptr && row_dest != nullptr, "qgemm_scatter_rows: NULL argument");
    TK_CHECK_ARG(ndest >= 1 && ndest <= kMaxRowDests, "qgemm_scatter_rows: 1..%d destinations",
                 kMaxRowDests);
    TK_CHECK_ARG(desc->batch == 1, "qgemm_scatter_rows: batch must be 1");
    TK_CHECK_ARG(rows_per_dest > 0 && rows_per_dest * ndest == desc->m,
                 "qgemm_scatter_rows: m (%lld) must equal ndest * rows_per_dest",
                 (long long)desc->m);
    TK_CHECK_ARG(desc->out_sm >= desc->n, "qgemm_scatter_rows: out_sm must be >= n");
    for (int i = 0; i < ndest; ++i)
        TK_CHECK_ARG(row_dest[i] != nullptr, "qgemm_scatter_rows: destination %d is NULL", i);
    const RowScatter sc = {row_dest, ndest, rows_per_dest};
    return run(desc, workspace, workspace_bytes, static_cast<cudaStream_t>(stream), Path::TensorCore,
               nullptr, &sc);
}

}  // extern "C"
