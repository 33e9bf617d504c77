// attention.cu -- fused scaled-dot-product attention on sm_100a tensor cores
// with the reference's int16-quantised composition semantics.
//
// The reference computes attention as separate launches
// (torch_kunlun/kunlun/attention.py:36-107): a per-slice quantised bmm
// q @ k^T (csrc/ops_nn.cpp:199-221), mul.Scalar by the scale, add of the
// causal / additive mask, softmax (csrc/ops_nn.cpp:73-83) and a per-slice
// quantised bmm with v, each a kernel writing and re-reading [L, S] tensors.
// Here the same arithmetic runs as:
//
//   attn_quant_kernel / attn_quant_staged_kernel
//                       per (batch, head) slice of q, k, v: max-abs, then
//                       int16 quantisation into int8 limb rows laid out for
//                       the tensor cores (v transposed); zeroes the slice's
//                       probability amax.  The staged form holds an fp16
//                       slice of up to 64 KB in shared memory (one HBM read).
//   attn_fused_kernel   fp16 slices of at most 512 queries and keys, head dim
//                       <= 128: one persistent thread-block cluster per slice
//                       keeps the scores in shared memory, exchanges the
//                       slice's largest probability through distributed
//                       shared memory and runs P v on the tensor cores
//                       (details above the kernel).
//   attn_stats_kernel   longer slices and fp32: S = q k^T on the tensor cores
//                       (three limb accumulators in TMEM); on the CUDA cores
//                       the exact dequantised, scaled, masked scores (each
//                       step rounded to T as the reference's separate launches
//                       round), written once as T, the row max and sum of
//                       exponentials, and the slice's largest probability --
//                       the per-slice amax with which the reference's second
//                       bmm quantises P.
//   attn_out_kernel     reads those scores back by TMA, forms
//                       P = T(exp(s - m) / l), quantises it with the slice
//                       scale into shared memory as limb tiles and
//                       accumulates P v on the tensor cores; the epilogue
//                       dequantises O and stores it through its strides.
// Both paths give identical bits.  Compared with the composition, the softmax
// pass, the probability tensor (written, read for its amax, read again to
// quantise) and its limb planes never reach HBM, and the score epilogue runs
// once; the fused path keeps the scores on chip as well.
//
// Limb layout ("64-interleaved"): an int16 row of 64*G values is stored as G
// chunks of 128 bytes, chunk g = [hi of values 64g..64g+63 | lo of the same],
// hi = q >> 8 (signed), lo = q & 255 (unsigned).  A 128-byte chunk is one
// 128B-swizzle row, so a tile of chunk rows is loaded by TMA with
// SWIZZLE_128B and consumed by tcgen05.mma kind::i8 through K-major
// descriptors: the hi part is K sub-blocks 0..1 (32 bytes each), the lo part
// sub-blocks 2..3.  Per 32-byte sub-block pair four MMAs produce
//   HH += hi*hi,  MID += hi*lo + lo*hi,  LL += lo*lo
// which recombine exactly as 65536*HH + 256*MID + LL.
//
// CTA roles of the statistics and output kernels (576 threads, one CTA per
// SM, persistent over 128-row query tiles):
//   warp 0      TMA producer (4-stage ring);
//   warp 1      TMEM owner and MMA issuer;
//   warps 2..17 CUDA-core work: warp w owns TMEM lane quarter w % 4 (32
//               query rows) and one quarter (16 keys) of each 64-key tile.
// Every wait is bounded (error word + abort flag); no TMA multicast is used.
#include <cuda.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "tk_internal.h"
#include "tk_numerics.cuh"
#include "tk_ptx.cuh"

namespace tk {
namespace {

constexpr int BM = 128;              // query rows per tile
constexpr int BKEY = 64;             // keys per tile
constexpr int EVT = 64;              // value columns per output tile
constexpr int STAGES = 4;
constexpr int NUM_SOFT_WARPS = 16;                  // four per TMEM lane quarter
constexpr int NUM_THREADS = 64 + 32 * NUM_SOFT_WARPS;
constexpr int SUBS = NUM_SOFT_WARPS / 4;             // warps sharing a lane quarter
constexpr int CW = 64 / SUBS;                        // key (or value) columns per warp
static_assert(CW == 16, "p_codes16_h and the score chunk layout take 16 keys per warp");
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t COL_S = 0;        // S: HH, MID, LL at +0, +64, +128
constexpr uint32_t COL_O = 256;      // O: HH, MID, LL at +256, +320, +384
constexpr int Q_CHUNK = BM * 128;    // bytes of one 128-row chunk tile
constexpr int K_CHUNK = BKEY * 128;
constexpr int V_TILE = EVT * 128;
constexpr int P_TILE = BM * 128;
constexpr float kMaskedValue = -1.0e4f;  // the reference's causal fill

constexpr uint32_t IDESC_SS = idesc_i8(BM, 64, true, true);
constexpr uint32_t IDESC_SU = idesc_i8(BM, 64, true, false);
constexpr uint32_t IDESC_US = idesc_i8(BM, 64, false, true);
constexpr uint32_t IDESC_UU = idesc_i8(BM, 64, false, false);

// Shared memory of the statistics kernel.
template <int G>
struct StatsSmem {
    static constexpr int STAGE_BYTES = G * K_CHUNK;
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_STAGE = OFF_Q + G * Q_CHUNK;
    static constexpr int OFF_RED = OFF_STAGE + STAGES * STAGE_BYTES;  // float[2][SUBS][2][BM]
    static constexpr int OFF_BAR = OFF_RED + 2 * SUBS * 2 * BM * 4;
    static constexpr int NUM_BARS = 2 * STAGES + 7;
    static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
    static constexpr int ALLOC = OFF_MISC + 16 + 1024;  // + slack for 1024-byte alignment
};

// Shared memory of the output kernel.
template <int DT>
struct OutSmem {
    static constexpr int S_BYTES = BM * BKEY * (DT == 0 ? 2 : 4);
    static constexpr int STAGE_BYTES = S_BYTES + V_TILE;
    static constexpr int OFF_STAGE = 0;
    static constexpr int OFF_P = OFF_STAGE + STAGES * STAGE_BYTES;
    static constexpr int OFF_BAR = OFF_P + 2 * P_TILE;
    static constexpr int NUM_BARS = 2 * STAGES + 7;
    static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
    static constexpr int ALLOC = OFF_MISC + 16 + 1024;
};

struct AttnParams {
    int B, H, L, S, Ev;
    int64_t Spad;   // keys per score row in the workspace (multiple of 64)
    int n_kt;       // key tiles of 64
    int m_tiles;    // query tiles of 128 per slice
    int ev_tiles;   // output column tiles of 64 (1 in the statistics kernel)
    int tiles;      // work items
    const float* amax;       // [3][B*H]: q, k, v
    unsigned* amax_p;        // [B*H] float bits of the slice's max probability
    float* row_max;          // [B*H*L]
    float* row_inv;          // [B*H*L] 1 / sum of exponentials
    void* scores;            // [B*H][L][Spad] T
    void* out;
    int64_t os[4];
    int out_vec;             // 16-byte vector stores of 32 consecutive columns
    const void* mask;
    int mask_vec;            // mask rows contiguous and 16-byte aligned: vector loads
    int64_t ms[4];
    int causal;
    float scale;
    int scale_h;             // scale is exactly a binary16 number
    unsigned* err;
};

__device__ __forceinline__ void decode(const AttnParams& p, int tile, int& bh, int& mt, int& evh) {
    evh = tile % p.ev_tiles;
    const int r = tile / p.ev_tiles;
    mt = r % p.m_tiles;
    bh = r / p.m_tiles;
}

// exp(x) as 2^(x log2 e) on the special-function unit.  Both kernels use the
// same function, so the largest probability found by the statistics kernel
// is exactly the one the output kernel quantises.
__device__ __forceinline__ float exp_fast(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x * 1.4426950408889634f));
    return y;
}

// The exact integer 65536*hh + 256*mid + ll of a score's limb accumulators
// as binary64, for head dims up to 128: the hi limbs lie in [-128, 127] and
// the lo limbs in [0, 255], so over at most 128 products |256*mid + ll| <
// 2^31 and the sum fits int32.  The two int32 values become binary64 through
// their bit patterns (2^52 + 2^31 + x has x + 2^31 in its low word) and one
// exact fused multiply-add joins them -- fp64-pipe work instead of 64-bit
// integer shifts and adds.
__device__ __forceinline__ double score_acc_to_double(uint32_t hh, uint32_t mid, uint32_t ll) {
    const int32_t t = static_cast<int32_t>(mid) * 256 + static_cast<int32_t>(ll);
    const double dh = __hiloint2double(0x43300000, static_cast<int>(hh ^ 0x80000000u)) - 4503601774854144.0;
    const double dt = __hiloint2double(0x43300000, static_cast<int>(static_cast<uint32_t>(t) ^ 0x80000000u)) -
                      4503601774854144.0;
    return __fma_rn(dh, 65536.0, dt);
}

// Probability codes of 16 consecutive fp16 scores of one row: P =
// T(exp(s - m) * inv) rounded to binary16 in pairs, then quantised with the
// slice scale inv_p (P <= max P, so quant_code_bits gives quant_one's code);
// hi and lo limb bytes packed four to a word.
__device__ __forceinline__ void p_codes16_h(const float (&s)[16], float m, float inv, float inv_p,
                                            uint32_t (&hw)[4], uint32_t (&lw)[4]) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        uint32_t r[4];
#pragma unroll
        for (int k = 0; k < 4; k += 2) {
            const float2 pr = __half22float2(__floats2half2_rn(exp_fast(s[4 * w + k] - m) * inv,
                                                               exp_fast(s[4 * w + k + 1] - m) * inv));
            r[k] = quant_code_bits(pr.x, inv_p);
            r[k + 1] = quant_code_bits(pr.y, inv_p);
        }
        pack_codes4(r[0], r[1], r[2], r[3], hw[w], lw[w]);
    }
}

// N consecutive scores j0..j0+N-1 of query row i in the reference
// composition: the exact limb dot product, T(acc * s_qk), T(. * scale), the
// causal -1e4 and the additive mask, each rounded to T; padding keys
// (j >= S) become -inf.  The conditions are uniform per call, so each step is
// a branch-free loop over the 32 elements.
template <int DT, int N>
__device__ __forceinline__ void scores_n(const uint32_t (&hh)[N], const uint32_t (&mid)[N],
                                         const uint32_t (&ll)[N], double sqk, const AttnParams& p,
                                         int64_t i, int64_t j0, const void* mask_row, float (&s)[N]) {
#pragma unroll
    for (int c = 0; c < N; ++c)
        s[c] = round_t_from_double(__dmul_rn(score_acc_to_double(hh[c], mid[c], ll[c]), sqk), DT);
    if (p.scale != 1.0f) {
#pragma unroll
        for (int c = 0; c < N; ++c) s[c] = round_t(__fmul_rn(s[c], p.scale), DT);
    }
    if (p.causal && j0 + N - 1 > i) {
#pragma unroll
        for (int c = 0; c < N; ++c) {
            const float t = round_t(__fadd_rn(s[c], kMaskedValue), DT);
            s[c] = (j0 + c > i) ? t : s[c];
        }
    }
    const bool full = j0 + N <= p.S;
    if (mask_row != nullptr) {
        float mv[N];
        if (full && p.mask_vec) {
            if constexpr (DT == 0) {
                const uint4* src = reinterpret_cast<const uint4*>(static_cast<const __half*>(mask_row) + j0);
#pragma unroll
                for (int k = 0; k < N / 8; ++k) {
                    const uint4 u = __ldg(src + k);
                    const __half2* h2 = reinterpret_cast<const __half2*>(&u);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 f = __half22float2(h2[e]);
                        mv[8 * k + 2 * e] = f.x;
                        mv[8 * k + 2 * e + 1] = f.y;
                    }
                }
            } else {
                const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(mask_row) + j0);
#pragma unroll
                for (int k = 0; k < N / 4; ++k) {
                    const float4 f = __ldg(src + k);
                    mv[4 * k] = f.x; mv[4 * k + 1] = f.y; mv[4 * k + 2] = f.z; mv[4 * k + 3] = f.w;
                }
            }
        } else {
#pragma unroll
            for (int c = 0; c < N; ++c) {
                const int64_t j = j0 + c < p.S ? j0 + c : p.S - 1;  // clamped: padding keys are overwritten below
                mv[c] = DT == 0 ? __half2float(__ldg(static_cast<const __half*>(mask_row) + j * p.ms[3]))
                                : __ldg(static_cast<const float*>(mask_row) + j * p.ms[3]);
            }
        }
#pragma unroll
        for (int c = 0; c < N; ++c) s[c] = round_t(__fadd_rn(s[c], mv[c]), DT);
    }
    if (!full) {
#pragma unroll
        for (int c = 0; c < N; ++c) s[c] = (j0 + c < p.S) ? s[c] : -INFINITY;
    }
}

// The binary16 form of scores_n: after the one binary64 -> binary16
// rounding every step is a packed binary16 operation.  A binary16 product or
// sum of two binary16 values rounded once equals the binary32 operation
// rounded to binary16 (products are exact in binary32; for sums binary32
// carries more than 2*11 + 2 significand bits), so the scale (when it is a
// binary16 number), the causal -1e4 and the mask need no conversions.
template <int N>
__device__ __forceinline__ void scores_h(const uint32_t (&hh)[N], const uint32_t (&mid)[N],
                                         const uint32_t (&ll)[N], double sqk, const AttnParams& p,
                                         int64_t i, int64_t j0, const void* mask_row, __half2 (&sh)[N / 2],
                                         const uint4* mask_pre = nullptr) {
#pragma unroll
    for (int j = 0; j < N / 2; ++j)
        sh[j] = __halves2half2(
            __double2half(__dmul_rn(score_acc_to_double(hh[2 * j], mid[2 * j], ll[2 * j]), sqk)),
            __double2half(__dmul_rn(score_acc_to_double(hh[2 * j + 1], mid[2 * j + 1], ll[2 * j + 1]), sqk)));
    if (p.scale != 1.0f) {
        if (p.scale_h) {
            const __half2 sc = __float2half2_rn(p.scale);
#pragma unroll
            for (int j = 0; j < N / 2; ++j) sh[j] = __hmul2(sh[j], sc);
        } else {
#pragma unroll
            for (int j = 0; j < N / 2; ++j) {
                const float2 f = __half22float2(sh[j]);
                sh[j] = __floats2half2_rn(__fmul_rn(f.x, p.scale), __fmul_rn(f.y, p.scale));
            }
        }
    }
    if (p.causal && j0 + N - 1 > i) {
        const __half2 neg = __float2half2_rn(kMaskedValue);
#pragma unroll
        for (int j = 0; j < N / 2; ++j) {
            const __half2 t = __hadd2(sh[j], neg);
            sh[j] = __halves2half2(j0 + 2 * j > i ? __low2half(t) : __low2half(sh[j]),
                                   j0 + 2 * j + 1 > i ? __high2half(t) : __high2half(sh[j]));
        }
    }
    const bool full = j0 + N <= p.S;
    if (mask_row != nullptr) {
        if (full && p.mask_vec) {
            const uint4* src = reinterpret_cast<const uint4*>(static_cast<const __half*>(mask_row) + j0);
#pragma unroll
            for (int k = 0; k < N / 8; ++k) {
                const uint4 u = mask_pre != nullptr ? mask_pre[k] : __ldg(src + k);
                const __half2* m2 = reinterpret_cast<const __half2*>(&u);
#pragma unroll
                for (int e = 0; e < 4; ++e) sh[4 * k + e] = __hadd2(sh[4 * k + e], m2[e]);
            }
        } else {
            const __half* mh = static_cast<const __half*>(mask_row);
#pragma unroll
            for (int j = 0; j < N / 2; ++j) {
                // clamped: padding keys are overwritten below
                const int64_t ja = j0 + 2 * j < p.S ? j0 + 2 * j : p.S - 1;
                const int64_t jb = j0 + 2 * j + 1 < p.S ? j0 + 2 * j + 1 : p.S - 1;
                sh[j] = __hadd2(sh[j], __halves2half2(__ldg(mh + ja * p.ms[3]), __ldg(mh + jb * p.ms[3])));
            }
        }
    }
    if (!full) {
        const __half ninf = __ushort_as_half(0xFC00);
#pragma unroll
        for (int j = 0; j < N / 2; ++j)
            sh[j] = __halves2half2(j0 + 2 * j < p.S ? __low2half(sh[j]) : ninf,
                                   j0 + 2 * j + 1 < p.S ? __high2half(sh[j]) : ninf);
    }
}

template <int DT, int N>
__device__ __forceinline__ void store_row_n(void* base, const float (&v)[N]) {
    if constexpr (DT == 0) {
        uint4* dst = static_cast<uint4*>(base);
#pragma unroll
        for (int c = 0; c < N / 8; ++c) {
            uint32_t w[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                __half2 h2 = __floats2half2_rn(v[8 * c + 2 * k], v[8 * c + 2 * k + 1]);
                w[k] = *reinterpret_cast<uint32_t*>(&h2);
            }
            dst[c] = make_uint4(w[0], w[1], w[2], w[3]);
        }
    } else {
        float4* dst = static_cast<float4*>(base);
#pragma unroll
        for (int c = 0; c < N / 4; ++c) dst[c] = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
    }
}

// N (16 or 32) consecutive TMEM columns of this warp's 32 lanes.
template <int N>
__device__ __forceinline__ void tmem_ld_cw(uint32_t taddr, uint32_t (&r)[N]) {
    if constexpr (N == 16) tmem_ld_32x32b_x16(taddr, r);
    else tmem_ld_32x32b_x32(taddr, r);
}

// ---- statistics kernel: scores, row max / sum, slice max probability ---------

template <int G, int DT>
__global__ void __launch_bounds__(NUM_THREADS, 1)
attn_stats_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const AttnParams p) {
    using L = StatsSmem<G>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
    uint64_t* stage_full = bars;
    uint64_t* stage_empty = bars + STAGES;
    uint64_t* q_full = bars + 2 * STAGES;
    uint64_t* q_empty = q_full + 1;
    uint64_t* s_full = q_full + 2;
    uint64_t* s_empty = q_full + 3;
    uint64_t* c_full = q_full + 4;   // [2] partials of the other key quarters published
    uint64_t* drain_bar = q_full + 6;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* red = reinterpret_cast<float*>(smem + L::OFF_RED);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(stage_full + s), 1);
            mbar_init(smem_u32(stage_empty + s), 1);
        }
        mbar_init(smem_u32(q_full), 1);
        mbar_init(smem_u32(q_empty), 1);
        mbar_init(smem_u32(s_full), 1);
        mbar_init(smem_u32(s_empty), NUM_SOFT_WARPS);
        mbar_init(smem_u32(c_full), NUM_SOFT_WARPS - 4);
        mbar_init(smem_u32(c_full + 1), NUM_SOFT_WARPS - 4);
        mbar_init(smem_u32(drain_bar), 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer: Q once per tile, K per key tile ----------------
        int stage = 0;
        uint32_t phase = 0;
        uint32_t last_phase[STAGES];
        bool used[STAGES];
        for (int s = 0; s < STAGES; ++s) { used[s] = false; last_phase[s] = 0; }
        int q_loads = 0;
        bool ok = true;
        int lt = 0;
        for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x, ++lt) {
            int bh, mt, evh;
            decode(p, tile, bh, mt, evh);
            if (!mbar_wait_bounded(smem_u32(q_empty), (static_cast<uint32_t>(lt) & 1u) ^ 1u,
                                   abort_flag, p.err, kDevErrWaitEmpty))
                break;
            if (lane == 0) {
                const uint32_t fb = smem_u32(q_full);
                mbar_arrive_expect_tx(fb, G * Q_CHUNK);
#pragma unroll
                for (int g = 0; g < G; ++g)
                    tma_load_3d(smem_u32(smem + L::OFF_Q + g * Q_CHUNK), &tmQ, fb, g * 128, mt * BM, bh);
            }
            __syncwarp();
            ++q_loads;
            for (int t = 0; t < p.n_kt; ++t) {
                if (!mbar_wait_bounded(smem_u32(stage_empty + stage), phase ^ 1u, abort_flag,
                                       p.err, kDevErrWaitEmpty)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    const uint32_t fb = smem_u32(stage_full + stage);
                    uint8_t* sb = smem + L::OFF_STAGE + stage * L::STAGE_BYTES;
                    mbar_arrive_expect_tx(fb, G * K_CHUNK);
#pragma unroll
                    for (int g = 0; g < G; ++g)
                        tma_load_3d(smem_u32(sb + g * K_CHUNK), &tmK, fb, g * 128, t * BKEY, bh);
                }
                __syncwarp();
                used[stage] = true;
                last_phase[stage] = phase;
                if (++stage == STAGES) { stage = 0; phase ^= 1u; }
            }
        }
        volatile int no_abort = 0;
        for (int s = 0; s < STAGES; ++s)
            if (used[s])
                mbar_wait_bounded(smem_u32(stage_full + s), last_phase[s], &no_abort, p.err,
                                  kDevErrWaitDrain);
        if (q_loads > 0)
            mbar_wait_bounded(smem_u32(q_full), static_cast<uint32_t>(q_loads - 1) & 1u, &no_abort,
                              p.err, kDevErrWaitDrain);
    } else if (warp == 1) {
        // ---------------- MMA issuer: S = Q K^T per key tile ----------------
        int stage = 0;
        uint32_t phase = 0;
        uint32_t n_s = 0;
        bool ok = true;
        int lt = 0;
        const uint32_t s_hh = tmem_base + COL_S, s_mid = s_hh + 64, s_ll = s_hh + 128;
        const uint32_t q_base = smem_u32(smem + L::OFF_Q);
        for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x, ++lt) {
            if (!mbar_wait_bounded(smem_u32(q_full), static_cast<uint32_t>(lt) & 1u, abort_flag,
                                   p.err, kDevErrWaitFull))
                break;
            for (int t = 0; t < p.n_kt; ++t) {
                if (!mbar_wait_bounded(smem_u32(stage_full + stage), phase, abort_flag, p.err,
                                       kDevErrWaitFull) ||
                    !mbar_wait_bounded(smem_u32(s_empty), (n_s & 1u) ^ 1u, abort_flag, p.err,
                                       kDevErrWaitAccEmpty)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t kb = smem_u32(smem + L::OFF_STAGE + stage * L::STAGE_BYTES);
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        const uint64_t a0 = smem_desc_kmajor_sw128(q_base + g * Q_CHUNK);
                        const uint64_t b0 = smem_desc_kmajor_sw128(kb + g * K_CHUNK);
#pragma unroll
                        for (int u = 0; u < 2; ++u) {
                            const uint64_t hi = static_cast<uint64_t>((u * 32) >> 4);
                            const uint64_t lo = static_cast<uint64_t>((64 + u * 32) >> 4);
                            const uint32_t acc = (g > 0 || u > 0) ? 1u : 0u;
                            tc_mma_i8(s_hh, a0 + hi, b0 + hi, IDESC_SS, acc);
                            tc_mma_i8(s_mid, a0 + hi, b0 + lo, IDESC_SU, acc);
                            tc_mma_i8(s_mid, a0 + lo, b0 + hi, IDESC_US, 1u);
                            tc_mma_i8(s_ll, a0 + lo, b0 + lo, IDESC_UU, acc);
                        }
                    }
                    tc_commit(smem_u32(s_full));
                    tc_commit(smem_u32(stage_empty + stage));
                }
                __syncwarp();
                ++n_s;
                if (++stage == STAGES) { stage = 0; phase ^= 1u; }
            }
            if (!ok) break;
            if (lane == 0) tc_commit(smem_u32(q_empty));
            __syncwarp();
        }
        if (lane == 0) tc_commit(smem_u32(drain_bar));
        __syncwarp();
        volatile int no_abort = 0;
        mbar_wait_bounded(smem_u32(drain_bar), 0, &no_abort, p.err, kDevErrWaitDrain);
    } else {
        // ---------------- scores and statistics (warps 2..17) ----------------
        const int quarter = warp & 3;
        const int sub = (warp - 2) >> 2;
        const int row = quarter * 32 + lane;
        const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
        const int BH = p.B * p.H;
        constexpr int ES = DT == 0 ? 2 : 4;
        uint32_t n_s = 0;
        int lt = 0;
        for (int tile = blockIdx.x; tile < p.tiles; tile += gridDim.x, ++lt) {
            int bh, mt, evh;
            decode(p, tile, bh, mt, evh);
            const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
            const int64_t i = static_cast<int64_t>(mt) * BM + row;
            const bool row_ok = i < p.L;
            const double sqk = dequant_scale(__ldg(p.amax + bh), __ldg(p.amax + BH + bh));
            const void* mask_row = nullptr;
            if (p.mask != nullptr && row_ok)
                mask_row = static_cast<const char*>(p.mask) + (b * p.ms[0] + h * p.ms[1] + i * p.ms[2]) * ES;
            char* srow = static_cast<char*>(p.scores) + ((static_cast<int64_t>(bh) * p.L + i) * p.Spad) * ES;
            float m_run = -INFINITY, l_run = 0.0f;
            bool ok = true;
            for (int t = 0; t < p.n_kt; ++t) {
                if (!mbar_wait_bounded(smem_u32(s_full), n_s & 1u, abort_flag, p.err,
                                       kDevErrWaitAccFull)) {
                    ok = false;
                    break;
                }
                ++n_s;
                tc_fence_after();
                uint32_t hh[CW], mid[CW], ll[CW];
                const uint32_t col = COL_S + CW * sub;
                tmem_ld_cw(t_lane + col, hh);
                tmem_ld_cw(t_lane + col + 64, mid);
                tmem_ld_cw(t_lane + col + 128, ll);
                tc_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(s_empty));
                const int64_t j0 = static_cast<int64_t>(t) * BKEY + CW * sub;
                float s[CW];
                if constexpr (DT == 0) {
                    __half2 sh[CW / 2];
                    scores_h<CW>(hh, mid, ll, sqk, p, i, j0, mask_row, sh);
                    if (row_ok) {
                        uint4* dst = reinterpret_cast<uint4*>(srow + j0 * ES);
                        const uint4* src = reinterpret_cast<const uint4*>(sh);
#pragma unroll
                        for (int k = 0; k < CW / 8; ++k) dst[k] = src[k];
                    }
#pragma unroll
                    for (int j = 0; j < CW / 2; ++j) {
                        const float2 f = __half22float2(sh[j]);
                        s[2 * j] = f.x;
                        s[2 * j + 1] = f.y;
                    }
                } else {
                    scores_n<DT, CW>(hh, mid, ll, sqk, p, i, j0, mask_row, s);
                    if (row_ok) store_row_n<DT, CW>(srow + j0 * ES, s);
                }
                float tmax = -INFINITY;
#pragma unroll
                for (int c = 0; c < CW; ++c) tmax = fmaxf(tmax, s[c]);
                const float m_new = fmaxf(m_run, tmax);
                if (m_new != -INFINITY) {
                    if (m_run != -INFINITY && m_new != m_run) l_run *= exp_fast(m_run - m_new);
                    m_run = m_new;
                    float acc = 0.0f;
#pragma unroll
                    for (int c = 0; c < CW; ++c) acc += exp_fast(s[c] - m_run);
                    l_run += acc;
                }
            }
            if (!ok) break;
            // Combine the key quarters of each row.  The warps of quarters
            // 1..SUBS-1 publish their partials in buffer lt & 1, rewritten two
            // work items later -- by then the quarter-0 warps have read it
            // (they release the next item's first S tile only after this
            // combine).
            const int rb = lt & 1;
            float* rm = red + rb * SUBS * 2 * BM;
            if (sub > 0) {
                rm[(sub * 2) * BM + row] = m_run;
                rm[(sub * 2 + 1) * BM + row] = l_run;
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(c_full + rb));
            } else {
                if (!mbar_wait_bounded(smem_u32(c_full + rb), (static_cast<uint32_t>(lt) >> 1) & 1u,
                                       abort_flag, p.err, kDevErrWaitFull))
                    break;
                float m = m_run;
#pragma unroll
                for (int q = 1; q < SUBS; ++q) m = fmaxf(m, rm[(q * 2) * BM + row]);
                float l = 0.0f;
                if (m_run != -INFINITY) l += l_run * exp_fast(m_run - m);
#pragma unroll
                for (int q = 1; q < SUBS; ++q) {
                    const float mq = rm[(q * 2) * BM + row], lq = rm[(q * 2 + 1) * BM + row];
                    if (mq != -INFINITY) l += lq * exp_fast(mq - m);
                }
                const float inv = 1.0f / l;
                unsigned bits = 0;
                if (row_ok) {
                    p.row_max[static_cast<int64_t>(bh) * p.L + i] = m;
                    p.row_inv[static_cast<int64_t>(bh) * p.L + i] = inv;
                    // the row's largest probability, T(exp(0) / l)
                    if (m != -INFINITY) bits = __float_as_uint(round_t(exp_fast(0.0f) * inv, DT));
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) bits = max(bits, __shfl_xor_sync(0xffffffffu, bits, o));
                if (lane == 0 && bits != 0) atomicMax(p.amax_p + bh, bits);
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

// ---- output kernel: P = softmax(scores), quantised, O = P V -------------------

template <int DT>
__global__ void __launch_bounds__(NUM_THREADS, 1)
attn_out_kernel(const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmV,
                const AttnParams p) {
    using L = OutSmem<DT>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
    uint64_t* stage_full = bars;
    uint64_t* stage_empty = bars + STAGES;
    uint64_t* p_full = bars + 2 * STAGES;  // [2]
    uint64_t* p_empty = p_full + 2;        // [2]
    uint64_t* o_full = p_full + 4;
    uint64_t* o_empty = p_full + 5;
    uint64_t* drain_bar = p_full + 6;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(stage_full + s), 1);
            mbar_init(smem_u32(stage_empty + s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(p_full + b), NUM_SOFT_WARPS);
            mbar_init(smem_u32(p_empty + b), 1);
        }
        mbar_init(smem_u32(o_full), 1);
        mbar_init(smem_u32(o_empty), NUM_SOFT_WARPS);
        mbar_init(smem_u32(drain_bar), 1);
        *abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmS);
        tma_prefetch_desc(&tmV);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer: score tile + V^T tile per key tile ----------------
        int stage = 0;
        uint32_t phase = 0;
        uint32_t last_phase[STAGES];
        bool used[STAGES];
        for (int s = 0; s < STAGES; ++s) { used[s] = false; last_phase[s] = 0; }
        bool ok = true;
        for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x) {
            int bh, mt, evh;
            decode(p, tile, bh, mt, evh);
            for (int t = 0; t < p.n_kt; ++t) {
                if (!mbar_wait_bounded(smem_u32(stage_empty + stage), phase ^ 1u, abort_flag,
                                       p.err, kDevErrWaitEmpty)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    const uint32_t fb = smem_u32(stage_full + stage);
                    uint8_t* sb = smem + L::OFF_STAGE + stage * L::STAGE_BYTES;
                    mbar_arrive_expect_tx(fb, L::STAGE_BYTES);
                    tma_load_3d(smem_u32(sb), &tmS, fb, t * BKEY, mt * BM, bh);
                    if (DT == 1)  // fp32 scores: a second 32-key box of 128-byte rows
                        tma_load_3d(smem_u32(sb + L::S_BYTES / 2), &tmS, fb, t * BKEY + 32, mt * BM, bh);
                    tma_load_3d(smem_u32(sb + L::S_BYTES), &tmV, fb, t * 128, evh * EVT, bh);
                }
                __syncwarp();
                used[stage] = true;
                last_phase[stage] = phase;
                if (++stage == STAGES) { stage = 0; phase ^= 1u; }
            }
        }
        volatile int no_abort = 0;
        for (int s = 0; s < STAGES; ++s)
            if (used[s])
                mbar_wait_bounded(smem_u32(stage_full + s), last_phase[s], &no_abort, p.err,
                                  kDevErrWaitDrain);
    } else if (warp == 1) {
        // ---------------- MMA issuer: O += P V per key tile ----------------
        int stage = 0;
        uint32_t phase = 0;
        uint32_t n_p = 0;
        bool ok = true;
        int lt = 0;
        const uint32_t o_hh = tmem_base + COL_O, o_mid = o_hh + 64, o_ll = o_hh + 128;
        for (int tile = blockIdx.x; tile < p.tiles && ok; tile += gridDim.x, ++lt) {
            for (int t = 0; t < p.n_kt; ++t) {
                const uint32_t buf = n_p & 1u;
                if (!mbar_wait_bounded(smem_u32(p_full + buf), (n_p >> 1) & 1u, abort_flag, p.err,
                                       kDevErrWaitFull) ||
                    !mbar_wait_bounded(smem_u32(stage_full + stage), phase, abort_flag, p.err,
                                       kDevErrWaitFull) ||
                    (t == 0 && !mbar_wait_bounded(smem_u32(o_empty), (static_cast<uint32_t>(lt) & 1u) ^ 1u,
                                                  abort_flag, p.err, kDevErrWaitAccEmpty))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (lane == 0) {
                    const uint64_t a0 = smem_desc_kmajor_sw128(smem_u32(smem + L::OFF_P + buf * P_TILE));
                    const uint64_t b0 = smem_desc_kmajor_sw128(
                        smem_u32(smem + L::OFF_STAGE + stage * L::STAGE_BYTES + L::S_BYTES));
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const uint64_t hi = static_cast<uint64_t>((u * 32) >> 4);
                        const uint64_t lo = static_cast<uint64_t>((64 + u * 32) >> 4);
                        const uint32_t acc = (t > 0 || u > 0) ? 1u : 0u;
                        tc_mma_i8(o_hh, a0 + hi, b0 + hi, IDESC_SS, acc);
                        tc_mma_i8(o_mid, a0 + hi, b0 + lo, IDESC_SU, acc);
                        tc_mma_i8(o_mid, a0 + lo, b0 + hi, IDESC_US, 1u);
                        tc_mma_i8(o_ll, a0 + lo, b0 + lo, IDESC_UU, acc);
                    }
                    tc_commit(smem_u32(p_empty + buf));
                    tc_commit(smem_u32(stage_empty + stage));
                    if (t == p.n_kt - 1) tc_commit(smem_u32(o_full));
                }
                __syncwarp();
                ++n_p;
                if (++stage == STAGES) { stage = 0; phase ^= 1u; }
            }
        }
        if (lane == 0) tc_commit(smem_u32(drain_bar));
        __syncwarp();
        volatile int no_abort = 0;
        mbar_wait_bounded(smem_u32(drain_bar), 0, &no_abort, p.err, kDevErrWaitDrain);
    } else {
        // ---------------- probabilities and output epilogue (warps 2..17) ----------------
        const int quarter = warp & 3;
        const int sub = (warp - 2) >> 2;
        const int row = quarter * 32 + lane;
        const int sw = row & 7;
        const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
        const int BH = p.B * p.H;
        int stage = 0;
        uint32_t phase = 0;
        uint32_t n_p = 0;
        int lt = 0;
        for (int tile = blockIdx.x; tile < p.tiles; tile += gridDim.x, ++lt) {
            int bh, mt, evh;
            decode(p, tile, bh, mt, evh);
            const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
            const int64_t i = static_cast<int64_t>(mt) * BM + row;
            const bool row_ok = i < p.L;
            // rows past L quantise to 0 (their scores are TMA zero fill)
            const float inv_p = row_ok ? quant_inv(__uint_as_float(p.amax_p[bh])) : 0.0f;
            float m_i = 0.0f, inv_i = 0.0f;
            if (row_ok) {
                m_i = p.row_max[static_cast<int64_t>(bh) * p.L + i];
                inv_i = p.row_inv[static_cast<int64_t>(bh) * p.L + i];
            }
            bool ok = true;
            for (int t = 0; t < p.n_kt; ++t) {
                if (!mbar_wait_bounded(smem_u32(stage_full + stage), phase, abort_flag, p.err,
                                       kDevErrWaitFull)) {
                    ok = false;
                    break;
                }
                const uint8_t* sb = smem + L::OFF_STAGE + stage * L::STAGE_BYTES;
                float s[CW];
                if constexpr (DT == 0) {
                    // the row's 128-byte line, 16-byte chunks swizzled by row & 7
                    const uint8_t* line = sb + row * 128;
#pragma unroll
                    for (int k = 0; k < CW / 8; ++k) {
                        const uint4 u = *reinterpret_cast<const uint4*>(line + ((((CW / 8) * sub + k) ^ sw) << 4));
                        const __half2* h2 = reinterpret_cast<const __half2*>(&u);
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float2 f = __half22float2(h2[e]);
                            s[8 * k + 2 * e] = f.x;
                            s[8 * k + 2 * e + 1] = f.y;
                        }
                    }
                } else {
                    // keys 32h..32h+31 are box h; within its 128-byte line,
                    // key 32h + c is float c
                    const int kb = CW * sub;
                    const uint8_t* line = sb + (kb / 32) * (L::S_BYTES / 2) + row * 128;
#pragma unroll
                    for (int k = 0; k < CW / 4; ++k) {
                        const float4 f = *reinterpret_cast<const float4*>(line + ((((kb % 32) / 4 + k) ^ sw) << 4));
                        s[4 * k] = f.x;
                        s[4 * k + 1] = f.y;
                        s[4 * k + 2] = f.z;
                        s[4 * k + 3] = f.w;
                    }
                }
                // P = T(exp(s - m) / l), quantised with the slice scale: the
                // probabilities are >= 0, so q is in [0, 32767] and the hi
                // limb in [0, 127].
                // (pr <= max P, so quant_code_bits gives quant_one's code)
                uint32_t hw[CW / 4], lw[CW / 4];
                if constexpr (DT == 0) {
                    p_codes16_h(s, m_i, inv_i, inv_p, hw, lw);
                } else {
#pragma unroll
                    for (int w = 0; w < CW / 4; ++w) {
                        uint32_t r[4];
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            r[k] = quant_code_bits(round_t(exp_fast(s[4 * w + k] - m_i) * inv_i, DT), inv_p);
                        pack_codes4(r[0], r[1], r[2], r[3], hw[w], lw[w]);
                    }
                }
                const uint32_t buf = n_p & 1u;
                if (!mbar_wait_bounded(smem_u32(p_empty + buf), ((n_p >> 1) & 1u) ^ 1u, abort_flag,
                                       p.err, kDevErrWaitEmpty)) {
                    ok = false;
                    break;
                }
                uint8_t* prow = smem + L::OFF_P + buf * P_TILE + row * 128;
#pragma unroll
                for (int k = 0; k < CW / 16; ++k) {
                    const int ch = (CW / 16) * sub + k;  // 16-key chunk of the hi part
                    *reinterpret_cast<uint4*>(prow + ((ch ^ sw) << 4)) =
                        make_uint4(hw[4 * k], hw[4 * k + 1], hw[4 * k + 2], hw[4 * k + 3]);
                    *reinterpret_cast<uint4*>(prow + (((ch + 4) ^ sw) << 4)) =
                        make_uint4(lw[4 * k], lw[4 * k + 1], lw[4 * k + 2], lw[4 * k + 3]);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(p_full + buf));
                ++n_p;
                if (++stage == STAGES) { stage = 0; phase ^= 1u; }
            }
            if (!ok) break;
            if (!mbar_wait_bounded(smem_u32(o_full), static_cast<uint32_t>(lt) & 1u, abort_flag, p.err,
                                   kDevErrWaitAccFull))
                break;
            tc_fence_after();
            uint32_t hh[CW], mid[CW], ll[CW];
            const uint32_t col = COL_O + CW * sub;
            tmem_ld_cw(t_lane + col, hh);
            tmem_ld_cw(t_lane + col + 64, mid);
            tmem_ld_cw(t_lane + col + 128, ll);
            tc_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(o_empty));
            if (row_ok) {
                const double spv = dequant_scale(__uint_as_float(p.amax_p[bh]), __ldg(p.amax + 2 * BH + bh));
                const int64_t e0 = static_cast<int64_t>(evh) * EVT + CW * sub;
                const int64_t obase = b * p.os[0] + h * p.os[1] + i * p.os[2];
                float o[CW];
#pragma unroll
                for (int c = 0; c < CW; ++c)
                    o[c] = round_t_from_double(__dmul_rn(limb_acc_to_double(hh[c], mid[c], ll[c]), spv), DT);
                if (p.out_vec && e0 + CW <= p.Ev) {
                    store_row_n<DT, CW>(static_cast<char*>(p.out) + (obase + e0) * (DT == 0 ? 2 : 4), o);
                } else {
#pragma unroll
                    for (int c = 0; c < CW; ++c)
                        if (e0 + c < p.Ev) store_t(p.out, DT, obase + (e0 + c) * p.os[3], o[c]);
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

// ---- fused kernel: scores resident in shared memory, one cluster per slice ----
//
// For fp16 slices with head dim <= 128 and at most 512 queries and keys, a
// cluster of ceil(L / 128) CTAs handles a (batch, head) slice, one CTA per
// 128 query rows; the clusters are persistent and walk the slices with a
// stride of the grid's cluster count.  Phase A computes S = Q K^T tile by
// tile on the tensor cores, forms the exact fp16 scores on the CUDA cores
// (scores_h) and keeps them in this CTA's shared memory (up to 128 KB) with
// an online row max and sum of exponentials.  The slice's largest
// probability (the scale of the reference's second bmm) is combined across
// the cluster through distributed shared memory while the scores turn into
// the binary16 probabilities in place.  Phase B converts each probability
// tile in place into the swizzled limb tile of the quantised P, and P V runs
// on the tensor cores while the CUDA-core warps already compute the next
// slice's scores; they dequantise O afterwards.  K and V^T tiles come
// through separate rings from two TMA warps, and S and P V are issued by two
// MMA warps, so the next slice's S tiles never queue behind this slice's P V.
// The scores are computed once and never reach HBM; the arithmetic (every
// rounding, the same exponential) is that of the statistics and output
// kernels above, so the results are identical.
constexpr int FUSED_MAX_KT = 8;                        // keys <= 512
constexpr int FUSED_THREADS = 128 + 32 * NUM_SOFT_WARPS;  // 4 role warps + 16 CUDA-core warps

template <int G>
struct FusedSmem {
    static constexpr int KSTAGES = G == 1 ? 4 : 2;    // K tiles of G * 8 KB
    static constexpr int VSTAGES = G == 1 ? 4 : 2;    // V^T tiles of 8 KB
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_K = OFF_Q + G * Q_CHUNK;
    static constexpr int OFF_V = OFF_K + KSTAGES * G * K_CHUNK;
    static constexpr int OFF_S = OFF_V + VSTAGES * V_TILE;            // key tile t at + t * P_TILE
    static constexpr int OFF_RED = OFF_S + FUSED_MAX_KT * P_TILE;     // float [SUBS][2][BM]
    static constexpr int OFF_BAR = OFF_RED + SUBS * 2 * BM * 4;
    // q_full, q_empty, k_full[], k_empty[], v_full[], v_empty[], s_full,
    // s_empty, comb, stats, cl[2], p_ready[8], p_free[8], o_full, o_empty,
    // drain_s, drain_o
    static constexpr int NUM_BARS = 2 + 2 * KSTAGES + 2 * VSTAGES + 6 + 2 * FUSED_MAX_KT + 4;
    // tmem slot, abort flag, cta max[2], slots[2][4]
    static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
    static constexpr int ALLOC = OFF_MISC + 64 + 1024;
    static_assert(ALLOC <= 232448, "shared memory budget");
    static_assert(OFF_S % 1024 == 0 && OFF_K % 1024 == 0 && OFF_V % 1024 == 0,
                  "128-byte swizzled tiles on 1024-byte boundaries");
};

// The largest probability of this CTA's rows, exchanged with the other CTAs
// of the cluster: slot crank of every CTA's slot array for the slice's
// parity, then an arrival on every CTA's barrier of that parity.
__device__ __forceinline__ void cluster_publish_max(unsigned v, int par, uint32_t crank, int cl,
                                                    volatile unsigned* slots, uint64_t* cl_bar) {
    const uint32_t slot_addr = smem_u32(const_cast<unsigned*>(slots) + par * 4 + crank);
    const uint32_t bar_addr = smem_u32(cl_bar + par);
    for (int r = 0; r < cl; ++r) {
        if (r == static_cast<int>(crank)) continue;
        st_shared_cluster_u32(mapa_shared(slot_addr, static_cast<uint32_t>(r)), v);
        mbar_arrive_remote(mapa_shared(bar_addr, static_cast<uint32_t>(r)));
    }
    slots[par * 4 + crank] = v;
    mbar_arrive(bar_addr);
}

template <int G>
__global__ void __launch_bounds__(FUSED_THREADS, 1)
attn_fused_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
    using L = FusedSmem<G>;
    constexpr int KS = L::KSTAGES, VS = L::VSTAGES;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
    uint64_t* q_full = bars;
    uint64_t* q_empty = bars + 1;             // Q read by the slice's last S MMA
    uint64_t* k_full = bars + 2;
    uint64_t* k_empty = k_full + KS;
    uint64_t* v_full = k_empty + KS;
    uint64_t* v_empty = v_full + VS;
    uint64_t* s_full = v_empty + VS;          // S tile in TMEM computed
    uint64_t* s_empty = s_full + 1;           // S tile read (16 warps)
    uint64_t* comb = s_full + 2;              // every warp's partial row statistics published (16 warps)
    uint64_t* stats = s_full + 3;             // this CTA's max probability formed (4 warps)
    uint64_t* cl_bar = s_full + 4;            // [2] the cluster's max probabilities gathered (CL arrivals)
    uint64_t* p_ready = s_full + 6;           // [FUSED_MAX_KT] P tile t written (16 warps)
    uint64_t* p_free = p_ready + FUSED_MAX_KT;  // [FUSED_MAX_KT] P V of tile t complete
    uint64_t* o_full = p_free + FUSED_MAX_KT;
    uint64_t* o_empty = o_full + 1;
    uint64_t* drain_s = o_full + 2;
    uint64_t* drain_o = o_full + 3;
    uint32_t* misc = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);
    uint32_t* tmem_slot = misc;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 1);
    unsigned* cta_max = misc + 2;             // [2] by slice parity
    volatile unsigned* slots = misc + 4;      // [2][4] max probability of each CTA, by slice parity
    float* red = reinterpret_cast<float*>(smem + L::OFF_RED);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int CL = p.m_tiles;
    const uint32_t crank = cluster_ctarank();
    const int mt = static_cast<int>(crank);
    const int n_cl = static_cast<int>(gridDim.x) / CL;
    const int cid = static_cast<int>(blockIdx.x) / CL;
    const int BH = p.B * p.H;
    const int n_slices = cid < BH ? (BH - cid + n_cl - 1) / n_cl : 0;
    const int n_kt = p.n_kt;

    if (threadIdx.x == 0) {
        mbar_init(smem_u32(q_full), 1);
        mbar_init(smem_u32(q_empty), 1);
        for (int s = 0; s < KS; ++s) {
            mbar_init(smem_u32(k_full + s), 1);
            mbar_init(smem_u32(k_empty + s), 1);
        }
        for (int s = 0; s < VS; ++s) {
            mbar_init(smem_u32(v_full + s), 1);
            mbar_init(smem_u32(v_empty + s), 1);
        }
        mbar_init(smem_u32(s_full), 1);
        mbar_init(smem_u32(s_empty), NUM_SOFT_WARPS);
        mbar_init(smem_u32(comb), NUM_SOFT_WARPS);
        mbar_init(smem_u32(stats), 4);
        mbar_init(smem_u32(cl_bar), static_cast<uint32_t>(CL));
        mbar_init(smem_u32(cl_bar + 1), static_cast<uint32_t>(CL));
        for (int t = 0; t < FUSED_MAX_KT; ++t) {
            mbar_init(smem_u32(p_ready + t), NUM_SOFT_WARPS);
            mbar_init(smem_u32(p_free + t), 1);
        }
        mbar_init(smem_u32(o_full), 1);
        mbar_init(smem_u32(o_empty), NUM_SOFT_WARPS);
        mbar_init(smem_u32(drain_s), 1);
        mbar_init(smem_u32(drain_o), 1);
        *abort_flag = 0;
        cta_max[0] = 0u;
        cta_max[1] = 0u;
        for (int r = 0; r < 8; ++r) slots[r] = 0u;
        fence_mbar_init();
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // every CTA of the cluster has initialised its barriers before any remote arrival
    cluster_sync_all();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA: per slice Q, then the K tiles ----------------
        int stage = 0;
        uint32_t phase = 0;
        uint32_t last_phase[KS];
        bool used[KS];
        for (int s = 0; s < KS; ++s) { used[s] = false; last_phase[s] = 0; }
        int q_loads = 0;
        bool ok = true;
        for (int it = 0; it < n_slices && ok; ++it) {
            const int bh = cid + it * n_cl;
            if (!mbar_wait_bounded(smem_u32(q_empty), (static_cast<uint32_t>(it) & 1u) ^ 1u, abort_flag, p.err,
                                   kDevErrWaitEmpty))
                break;
            if (lane == 0) {
                mbar_arrive_expect_tx(smem_u32(q_full), G * Q_CHUNK);
#pragma unroll
                for (int g = 0; g < G; ++g)
                    tma_load_3d(smem_u32(smem + L::OFF_Q + g * Q_CHUNK), &tmQ, smem_u32(q_full), g * 128, mt * BM, bh);
            }
            __syncwarp();
            ++q_loads;
            for (int t = 0; t < n_kt; ++t) {
                if (!mbar_wait_bounded(smem_u32(k_empty + stage), phase ^ 1u, abort_flag, p.err, kDevErrWaitEmpty)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    const uint32_t fb = smem_u32(k_full + stage);
                    const uint32_t dst = smem_u32(smem + L::OFF_K + stage * G * K_CHUNK);
                    mbar_arrive_expect_tx(fb, G * K_CHUNK);
#pragma unroll
                    for (int g = 0; g < G; ++g) tma_load_3d(dst + g * K_CHUNK, &tmK, fb, g * 128, t * BKEY, bh);
                }
                __syncwarp();
                used[stage] = true;
                last_phase[stage] = phase;
                if (++stage == KS) { stage = 0; phase ^= 1u; }
            }
        }
        volatile int no_abort = 0;
        for (int s = 0; s < KS; ++s)
            if (used[s])
                mbar_wait_bounded(smem_u32(k_full + s), last_phase[s], &no_abort, p.err, kDevErrWaitDrain);
        if (q_loads > 0)
            mbar_wait_bounded(smem_u32(q_full), static_cast<uint32_t>(q_loads - 1) & 1u, &no_abort, p.err,
                              kDevErrWaitDrain);
    } else if (warp == 2) {
        // ---------------- TMA: per slice the V^T tiles ----------------
        int stage = 0;
        uint32_t phase = 0;
        uint32_t last_phase[VS];
        bool used[VS];
        for (int s = 0; s < VS; ++s) { used[s] = false; last_phase[s] = 0; }
        bool ok = true;
        for (int it = 0; it < n_slices && ok; ++it) {
            const int bh = cid + it * n_cl;
            for (int j = 0; j < p.ev_tiles * n_kt; ++j) {
                if (!mbar_wait_bounded(smem_u32(v_empty + stage), phase ^ 1u, abort_flag, p.err, kDevErrWaitEmpty)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    const uint32_t fb = smem_u32(v_full + stage);
                    mbar_arrive_expect_tx(fb, V_TILE);
                    tma_load_3d(smem_u32(smem + L::OFF_V + stage * V_TILE), &tmV, fb, (j % n_kt) * 128,
                                (j / n_kt) * EVT, bh);
                }
                __syncwarp();
                used[stage] = true;
                last_phase[stage] = phase;
                if (++stage == VS) { stage = 0; phase ^= 1u; }
            }
        }
        volatile int no_abort = 0;
        for (int s = 0; s < VS; ++s)
            if (used[s])
                mbar_wait_bounded(smem_u32(v_full + s), last_phase[s], &no_abort, p.err, kDevErrWaitDrain);
    } else if (warp == 1) {
        // ---------------- MMA: S = Q K^T per key tile, running ahead into the next slice ----------------
        int stage = 0;
        uint32_t phase = 0;
        uint32_t n_s = 0;
        bool ok = true;
        const uint32_t s_hh = tmem_base + COL_S, s_mid = s_hh + 64, s_ll = s_hh + 128;
        const uint32_t q_base = smem_u32(smem + L::OFF_Q);
        for (int it = 0; it < n_slices && ok; ++it) {
            if (!mbar_wait_bounded(smem_u32(q_full), static_cast<uint32_t>(it) & 1u, abort_flag, p.err,
                                   kDevErrWaitFull))
                break;
            for (int t = 0; t < n_kt; ++t) {
                // the S columns are single-buffered: the CUDA-core warps release
                // them right after their TMEM loads, before the scores' arithmetic
                if (!mbar_wait_bounded(smem_u32(k_full + stage), phase, abort_flag, p.err, kDevErrWaitFull) ||
                    !mbar_wait_bounded(smem_u32(s_empty), (n_s & 1u) ^ 1u, abort_flag, p.err, kDevErrWaitAccEmpty)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t kb = smem_u32(smem + L::OFF_K + stage * G * K_CHUNK);
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        const uint64_t q0 = smem_desc_kmajor_sw128(q_base + g * Q_CHUNK);
                        const uint64_t b0 = smem_desc_kmajor_sw128(kb + g * K_CHUNK);
#pragma unroll
                        for (int u = 0; u < 2; ++u) {
                            const uint64_t hi = static_cast<uint64_t>((u * 32) >> 4);
                            const uint64_t lo = static_cast<uint64_t>((64 + u * 32) >> 4);
                            const uint32_t acc = (g > 0 || u > 0) ? 1u : 0u;
                            tc_mma_i8(s_hh, q0 + hi, b0 + hi, IDESC_SS, acc);
                            tc_mma_i8(s_mid, q0 + hi, b0 + lo, IDESC_SU, acc);
                            tc_mma_i8(s_mid, q0 + lo, b0 + hi, IDESC_US, 1u);
                            tc_mma_i8(s_ll, q0 + lo, b0 + lo, IDESC_UU, acc);
                        }
                    }
                    tc_commit(smem_u32(s_full));
                    tc_commit(smem_u32(k_empty + stage));
                    if (t == n_kt - 1) tc_commit(smem_u32(q_empty));
                }
                __syncwarp();
                ++n_s;
                if (++stage == KS) { stage = 0; phase ^= 1u; }
            }
        }
        if (lane == 0) tc_commit(smem_u32(drain_s));
        __syncwarp();
        volatile int no_abort = 0;
        mbar_wait_bounded(smem_u32(drain_s), 0, &no_abort, p.err, kDevErrWaitDrain);
    } else if (warp == 3) {
        // ---------------- MMA: O += P V, and the cluster exchange ----------------
        int stage = 0;
        uint32_t phase = 0;
        uint32_t n_o = 0;
        bool ok = true;
        const uint32_t o_hh = tmem_base + COL_O, o_mid = o_hh + 64, o_ll = o_hh + 128;
        for (int it = 0; it < n_slices && ok; ++it) {
            const int par = it & 1;
            // Exchange this CTA's largest probability with the cluster.  Slots
            // and barriers alternate with the slice's parity, so a CTA that runs
            // a slice ahead never touches what a slower one still reads.
            if (lane == 0) {
                mbar_wait_bounded(smem_u32(stats), static_cast<uint32_t>(par), abort_flag, p.err, kDevErrWaitFull);
                const unsigned v = *reinterpret_cast<volatile unsigned*>(cta_max + par);
                *reinterpret_cast<volatile unsigned*>(cta_max + par) = 0u;  // for the slice after next
                cluster_publish_max(v, par, crank, CL, slots, cl_bar);
            }
            __syncwarp();
            for (int evh = 0; evh < p.ev_tiles && ok; ++evh) {
                if (!mbar_wait_bounded(smem_u32(o_empty), (n_o & 1u) ^ 1u, abort_flag, p.err, kDevErrWaitAccEmpty)) {
                    ok = false;
                    break;
                }
                for (int t = 0; t < n_kt; ++t) {
                    if (!mbar_wait_bounded(smem_u32(p_ready + t), static_cast<uint32_t>(par), abort_flag, p.err,
                                           kDevErrWaitFull) ||
                        !mbar_wait_bounded(smem_u32(v_full + stage), phase, abort_flag, p.err, kDevErrWaitFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (lane == 0) {
                        const uint64_t a0 = smem_desc_kmajor_sw128(smem_u32(smem + L::OFF_S + t * P_TILE));
                        const uint64_t b0 = smem_desc_kmajor_sw128(smem_u32(smem + L::OFF_V + stage * V_TILE));
#pragma unroll
                        for (int u = 0; u < 2; ++u) {
                            const uint64_t hi = static_cast<uint64_t>((u * 32) >> 4);
                            const uint64_t lo = static_cast<uint64_t>((64 + u * 32) >> 4);
                            const uint32_t acc = (t > 0 || u > 0) ? 1u : 0u;
                            tc_mma_i8(o_hh, a0 + hi, b0 + hi, IDESC_SS, acc);
                            tc_mma_i8(o_mid, a0 + hi, b0 + lo, IDESC_SU, acc);
                            tc_mma_i8(o_mid, a0 + lo, b0 + hi, IDESC_US, 1u);
                            tc_mma_i8(o_ll, a0 + lo, b0 + lo, IDESC_UU, acc);
                        }
                        tc_commit(smem_u32(v_empty + stage));
                        if (evh == p.ev_tiles - 1) tc_commit(smem_u32(p_free + t));
                        if (t == n_kt - 1) tc_commit(smem_u32(o_full));
                    }
                    __syncwarp();
                    if (++stage == VS) { stage = 0; phase ^= 1u; }
                }
                ++n_o;
            }
        }
        if (lane == 0) tc_commit(smem_u32(drain_o));
        __syncwarp();
        volatile int no_abort = 0;
        mbar_wait_bounded(smem_u32(drain_o), 0, &no_abort, p.err, kDevErrWaitDrain);
    } else {
        // ---------------- scores, statistics, P and the output (warps 4..19) ----------------
        const int quarter = warp & 3;
        const int sub = (warp - 4) >> 2;
        const int row = quarter * 32 + lane;
        const int sw = row & 7;
        const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
        const int64_t i = static_cast<int64_t>(mt) * BM + row;
        const bool row_ok = i < p.L;
        uint8_t* line0 = smem + L::OFF_S + row * 128;
        uint32_t n_s = 0, n_o = 0;
        bool ok = true;
        // With one output tile the dequantisation of a slice's O waits until
        // the next slice's scores are formed, so P V runs meanwhile; with more,
        // the later output tiles reuse the accumulator and it runs at once.
        const bool defer = p.ev_tiles == 1;
        // O of slice (b, h): dequantise with the slice's P and v scales, store
        auto epilogue = [&](int b, int h, float pmax, float amax_v) {
            for (int evh = 0; evh < p.ev_tiles; ++evh) {
                if (!mbar_wait_bounded(smem_u32(o_full), n_o & 1u, abort_flag, p.err, kDevErrWaitAccFull)) {
                    ok = false;
                    return;
                }
                ++n_o;
                tc_fence_after();
                uint32_t hh[CW], mid[CW], ll[CW];
                const uint32_t col = COL_O + CW * sub;
                tmem_ld_cw(t_lane + col, hh);
                tmem_ld_cw(t_lane + col + 64, mid);
                tmem_ld_cw(t_lane + col + 128, ll);
                tc_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(o_empty));
                if (row_ok) {
                    const double spv = dequant_scale(pmax, amax_v);
                    const int64_t e0 = static_cast<int64_t>(evh) * EVT + CW * sub;
                    const int64_t obase = b * p.os[0] + h * p.os[1] + i * p.os[2];
                    float o[CW];
#pragma unroll
                    for (int c = 0; c < CW; ++c)
                        o[c] = round_t_from_double(__dmul_rn(limb_acc_to_double(hh[c], mid[c], ll[c]), spv), 0);
                    if (p.out_vec && e0 + CW <= p.Ev) {
                        store_row_n<0, CW>(static_cast<char*>(p.out) + (obase + e0) * 2, o);
                    } else {
#pragma unroll
                        for (int c = 0; c < CW; ++c)
                            if (e0 + c < p.Ev) store_t(p.out, 0, obase + (e0 + c) * p.os[3], o[c]);
                    }
                }
            }
        };
        int prev_b = 0, prev_h = 0;
        float prev_pmax = 0.0f, prev_av = 0.0f;
        bool have_prev = false;
        // the slice's q, k, v scales, loaded one slice ahead
        float aq = 0.0f, ak = 0.0f, av = 0.0f;
        if (n_slices > 0) {
            aq = __ldg(p.amax + cid);
            ak = __ldg(p.amax + BH + cid);
            av = __ldg(p.amax + 2 * BH + cid);
        }
        for (int it = 0; it < n_slices && ok; ++it) {
            const int bh = cid + it * n_cl;
            const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
            const int par = it & 1;
            const double sqk = dequant_scale(aq, ak);
            const float amax_v = av;
            if (it + 1 < n_slices) {
                aq = __ldg(p.amax + bh + n_cl);
                ak = __ldg(p.amax + BH + bh + n_cl);
                av = __ldg(p.amax + 2 * BH + bh + n_cl);
            }
            const void* mask_row = nullptr;
            if (p.mask != nullptr && row_ok)
                mask_row = static_cast<const char*>(p.mask) + (b * p.ms[0] + h * p.ms[1] + i * p.ms[2]) * 2;
            float m_run = -INFINITY, l_run = 0.0f;
            for (int t = 0; t < n_kt; ++t) {
                const int64_t j0 = static_cast<int64_t>(t) * BKEY + CW * sub;
                // this tile's mask values are loaded before the wait for S
                uint4 mpre[CW / 8];
                const bool pre = mask_row != nullptr && p.mask_vec && j0 + CW <= p.S;
                if (pre) {
                    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const __half*>(mask_row) + j0);
#pragma unroll
                    for (int k = 0; k < CW / 8; ++k) mpre[k] = __ldg(src + k);
                }
                if (!mbar_wait_bounded(smem_u32(s_full), n_s & 1u, abort_flag, p.err, kDevErrWaitAccFull)) {
                    ok = false;
                    break;
                }
                ++n_s;
                tc_fence_after();
                uint32_t hh[CW], mid[CW], ll[CW];
                const uint32_t col = COL_S + CW * sub;
                tmem_ld_cw(t_lane + col, hh);
                tmem_ld_cw(t_lane + col + 64, mid);
                tmem_ld_cw(t_lane + col + 128, ll);
                tc_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(s_empty));
                __half2 sh[CW / 2];
                scores_h<CW>(hh, mid, ll, sqk, p, i, j0, mask_row, sh, pre ? mpre : nullptr);
                // the previous slice's P tile t has been read by its P V
                if (it > 0 &&
                    !mbar_wait_bounded(smem_u32(p_free + t), static_cast<uint32_t>(par ^ 1), abort_flag, p.err,
                                       kDevErrWaitEmpty)) {
                    ok = false;
                    break;
                }
                // keys j0..j0+7 go to 16-byte chunk sub of the row's line, keys
                // j0+8..j0+15 to chunk 4 + sub: the chunks that later hold this
                // warp's hi and lo limbs of P, so each warp converts its own bytes
                uint8_t* line = line0 + t * P_TILE;
                const uint4* src = reinterpret_cast<const uint4*>(sh);
                *reinterpret_cast<uint4*>(line + ((sub ^ sw) << 4)) = src[0];
                *reinterpret_cast<uint4*>(line + (((4 + sub) ^ sw) << 4)) = src[1];
                float s[CW];
#pragma unroll
                for (int j = 0; j < CW / 2; ++j) {
                    const float2 f = __half22float2(sh[j]);
                    s[2 * j] = f.x;
                    s[2 * j + 1] = f.y;
                }
                float tmax = -INFINITY;
#pragma unroll
                for (int c = 0; c < CW; ++c) tmax = fmaxf(tmax, s[c]);
                const float m_new = fmaxf(m_run, tmax);
                if (m_new != -INFINITY) {
                    if (m_run != -INFINITY && m_new != m_run) l_run *= exp_fast(m_run - m_new);
                    m_run = m_new;
                    float acc = 0.0f;
#pragma unroll
                    for (int c = 0; c < CW; ++c) acc += exp_fast(s[c] - m_run);
                    l_run += acc;
                }
            }
            if (!ok) break;
            if (have_prev) {
                epilogue(prev_b, prev_h, prev_pmax, prev_av);
                have_prev = false;
                if (!ok) break;
            }
            // Every warp publishes its partial (m, l); each warp then combines
            // the four partials of its rows in the statistics kernel's order
            // (key quarter 0 first), so all four warps of a row hold the same
            // m and 1/l.  red is rewritten only in the next slice, after every
            // warp has passed this slice's P tiles.
            red[(sub * 2) * BM + row] = m_run;
            red[(sub * 2 + 1) * BM + row] = l_run;
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(comb));
            if (!mbar_wait_bounded(smem_u32(comb), static_cast<uint32_t>(par), abort_flag, p.err, kDevErrWaitFull)) {
                ok = false;
                break;
            }
            const float m0 = red[row], l0 = red[BM + row];
            float m_i = m0;
#pragma unroll
            for (int q = 1; q < SUBS; ++q) m_i = fmaxf(m_i, red[(q * 2) * BM + row]);
            float l = 0.0f;
            if (m0 != -INFINITY) l += l0 * exp_fast(m0 - m_i);
#pragma unroll
            for (int q = 1; q < SUBS; ++q) {
                const float mq = red[(q * 2) * BM + row], lq = red[(q * 2 + 1) * BM + row];
                if (mq != -INFINITY) l += lq * exp_fast(mq - m_i);
            }
            const float inv_i = 1.0f / l;
            if (sub == 0) {
                // the row's largest probability, T(exp(0) / l)
                unsigned bits = 0;
                if (row_ok && m_i != -INFINITY) bits = __float_as_uint(round_t(exp_fast(0.0f) * inv_i, 0));
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) bits = max(bits, __shfl_xor_sync(0xffffffffu, bits, o));
                if (lane == 0) {
                    if (bits != 0u) atomicMax(cta_max + par, bits);
                    mbar_arrive(smem_u32(stats));
                }
            }
            // While the cluster exchanges, P = T(exp(s - m) / l) replaces the
            // scores in place (binary16, as the reference's softmax output)
            for (int t = 0; t < n_kt; ++t) {
                uint4* c0 = reinterpret_cast<uint4*>(line0 + t * P_TILE + ((sub ^ sw) << 4));
                uint4* c1 = reinterpret_cast<uint4*>(line0 + t * P_TILE + (((4 + sub) ^ sw) << 4));
                uint4 c[2] = {*c0, *c1};
                __half2* hv = reinterpret_cast<__half2*>(c);
#pragma unroll
                for (int e = 0; e < CW / 2; ++e) {
                    const float2 f = __half22float2(hv[e]);
                    hv[e] = __floats2half2_rn(exp_fast(f.x - m_i) * inv_i, exp_fast(f.y - m_i) * inv_i);
                }
                *c0 = c[0];
                *c1 = c[1];
            }
            // barrier par completes for the (it >> 1)-th time in this slice
            if (!mbar_wait_bounded_cluster(smem_u32(cl_bar + par), (static_cast<uint32_t>(it) >> 1) & 1u, abort_flag,
                                           p.err, kDevErrWaitCluster)) {
                ok = false;
                break;
            }
            unsigned pm = 0;
            for (int r = 0; r < CL; ++r) pm = max(pm, slots[par * 4 + r]);
            const float pmax = __uint_as_float(pm);
            // rows past L quantise to 0
            const float inv_p = row_ok ? quant_inv(pmax) : 0.0f;
            // each P tile becomes its quantised limb tile in place: the warp's
            // 16 keys' hi limbs in chunk sub, lo limbs in chunk 4 + sub (P <=
            // max P, so quant_code_bits gives quant_one's code)
            for (int t = 0; t < n_kt; ++t) {
                uint4* c0 = reinterpret_cast<uint4*>(line0 + t * P_TILE + ((sub ^ sw) << 4));
                uint4* c1 = reinterpret_cast<uint4*>(line0 + t * P_TILE + (((4 + sub) ^ sw) << 4));
                uint4 c[2] = {*c0, *c1};
                const __half2* hv = reinterpret_cast<const __half2*>(c);
                uint32_t hw[CW / 4], lw[CW / 4];
#pragma unroll
                for (int w = 0; w < CW / 4; ++w) {
                    const float2 a = __half22float2(hv[2 * w]), b2 = __half22float2(hv[2 * w + 1]);
                    pack_codes4(quant_code_bits(a.x, inv_p), quant_code_bits(a.y, inv_p),
                                quant_code_bits(b2.x, inv_p), quant_code_bits(b2.y, inv_p), hw[w], lw[w]);
                }
                *c0 = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                *c1 = make_uint4(lw[0], lw[1], lw[2], lw[3]);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(p_ready + t));
            }
            if (defer) {
                prev_b = b;
                prev_h = h;
                prev_pmax = pmax;
                prev_av = amax_v;
                have_prev = true;
            } else {
                epilogue(b, h, pmax, amax_v);
            }
        }
        if (have_prev && ok) epilogue(prev_b, prev_h, prev_pmax, prev_av);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
    // no CTA leaves while another CTA of the cluster may still write to it
    cluster_sync_all();
}

// ---- quantisation of q, k, v into limb rows ---------------------------------

struct QuantParams {
    const void* src[3];
    int64_t st[3][4];
    int rows[3], cols[3];
    int H, BH;
    int vec[3];         // columns contiguous, 16-byte aligned rows: vector loads
    float* amax;        // [3][BH]
    unsigned* amax_p;   // [BH], zeroed here
    uint8_t* dst[3];
    int64_t ld[3];      // bytes per limb row
    int64_t slice[3];   // bytes per slice
};

constexpr int QT_THREADS = 256;
constexpr int QT_MAX_EV = 256;

template <typename T> __device__ __forceinline__ float ldx(const T* p, int64_t i);
template <> __device__ __forceinline__ float ldx<__half>(const __half* p, int64_t i) { return __half2float(__ldg(p + i)); }
template <> __device__ __forceinline__ float ldx<float>(const float* p, int64_t i) { return __ldg(p + i); }

// 8 consecutive elements from a 16-byte aligned address.
__device__ __forceinline__ void ld8(const __half* p, float* v) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    const __half2* h2 = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(h2[e]);
        v[2 * e] = f.x;
        v[2 * e + 1] = f.y;
    }
}
__device__ __forceinline__ void ld8(const float* p, float* v) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ void pack16(const int (&q)[16], uint4& hi, uint4& lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        h[w] = 0;
        l[w] = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            h[w] |= static_cast<uint32_t>((q[4 * w + k] >> 8) & 0xFF) << (8 * k);
            l[w] |= static_cast<uint32_t>(q[4 * w + k] & 0xFF) << (8 * k);
        }
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

template <typename T>
__global__ void __launch_bounds__(QT_THREADS)
attn_quant_kernel(QuantParams p) {
    __shared__ unsigned red[QT_THREADS / 32];
    __shared__ int16_t tile[BKEY][QT_MAX_EV + 2];
    const int bh = blockIdx.x, z = blockIdx.y;
    const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
    const T* x = static_cast<const T*>(p.src[z]) + b * p.st[z][0] + h * p.st[z][1];
    const int64_t sr = p.st[z][2], sc = p.st[z][3];
    const int rows = p.rows[z], cols = p.cols[z];
    const bool vec = p.vec[z] != 0;

    unsigned mx = 0;  // max of |x| bit patterns: NaN dominates, then Inf
    if (vec) {
        const int pcs = cols / 8;
        for (int it = threadIdx.x; it < rows * pcs; it += QT_THREADS) {
            const int r = it / pcs, pc = it - (it / pcs) * pcs;
            float v[8];
            ld8(x + r * sr + pc * 8, v);
#pragma unroll
            for (int e = 0; e < 8; ++e) mx = max(mx, __float_as_uint(fabsf(v[e])));
        }
    } else {
        for (int it = threadIdx.x; it < rows * cols; it += QT_THREADS) {
            const int r = it / cols, c = it - (it / cols) * cols;
            mx = max(mx, __float_as_uint(fabsf(ldx<T>(x, r * sr + c * sc))));
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = 0;
#pragma unroll
    for (int w = 0; w < QT_THREADS / 32; ++w) mx = max(mx, red[w]);
    const float amax = __uint_as_float(mx);
    if (threadIdx.x == 0) {
        p.amax[z * p.BH + bh] = amax;
        if (z == 0) p.amax_p[bh] = 0u;
    }
    const float inv = quant_inv(amax);
    uint8_t* out = p.dst[z] + bh * p.slice[z];
    const int64_t ld = p.ld[z];

    if (z < 2) {
        // rows x (ld / 2) values in 16-value pieces: hi at g*128 + c%64, lo at +64
        const int pieces = static_cast<int>(ld / 32);
        for (int it = threadIdx.x; it < rows * pieces; it += QT_THREADS) {
            const int r = it / pieces, pc = it - (it / pieces) * pieces;
            const int c0 = pc * 16;
            float v[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) v[e] = 0.0f;
            if (inv != 0.0f) {  // inv == 0 (amax 0 or not finite): every code is 0
                if (vec && c0 + 16 <= cols) {
                    ld8(x + r * sr + c0, v);
                    ld8(x + r * sr + c0 + 8, v + 8);
                } else {
#pragma unroll
                    for (int e = 0; e < 16; ++e)
                        if (c0 + e < cols) v[e] = ldx<T>(x, r * sr + (c0 + e) * sc);
                }
            }
            uint32_t cb[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) cb[e] = quant_code_bits(v[e], inv);
            uint4 hi, lo;
            pack_codes4(cb[0], cb[1], cb[2], cb[3], hi.x, lo.x);
            pack_codes4(cb[4], cb[5], cb[6], cb[7], hi.y, lo.y);
            pack_codes4(cb[8], cb[9], cb[10], cb[11], hi.z, lo.z);
            pack_codes4(cb[12], cb[13], cb[14], cb[15], hi.w, lo.w);
            uint8_t* dst = out + r * ld + (c0 / 64) * 128 + (c0 % 64);
            *reinterpret_cast<uint4*>(dst) = hi;
            *reinterpret_cast<uint4*>(dst + 64) = lo;
        }
    } else {
        // v^T: row e holds, per key tile kt, [hi of keys 64kt.. | lo of the same]
        const int n_kt = static_cast<int>(ld / 128);
        for (int kt = 0; kt < n_kt; ++kt) {
            if (vec) {
                const int pcs = cols / 8;
                for (int it = threadIdx.x; it < BKEY * pcs; it += QT_THREADS) {
                    const int kk = it / pcs, pc = it - (it / pcs) * pcs;
                    const int j = kt * BKEY + kk;
                    float v[8];
                    if (j < rows) {
                        ld8(x + j * sr + pc * 8, v);
                    } else {
#pragma unroll
                        for (int e = 0; e < 8; ++e) v[e] = 0.0f;
                    }
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        tile[kk][pc * 8 + e] =
                            inv != 0.0f ? static_cast<int16_t>(quant_code_bits(v[e], inv) & 0xFFFFu) : int16_t(0);
                }
            } else {
                for (int it = threadIdx.x; it < BKEY * cols; it += QT_THREADS) {
                    const int kk = it / cols, e = it - (it / cols) * cols;
                    const int j = kt * BKEY + kk;
                    tile[kk][e] = static_cast<int16_t>(j < rows ? quant_one(ldx<T>(x, j * sr + e * sc), inv) : 0);
                }
            }
            __syncthreads();
            for (int it = threadIdx.x; it < cols * 4; it += QT_THREADS) {
                const int e = it >> 2, pc = it & 3;
                int q[16];
#pragma unroll
                for (int k = 0; k < 16; ++k) q[k] = tile[pc * 16 + k][e];
                uint4 hi, lo;
                pack16(q, hi, lo);
                uint8_t* dst = out + e * ld + kt * 128 + pc * 16;
                *reinterpret_cast<uint4*>(dst) = hi;
                *reinterpret_cast<uint4*>(dst + 64) = lo;
            }
            __syncthreads();
        }
    }
}

// The same quantisation with the whole slice staged in shared memory (fp16
// slices of at most 32 KB elements, e.g. 512 x 64): the slice crosses HBM
// once -- loaded with eight 16-byte loads in flight per thread while its
// max-abs is folded -- and the codes are formed from shared memory.  Codes,
// layouts and the max-abs convention are those of attn_quant_kernel.
constexpr int QS_MAX_BYTES = 64 * 1024;

__global__ void __launch_bounds__(QT_THREADS)
attn_quant_staged_kernel(QuantParams p) {
    extern __shared__ __align__(16) uint8_t qsm[];
    __shared__ unsigned red[QT_THREADS / 32];
    const __half* raw = reinterpret_cast<const __half*>(qsm);
    const int bh = blockIdx.x, z = blockIdx.y;
    const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
    const __half* x = static_cast<const __half*>(p.src[z]) + b * p.st[z][0] + h * p.st[z][1];
    const int64_t sr = p.st[z][2];
    const int rows = p.rows[z], cols = p.cols[z];
    const int pcs = cols / 8;  // 16-byte pieces per row (cols % 8 == 0, rows 16-byte aligned)
    const int n = rows * pcs;
    unsigned mx = 0;  // max of |x| bit patterns: NaN dominates, then Inf
    for (int it0 = threadIdx.x; it0 < n; it0 += 8 * QT_THREADS) {
        uint4 u[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int it = it0 + k * QT_THREADS;
            if (it < n) {
                const int r = it / pcs, pc = it - (it / pcs) * pcs;
                u[k] = __ldg(reinterpret_cast<const uint4*>(x + r * sr + pc * 8));
            }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int it = it0 + k * QT_THREADS;
            if (it < n) {
                reinterpret_cast<uint4*>(qsm)[it] = u[k];
                const __half2* h2 = reinterpret_cast<const __half2*>(&u[k]);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __half22float2(h2[e]);
                    mx = max(mx, max(__float_as_uint(fabsf(f.x)), __float_as_uint(fabsf(f.y))));
                }
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = 0;
#pragma unroll
    for (int w = 0; w < QT_THREADS / 32; ++w) mx = max(mx, red[w]);
    const float amax = __uint_as_float(mx);
    if (threadIdx.x == 0) {
        p.amax[z * p.BH + bh] = amax;
        if (z == 0) p.amax_p[bh] = 0u;
    }
    const float inv = quant_inv(amax);
    uint8_t* out = p.dst[z] + bh * p.slice[z];
    const int64_t ld = p.ld[z];
    if (z < 2) {
        // rows x (ld / 2) values in 16-value pieces: hi at g*128 + c%64, lo at +64
        const int pieces = static_cast<int>(ld / 32);
        for (int it = threadIdx.x; it < rows * pieces; it += QT_THREADS) {
            const int r = it / pieces, pc = it - (it / pieces) * pieces;
            const int c0 = pc * 16;
            uint32_t cb[16];
            if (inv != 0.0f && c0 + 16 <= cols) {
                const uint4* src = reinterpret_cast<const uint4*>(raw + r * cols + c0);
                const uint4 a = src[0], b2 = src[1];
                const __half2* ha = reinterpret_cast<const __half2*>(&a);
                const __half2* hb = reinterpret_cast<const __half2*>(&b2);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 fa = __half22float2(ha[e]), fb = __half22float2(hb[e]);
                    cb[2 * e] = quant_code_bits(fa.x, inv);
                    cb[2 * e + 1] = quant_code_bits(fa.y, inv);
                    cb[8 + 2 * e] = quant_code_bits(fb.x, inv);
                    cb[8 + 2 * e + 1] = quant_code_bits(fb.y, inv);
                }
            } else {
#pragma unroll
                for (int e = 0; e < 16; ++e)
                    cb[e] = quant_code_bits(
                        (inv != 0.0f && c0 + e < cols) ? __half2float(raw[r * cols + c0 + e]) : 0.0f, inv);
            }
            uint4 hi, lo;
            pack_codes4(cb[0], cb[1], cb[2], cb[3], hi.x, lo.x);
            pack_codes4(cb[4], cb[5], cb[6], cb[7], hi.y, lo.y);
            pack_codes4(cb[8], cb[9], cb[10], cb[11], hi.z, lo.z);
            pack_codes4(cb[12], cb[13], cb[14], cb[15], hi.w, lo.w);
            uint8_t* dst = out + r * ld + (c0 / 64) * 128 + (c0 % 64);
            *reinterpret_cast<uint4*>(dst) = hi;
            *reinterpret_cast<uint4*>(dst + 64) = lo;
        }
    } else {
        // v^T: row e holds, per key tile kt, [hi of keys 64kt.. | lo of the same]
        const int n_kt = static_cast<int>(ld / 128);
        for (int it = threadIdx.x; it < n_kt * cols * 4; it += QT_THREADS) {
            const int kt = it / (cols * 4), rem = it - kt * (cols * 4);
            const int e = rem >> 2, pc = rem & 3;
            int q[16];
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                const int j = kt * BKEY + pc * 16 + k;
                const float v = (inv != 0.0f && j < rows) ? __half2float(raw[j * cols + e]) : 0.0f;
                q[k] = static_cast<int>(static_cast<int16_t>(quant_code_bits(v, inv) & 0xFFFFu));
            }
            uint4 hi, lo;
            pack16(q, hi, lo);
            uint8_t* dst = out + e * ld + kt * 128 + pc * 16;
            *reinterpret_cast<uint4*>(dst) = hi;
            *reinterpret_cast<uint4*>(dst + 64) = lo;
        }
    }
}

// ---- host side ---------------------------------------------------------------

struct Layout {
    int G;
    int64_t BH, Spad, ldq, ldv;
    size_t off_amax, off_amax_p, off_max, off_inv, off_q, off_k, off_v, off_s, total;
};

// Slices the fused kernel takes: fp16, head dim <= 128, at most 512 queries
// and keys (the scores of 128 queries fit in shared memory, the slice's CTAs
// in one portable cluster).
bool fused_ok(const tk_sdpa_desc_t& d) {
    return d.dtype == TK_DTYPE_F16 && d.e <= 128 && d.l <= BM * 4 && d.s <= BKEY * FUSED_MAX_KT;
}

Layout layout_of(const tk_sdpa_desc_t& d) {
    Layout l;
    l.G = static_cast<int>(ceil_div(d.e, 64));
    l.BH = d.batch * d.heads;
    l.Spad = static_cast<int64_t>(round_up(static_cast<size_t>(d.s), BKEY));
    l.ldq = 128 * l.G;
    l.ldv = 2 * l.Spad;
    const size_t es = dtype_size(d.dtype);
    size_t o = 0;
    auto take = [&](size_t bytes) {
        const size_t at = o;
        o = round_up(o + bytes, 1024);
        return at;
    };
    l.off_amax = take(3 * l.BH * sizeof(float));
    l.off_amax_p = take(l.BH * sizeof(unsigned));
    l.off_max = take(l.BH * d.l * sizeof(float));
    l.off_inv = take(l.BH * d.l * sizeof(float));
    l.off_q = take(static_cast<size_t>(l.BH * d.l * l.ldq));
    l.off_k = take(static_cast<size_t>(l.BH * d.s * l.ldq));
    l.off_v = take(static_cast<size_t>(l.BH * d.ev * l.ldv));
    l.off_s = take(fused_ok(d) ? 0 : static_cast<size_t>(l.BH * d.l * l.Spad) * es);
    l.total = o + 1024;  // base alignment slack
    return l;
}

int validate(const tk_sdpa_desc_t* d) {
    TK_CHECK_ARG(d != nullptr, "tk_sdpa_q16: NULL descriptor");
    TK_CHECK_ARG(d->dtype == TK_DTYPE_F16 || d->dtype == TK_DTYPE_F32, "tk_sdpa_q16: bad dtype");
    TK_CHECK_ARG(d->batch >= 0 && d->heads >= 0 && d->l >= 0 && d->s >= 0 && d->e >= 0 && d->ev >= 0,
                 "tk_sdpa_q16: negative size");
    if (d->e > 128) TK_FAIL(TK_ERR_UNSUPPORTED, "tk_sdpa_q16: head dim %lld > 128", (long long)d->e);
    if (d->ev > QT_MAX_EV)
        TK_FAIL(TK_ERR_UNSUPPORTED, "tk_sdpa_q16: value dim %lld > %d", (long long)d->ev, QT_MAX_EV);
    if (d->s > 32768)
        TK_FAIL(TK_ERR_UNSUPPORTED, "tk_sdpa_q16: %lld keys exceed the exact int32 limb sums (32768)",
                (long long)d->s);
    TK_CHECK_ARG(d->batch * d->heads < (1LL << 31) && d->l < (1LL << 31), "tk_sdpa_q16: too large");
    return TK_OK;
}

int make_map(CUtensorMap* map, CUtensorMapDataType type, size_t esize, const void* base, int64_t d0,
             int64_t d1, int64_t d2, uint32_t box0, uint32_t box1) {
    EncodeTiledFn enc = tensor_map_encoder();
    if (enc == nullptr) TK_FAIL(TK_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(d0), static_cast<cuuint64_t>(d1),
                          static_cast<cuuint64_t>(d2)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(d0 * esize), static_cast<cuuint64_t>(d0 * d1 * esize)};
    cuuint32_t box[3] = {box0, box1, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, type, 3, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) TK_FAIL(TK_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return TK_OK;
}

// One attribute call per kernel instantiation and device (the template is
// keyed by the kernel itself, not its signature, which several share).
template <auto Kernel>
int set_smem(int bytes, int dev) {
    static std::once_flag once[64];
    static cudaError_t err[64];
    const int slot = std::min(dev, 63);
    std::call_once(once[slot], [&] {
        err[slot] = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    });
    if (err[slot] != cudaSuccess)
        TK_FAIL(TK_ERR_CUDA, "attention smem attribute: %s", cudaGetErrorString(err[slot]));
    return TK_OK;
}

template <int G, int DT>
int run_attention(const CUtensorMap& tq, const CUtensorMap& tk_, const CUtensorMap& ts,
                  const CUtensorMap& tv, AttnParams p, int ev_tiles, int dev, cudaStream_t stream) {
    const int sms = sm_count(dev);
    p.ev_tiles = 1;
    p.tiles = p.B * p.H * p.m_tiles;
    int rc = set_smem<attn_stats_kernel<G, DT>>(StatsSmem<G>::ALLOC, dev);
    if (rc) return rc;
    attn_stats_kernel<G, DT><<<std::min(p.tiles, sms), NUM_THREADS, StatsSmem<G>::ALLOC, stream>>>(tq, tk_, p);
    rc = launch_status("attention statistics");
    if (rc) return rc;
    p.ev_tiles = ev_tiles;
    p.tiles = p.B * p.H * p.m_tiles * ev_tiles;
    rc = set_smem<attn_out_kernel<DT>>(OutSmem<DT>::ALLOC, dev);
    if (rc) return rc;
    attn_out_kernel<DT><<<std::min(p.tiles, sms), NUM_THREADS, OutSmem<DT>::ALLOC, stream>>>(ts, tv, p);
    return launch_status("attention output");
}

// Clusters of `cl` CTAs of the fused kernel that fit on device `dev` at
// once (one CTA per SM), queried once per (device, cluster size).
template <int G>
int max_fused_clusters(int cl, int dev) {
    static std::once_flag once[64][5];
    static int count[64][5];
    const int slot = std::min(dev, 63);
    std::call_once(once[slot][cl], [&] {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(static_cast<unsigned>(cl * 1024));
        cfg.blockDim = dim3(FUSED_THREADS);
        cfg.dynamicSmemBytes = FusedSmem<G>::ALLOC;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = static_cast<unsigned>(cl);
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, attn_fused_kernel<G>, &cfg) != cudaSuccess || n <= 0) {
            (void)cudaGetLastError();
            n = std::max(1, sm_count(dev) / cl);
        }
        count[slot][cl] = n;
    });
    return count[slot][cl];
}

template <int G>
int run_fused(const CUtensorMap& tq, const CUtensorMap& tk_, const CUtensorMap& tv, AttnParams p,
              int ev_tiles, int dev, cudaStream_t stream) {
    using L = FusedSmem<G>;
    p.ev_tiles = ev_tiles;
    p.tiles = p.B * p.H * p.m_tiles;
    int rc = set_smem<attn_fused_kernel<G>>(L::ALLOC, dev);
    if (rc) return rc;
    // persistent clusters: as many as fit on the device at once
    const int n_cl = std::min(p.B * p.H, max_fused_clusters<G>(p.m_tiles, dev));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(n_cl * p.m_tiles));
    cfg.blockDim = dim3(FUSED_THREADS);
    cfg.dynamicSmemBytes = L::ALLOC;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(p.m_tiles);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, attn_fused_kernel<G>, tq, tk_, tv, p);
    if (e != cudaSuccess) TK_FAIL(TK_ERR_CUDA, "fused attention launch: %s", cudaGetErrorString(e));
    return launch_status("fused attention");
}

// Innermost stride 1 and every other stride and the base 16-byte aligned, so
// runs of `cols` (a multiple of 8) elements load and store as vectors.
bool vec_ok(const void* ptr, const int64_t* st, int64_t cols, size_t es) {
    const int64_t v = static_cast<int64_t>(16 / es);
    return st[3] == 1 && cols % 8 == 0 && reinterpret_cast<uintptr_t>(ptr) % 16 == 0 &&
           st[0] % v == 0 && st[1] % v == 0 && st[2] % v == 0;
}

}  // namespace
}  // namespace tk

extern "C" {

size_t tk_sdpa_workspace_size(const tk_sdpa_desc_t* desc) {
    if (tk::validate(desc) != TK_OK) return 0;
    return tk::layout_of(*desc).total;
}

int tk_sdpa_q16(const tk_sdpa_desc_t* desc, void* workspace, size_t workspace_bytes, void* stream_) {
    using namespace tk;
    int rc = validate(desc);
    if (rc) return rc;
    const tk_sdpa_desc_t& d = *desc;
    if (d.batch == 0 || d.heads == 0 || d.l == 0 || d.ev == 0) return TK_OK;
    TK_CHECK_ARG(d.s > 0 && d.e > 0, "tk_sdpa_q16: empty key or head dimension");
    TK_CHECK_ARG(d.q && d.k && d.v && d.out, "tk_sdpa_q16: NULL tensor");
    const Layout l = layout_of(d);
    if (workspace == nullptr || workspace_bytes < l.total)
        TK_FAIL(TK_ERR_WORKSPACE, "tk_sdpa_q16: workspace of %zu bytes, %zu needed", workspace_bytes,
                l.total);
    uint8_t* ws = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(workspace) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    const int dev = current_device();
    const size_t es = dtype_size(d.dtype);

    QuantParams qp;
    const void* srcs[3] = {d.q, d.k, d.v};
    const int64_t* strs[3] = {d.q_strides, d.k_strides, d.v_strides};
    const int64_t rows[3] = {d.l, d.s, d.s}, cols[3] = {d.e, d.e, d.ev};
    uint8_t* dsts[3] = {ws + l.off_q, ws + l.off_k, ws + l.off_v};
    const int64_t lds[3] = {l.ldq, l.ldq, l.ldv};
    const int64_t slices[3] = {d.l * l.ldq, d.s * l.ldq, d.ev * l.ldv};
    for (int z = 0; z < 3; ++z) {
        qp.src[z] = srcs[z];
        for (int a = 0; a < 4; ++a) qp.st[z][a] = strs[z][a];
        qp.rows[z] = static_cast<int>(rows[z]);
        qp.cols[z] = static_cast<int>(cols[z]);
        qp.vec[z] = vec_ok(srcs[z], strs[z], cols[z], es) ? 1 : 0;
        qp.dst[z] = dsts[z];
        qp.ld[z] = lds[z];
        qp.slice[z] = slices[z];
    }
    qp.H = static_cast<int>(d.heads);
    qp.BH = static_cast<int>(l.BH);
    qp.amax = reinterpret_cast<float*>(ws + l.off_amax);
    qp.amax_p = reinterpret_cast<unsigned*>(ws + l.off_amax_p);
    const dim3 qgrid(static_cast<unsigned>(l.BH), 3);
    // fp16 slices whose rows are contiguous 16-byte aligned runs and that fit
    // 64 KB are staged in shared memory (one HBM read)
    const int64_t stage_bytes = std::max(d.l * d.e, std::max(d.s * d.e, d.s * d.ev)) * 2;
    const bool staged = d.dtype == TK_DTYPE_F16 && stage_bytes <= QS_MAX_BYTES && qp.vec[0] && qp.vec[1] && qp.vec[2];
    if (staged) {
        rc = set_smem<attn_quant_staged_kernel>(QS_MAX_BYTES, dev);
        if (rc) return rc;
        attn_quant_staged_kernel<<<qgrid, QT_THREADS, static_cast<size_t>(stage_bytes), stream>>>(qp);
    } else if (d.dtype == TK_DTYPE_F16) {
        attn_quant_kernel<__half><<<qgrid, QT_THREADS, 0, stream>>>(qp);
    } else {
        attn_quant_kernel<float><<<qgrid, QT_THREADS, 0, stream>>>(qp);
    }
    rc = launch_status("attention quantise");
    if (rc) return rc;

    const CUtensorMapDataType stype =
        d.dtype == TK_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    CUtensorMap tq, tk_, tv, ts;
    rc = make_map(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ws + l.off_q, l.ldq, d.l, l.BH, 128, BM);
    if (!rc) rc = make_map(&tk_, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ws + l.off_k, l.ldq, d.s, l.BH, 128, BKEY);
    if (!rc) rc = make_map(&tv, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ws + l.off_v, l.ldv, d.ev, l.BH, 128, EVT);
    const bool fused = fused_ok(d);
    if (!rc && !fused)
        rc = make_map(&ts, stype, es, ws + l.off_s, l.Spad, d.l, l.BH, static_cast<uint32_t>(128 / es), BM);
    if (rc) return rc;

    AttnParams p;
    p.B = static_cast<int>(d.batch);
    p.H = static_cast<int>(d.heads);
    p.L = static_cast<int>(d.l);
    p.S = static_cast<int>(d.s);
    p.Ev = static_cast<int>(d.ev);
    p.Spad = l.Spad;
    p.n_kt = static_cast<int>(ceil_div(d.s, BKEY));
    p.m_tiles = static_cast<int>(ceil_div(d.l, BM));
    p.amax = qp.amax;
    p.amax_p = qp.amax_p;
    p.row_max = reinterpret_cast<float*>(ws + l.off_max);
    p.row_inv = reinterpret_cast<float*>(ws + l.off_inv);
    p.scores = ws + l.off_s;
    p.out = d.out;
    for (int a = 0; a < 4; ++a) {
        p.os[a] = d.out_strides[a];
        p.ms[a] = d.mask_strides[a];
    }
    p.out_vec = vec_ok(d.out, d.out_strides, CW, es) ? 1 : 0;
    p.mask = d.mask;
    p.mask_vec = d.mask != nullptr && vec_ok(d.mask, d.mask_strides, CW, es) ? 1 : 0;
    p.causal = d.causal ? 1 : 0;
    p.scale = d.scale;
    p.scale_h = __half2float(__float2half_rn(d.scale)) == d.scale ? 1 : 0;
    p.err = device_error_word(dev);
    const int ev_tiles = static_cast<int>(ceil_div(d.ev, EVT));
    TK_CHECK_ARG(l.BH * p.m_tiles * ev_tiles < (1LL << 31), "tk_sdpa_q16: too many tiles");
    if (fused) return l.G == 1 ? run_fused<1>(tq, tk_, tv, p, ev_tiles, dev, stream)
                               : run_fused<2>(tq, tk_, tv, p, ev_tiles, dev, stream);
    if (l.G == 1)
        return d.dtype == TK_DTYPE_F16 ? run_attention<1, 0>(tq, tk_, ts, tv, p, ev_tiles, dev, stream)
                                       : run_attention<1, 1>(tq, tk_, ts, tv, p, ev_tiles, dev, stream);
    return d.dtype == TK_DTYPE_F16 ? run_attention<2, 0>(tq, tk_, ts, tv, p, ev_tiles, dev, stream)
                                   : run_attention<2, 1>(tq, tk_, ts, tv, p, ev_tiles, dev, stream);
}

}  // extern "C"
