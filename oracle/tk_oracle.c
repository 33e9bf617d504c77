/*
 * tk_oracle.c -- CPU restatement of torch_kunlun's int16-quantised dense path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped package links, loads or
 * calls this file; only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg use it, and only as the checker.
 *
 * Parity status: unpinned at bit level.  The reference computes in Baidu's
 * closed XDNN library (calls at csrc/ops.cpp:224 fc, csrc/ops.cpp:264
 * conv2d, csrc/ops_nn.cpp:214 per-slice fc for bmm) and its test-suite holds
 * no golden vectors.  The documented semantics (README.md:72-74 of the
 * reference's numerics notes, TODO.md:188-197: "XDNN scales each operand by its
 * per-tensor max into int16 ... and dequantizes with a single scale (XFP16
 * uses 1/32767^2)") are turned into the exact contract below; the tolerance
 * tests of the reference (tests/test_numeric_semantics.py:49-57,
 * tests/test_runtime.py:53-79) are re-run against it in tests/.
 *
 * The contract (every step IEEE-754, round-to-nearest-even, no contraction):
 *
 *   amax      = max_i |float(x_i)|                 (NaN dominates)
 *   inv       = fp32(32767.0f / amax)              (0 when amax is 0 or not finite)
 *   q_i       = clamp(rint(fp32(float(x_i) * inv)), -32767, 32767)
 *   acc[m,n]  = sum_k qa[m,k] * qb[k,n]            exact in int64
 *   s         = fp64(fp64(amax_a) * fp64(amax_b)) / 1073676289.0   (= 32767^2)
 *   r         = T(fp64(acc) * s)                   T = fp16 or fp32 (one rounding)
 *   alpha!=1: r = T(float(r) * alpha)              (reference addmm: mm, then scale)
 *   bias:     r = T(float(r) + float(bias[n]))     (reference linear: fc, then add)
 *   beta!=0:  b = beta==1 ? addend : T(float(addend)*beta);  r = T(float(r) + float(b))
 *   act:      relu(r) = r > 0 || isnan(r) ? r : +0
 *
 * bmm quantises every batch slice with its own amax (csrc/ops_nn.cpp:213-220:
 * one fc call per slice, each with null max pointers); conv2d quantises the
 * whole input and the whole weight once (csrc/ops.cpp:264-269) and adds the
 * bias afterwards (csrc/ops.cpp:271-283).
 *
 * Build: see oracle/Makefile (gcc -O2 -fno-fast-math -ffp-contract=off).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define TKO_F16 0
#define TKO_F32 1

#define TKO_ACT_NONE 0
#define TKO_ACT_RELU 1

/* ---- IEEE helpers, written from the binary16/binary64 definitions ------ */

float tko_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0x1F) {
        bits = sign | 0x7F800000u | (man << 13);
    } else if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            /* subnormal: value = man * 2^-24, exact in binary32 */
            float v = (float)man * 5.9604644775390625e-08f;
            memcpy(&bits, &v, 4);
            bits |= sign;
        }
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* Correctly rounded (nearest-even) binary64 -> binary16. */
uint16_t tko_f64_to_f16(double d) {
    uint64_t b;
    memcpy(&b, &d, 8);
    uint16_t sign = (uint16_t)((b >> 48) & 0x8000u);
    uint64_t a = b & 0x7FFFFFFFFFFFFFFFull;
    if (a >= 0x7FF0000000000000ull) {
        return (uint16_t)(sign | (a == 0x7FF0000000000000ull ? 0x7C00u : 0x7E00u));
    }
    int e = (int)(a >> 52) - 1023;
    if (e < -25) {
        return sign; /* below half the smallest subnormal (2^-25): rounds to 0 */
    }
    uint64_t sig = (a & 0xFFFFFFFFFFFFFull) | (1ull << 52);
    int shift = 42 + (e < -14 ? (-14 - e) : 0);
    uint64_t q = sig >> shift;
    uint64_t rem = sig & ((1ull << shift) - 1);
    uint64_t half = 1ull << (shift - 1);
    if (rem > half || (rem == half && (q & 1u))) {
        q++;
    }
    if (e < -14) {
        /* subnormal result; q == 1024 is the smallest normal, same bits */
        return (uint16_t)(sign | q);
    }
    if (q == 2048u) {
        q = 1024u;
        e++;
    }
    if (e > 15) {
        return (uint16_t)(sign | 0x7C00u);
    }
    return (uint16_t)(sign | ((uint32_t)(e + 15) << 10) | (q & 0x3FFu));
}

uint16_t tko_f32_to_f16(float f) {
    return tko_f64_to_f16((double)f); /* binary32 -> binary64 is exact */
}

static float load_as_f32(const void* p, int dtype, int64_t i) {
    if (dtype == TKO_F16) {
        return tko_f16_to_f32(((const uint16_t*)p)[i]);
    }
    return ((const float*)p)[i];
}

/* Round a binary64 value to the output type T and return it widened to fp32. */
static float round_to_t(double v, int dtype) {
    if (dtype == TKO_F16) {
        return tko_f16_to_f32(tko_f64_to_f16(v));
    }
    return (float)v;
}

static void store_t(void* p, int dtype, int64_t i, float v) {
    if (dtype == TKO_F16) {
        ((uint16_t*)p)[i] = tko_f64_to_f16((double)v);
    } else {
        ((float*)p)[i] = v;
    }
}

/* ---- quantisation ------------------------------------------------------- */

/* max |x| over a strided 2-D view (rows x cols).  NaN dominates: the max is
 * taken over the bit patterns of |x|, which orders all non-negative floats
 * and places every NaN above +Inf. */
float tko_amax2d(const void* x, int dtype, int64_t rows, int64_t cols,
                 int64_t srow, int64_t scol) {
    uint32_t best = 0;
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t c = 0; c < cols; ++c) {
            float v = load_as_f32(x, dtype, r * srow + c * scol);
            uint32_t bits;
            memcpy(&bits, &v, 4);
            bits &= 0x7FFFFFFFu;
            if (bits > best) best = bits;
        }
    }
    float out;
    memcpy(&out, &best, 4);
    return out;
}

float tko_amax(const void* x, int dtype, int64_t n) {
    return tko_amax2d(x, dtype, 1, n, 0, 1);
}

float tko_quant_inv(float amax) {
    if (!(amax > 0.0f) || isinf(amax)) {
        return 0.0f; /* zero, NaN or Inf: every q is 0 */
    }
    return 32767.0f / amax;
}

static int16_t quant_one(float v, float inv) {
    float t = v * inv;
    if (isnan(t)) return 0;
    float r = nearbyintf(t); /* default rounding mode: nearest-even */
    if (r > 32767.0f) r = 32767.0f;
    if (r < -32767.0f) r = -32767.0f;
    return (int16_t)r;
}

/* q[r*cols + c] = quant(x[r*srow + c*scol]) for a strided 2-D view. */
void tko_quant2d(const void* x, int dtype, int64_t rows, int64_t cols,
                 int64_t srow, int64_t scol, float amax, int16_t* q) {
    float inv = tko_quant_inv(amax);
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t c = 0; c < cols; ++c) {
            q[r * cols + c] = quant_one(load_as_f32(x, dtype, r * srow + c * scol), inv);
        }
    }
}

void tko_quant(const void* x, int dtype, int64_t n, float amax, int16_t* q) {
    tko_quant2d(x, dtype, 1, n, 0, 1, amax, q);
}

/* Signed high limb and unsigned low limb: q = 256 * hi + lo. */
void tko_limbs(const int16_t* q, int64_t n, int8_t* hi, uint8_t* lo) {
    for (int64_t i = 0; i < n; ++i) {
        int32_t v = q[i];
        hi[i] = (int8_t)(v >> 8);   /* arithmetic shift: floor(v / 256) */
        lo[i] = (uint8_t)(v & 0xFF);
    }
}

/* ---- integer GEMM --------------------------------------------------------- */

/* acc[m*N+n] = sum_k qa[m*sam + k*sak] * qb[k*sbk + n*sbn], exact int64. */
void tko_gemm_i16(int64_t M, int64_t N, int64_t K,
                  const int16_t* qa, int64_t sam, int64_t sak,
                  const int16_t* qb, int64_t sbk, int64_t sbn, int64_t* acc) {
    for (int64_t m = 0; m < M; ++m) {
        for (int64_t n = 0; n < N; ++n) {
            int64_t s = 0;
            const int16_t* pa = qa + m * sam;
            const int16_t* pb = qb + n * sbn;
            for (int64_t k = 0; k < K; ++k) {
                s += (int64_t)pa[k * sak] * (int64_t)pb[k * sbk];
            }
            acc[m * N + n] = s;
        }
    }
}

double tko_dequant_scale(float amax_a, float amax_b) {
    return ((double)amax_a * (double)amax_b) / 1073676289.0;
}

/* ---- epilogue ------------------------------------------------------------- */

/*
 * out[m*ldo + n] = epilogue(acc[m*N + n]) following the contract in the
 * file header.  bias is [N] (may be NULL); addend is read at
 * addend[m*add_sm + n*add_sn] (may be NULL; strides of 0 broadcast).
 */
void tko_epilogue(int dtype, int64_t M, int64_t N, const int64_t* acc,
                  float amax_a, float amax_b, float alpha,
                  const void* bias, const void* addend, int64_t add_sm,
                  int64_t add_sn, float beta, int act, void* out, int64_t ldo) {
    double s = tko_dequant_scale(amax_a, amax_b);
    for (int64_t m = 0; m < M; ++m) {
        for (int64_t n = 0; n < N; ++n) {
            float r = round_to_t((double)acc[m * N + n] * s, dtype);
            if (alpha != 1.0f) {
                r = round_to_t((double)(r * alpha), dtype);
            }
            if (bias != NULL) {
                r = round_to_t((double)(r + load_as_f32(bias, dtype, n)), dtype);
            }
            if (addend != NULL && beta != 0.0f) {
                float b = load_as_f32(addend, dtype, m * add_sm + n * add_sn);
                if (beta != 1.0f) {
                    b = round_to_t((double)(b * beta), dtype);
                }
                r = round_to_t((double)(r + b), dtype);
            }
            if (act == TKO_ACT_RELU) {
                if (!(r > 0.0f) && !isnan(r)) r = 0.0f;
            }
            store_t(out, dtype, m * ldo + n, r);
        }
    }
}

/* ---- direct conv2d on quantised NCHW / OIHW tensors ---------------------- */

/*
 * acc[((b*F + f)*OH + oh)*OW + ow] =
 *   sum_{c in group, r, s} qx[b, c, oh*sh - ph + r*dh, ow*sw - pw + s*dw] * qw[f, c', r, s]
 * Out-of-range input positions contribute 0 (zero padding).
 */
void tko_conv2d_i16(int64_t NB, int64_t C, int64_t H, int64_t W, int64_t F,
                    int64_t KH, int64_t KW, int64_t sh, int64_t sw, int64_t ph,
                    int64_t pw, int64_t dh, int64_t dw, int64_t groups,
                    const int16_t* qx, const int16_t* qw, int64_t* acc) {
    int64_t OH = (H + 2 * ph - dh * (KH - 1) - 1) / sh + 1;
    int64_t OW = (W + 2 * pw - dw * (KW - 1) - 1) / sw + 1;
    int64_t cg = C / groups, fg = F / groups;
    for (int64_t b = 0; b < NB; ++b) {
        for (int64_t f = 0; f < F; ++f) {
            int64_t g = f / fg;
            for (int64_t oh = 0; oh < OH; ++oh) {
                for (int64_t ow = 0; ow < OW; ++ow) {
                    int64_t s = 0;
                    for (int64_t c = 0; c < cg; ++c) {
                        int64_t ci = g * cg + c;
                        for (int64_t r = 0; r < KH; ++r) {
                            int64_t ih = oh * sh - ph + r * dh;
                            if (ih < 0 || ih >= H) continue;
                            for (int64_t t = 0; t < KW; ++t) {
                                int64_t iw = ow * sw - pw + t * dw;
                                if (iw < 0 || iw >= W) continue;
                                s += (int64_t)qx[((b * C + ci) * H + ih) * W + iw] *
                                     (int64_t)qw[((f * cg + c) * KH + r) * KW + t];
                            }
                        }
                    }
                    acc[((b * F + f) * OH + oh) * OW + ow] = s;
                }
            }
        }
    }
}
