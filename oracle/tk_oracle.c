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
 *   act:      relu(r) = r > 0 || isnan(r) ? r : +0;  gelu / gelu_tanh / silu:
 *             r = T(act(float(r))) with act evaluated in binary64 (libm)
 *
 * bmm quantises every batch slice with its own amax (csrc/ops_nn.cpp:213-220:
 * one fc call per slice, each with null max pointers); conv2d quantises the
 * whole input and the whole weight once (csrc/ops.cpp:264-269) and adds the
 * bias afterwards (csrc/ops.cpp:271-283).
 *
 * Build: see oracle/Makefile (gcc -O2 -fno-fast-math -ffp-contract=off
 * -pthread).  The large elementwise loops (amax, quantise, limbs, epilogue)
 * are split over the host cores by tko_parallel: each thread takes a
 * contiguous index range and the only cross-thread combination is a max, so
 * results do not depend on the thread count.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#define TKO_F16 0
#define TKO_F32 1

#define TKO_ACT_NONE 0
#define TKO_ACT_RELU 1
#define TKO_ACT_GELU 2      /* erf form */
#define TKO_ACT_GELU_TANH 3 /* tanh approximation */
#define TKO_ACT_SILU 4

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

/* ---- host threads -------------------------------------------------------- */

/* fn(ctx, begin, end, tid) over [0, n) split into contiguous ranges, one per
 * host thread (TKO_THREADS overrides the count), each range at least `grain`
 * items (small n runs inline). */
typedef void (*tko_range_fn)(void* ctx, int64_t begin, int64_t end, int tid);

#define TKO_MAX_THREADS 256

struct tko_job {
    tko_range_fn fn;
    void* ctx;
    int64_t begin, end;
    int tid;
};

static void* tko_job_main(void* p) {
    struct tko_job* j = (struct tko_job*)p;
    j->fn(j->ctx, j->begin, j->end, j->tid);
    return NULL;
}

int tko_num_threads(void) {
    const char* e = getenv("TKO_THREADS");
    long n = e != NULL ? atol(e) : sysconf(_SC_NPROCESSORS_ONLN);
    if (n < 1) n = 1;
    if (n > TKO_MAX_THREADS) n = TKO_MAX_THREADS;
    return (int)n;
}

static void tko_parallel(int64_t n, int64_t grain, tko_range_fn fn, void* ctx) {
    int t = tko_num_threads();
    if (grain < 1) grain = 1;
    if (n < (int64_t)t * grain) t = (int)(n / grain) + 1;
    if (t <= 1) {
        fn(ctx, 0, n, 0);
        return;
    }
    pthread_t th[TKO_MAX_THREADS];
    struct tko_job jobs[TKO_MAX_THREADS];
    int started[TKO_MAX_THREADS];
    for (int i = 0; i < t; ++i) {
        jobs[i].fn = fn;
        jobs[i].ctx = ctx;
        jobs[i].begin = n * i / t;
        jobs[i].end = n * (i + 1) / t;
        jobs[i].tid = i;
        started[i] = i > 0 && pthread_create(&th[i], NULL, tko_job_main, &jobs[i]) == 0;
    }
    tko_job_main(&jobs[0]);
    for (int i = 1; i < t; ++i) {
        if (started[i]) {
            pthread_join(th[i], NULL);
        } else {
            tko_job_main(&jobs[i]); /* thread creation failed: run the range here */
        }
    }
}

/* ---- quantisation ------------------------------------------------------- */

/* max |x| over a strided 2-D view (rows x cols).  NaN dominates: the max is
 * taken over the bit patterns of |x|, which orders all non-negative floats
 * and places every NaN above +Inf. */
struct tko_view2d {
    const void* x;
    int dtype;
    int64_t cols, srow, scol;
    float inv;
    int16_t* q;
    uint32_t best[TKO_MAX_THREADS];
};

static void amax_range(void* p, int64_t begin, int64_t end, int tid) {
    struct tko_view2d* v = (struct tko_view2d*)p;
    uint32_t best = 0;
    int64_t r = begin / v->cols, c = begin % v->cols;
    for (int64_t i = begin; i < end; ++i) {
        float f = load_as_f32(v->x, v->dtype, r * v->srow + c * v->scol);
        uint32_t bits;
        memcpy(&bits, &f, 4);
        bits &= 0x7FFFFFFFu;
        if (bits > best) best = bits;
        if (++c == v->cols) { c = 0; ++r; }
    }
    v->best[tid] = best;
}

float tko_amax2d(const void* x, int dtype, int64_t rows, int64_t cols,
                 int64_t srow, int64_t scol) {
    uint32_t best = 0;
    if (rows > 0 && cols > 0) {
        struct tko_view2d* v = (struct tko_view2d*)calloc(1, sizeof(struct tko_view2d));
        v->x = x;
        v->dtype = dtype;
        v->cols = cols;
        v->srow = srow;
        v->scol = scol;
        tko_parallel(rows * cols, 65536, amax_range, v);
        for (int i = 0; i < TKO_MAX_THREADS; ++i)
            if (v->best[i] > best) best = v->best[i];
        free(v);
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
static void quant_range(void* p, int64_t begin, int64_t end, int tid) {
    (void)tid;
    struct tko_view2d* v = (struct tko_view2d*)p;
    int64_t r = begin / v->cols, c = begin % v->cols;
    for (int64_t i = begin; i < end; ++i) {
        v->q[i] = quant_one(load_as_f32(v->x, v->dtype, r * v->srow + c * v->scol), v->inv);
        if (++c == v->cols) { c = 0; ++r; }
    }
}

void tko_quant2d(const void* x, int dtype, int64_t rows, int64_t cols,
                 int64_t srow, int64_t scol, float amax, int16_t* q) {
    if (rows <= 0 || cols <= 0) return;
    struct tko_view2d* v = (struct tko_view2d*)calloc(1, sizeof(struct tko_view2d));
    v->x = x;
    v->dtype = dtype;
    v->cols = cols;
    v->srow = srow;
    v->scol = scol;
    v->inv = tko_quant_inv(amax);
    v->q = q;
    tko_parallel(rows * cols, 65536, quant_range, v);
    free(v);
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

/* ---- floating-point ops, in binary64 with libm ------------------------------
 * The reference runs these through XDNN (gelu / approximate_gelu
 * csrc/ops_nn.cpp:132-147, swish csrc/ops_extra.cpp:71, softmax
 * csrc/ops_nn.cpp:73-83, layer_norm csrc/ops_nn.cpp:85-130); only their
 * mathematical definitions are restated here, each evaluated in binary64 and
 * rounded once to the output type.  The device evaluates the same formulas
 * in binary32, so the two agree within the bounds the tests state. */

/*   gelu (erf):  0.5 x (1 + erf(x / sqrt(2)))
 *   gelu (tanh): 0.5 x (1 + tanh(sqrt(2 / pi) (x + 0.044715 x^3)))
 *   silu:        x / (1 + exp(-x)) */
double tko_act64(double x, int act) {
    switch (act) {
        case TKO_ACT_RELU: return (x > 0.0 || isnan(x)) ? x : 0.0;
        case TKO_ACT_GELU: return 0.5 * x * (1.0 + erf(x * 0.70710678118654752440));
        case TKO_ACT_GELU_TANH:
            return 0.5 * x * (1.0 + tanh(0.79788456080286535588 * (x + 0.044715 * x * x * x)));
        case TKO_ACT_SILU: return x / (1.0 + exp(-x));
        default: return x;
    }
}

struct tko_ew_job {
    const void* a;
    const void* b;
    void* out;
    int dtype, act;
};

static void act_range(void* p, int64_t begin, int64_t end, int tid) {
    (void)tid;
    const struct tko_ew_job* j = (const struct tko_ew_job*)p;
    for (int64_t i = begin; i < end; ++i)
        store_t(j->out, j->dtype, i, round_to_t(tko_act64(load_as_f32(j->a, j->dtype, i), j->act), j->dtype));
}

/* out[i] = T(act(x[i])). */
void tko_act(const void* x, int dtype, int64_t n, int act, void* out) {
    struct tko_ew_job j = {x, NULL, out, dtype, act};
    if (n > 0) tko_parallel(n, 16384, act_range, &j);
}

static void silu_mul_range(void* p, int64_t begin, int64_t end, int tid) {
    (void)tid;
    const struct tko_ew_job* j = (const struct tko_ew_job*)p;
    for (int64_t i = begin; i < end; ++i) {
        const float h = round_to_t(tko_act64(load_as_f32(j->a, j->dtype, i), TKO_ACT_SILU), j->dtype);
        store_t(j->out, j->dtype, i, round_to_t((double)h * (double)load_as_f32(j->b, j->dtype, i), j->dtype));
    }
}

/* out[i] = T(T(silu(gate[i])) * up[i]): the reference's swish, stored as T,
 * then mul (csrc/ops_extra.cpp:71, csrc/autograd.cpp:60-71). */
void tko_silu_mul(const void* gate, const void* up, int dtype, int64_t n, void* out) {
    struct tko_ew_job j = {gate, up, out, dtype, TKO_ACT_SILU};
    if (n > 0) tko_parallel(n, 16384, silu_mul_range, &j);
}

struct tko_row_job {
    const void* x;
    const void* gamma;
    const void* beta;
    void* out;
    float* mean;
    float* rstd;
    int64_t cols;
    double eps;
    int dtype, out_dtype, wdtype;
};

static void softmax_range(void* p, int64_t begin, int64_t end, int tid) {
    (void)tid;
    const struct tko_row_job* j = (const struct tko_row_job*)p;
    const int64_t n = j->cols;
    double* e = (double*)malloc(sizeof(double) * (size_t)(n > 0 ? n : 1));
    for (int64_t r = begin; r < end; ++r) {
        double m = -INFINITY;
        for (int64_t c = 0; c < n; ++c) {
            const double v = load_as_f32(j->x, j->dtype, r * n + c);
            if (v > m || isnan(v)) m = v;
        }
        double s = 0.0;
        for (int64_t c = 0; c < n; ++c) {
            const double v = load_as_f32(j->x, j->dtype, r * n + c);
            e[c] = (v == -INFINITY) ? 0.0 : exp(v - m);
            s += e[c];
        }
        for (int64_t c = 0; c < n; ++c) store_t(j->out, j->out_dtype, r * n + c, round_to_t(e[c] / s, j->out_dtype));
    }
    free(e);
}

/* Softmax over the last axis of [rows, cols]: m = max, e = exp(x - m),
 * y = T(e / sum e), all in binary64. */
void tko_softmax(const void* x, int dtype, int64_t rows, int64_t cols, int out_dtype, void* out) {
    struct tko_row_job j = {x, NULL, NULL, out, NULL, NULL, cols, 0.0, dtype, out_dtype, dtype};
    if (rows > 0 && cols > 0) tko_parallel(rows, 64, softmax_range, &j);
}

static void layer_norm_range(void* p, int64_t begin, int64_t end, int tid) {
    (void)tid;
    const struct tko_row_job* j = (const struct tko_row_job*)p;
    const int64_t n = j->cols;
    for (int64_t r = begin; r < end; ++r) {
        double mu = 0.0, var = 0.0;
        for (int64_t c = 0; c < n; ++c) mu += load_as_f32(j->x, j->dtype, r * n + c);
        mu /= (double)n;
        for (int64_t c = 0; c < n; ++c) {
            const double d = load_as_f32(j->x, j->dtype, r * n + c) - mu;
            var += d * d;
        }
        var /= (double)n;
        const double rs = 1.0 / sqrt(var + j->eps);
        if (j->mean) j->mean[r] = (float)mu;
        if (j->rstd) j->rstd[r] = (float)rs;
        for (int64_t c = 0; c < n; ++c) {
            double y = (load_as_f32(j->x, j->dtype, r * n + c) - mu) * rs;
            if (j->gamma) y *= load_as_f32(j->gamma, j->wdtype, c);
            if (j->beta) y += load_as_f32(j->beta, j->wdtype, c);
            store_t(j->out, j->dtype, r * n + c, round_to_t(y, j->dtype));
        }
    }
}

/* LayerNorm over the last axis: mean and biased variance in binary64,
 * y = T((x - mean) / sqrt(var + eps) * gamma + beta); mean / rstd rows as
 * fp32 when the pointers are non-NULL. */
void tko_layer_norm(const void* x, int dtype, int64_t rows, int64_t cols, const void* gamma,
                    const void* beta, int wdtype, double eps, void* out, float* mean, float* rstd) {
    struct tko_row_job j = {x, gamma, beta, out, mean, rstd, cols, eps, dtype, dtype, wdtype};
    if (rows > 0 && cols > 0) tko_parallel(rows, 64, layer_norm_range, &j);
}

/* ---- integer GEMM --------------------------------------------------------- */

struct tko_gemm_job {
    int64_t N, K, sam, sak, sbk, sbn;
    const int16_t* qa;
    const int16_t* qb;
    int64_t* acc;
};

static void gemm_range(void* p, int64_t begin, int64_t end, int tid) {
    (void)tid;
    const struct tko_gemm_job* j = (const struct tko_gemm_job*)p;
    for (int64_t i = begin; i < end; ++i) {
        const int64_t m = i / j->N, n = i - m * j->N;
        const int16_t* pa = j->qa + m * j->sam;
        const int16_t* pb = j->qb + n * j->sbn;
        int64_t s = 0;
        for (int64_t k = 0; k < j->K; ++k) {
            s += (int64_t)pa[k * j->sak] * (int64_t)pb[k * j->sbk];
        }
        j->acc[i] = s;
    }
}

/* acc[m*N+n] = sum_k qa[m*sam + k*sak] * qb[k*sbk + n*sbn], exact int64
 * (whole output elements per thread). */
void tko_gemm_i16(int64_t M, int64_t N, int64_t K,
                  const int16_t* qa, int64_t sam, int64_t sak,
                  const int16_t* qb, int64_t sbk, int64_t sbn, int64_t* acc) {
    struct tko_gemm_job j = {N, K, sam, sak, sbk, sbn, qa, qb, acc};
    if (M <= 0 || N <= 0) return;
    tko_parallel(M * N, 65536 / (K > 0 ? K : 1), gemm_range, &j);
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
struct tko_epi_job {
    int dtype, act;
    int64_t N, add_sm, add_sn, ldo;
    const int64_t* acc;
    double s;
    float alpha, beta;
    const void* bias;
    const void* addend;
    void* out;
};

static void epilogue_range(void* p, int64_t begin, int64_t end, int tid) {
    (void)tid;
    const struct tko_epi_job* j = (const struct tko_epi_job*)p;
    const int dtype = j->dtype;
    for (int64_t i = begin; i < end; ++i) {
        const int64_t m = i / j->N, n = i - m * j->N;
        float r = round_to_t((double)j->acc[i] * j->s, dtype);
        if (j->alpha != 1.0f) {
            r = round_to_t((double)(r * j->alpha), dtype);
        }
        if (j->bias != NULL) {
            r = round_to_t((double)(r + load_as_f32(j->bias, dtype, n)), dtype);
        }
        if (j->addend != NULL && j->beta != 0.0f) {
            float b = load_as_f32(j->addend, dtype, m * j->add_sm + n * j->add_sn);
            if (j->beta != 1.0f) {
                b = round_to_t((double)(b * j->beta), dtype);
            }
            r = round_to_t((double)(r + b), dtype);
        }
        if (j->act == TKO_ACT_RELU) {
            if (!(r > 0.0f) && !isnan(r)) r = 0.0f;
        } else if (j->act != TKO_ACT_NONE) {
            r = round_to_t(tko_act64((double)r, j->act), dtype);
        }
        store_t(j->out, dtype, m * j->ldo + n, r);
    }
}

void tko_epilogue(int dtype, int64_t M, int64_t N, const int64_t* acc,
                  float amax_a, float amax_b, float alpha,
                  const void* bias, const void* addend, int64_t add_sm,
                  int64_t add_sn, float beta, int act, void* out, int64_t ldo) {
    struct tko_epi_job j = {dtype, act, N, add_sm, add_sn, ldo, acc,
                            tko_dequant_scale(amax_a, amax_b), alpha, beta, bias, addend, out};
    if (M <= 0 || N <= 0) return;
    tko_parallel(M * N, 16384, epilogue_range, &j);
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
