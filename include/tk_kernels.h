/*
 * tk_kernels.h -- C ABI of libtk_kernels.so, the sm_100a kernel library behind
 * torch_kunlun's dense-op hot path.
 *
 * Conventions (every entry point):
 *   - returns int status: 0 (TK_OK) on success, > 0 on error; the message of
 *     the last error on the calling thread is tk_last_error_string();
 *   - no C++ exceptions cross the boundary; no allocation: device scratch is
 *     a caller-provided workspace sized by the matching *_workspace_size call;
 *   - all pointers are device pointers unless stated; `stream` is a
 *     cudaStream_t (NULL = legacy default stream of the current device);
 *   - work is enqueued asynchronously on `stream`; nothing synchronises;
 *   - some kernels are launched with programmatic dependent launch: they may
 *     be placed while the previous kernel on `stream` is still running, but
 *     touch global memory only after it has completed, so stream order holds
 *     exactly as for ordinary launches;
 *   - element strides are in elements, not bytes;
 *   - functions are reentrant and keep no per-call global state, except
 *     tk_qgemm_noalloc, whose scratch is one array shared by all its calls.
 *
 * Each function names the reference interface it replaces: the reference
 * calls Baidu XDNN (baidu::xpu::api::*) from the files cited.
 */
#ifndef TK_KERNELS_H
#define TK_KERNELS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TK_ABI_VERSION 1

#if defined(__GNUC__)
#define TK_API __attribute__((visibility("default")))
#else
#define TK_API
#endif

typedef enum {
    TK_OK = 0,
    TK_ERR_INVALID_ARG = 1,
    TK_ERR_UNSUPPORTED = 2,
    TK_ERR_CUDA = 3,
    TK_ERR_WORKSPACE = 4,
    TK_ERR_DEVICE = 5
} tk_status_t;

typedef enum { TK_DTYPE_F16 = 0, TK_DTYPE_F32 = 1 } tk_dtype_t;

typedef enum {
    TK_ACT_NONE = 0,
    TK_ACT_RELU = 1,
    TK_ACT_GELU = 2,      /* erf form */
    TK_ACT_GELU_TANH = 3, /* tanh approximation */
    TK_ACT_SILU = 4,
    /* The gated-MLP activation (silu(gate) * up) fused into the up
     * projection: the addend operand holds the gate, and the epilogue
     * multiplies by T(silu(gate)) instead of adding (beta must be 1); each
     * product rounds once to T, as the separate swish + mul.  fp16 output on
     * the vector epilogue path only (16-byte aligned out, bias and gate rows,
     * unit column stride, N a multiple of 16, no split reduction). */
    TK_ACT_SILU_GATE = 5
} tk_act_t;

/* ---- library ------------------------------------------------------------- */

TK_API int tk_abi_version(void);
TK_API const char* tk_last_error_string(void);

/* Reads and clears the device-side error word of `device` (a bounded wait
 * inside a kernel that timed out records a code there).  Synchronises the
 * device.  *code_out = 0 means no error was recorded. */
TK_API int tk_device_error(int device, unsigned* code_out);

/* ---- quantisation ----------------------------------------------------------
 * Replaces the max-abs and int16-quantise steps that XDNN performs inside
 * fc/conv2d when the max pointers are null (csrc/ops.cpp:224-227,
 * csrc/ops.cpp:264-268, csrc/ops_nn.cpp:214-218).
 */

/* amax_out[s] = max |x[s*slice_stride + i]|, i in [0, slice_len), NaN
 * dominating.  Each slice is a dense memory range of slice_len elements. */
TK_API int tk_amax(tk_dtype_t dtype, const void* x, int64_t nslices, int64_t slice_stride,
            int64_t slice_len, float* amax_out, void* stream);

/* Quantise a batch of strided [rows, cols] views to int16 with scale
 * 32767/amax[b * amax_stride] and store them as two limb planes,
 * q = 256*hi + lo: limbs + ((b*2 + 0)*rows + r)*ld holds the signed high
 * limbs and plane 1 the unsigned low limbs, ld = round_up(cols, 16); columns
 * [cols, ld) are written as zero.  View element (b, r, c) is at
 * x[b*sb + r*sr + c*sc]. */
TK_API int tk_quantize_limbs(tk_dtype_t dtype, const void* x, int64_t batch, int64_t rows,
                      int64_t cols, int64_t sb, int64_t sr, int64_t sc, const float* amax,
                      int64_t amax_stride, int8_t* limbs, void* stream);

/* ---- quantised GEMM ---------------------------------------------------------
 * Replaces baidu::xpu::api::fc<T,T,T,TGEMM> as called by fc_impl
 * (csrc/ops.cpp:210-230, mm and linear), by bmm_impl (csrc/ops_nn.cpp:199-221,
 * one fc per slice), and the separate epilogue launches that follow it: the
 * bias add of linear (csrc/ops.cpp:491-493), the alpha/beta scale and add of
 * addmm (csrc/autograd.cpp:192-218) and baddbmm
 * (csrc/linalg_extra.cpp:85-93), and activations (csrc/ops.cpp:151-160,
 * csrc/ops_nn.cpp:132-147, csrc/ops_extra.cpp:71).
 *
 *   out[b][m][n] = epilogue( sum_k q(A[b][m][k]) * q(B[b][n][k]) )
 *
 * A element (b,m,k) is at a[b*a_sb + m*a_sm + k*a_sk]; B element (b,n,k) at
 * b[b*b_sb + n*b_sn + k*b_sk] (so a row-major W[N,K] of linear has
 * b_sn = K, b_sk = 1 and a row-major [K,N] operand of mm has b_sn = 1,
 * b_sk = N).  out has unit stride along n.  With per_slice_scales = 1 every
 * batch slice of A and of B gets its own amax (bmm); with 0 one amax covers
 * the whole operand (every slice must then be laid out densely).
 * The epilogue (in order): dequantise and round to dtype; if alpha != 1
 * multiply by alpha and round; if bias add bias[n] and round; if addend and
 * beta != 0 add beta*addend (addend element (b,m,n) at
 * addend[b*add_sb + m*add_sm + n*add_sn], strides may be 0 to broadcast) and
 * round; apply act (TK_ACT_SILU_GATE replaces the addend step: multiply by
 * T(silu(addend)) and round).  K is any size: reductions longer than 32768 (and long
 * reductions with few output tiles) are split into chunks whose exact int64
 * sums are added in the workspace before the one dequantising rounding.
 */
typedef struct {
    tk_dtype_t dtype;
    int64_t batch, m, n, k;
    const void* a;
    int64_t a_sb, a_sm, a_sk;
    const void* b;
    int64_t b_sb, b_sn, b_sk;
    void* out;
    int64_t out_sb, out_sm;
    const void* bias;
    const void* addend;
    int64_t add_sb, add_sm, add_sn;
    float alpha, beta;
    tk_act_t act;
    int per_slice_scales;
    /* Optional precomputed amax (device, one float per slice or one per
     * operand); NULL means computed by the call (the reference's null
     * x_maxptr / w_maxptr, csrc/ops.cpp:227). */
    const float* amax_a;
    const float* amax_b;
    /* Optional (device, one float): receives max |out| over the whole output
     * after the epilogue (NaN above everything), the scale the next quantised
     * op on out would compute -- folded into the epilogue for fp16 outputs on
     * the vector path, else one extra pass over out (which must then be
     * contiguous).  NULL: not computed. */
    float* amax_out;
} tk_qgemm_desc_t;

TK_API size_t tk_qgemm_workspace_size(const tk_qgemm_desc_t* desc);
TK_API int tk_qgemm(const tk_qgemm_desc_t* desc, void* workspace, size_t workspace_bytes,
             void* stream);

/* The GEMM and epilogue alone, on operands already quantised by
 * tk_quantize_limbs (layout [batch][2][rows][round_up(k,16)]) with the amax
 * values they were quantised with (one per slice when per_slice_scales, else
 * one per operand).  desc->a and desc->b are ignored.  Lets a caller keep the
 * quantised form of an operand that does not change between calls (weights)
 * -- XDNN's fc accepts precomputed max pointers for the same purpose
 * (csrc/ops.cpp:227 passes them as null).  K must be <= 32768 (no workspace
 * for a split reduction).  amax_out is supported when the epilogue is the
 * fp16 vector path (it is folded into the epilogue). */
TK_API int tk_qgemm_from_limbs(const tk_qgemm_desc_t* desc, const int8_t* a_limbs,
                               const int8_t* b_limbs, const float* amax_a, const float* amax_b,
                               void* stream);

/* tk_qgemm for callers that cannot allocate device memory (for example a
 * host application or inference server that owns all device memory, passes
 * this library only its inputs and outputs, and forbids allocation after
 * start-up).  No counterpart in the reference: XDNN's fc draws its scratch
 * from the per-device context the reference creates.  Same contract and
 * results as tk_qgemm, but the scratch is a fixed 64 MiB array inside the
 * library's device image (held by every GPU that loads the library until
 * exit), so the call allocates nothing.  Problems whose
 * tk_qgemm_workspace_size exceeds 64 MiB - 1 KiB are rejected with
 * TK_ERR_WORKSPACE.  All calls share the array: calls that overlap on the
 * GPU race; calls ordered on one stream are safe.  The first call on a
 * device does a one-time set-up (device address lookup); make it before any
 * stream capture.  `stream` must belong to the current device (the scratch
 * used is the current device's); a stream of another device is rejected with
 * TK_ERR_INVALID_ARG, as are descriptors tk_qgemm rejects. */
TK_API int tk_qgemm_noalloc(const tk_qgemm_desc_t* desc, void* stream);

/* tk_qgemm (batch 1) with the output rows scattered over destination buffers:
 * rows [q*rows_per_dest, (q+1)*rows_per_dest) are stored at row_dest[q]
 * (row stride out_sm, local row m - q*rows_per_dest) and out is ignored.
 * row_dest entries are device pointers valid on the calling GPU, typically
 * other GPUs' buffers opened through CUDA IPC: a row-parallel linear writes
 * each row block straight into the rank that owns it over NVLink while the
 * GEMM runs, and that rank sums its slots with tk_reduce_sum.  Replaces the
 * fc + bkcl reduce_scatter pair of a row-parallel linear (csrc/ops.cpp:210-230,
 * csrc/xccl.cpp:111-163).  1 <= ndest <= 8, m == ndest * rows_per_dest. */
TK_API int tk_qgemm_scatter_rows(const tk_qgemm_desc_t* desc, void* const* row_dest, int ndest,
                                 int64_t rows_per_dest, void* workspace, size_t workspace_bytes,
                                 void* stream);

/* Same contract computed by a plain CUDA-core kernel (one output per thread).
 * Used to cross-check the tensor-core path on the device; not fast. */
TK_API int tk_qgemm_simt(const tk_qgemm_desc_t* desc, void* workspace, size_t workspace_bytes,
                  void* stream);

/* Debug view of the tensor-core GEMM: writes the three int32 limb-product
 * accumulators (hi*hi, hi*lo + lo*hi, lo*lo) of slice 0 to acc3
 * ([3][m][n], int32) in addition to out. */
TK_API int tk_qgemm_debug(const tk_qgemm_desc_t* desc, void* workspace, size_t workspace_bytes,
                   int32_t* acc3, void* stream);

/* ---- quantised conv2d --------------------------------------------------------
 * Replaces baidu::xpu::api::conv2d<T,T,T,TGEMM> and the bias broadcast_add of
 * conv2d_impl (csrc/ops.cpp:237-285): NCHW input x [n,c,h,w], OIHW weight
 * [f, c/groups, kh, kw], optional bias [f], NCHW output [n,f,oh,ow], all
 * contiguous.  The whole input and the whole weight are quantised with one
 * scale each; the bias is added after the output is rounded to dtype.
 * (c/groups)*kh*kw must be <= 32768.
 */
typedef struct {
    tk_dtype_t dtype;
    int64_t n, c, h, w, f, kh, kw;
    int64_t stride_h, stride_w, pad_h, pad_w, dil_h, dil_w, groups;
    const void* x;
    const void* weight;
    const void* bias;
    void* out;
    const float* amax_x; /* optional precomputed per-tensor amax (device) */
    const float* amax_w;
} tk_conv2d_desc_t;

TK_API size_t tk_conv2d_workspace_size(const tk_conv2d_desc_t* desc);
TK_API int tk_conv2d_q16(const tk_conv2d_desc_t* desc, void* workspace, size_t workspace_bytes,
                         void* stream);

/* ---- quantised conv3d --------------------------------------------------------
 * Replaces baidu::xpu::api::conv3d<T,T,T,TGEMM> and the bias add of conv3d
 * (csrc/ops_nn_extra.cpp:88-121) with the conv2d contract above: NCDHW input
 * [n,c,d,h,w], OIDHW weight [f, c/groups, kd, kh, kw], optional bias [f],
 * NCDHW output, one scale per tensor, bias added after rounding.
 * (c/groups)*kd*kh*kw must be <= 32768.  tk_conv2d_q16 is this call with
 * d = kd = 1. */
typedef struct {
    tk_dtype_t dtype;
    int64_t n, c, d, h, w, f, kd, kh, kw;
    int64_t stride_d, stride_h, stride_w, pad_d, pad_h, pad_w, dil_d, dil_h, dil_w, groups;
    const void* x;
    const void* weight;
    const void* bias;
    void* out;
    const float* amax_x; /* optional precomputed per-tensor amax (device) */
    const float* amax_w;
} tk_conv3d_desc_t;

TK_API size_t tk_conv3d_workspace_size(const tk_conv3d_desc_t* desc);
TK_API int tk_conv3d_q16(const tk_conv3d_desc_t* desc, void* workspace, size_t workspace_bytes,
                         void* stream);

/* ---- convolution weight gradient --------------------------------------------
 * Replaces the weight-gradient half of conv2d_grad (csrc/autograd.cpp:621-682)
 * and of the conv3d / conv_transpose2d backward
 * (csrc/autograd_nn_extra.cpp:427-690) under the same contract as the forward
 * convolution: x (NCDHW [n,c,d,h,w]) and grad_out ([n,f,od,oh,ow], the
 * forward's output shape) are each quantised with one per-tensor scale, and
 *   grad_weight[f][c][t][r][s] = T( scale * sum_{n,od,oh,ow} q(grad_out)[n][f][od][oh][ow]
 *                                  * q(x)[n][g*C/groups + c][od*sd + t*dd - pd][oh*sh + r*dh - ph][ow*sw + s*dw - pw] )
 * (zero outside the input, f in group g), an exact integer sum of any length
 * rounded once.  grad_weight is contiguous [f, c/groups, kd, kh, kw].  A 2-D
 * convolution is d = kd = 1. */
typedef struct {
    tk_dtype_t dtype;
    int64_t n, c, d, h, w, f, kd, kh, kw;
    int64_t stride_d, stride_h, stride_w, pad_d, pad_h, pad_w, dil_d, dil_h, dil_w, groups;
    const void* x;        /* forward input [n, c, d, h, w] */
    const void* grad_out; /* gradient of the forward output [n, f, od, oh, ow] */
    void* grad_weight;    /* [f, c/groups, kd, kh, kw] */
    const float* amax_x;  /* optional precomputed per-tensor amax (device) */
    const float* amax_g;
} tk_conv3d_wgrad_desc_t;

TK_API size_t tk_conv3d_wgrad_workspace_size(const tk_conv3d_wgrad_desc_t* desc);
TK_API int tk_conv3d_wgrad_q16(const tk_conv3d_wgrad_desc_t* desc, void* workspace,
                               size_t workspace_bytes, void* stream);

/* ---- reduction ---------------------------------------------------------------
 * out[o][i] = sum_r x[o][r][i] over a contiguous [outer, red, inner] tensor,
 * accumulated in fp32 in a fixed order (deterministic) and rounded once to
 * out_dtype (fp16 input may produce fp32 output).  Replaces xdnn::reduce_sum
 * of the bias gradients (csrc/autograd.cpp:407-412) and of sum over dims. */
TK_API int tk_reduce_sum(tk_dtype_t in_dtype, tk_dtype_t out_dtype, const void* x, int64_t outer,
                         int64_t red, int64_t inner, void* out, void* stream);

/* ---- fused scaled-dot-product attention -------------------------------------
 * out = softmax(T(T(T(q k^T) * scale) + mask)) v over [batch, heads] slices,
 * with the reference's composition semantics
 * (torch_kunlun/kunlun/attention.py:36-107, csrc/ops_nn.cpp:199-221): per-slice
 * max-abs int16 quantisation of q, k, v and of the softmax output P, exact
 * integer MAC, dequantisation, every intermediate rounded to T where the
 * reference writes a T tensor.  The causal mask adds -1e4 above the diagonal
 * and the additive mask (type T, any broadcast strides) is added after it as
 * a separately rounded add.  The [L, S] scores never reach HBM: a statistics
 * pass (row max and sum of exponentials, the slice's max probability) and an
 * output pass recompute them on the tensor cores.
 * Limits: e <= 128, s <= 32768.  Strides are in elements over
 * (batch, heads, row, column); mask strides may be 0 (broadcast). */
typedef struct {
    tk_dtype_t dtype;
    int64_t batch, heads, l, s, e, ev;
    const void* q;
    int64_t q_strides[4];
    const void* k;
    int64_t k_strides[4];
    const void* v;
    int64_t v_strides[4];
    void* out;
    int64_t out_strides[4];
    const void* mask; /* NULL = none */
    int64_t mask_strides[4];
    int causal;
    float scale; /* multiplier of q k^T; the reference passes 1/sqrt(e) */
} tk_sdpa_desc_t;

TK_API size_t tk_sdpa_workspace_size(const tk_sdpa_desc_t* desc);
TK_API int tk_sdpa_q16(const tk_sdpa_desc_t* desc, void* workspace, size_t workspace_bytes,
                       void* stream);

/* ---- row ops ------------------------------------------------------------------
 * Softmax over the last dimension of a contiguous [rows, cols] tensor
 * (xdnn::softmax, csrc/ops_nn.cpp:73-83); out_dtype may be fp32 for fp16
 * input (aten _softmax half_to_float). */
TK_API int tk_softmax(tk_dtype_t in_dtype, tk_dtype_t out_dtype, const void* x, void* y,
                      int64_t rows, int64_t cols, void* stream);

/* LayerNorm over the last `cols` elements of each row, optional gamma/beta of
 * wdtype, writing fp32 mean and rstd per row when the pointers are non-NULL
 * (xdnn::layer_norm, csrc/ops_nn.cpp:85-130). */
TK_API int tk_layer_norm(tk_dtype_t dtype, tk_dtype_t wdtype, const void* x, const void* gamma,
                         const void* beta, void* y, float* mean, float* rstd, int64_t rows,
                         int64_t cols, float eps, void* stream);

/* ---- data movement and elementwise ops -----------------------------------
 * Scalar type codes of tk_copy_strided / tk_fill_strided. */
typedef enum {
    TK_T_BOOL = 0, TK_T_U8 = 1, TK_T_I8 = 2, TK_T_I16 = 3, TK_T_I32 = 4, TK_T_I64 = 5,
    TK_T_F16 = 6, TK_T_BF16 = 7, TK_T_F32 = 8, TK_T_F64 = 9
} tk_scalar_t;

/* dst[i] = convert(src[i]) over an ndim <= 8 strided index space.  Replaces
 * the host-staged copy_ / materialize_private_contiguous of the reference
 * (csrc/ops.cpp:289-418), which copies non-contiguous views through CPU
 * memory; conversion is by value (float -> int truncates). */
TK_API int tk_copy_strided(void* dst, int dst_type, const void* src, int src_type, int ndim,
                           const int64_t* sizes, const int64_t* dst_strides,
                           const int64_t* src_strides, void* stream);

/* Fill a strided view with one value (float types use `value`, integer types
 * `ivalue`).  Replaces xdnn::constant and the host-pattern fill of
 * csrc/ops.cpp:162-208. */
TK_API int tk_fill_strided(void* dst, int type, double value, int64_t ivalue, int ndim,
                           const int64_t* sizes, const int64_t* strides, void* stream);

typedef enum {
    TK_BIN_ADD = 0,
    TK_BIN_SUB = 1,
    TK_BIN_MUL = 2,
    TK_BIN_DIV = 3,
    TK_BIN_THRESHOLD_BACKWARD = 4 /* out = b > alpha ? a : 0 (relu_grad, csrc/autograd.cpp:320-335) */
} tk_binop_t;

/* out[i] = a[i] op (alpha * b[i]) (alpha applies to add/sub) computed in fp32
 * and rounded once, over a broadcast index space (strides 0 broadcast); out
 * is contiguous.  Replaces xdnn add/broadcast_add/sub/mul
 * (csrc/ops.cpp:117-149, csrc/autograd.cpp:40-100). */
TK_API int tk_binary(int op, tk_dtype_t dtype, const void* a, const int64_t* a_strides,
                     const void* b, const int64_t* b_strides, void* out, int ndim,
                     const int64_t* sizes, float alpha, void* stream);

typedef enum {
    TK_UN_RELU = 0, TK_UN_GELU = 1, TK_UN_GELU_TANH = 2, TK_UN_SILU = 3, TK_UN_SCALE = 4
} tk_unop_t;

/* y[i] = op(x[i]) on n contiguous elements; TK_UN_SCALE is x*p0 + p1.
 * Replaces xdnn relu (csrc/ops.cpp:151-160), gelu / approximate_gelu
 * (csrc/ops_nn.cpp:132-147), swish (csrc/ops_extra.cpp:71) and scale
 * (csrc/autograd.cpp:586-601). */
TK_API int tk_unary(int op, tk_dtype_t dtype, const void* x, void* y, int64_t n, float p0,
                    float p1, void* stream);

/* y = T(silu(gate)) * up, rounded like the reference's swish followed by mul. */
TK_API int tk_silu_mul(tk_dtype_t dtype, const void* gate, const void* up, void* y, int64_t n,
                       void* stream);

/* tk_silu_mul that also writes amax_out[0] = max |y| (device fp32, NaN
 * dominating): the per-tensor scale with which the reference's next fc
 * quantises the gated activation (csrc/ops.cpp:224-227 with a null max
 * pointer), without a second pass over y.  Replaces swish + mul
 * (csrc/ops_extra.cpp:71, csrc/autograd.cpp:60-71) and that max-find. */
TK_API int tk_silu_mul_amax(tk_dtype_t dtype, const void* gate, const void* up, void* y, int64_t n,
                            float* amax_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TK_KERNELS_H */
