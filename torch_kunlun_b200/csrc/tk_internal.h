// tk_internal.h -- shared host-side helpers of libtk_kernels.so.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>
#include <utility>

#include "../../include/tk_kernels.h"

namespace tk {

// Thread-local last-error message; set by fail() and returned by
// tk_last_error_string().
void set_error(const char* fmt, ...);

inline int fail_status(int status) { return status; }

#define TK_FAIL(status, ...)          \
    do {                              \
        ::tk::set_error(__VA_ARGS__); \
        return (status);              \
    } while (0)

#define TK_CHECK_ARG(cond, ...)                                  \
    do {                                                         \
        if (!(cond)) TK_FAIL(TK_ERR_INVALID_ARG, __VA_ARGS__);   \
    } while (0)

#define TK_CUDA_TRY(expr)                                                              \
    do {                                                                               \
        cudaError_t _e = (expr);                                                       \
        if (_e != cudaSuccess)                                                         \
            TK_FAIL(TK_ERR_CUDA, "%s failed: %s", #expr, cudaGetErrorString(_e));      \
    } while (0)

// Status of the most recent kernel launch on this thread.
inline int launch_status(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) TK_FAIL(TK_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
    return TK_OK;
}

int current_device();
int sm_count(int device);
// Device address of the per-device error word that bounded waits write.
unsigned* device_error_word(int device);

inline size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Launch with programmatic stream serialisation: the kernel may be placed
// while the kernel before it on the stream drains; it waits (pdl_wait) before
// reading anything that kernel wrote.  Returns the launch's own error code.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

inline size_t dtype_size(tk_dtype_t dt) { return dt == TK_DTYPE_F16 ? 2 : 4; }

// One GEMM operand to quantise: a [batch][rows][cols] strided view, one amax
// per slice (per_slice) or for the whole operand, written to amax_out unless
// given_amax is set, and limb planes [batch][2][rows][round_up(cols,16)].
struct QuantOperand {
    const void* x;
    int64_t batch, rows, cols, sb, sr, sc;
    bool per_slice;
    const float* given_amax;
    float* amax_out;
    int8_t* limbs;
};
int quantise_operands(tk_dtype_t dt, const QuantOperand* ops, int nops, cudaStream_t stream);

// cuTensorMapEncodeTiled, resolved once through the runtime's driver entry
// point query (NULL when unavailable).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn tensor_map_encoder();

// The argument checks of tk_qgemm (sizes, dtype, activation, output pointer).
int qgemm_validate(const tk_qgemm_desc_t& d);

}  // namespace tk
