/*
 * nert_b200.h — the C ABI of the B200 execution layer for NERT.
 *
 * Plain pointers and sizes only: no C++ or torch types cross this boundary.
 * Every entry point returns NB2_OK (0) or a negative status; the message of
 * the last failure on the calling thread is nb2_last_error().
 *
 * Op rows take DEVICE pointers, launch on the device's stream (one non-blocking
 * stream per GPU) and return without synchronising. Results become visible to
 * the host through nb2_memcpy_d2h / nb2_device_synchronize, which also report
 * errors that kernels recorded on the device (NB2_ERR_DEVICE) instead of
 * trapping. Each row replaces one row of the reference's CUDA kernel table
 * (src/cuda/table.cu:103-189), which the reference reaches only through the
 * C++ KernelFn seam (include/nert/device.hpp:30-31); the C++ shim in
 * nert_b200/device/b200_device.cpp binds these entry points to that seam.
 */
#ifndef NERT_B200_H
#define NERT_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NB2_OK 0
#define NB2_ERR_INVALID -1     /* bad argument, attribute or shape */
#define NB2_ERR_CUDA -2        /* a CUDA runtime/driver call failed */
#define NB2_ERR_DEVICE -3      /* a kernel recorded an error (index out of range, bounded wait expired) */
#define NB2_ERR_UNSUPPORTED -4 /* a valid request this layer does not implement */
#define NB2_ERR_NOMEM -5

/* precision of Conv/Gemm/MatMul contractions */
#define NB2_PREC_3XTF32 0 /* fp32-accurate split (default) */
#define NB2_PREC_1XTF32 1 /* opt-in single tf32 pass */

/* fused epilogue activations */
#define NB2_ACT_NONE 0
#define NB2_ACT_RELU 1
#define NB2_ACT_SILU 2    /* x * sigmoid(x) */
#define NB2_ACT_SIGMOID 3

/* unary ops (nb2_unary) */
#define NB2_UNARY_RELU 0
#define NB2_UNARY_SIGMOID 1
#define NB2_UNARY_ERF 2
#define NB2_UNARY_SQRT 3
#define NB2_UNARY_NEG 4
#define NB2_UNARY_ABS 5
#define NB2_UNARY_EXP 6
#define NB2_UNARY_TANH 7
#define NB2_UNARY_IDENTITY 8
#define NB2_UNARY_SILU 9
#define NB2_UNARY_GELU_ERF 10

/* binary ops (nb2_binary) */
#define NB2_BINARY_ADD 0
#define NB2_BINARY_SUB 1
#define NB2_BINARY_MUL 2
#define NB2_BINARY_DIV 3
#define NB2_BINARY_POW 4

/* element types */
#define NB2_F32 0
#define NB2_I64 1
#define NB2_BOOL 2

typedef struct nb2_device nb2_device;

/* 2-D convolution geometry, NCHW (a 1-D conv uses h = kh = oh = 1). */
typedef struct nb2_conv_geom {
    int64_t n, c, h, w;       /* input X [n, c, h, w] */
    int64_t m, kh, kw;        /* weight W [m, c/group, kh, kw] */
    int64_t oh, ow;           /* output Y [n, m, oh, ow] */
    int64_t stride_h, stride_w;
    int64_t pad_top, pad_left, pad_bottom, pad_right;
    int64_t dil_h, dil_w;
    int64_t group;
} nb2_conv_geom;

/* ---- errors and devices ------------------------------------------------ */

/* Message of the last failing call on this thread ("" if none). */
const char* nb2_last_error(void);

/* The process-lifetime context of GPU `ordinal` (replaces the reference's
 * process singleton CudaDevice(), src/cuda_device.cpp:98-102, one per GPU). */
int nb2_device_open(int ordinal, nb2_device** out);
int nb2_device_ordinal(const nb2_device* dev);
/* The device's cudaStream_t, as an opaque pointer. */
void* nb2_device_stream(nb2_device* dev);
int nb2_device_set_precision(nb2_device* dev, int precision);
int nb2_device_get_precision(const nb2_device* dev);
/* Wait for the device's stream; NB2_ERR_DEVICE if a kernel recorded an error. */
int nb2_device_synchronize(nb2_device* dev);

/* Device memory (replaces CudaAllocator, src/cuda_device.cpp:30-51):
 * 256-byte aligned, null on bytes <= 0. */
int nb2_device_malloc(nb2_device* dev, int64_t bytes, void** out);
int nb2_device_free(nb2_device* dev, void* ptr);

/* Copies (replace CudaTransfer, src/cuda_device.cpp:53-72; bytes == 0 is a
 * no-op). h2d returns once `src` may be reused (staged through pinned memory,
 * ordered on the device stream); d2h returns with `dst` filled and reports
 * device-recorded errors. */
int nb2_memcpy_h2d(nb2_device* dev, void* dst, const void* src, int64_t bytes);
int nb2_memcpy_d2h(nb2_device* dev, void* dst, const void* src, int64_t bytes);
int nb2_memcpy_d2d(nb2_device* dev, void* dst, const void* src, int64_t bytes);

/* ---- contraction rows (tcgen05) ------------------------------------------ */

/* Conv row: src/kernels/conv.cpp:138-295 semantics (cross-correlation,
 * groups, strides, dilations, explicit begin/end pads, optional bias [m]),
 * plus an optional fused residual add (same shape as Y) and activation.
 * The weight is split/packed per call into the device workspace. */
int nb2_conv2d(nb2_device* dev, const nb2_conv_geom* g, const float* x, const float* w, const float* bias,
               const float* residual, int act, float* y);
/* Packed-weight form for callers that keep weights resident: pack once,
 * run many times. */
int nb2_conv2d_packed_size(const nb2_conv_geom* g, int64_t* bytes);
int nb2_conv2d_pack(nb2_device* dev, const nb2_conv_geom* g, const float* w, void* packed);
int nb2_conv2d_run_packed(nb2_device* dev, const nb2_conv_geom* g, const float* x, const void* packed,
                          const float* bias, const float* residual, int act, float* y);

/* Gemm row: src/kernels/gemm.cpp:59-137 — Y[m,n] = alpha*op(A)op(B) +
 * beta*C with C absent (c_rank 0), [n] (c_rank 1) or [m,n] (c_rank 2), then
 * an optional activation. A is [m,k] ([k,m] if trans_a), B is [k,n]
 * ([n,k] if trans_b), all row-major and contiguous. */
int nb2_gemm(nb2_device* dev, const float* a, const float* b, const float* c, int c_rank, float* y, int64_t m,
             int64_t n, int64_t k, int trans_a, int trans_b, float alpha, float beta, int act);

/* MatMul row: src/kernels/mat_mul.cpp:79-169 — NumPy matmul with 1-D
 * promotion. Batch dims must match the output's or be all ones/absent. */
int nb2_matmul(nb2_device* dev, const float* a, const int64_t* a_dims, int a_rank, const float* b,
               const int64_t* b_dims, int b_rank, float* y);

/* ---- bandwidth rows ------------------------------------------------------ */

int nb2_unary(nb2_device* dev, int op, const float* x, float* y, int64_t count);
/* y = a (op) b with NumPy broadcasting (src/kernels/add.cpp:96-130); dtype
 * NB2_F32 or NB2_I64 (int64 Div truncates toward zero). */
int nb2_binary(nb2_device* dev, int op, int dtype, const void* a, const int64_t* a_dims, int a_rank, const void* b,
               const int64_t* b_dims, int b_rank, void* y, const int64_t* y_dims, int y_rank);
/* MaxPool 2-D (src/kernels/max_pool.cpp:138-239): x [n,c,h,w] -> y [n,c,oh,ow]. */
int nb2_maxpool2d(nb2_device* dev, const float* x, const int64_t x_dims[4], float* y, const int64_t y_dims[4],
                  const int64_t kernel[2], const int64_t strides[2], const int64_t pads[4], const int64_t dilations[2]);
/* Mean over the trailing `inner` elements of `rows` rows, double accumulation
 * (GlobalAveragePool, src/kernels/global_average_pool.cpp:32-68). */
int nb2_row_mean(nb2_device* dev, const float* x, int64_t rows, int64_t inner, float* y);

#ifdef __cplusplus
}
#endif

#endif /* NERT_B200_H */
