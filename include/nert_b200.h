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
/* Bound, in SM clock ticks, after which a tensor-core kernel's pipeline wait
 * gives up, records a device error (NB2_ERR_DEVICE, "bounded wait expired",
 * at the next synchronisation) and unwinds instead of hanging; cycles <= 0
 * restores the default (about one second). No counterpart in the reference,
 * whose CUDA rows synchronise after every launch (src/cuda/relu.cu:68). */
int nb2_device_set_wait_bound(nb2_device* dev, int64_t cycles);
int64_t nb2_device_get_wait_bound(const nb2_device* dev);
/* Schedule the host chose for the most recent Conv/Gemm/MatMul launch on this
 * device: output tile width (64 or 128), whether two tiles were kept in flight
 * (MMA issuers on alternate tiles), the number of K slices (1 = unsplit; 0 =
 * the balanced split, every CTA an equal span of all (tile, K block) pairs),
 * the A-operand mode and the number of output tiles. Any pointer may be null.
 * Diagnostics for tests and tuning; the reference has no counterpart (cuDNN
 * and cuBLAS pick their algorithms internally, src/cuda/conv.cu:230-530). */
int nb2_device_last_contraction(const nb2_device* dev, int* tile_n, int* two_in_flight, int* k_slices, int* a_mode,
                                int64_t* tiles);

/* 1 when kernels can read `ptr` directly (device, managed or pinned host
 * memory), 0 for ordinary pageable host memory or null. The nert::Device rows
 * use it to stage host views (the reference's FoldConstants hands every
 * device's rows host initializer bytes, src/constant_folding.cpp:32-95). No
 * counterpart in the reference. */
int nb2_pointer_on_device(const void* ptr);

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

/* ConvTranspose geometry, NCHW: x [n,c,h,w], w [c, m/group, kh, kw],
 * y [n,m,oh,ow] with oh = stride_h*(h-1) + out_pad_h + dil_h*(kh-1) + 1 -
 * pad_top - pad_bottom (and the same for the width). */
typedef struct nb2_convt_geom {
    int64_t n, c, h, w;
    int64_t m, kh, kw;
    int64_t oh, ow;
    int64_t stride_h, stride_w;
    int64_t pad_top, pad_left, pad_bottom, pad_right;
    int64_t dil_h, dil_w;
    int64_t out_pad_h, out_pad_w;
    int64_t group;
} nb2_convt_geom;

/* ConvTranspose row: src/kernels/conv_transpose.cpp (explicit pads,
 * output_padding, dilations, groups, optional bias [m]), computed as a
 * stride-1 Conv on the tensor cores over the input with stride-1 zeros
 * inserted, with the weight transposed per group and flipped. Pads above
 * dil*(k-1) are NB2_ERR_UNSUPPORTED. Scratch comes from the device workspace. */
int nb2_conv_transpose2d(nb2_device* dev, const nb2_convt_geom* g, const float* x, const float* w, const float* bias,
                         float* y);

/* Conv for callers that cannot allocate device memory (no counterpart in the
 * reference). Same semantics and validation as nb2_conv2d, but the weight is
 * packed into a fixed 8 MiB static device array (per GPU, held until exit)
 * instead of the growable workspace, so the call performs no cudaMalloc,
 * cudaFree or other allocation: for a plug-in inside a host framework that
 * owns all device memory, or a service on a fixed memory budget. It never splits K (the
 * split-K buffer is shared and growable), so it launches one contraction
 * kernel whatever the layer. Weights whose packed form exceeds
 * nb2_conv2d_noalloc_capacity() bytes are rejected (NB2_ERR_INVALID).
 * The first call on a device resolves the array's device address, so make it
 * before any stream capture. All calls share the array and leave their data
 * in it; calls whose kernels overlap on one GPU would race on it. */
int nb2_conv2d_noalloc(nb2_device* dev, const nb2_conv_geom* g, const float* x, const float* w, const float* bias,
                       const float* residual, int act, float* y);
int64_t nb2_conv2d_noalloc_capacity(void);

/* Gemm row: src/kernels/gemm.cpp:59-137 — Y[m,n] = alpha*op(A)op(B) +
 * beta*C with C absent (c_rank 0), [n] (c_rank 1) or [m,n] (c_rank 2), then
 * an optional activation. A is [m,k] ([k,m] if trans_a), B is [k,n]
 * ([n,k] if trans_b), all row-major and contiguous. */
int nb2_gemm(nb2_device* dev, const float* a, const float* b, const float* c, int c_rank, float* y, int64_t m,
             int64_t n, int64_t k, int trans_a, int trans_b, float alpha, float beta, int act);

/* Packed-B form of the Gemm row for callers that keep B resident (a weight):
 * pack op(B) ([k,n], or [n,k] stored when trans_b) once into
 * nb2_gemm_packed_size bytes of device memory, then run many times with the
 * same semantics as nb2_gemm. A MatMul with a rank-2 B is the same
 * contraction with m = the product of A's leading dimensions. */
int nb2_gemm_packed_size(int64_t n, int64_t k, int64_t* bytes);
int nb2_gemm_pack(nb2_device* dev, const float* b, int64_t n, int64_t k, int trans_b, void* packed);
int nb2_gemm_run_packed(nb2_device* dev, const float* a, const void* packed_b, const float* c, int c_rank, float* y,
                        int64_t m, int64_t n, int64_t k, int trans_a, float alpha, float beta, int act);

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
/* Fused attention, the chain MatMul(Q, K^T) -> Div/Mul by a scalar ->
 * Softmax(axis -1) -> MatMul(., V) (src/kernels/mat_mul.cpp:79-169,
 * div.cpp, softmax.cpp:47-120) in one launch, one CTA per (batch, head), on
 * the tcgen05 tensor cores with the 3xTF32 split. Element (token t, dim j)
 * of head (b, h) is at b*s[0] + h*s[1] + t*s[2] + j*s[3] of q, k and v (so a
 * K^T operand [.., d, T] has s[2] = 1, s[3] = T); output row (b, h, t) at
 * b*o[0] + h*o[1] + t*o[2], its head_dim values contiguous (o = {T*H*D, D,
 * H*D} writes the merged [B, T, H*D] layout). scale_mode 0: no scale, 1:
 * multiply by `scale`, 2: divide by `scale`. head_dim 64, 1 <= tokens <= 208. */
int nb2_attention(nb2_device* dev, const float* q, const float* k, const float* v, float* out, int64_t batch,
                  int64_t heads, int64_t tokens, int64_t head_dim, const int64_t q_strides[4],
                  const int64_t k_strides[4], const int64_t v_strides[4], const int64_t out_strides[3],
                  int scale_mode, float scale);
/* SPPF, the YOLO spatial-pyramid block as one pass: y [n,(chain+1)*c,h,w] =
 * Concat over channels of [x, m1, ..., m_chain], m_l the k x k stride-1
 * pad-k/2 MaxPool of m_{l-1} (m0 = x) with the reference's MaxPool semantics
 * (src/kernels/max_pool.cpp:207-235) and Concat layout (src/kernels/concat.cpp).
 * Replaces `chain` MaxPool rows and one Concat row; k odd, h*w <= 6144. */
int nb2_sppf(nb2_device* dev, const float* x, const int64_t x_dims[4], float* y, int64_t k, int64_t chain);
/* AveragePool 2-D (src/kernels/average_pool.cpp:128-225): x [n,c,h,w] ->
 * y [n,c,oh,ow], explicit pads {top, left, bottom, right}; the divisor counts
 * the padded window when count_include_pad, else the in-range taps. */
int nb2_avgpool2d(nb2_device* dev, const float* x, const int64_t x_dims[4], float* y, const int64_t y_dims[4],
                  const int64_t kernel[2], const int64_t strides[2], const int64_t pads[4], int count_include_pad);
/* Mean over the trailing `inner` elements of `rows` rows, double accumulation
 * (GlobalAveragePool, src/kernels/global_average_pool.cpp:32-68). */
int nb2_row_mean(nb2_device* dev, const float* x, int64_t rows, int64_t inner, float* y);
/* Softmax over the middle axis of an [outer, len, inner] view
 * (src/kernels/softmax.cpp:47-120). */
int nb2_softmax(nb2_device* dev, const float* x, float* y, int64_t outer, int64_t len, int64_t inner);
/* LayerNormalization over rows of length d (src/kernels/layer_normalization.cpp:77-160);
 * bias, mean and inv_std may be null. */
int nb2_layernorm(nb2_device* dev, const float* x, const float* scale, const float* bias, float* y, float* mean,
                  float* inv_std, int64_t rows, int64_t d, float epsilon);
/* Transpose (src/kernels/transpose.cpp:54): y = permute(x, perm); elem_bytes 1, 4 or 8. */
int nb2_transpose(nb2_device* dev, const void* x, void* y, const int64_t* dims, const int64_t* perm, int rank,
                  int elem_bytes);
/* Concat / Split (src/kernels/concat.cpp:64, split.cpp:65) as one launch:
 * `parts` blocks of parts_len[i]*inner elements per outer row. concat=1
 * gathers parts[] into whole, concat=0 scatters whole into parts[]. */
int nb2_concat_split(nb2_device* dev, int concat, void* whole, void* const* parts, const int64_t* parts_len,
                     int n_parts, int64_t outer, int64_t inner, int elem_bytes);
/* Slice (src/kernels/slice.cpp) with resolved per-axis starts and steps. */
int nb2_slice(nb2_device* dev, const void* x, void* y, const int64_t* in_dims, const int64_t* out_dims,
              const int64_t* starts, const int64_t* steps, int rank, int elem_bytes);
/* Gather (src/kernels/gather.cpp:49-129) on an [outer, axis_len, inner] view
 * with int64 indices; out-of-range indices surface as NB2_ERR_DEVICE at the
 * next synchronisation (no device trap). */
int nb2_gather(nb2_device* dev, const void* x, const int64_t* indices, void* y, int64_t outer, int64_t axis_len,
               int64_t inner, int64_t n_indices, int elem_bytes);
/* TopK largest/sorted along the last axis of [rows, len] (src/kernels/top_k.cpp:53-142):
 * values and int64 indices ordered by (value desc, index asc); any k <= len. */
int nb2_topk(nb2_device* dev, const float* x, float* values, int64_t* indices, int64_t rows, int64_t len, int64_t k);
/* Resize nearest/linear (src/kernels/resize.cpp:162-): mode 0 nearest, 1 linear;
 * transform 0 half_pixel, 1 pytorch_half_pixel, 2 align_corners, 3 asymmetric;
 * nearest_mode 0 round_prefer_floor, 1 round_prefer_ceil, 2 floor, 3 ceil.
 * `scales` are the per-axis factors of the coordinate transform. */
int nb2_resize(nb2_device* dev, const void* x, void* y, const int64_t* in_dims, const int64_t* out_dims,
               const double* scales, int rank, int mode, int transform, int nearest_mode, int dtype);
/* Cast between NB2_F32 / NB2_I64 / NB2_BOOL (float -> int64 truncates). */
int nb2_cast(nb2_device* dev, const void* x, int from_dtype, void* y, int to_dtype, int64_t count);

/* ---- engine: whole graphs ------------------------------------------------ */

/* One ONNX graph bound to one GPU and one concrete input shape: the B200
 * counterpart of nert::Model (include/nert/executor.hpp:57-122,
 * src/executor.cpp:202-560). Construction parses the ONNX bytes, infers
 * shapes, fuses Conv/Gemm/MatMul epilogues (Relu, residual Add, SiLU, bias),
 * plans one arena, uploads weights once (Conv/Gemm weights pre-split for the
 * tensor cores) and allocates every device buffer; a run allocates nothing.
 * Errors: NB2_ERR_INVALID for a graph the engine cannot run (unknown op,
 * unsupported form), NB2_ERR_DEVICE for a device-recorded run-time error. */
typedef struct nb2_model nb2_model;

#define NB2_MODEL_NO_FUSION 1 /* run every node as its own row */
#define NB2_MODEL_NO_GRAPH 2  /* launch rows one by one instead of a CUDA-graph replay */
/* Keep every activation NCHW. By default a Conv trunk whose tensors only meet
 * Conv (group 1, C % 4 == 0 inputs), MaxPool, GlobalAveragePool, Concat,
 * Split, 4-D Resize and layout-free elementwise rows is kept channels-last
 * (NHWC) inside the arena; graph inputs and outputs are NCHW either way. */
#define NB2_MODEL_NCHW_ONLY 4
/* Run attention chains (MatMul Q K^T, scale, Softmax, MatMul with V) as
 * separate rows instead of the fused attention step. */
#define NB2_MODEL_NO_ATTENTION 8

int nb2_model_create(const void* onnx, int64_t size, int n_inputs, const char* const* input_names,
                     const int64_t* dims_flat, const int* ranks, int ordinal, int flags, nb2_model** out);
int nb2_model_destroy(nb2_model* m);
int nb2_model_num_io(const nb2_model* m, int* n_inputs, int* n_outputs);
/* name / dtype (NB2_F32, NB2_I64, NB2_BOOL) / dims (up to 8) / device buffer
 * of input or output i. */
int nb2_model_io(const nb2_model* m, int is_output, int i, const char** name, int* dtype, int* rank, int64_t* dims8,
                 void** device_ptr);
/* End to end (Model::Run): copy every input from host memory (pinned memory
 * from nb2_host_alloc makes the copies asynchronous), run, copy every output
 * back, synchronise. Inputs/outputs in declaration order. */
int nb2_model_run(nb2_model* m, const void* const* host_inputs, void* const* host_outputs);
/* nb2_model_run without the final synchronise (host buffers must stay valid
 * until nb2_model_synchronize returns). */
int nb2_model_run_async(nb2_model* m, const void* const* host_inputs, void* const* host_outputs);
/* Device-resident run: the inputs are already in the model's input buffers
 * (nb2_model_io); returns once the work is queued. */
int nb2_model_launch(nb2_model* m);
int nb2_model_synchronize(nb2_model* m);
int nb2_model_stats(const nb2_model* m, int64_t* kernels_per_run, int64_t* arena_bytes, int64_t* weight_bytes,
                    int64_t* fused_groups, int64_t* exec_nodes);
/* One eager pass with a CUDA event between rows: per-row labels
 * (label_len bytes each) and milliseconds; *count = number of rows. */
int nb2_model_profile(nb2_model* m, int max_steps, char* labels, int label_len, float* ms, int* count);
int nb2_model_stream(const nb2_model* m, void** stream);

/* ---- batch sharding over several GPUs ----------------------------------- */

/* Contiguous slices of `batch` images over `n_shards` GPUs: shard i takes
 * counts[i] images starting at offsets[i]; the first batch % n_shards shards
 * take one image more. Host only. */
int nb2_shard_plan(int64_t batch, int n_shards, int64_t* offsets, int64_t* counts);

/* One graph run batch-sharded over several GPUs: a plan per GPU for its slice
 * of the batch (every input leads with the same batch dimension; the graph
 * must be valid at each slice's batch and every output must lead with the
 * batch dimension), one host thread and stream per shard, the slices copied
 * from and into the caller's host buffers at offset first-image x bytes per
 * image. `ordinals[i]` is the GPU of shard i; shards may share a GPU (then
 * CUDA-graph replay is required). No data crosses between GPUs: every op on
 * the path is per image once BatchNormalization is folded. The reference
 * binds one Model to one process-wide device (src/cuda_device.cpp:98-102,
 * src/executor.cpp:202-225); this has no counterpart there. */
typedef struct nb2_sharded nb2_sharded;
int nb2_sharded_create(const void* onnx, int64_t size, int n_inputs, const char* const* input_names,
                       const int64_t* dims_flat, const int* ranks, const int* ordinals, int n_shards, int flags,
                       nb2_sharded** out);
int nb2_sharded_destroy(nb2_sharded* s);
int nb2_sharded_num_io(const nb2_sharded* s, int* n_inputs, int* n_outputs);
/* name / dtype / global dims (up to 8) of input or output i */
int nb2_sharded_io(const nb2_sharded* s, int is_output, int i, const char** name, int* dtype, int* rank,
                   int64_t* dims8);
int nb2_sharded_shard(const nb2_sharded* s, int i, int* ordinal, int64_t* batch_offset, int64_t* batch_count);
/* Scatter, run every shard concurrently, gather; returns when all are done. */
int nb2_sharded_run(nb2_sharded* s, const void* const* host_inputs, void* const* host_outputs);

/* Host-only planning (no GPU needed): shapes, fused row list and arena plan
 * of a graph as JSON; *needed is the byte size including the terminator. */
int nb2_graph_analyze(const void* onnx, int64_t size, int n_inputs, const char* const* input_names,
                      const int64_t* dims_flat, const int* ranks, int flags, char* buf, int64_t cap, int64_t* needed);

/* Pinned host memory for inputs/outputs that cross PCIe every run. */
int nb2_host_alloc(int64_t bytes, void** out);
int nb2_host_free(void* p);

#ifdef __cplusplus
}
#endif

#endif /* NERT_B200_H */
