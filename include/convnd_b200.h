/*
 * convnd_b200.h — C ABI of the B200 (sm_100a) N-dimensional dense convolution library.
 *
 * The library replaces the reference's native CUDA backend of torch-convnd 0.5.0
 * (src/torch_convnd/csrc/convnd.cpp, convnd_cuda.cu, convnd_mixed.cpp). The reference
 * exposes the path only as two PyTorch dispatcher operators,
 *
 *   torch_convnd::conv_nd(Tensor input, Tensor weight, Tensor? bias, int[] stride,
 *                         int[] padding, int[] dilation, int groups, int workspace_bytes)
 *   torch_convnd::conv_nd_backward(Tensor grad_output, Tensor input, Tensor weight,
 *                         int[] stride, int[] padding, int[] dilation, int groups,
 *                         int workspace_bytes, bool[3] output_mask)
 *
 * (schemas: src/torch_convnd/_operators.py:47-56; C++ kernels: convnd.cpp:305-415).
 * This header carries the same contract through plain pointers and sizes, so that any
 * host (the bundled PyTorch shim, ctypes, cgo, JNI) can drive the kernels. No torch types
 * appear here. All tensors are dense and in device memory; activations are channels-first
 * ([N, C, d0, d1, ...]), exactly as the reference's operators see them after
 * `.contiguous()`, unless cnd_problem.layout marks them channels-last.
 *
 * Error convention: every entry point returns CND_OK (0) or a negative status; the
 * message of the last failure on the calling thread is returned by cnd_last_error().
 * Validation failures use the reference's own TORCH_CHECK texts (convnd.cpp:19-100).
 */
#ifndef CONVND_B200_H
#define CONVND_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(_WIN32)
#define CND_API __declspec(dllexport)
#else
#define CND_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* PyTorch tensors have at most 64 dimensions: batch, channels and 62 spatial axes
 * (reference: csrc/convnd.h:10-11, kMaxSpatialDims). */
#define CND_MAX_RANK 62

/* Status codes. */
#define CND_OK 0
#define CND_ERR_INVALID (-1)     /* bad geometry / arguments (reference TORCH_CHECK texts) */
#define CND_ERR_UNSUPPORTED (-2) /* dtype or layout that the library does not implement  */
#define CND_ERR_CUDA (-3)        /* a CUDA runtime/driver call failed                     */
#define CND_ERR_WORKSPACE (-4)   /* caller-provided workspace is smaller than required    */
#define CND_ERR_TIMEOUT (-5)     /* a bounded in-kernel wait expired (see cnd_device_status) */

/* Element types (the reference accepts float16, bfloat16, float32, float64:
 * convnd.cpp:40-42). */
typedef enum cnd_dtype {
  CND_F16 = 0,
  CND_BF16 = 1,
  CND_F32 = 2,
  CND_F64 = 3
} cnd_dtype;

/* How float32 problems use the tensor cores.
 *   CND_FP32_3XTF32: error-compensated split products (default): each fp32 operand is
 *                    split into a TF32 "big" part and a TF32 remainder and three
 *                    kind::tf32 MMAs form each product; input-gradient passes over 16
 *                    or more gradient channels, and every weight gradient, split into
 *                    bfloat16 hi + lo parts instead (three kind::f16 MMAs, ~16
 *                    significant bits per operand, inside fp32's rtol 1e-3 bar).
 *   CND_FP32_TF32:   one kind::tf32 MMA per forward / input-gradient product (what
 *                    cuBLAS does under allow_tf32=True in the reference's bmm calls,
 *                    convnd.cpp:334); weight gradients as above.
 *   CND_FP32_SIMT:   exact fp32 CUDA-core path (no tensor cores). */
typedef enum cnd_fp32_mode {
  CND_FP32_3XTF32 = 0,
  CND_FP32_TF32 = 1,
  CND_FP32_SIMT = 2
} cnd_fp32_mode;

/* Memory layouts of the activation tensors (cnd_problem.layout, a bit set). By default
 * every activation is dense channels-first [N, C, d0, d1, ...] (what the reference's
 * operators see after `.contiguous()`). A set bit makes that tensor dense channels-last,
 * [N, d0, d1, ..., C] in memory (PyTorch's channels_last strides of the same logical
 * shape), which the tensor-core passes read without a layout pass when its channel rows
 * already have the kernels' width (16-bit, 16/32/64 or a multiple of 64 channels, one
 * group or thin groups run dense) and write directly:
 *   CND_LAYOUT_X_CL: x (forward, backward) and dx (backward);
 *   CND_LAYOUT_Y_CL: y (forward) and dy (backward).
 * Weights, biases and their gradients have no layout choice. */
#define CND_LAYOUT_X_CL 1
#define CND_LAYOUT_Y_CL 2

/* Activation fused into the epilogue (also carried in cnd_problem.layout, bits 8-15, so
 * that the workspace size functions see it). CND_ACT_GELU is PyTorch's exact GELU,
 * 0.5 * v * (1 + erf(v / sqrt(2))). Used by cnd_forward_act / cnd_backward_act only. */
#define CND_ACT_NONE 0
#define CND_ACT_GELU 1
#define CND_LAYOUT_ACT_SHIFT 8

/* Convolution problem. Mirrors the reference's `Geometry` record (csrc/convnd.h:13-27)
 * plus batch size, dtype and activation layouts. Filled and validated by
 * cnd_problem_init (which sets layout to 0, channels-first). */
typedef struct cnd_problem {
  int32_t rank;           /* spatial rank, 1..62 */
  int32_t dtype;          /* cnd_dtype */
  int32_t fp32_mode;      /* cnd_fp32_mode, only read for CND_F32 */
  int32_t layout;         /* CND_LAYOUT_* bits; 0 = every activation channels-first */
  int64_t batch;
  int64_t channels;        /* input channels (all groups) */
  int64_t output_channels; /* output channels (all groups) */
  int64_t groups;
  int64_t input_volume;
  int64_t output_volume;
  int64_t kernel_volume;
  int64_t input[CND_MAX_RANK];
  int64_t output[CND_MAX_RANK];
  int64_t kernel[CND_MAX_RANK];
  int64_t stride[CND_MAX_RANK];
  int64_t padding[CND_MAX_RANK];
  int64_t dilation[CND_MAX_RANK];
} cnd_problem;

/* Validate a geometry and derive output extents and volumes.
 * Replaces make_geometry (reference csrc/convnd.cpp:33-87): same checks, same order, same
 * messages ("groups must be positive", "kernel exceeds padded input", "... overflows
 * int64", ...). `input_shape` is [N, C, d0..], `weight_shape` is [Cout, C/groups, k0..];
 * both have rank+2 entries. */
CND_API int cnd_problem_init(cnd_problem* problem, int32_t rank, const int64_t* input_shape,
                     const int64_t* weight_shape, const int64_t* stride,
                     const int64_t* padding, const int64_t* dilation, int64_t groups,
                     int32_t dtype);

/* The reference's patch-budget rule (tile_size, csrc/convnd.cpp:89-100): fails with
 * "workspace_bytes is too small for one output position; requires at least <n>" when the
 * budget cannot hold one output position's patch column. The B200 kernels never
 * materialise patches, so the budget is only validated to keep the operator contract. */
CND_API int cnd_check_workspace_budget(const cnd_problem* problem, int64_t element_size,
                               int64_t workspace_bytes);

/* Device scratch bytes that cnd_forward / cnd_backward need for `problem`
 * (channels-last operand copies, packed weights, split-K partials). */
CND_API size_t cnd_forward_workspace_size(const cnd_problem* problem);
CND_API size_t cnd_backward_workspace_size(const cnd_problem* problem, const int32_t output_mask[3]);

/* Forward: y = conv(x, w) + b. Replaces torch_convnd::conv_nd's CUDA kernel
 * (reference csrc/convnd.cpp:305-343). x: [N, C, in...], w: [Cout, C/g, k...],
 * b: [Cout] or NULL, y: [N, Cout, out...]; all of `problem->dtype`, contiguous.
 * `stream` is a cudaStream_t (NULL = legacy default stream). */
CND_API int cnd_forward(const cnd_problem* problem, const void* x, const void* w, const void* b,
                void* y, void* workspace, size_t workspace_bytes, void* stream);

/* Capacity of the static device scratch that cnd_forward_noalloc uses (bytes). */
#define CND_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)

/* Forward without any device allocation by the caller or the library.
 * For callers that cannot allocate device memory: hosts that drive this C ABI through
 * thin bindings that hold no device allocator of their own (cgo, JNI, N-API or ctypes
 * code that only has the input/output pointers it was handed), and processes whose
 * device memory belongs to another allocator with a fixed budget (a serving process
 * where a PyTorch caching allocator or a pre-sized pool owns the GPU), for which an extra
 * workspace allocation would fail or fragment the pool.
 * This variant has no counterpart in the reference. It computes exactly what
 * cnd_forward computes, using as workspace a file-scope device array of
 * CND_NOALLOC_SCRATCH_BYTES that every GPU which loads this library keeps until process
 * exit. Problems whose workspace (cnd_forward_workspace_size) exceeds that size are
 * rejected with CND_ERR_WORKSPACE and a message naming both sizes. The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress) with that device
 * current, so make that first call before any stream capture. All calls share the one
 * array and it keeps the last call's contents (every byte a call reads is written by
 * the same call first); calls that overlap on the GPU, e.g. on two streams at once,
 * race on it. */
CND_API int cnd_forward_noalloc(const cnd_problem* problem, const void* x, const void* w,
                                const void* b, void* y, void* stream);

/* Backward: fills the gradients selected by output_mask = {dx, dw, db}.
 * Replaces torch_convnd::conv_nd_backward's CUDA kernel (reference
 * csrc/convnd.cpp:345-415 for fp32/fp64 and csrc/convnd_mixed.cpp:11-59 for fp16/bf16).
 * dx has x's shape, dw has w's shape, db has Cout entries, all of `problem->dtype`.
 * Low-precision gradients accumulate in fp32 and are rounded once, as the reference's
 * mixed backward does. Pointers whose mask entry is 0 may be NULL. */
CND_API int cnd_backward(const cnd_problem* problem, const void* dy, const void* x, const void* w,
                 void* dx, void* dw, void* db, const int32_t output_mask[3],
                 void* workspace, size_t workspace_bytes, void* stream);

/* Convolution with a fused activation (no counterpart in the reference, whose callers
 * run the activation as a separate pass: the c5 training step's GELU between layers).
 * cnd_forward_act writes y = act(conv(x, w) + b) and, when `pre` is not NULL, the
 * pre-activation conv(x, w) + b to `pre` (same shape and layout as y), both from the fp32
 * accumulators of one epilogue. cnd_backward_act takes the gradient of y, multiplies it
 * by act'(pre) while packing it (the activation's backward, in fp32, rounded once to the
 * problem's dtype as an eager activation backward would), and runs the convolution's
 * backward on that product: dx, dw and db of conv + activation. `activation` is a
 * CND_ACT_* value; set it in problem->layout (activation << CND_LAYOUT_ACT_SHIFT) too
 * before asking for workspace sizes. */
CND_API int cnd_forward_act(const cnd_problem* problem, const void* x, const void* w,
                            const void* b, void* y, void* pre, int32_t activation,
                            void* workspace, size_t workspace_bytes, void* stream);
CND_API int cnd_backward_act(const cnd_problem* problem, const void* dy, const void* pre,
                             int32_t activation, const void* x, const void* w, void* dx,
                             void* dw, void* db, const int32_t output_mask[3],
                             void* workspace, size_t workspace_bytes, void* stream);

/* Which kernel family cnd_forward / cnd_backward would use for `problem`:
 * bit 0 = forward on tcgen05, bit 1 = dgrad on tcgen05, bit 2 = wgrad on tcgen05.
 * A clear bit means the generic CUDA-core kernels run that pass. */
CND_API int cnd_fast_path_mask(const cnd_problem* problem);

/* Writes a one-line-per-pass text description of how the library would run `problem`
 * (kernel family, tile shape, halo and pipeline choices) into `buffer` (NUL-terminated,
 * truncated to `size`). Returns the number of characters the full text needs. */
CND_API int cnd_plan_summary(const cnd_problem* problem, char* buffer, size_t size);

/* Reads and clears the library's device error word (set by a bounded wait that expired
 * inside a kernel). Returns CND_OK, or CND_ERR_TIMEOUT with the failing site in the
 * message. Synchronises `stream`. */
CND_API int cnd_device_status(void* stream);

/* Number of kernels the library launched (all threads) since the last reset. */
CND_API int64_t cnd_launch_count(int32_t reset);

/* Process-wide default for how float32 problems use the tensor cores (cnd_fp32_mode);
 * cnd_problem_init copies it into each problem. Returns the previous value. */
CND_API int cnd_set_default_fp32_mode(int32_t mode);

/* Test support for the bounded-wait failure path: launches one small forward kernel
 * whose producer never issues a load, so the MMA thread's wait expires after
 * `timeout_ms`; the kernel then returns normally with the device error word set.
 * Returns CND_ERR_TIMEOUT when that path works (no fault, no hang), another status
 * otherwise. Allocates and frees its own small buffers. */
CND_API int cnd_debug_stall_test(int32_t timeout_ms, void* stream);

/* Benchmark support. While enabled, every pass the library launches is bracketed by a
 * pair of CUDA events recorded on its launching stream. cnd_collect_kernel_timings
 * synchronises those events, writes up to `capacity` (kind, milliseconds) records and
 * clears the list; it returns the number written. Kinds: 1 forward pass (tcgen05),
 * 2 dgrad pass (tcgen05), 3 wgrad pass (tcgen05), 4 activation pack, 5 weight pack,
 * 6 reductions, 7 generic CUDA-core kernel. */
CND_API int cnd_set_kernel_timing(int32_t enable);
CND_API int cnd_collect_kernel_timings(int32_t* kinds, float* milliseconds, int32_t capacity);

/* Message of the last failure on the calling thread ("" if none). */
CND_API const char* cnd_last_error(void);

/* Library version string. */
CND_API const char* cnd_version(void);

#ifdef __cplusplus
}
#endif

#endif /* CONVND_B200_H */
