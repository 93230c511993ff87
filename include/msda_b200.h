/*
 * msda_b200 -- C ABI of the B200 (sm_100a) multi-scale deformable attention
 * (MSDA) kernels.
 *
 * The library is the native replacement for the CUDA half of the reference
 * operator roulbac/msda-triton: the Triton kernels in src/msda_triton/kernels.py
 * and the launches in src/msda_triton/ops.py. Every entry point takes plain
 * device pointers, sizes and a cudaStream_t passed as void*; no C++ exception
 * and no framework type crosses this boundary.
 *
 * Tensor layouts (all contiguous, row-major; identical to the reference):
 *   value              (B, S, M, D)          dtype
 *   spatial_shapes     (L, 2)  int64         (H_l, W_l), on the device
 *   level_start_index  (L,)    int64         on the device
 *   sampling_locations (B, Q, M, L, K, 2)    dtype, normalised (x, y)
 *   attention_weights  (B, Q, M, L, K)       dtype
 *   output / grad_out  (B, Q, M, D)          dtype (the host views it as (B, Q, M*D))
 *
 * Ownership: the caller allocates every buffer, including the optional
 * backward workspace; the library never allocates device memory.
 * Threading: apart from a thread-local error string and the static scratch
 * array of msda_backward_noalloc (described there), the library holds no
 * state; every call enqueues its work on the given stream with no host
 * synchronisation.
 * Errors: every entry point returns an msda_status (0 = success); the message
 * of the last failure on the calling thread is available from
 * msda_last_error(). A CUDA launch error is reported as MSDA_ERR_CUDA.
 */
#ifndef MSDA_B200_H_
#define MSDA_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MSDA_API __attribute__((visibility("default")))
#else
#define MSDA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Element type of value / sampling_locations / attention_weights / outputs.
 * Mirrors the dtype set accepted by src/msda_triton/ops.py:17 (_FLOAT_DTYPES). */
typedef enum msda_dtype {
  MSDA_DTYPE_F32 = 0,
  MSDA_DTYPE_F16 = 1,
  MSDA_DTYPE_BF16 = 2
} msda_dtype;

typedef enum msda_status {
  MSDA_OK = 0,
  MSDA_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad size, misaligned buffer */
  MSDA_ERR_UNSUPPORTED = 2,      /* dtype / head dim / level count outside what is built */
  MSDA_ERR_CUDA = 3              /* a CUDA call or kernel launch failed */
} msda_status;

/* Backward flags. */
/* Accumulate grad_value in fp32 and round to the value dtype once (the
 * fp32_grad_accum=True path of src/msda_triton/ops.py:76-92). Without it
 * fp16/bf16 gradients are added with native packed fp16x2/bf16x2 reductions
 * (fp32 inputs always accumulate in fp32). */
#define MSDA_BWD_FP32_ACCUM 1u
/* Force the grad_value algorithm (tests and benchmarks; default: automatic).
 * SCATTER: one pass over sampling points with vector `red.global` adds
 *   (fp32 workspace + downcast when MSDA_BWD_FP32_ACCUM is set for fp16/bf16,
 *   native packed fp16x2/bf16x2 adds otherwise).
 * COUNTED: hit-counted scatter -- a first pass counts the bilinear hits of
 *   the grad_value rows of the sparse levels (levels with fewer than two
 *   corner hits per row on average) and flags the rows of the dense levels;
 *   rows hit once get their single contribution stored, rows hit more often
 *   and flagged rows accumulate in fp32 rows of the workspace; a last pass
 *   writes zeros / rounds the fp32 rows. Same result as fp32 accumulation,
 *   with fp32 traffic only where rows are hit more than once (the automatic
 *   choice for fp32 accumulation when sampling is sparse, Q*L*K <= 2*S).
 * Flag bit 4u is unused; msda_backward rejects flag bits it does not know
 * with MSDA_ERR_INVALID_ARGUMENT. */
#define MSDA_BWD_FORCE_SCATTER 2u
#define MSDA_BWD_FORCE_COUNTED 8u
/* Deterministic grad_value (no counterpart in the reference, which documents
 * its backward as nondeterministic, README.md:179 and ops.py:135-138):
 * contributions a * w_c * g are rounded once to 64-bit fixed point and
 * accumulated with integer reductions, whose sum does not depend on the
 * order the atomics land in, then each element is rounded once to the
 * value dtype (the hit-counted algorithm stores rows hit once and reduces
 * rows hit exactly twice in fp32: two commutative adds into zero are
 * order-independent too). Results are bitwise reproducible from run to run for the same
 * inputs. The fixed-point scale is set on the device from max|attention
 * weight| (1 for the fused prologue's softmax weights) and max|grad_output|
 * so that no row sum can overflow; one contribution's rounding error is below
 * 2^-45 of the largest possible contribution for Q*K <= 2^17 (finer than
 * fp32 accumulation). Inputs with non-finite values fall back to fp32
 * atomics (Inf / NaN propagate as in fp32 accumulation; no determinism
 * claim then). Takes the hit-counted algorithm for sparse sampling
 * (Q*L*K <= 2*S), else the scatter; MSDA_BWD_FORCE_SCATTER / _COUNTED pick
 * one. MSDA_BWD_FP32_ACCUM is implied.
 * fp16 / bf16 values in the hit-counted algorithm need no absmax pass and
 * reduce most rows in 4-byte words: the count pass also records, per
 * grad_value row, a bound on its contributions (max |attention weight| *
 * max |grad_output row| over the points hitting it). A row with 2 to 32
 * hits gets every contribution rounded once to an integer multiple of 2^-F,
 * 2^F chosen from that bound and the hit count so that every partial sum is
 * an integer below 2^24: exact in fp32, hence order-independent, on a grid of
 * at most 2^-19 of the bound; the reductions move the bytes of fp32
 * accumulation. Busier rows take 64-bit integers on a per-row scale from the
 * same bound (a grid of 2^-51 of it).
 * Needs a workspace (msda_backward_workspace_size with this flag). */
#define MSDA_BWD_DETERMINISTIC 16u
/* Sibling gathers only (msda_grid_sample_backward, msda_roi_align_backward;
 * msda_backward rejects it): grad_input is written (N, C, H, W) contiguous
 * instead of (N, H, W, C). The reductions then always go into the NHWC
 * workspace (fp32, 64-bit fixed point, or the data type when neither
 * MSDA_BWD_FP32_ACCUM nor MSDA_BWD_DETERMINISTIC applies), and one pass
 * converts and transposes it into grad_input: the NCHW gradient of an NCHW
 * input without a separate msda_transpose call. The workspace size queries
 * take the same flag. */
#define MSDA_BWD_GRAD_INPUT_NCHW 32u

/* Library version string, e.g. "msda_b200 0.1.0 sm_100a". */
MSDA_API const char* msda_version(void);

/* Message of the last failed call on this thread ("" after a success). */
MSDA_API const char* msda_last_error(void);

/*
 * Forward: output[b,q,m,:] = sum_{l,k} attn[b,q,m,l,k] *
 *                            bilinear(value[b, level l, m, :], loc[b,q,m,l,k,:])
 * Replaces the launch of _msda_forward_kernel in _MSDAFunction.forward
 * (src/msda_triton/ops.py:46-52; kernel src/msda_triton/kernels.py:58-163).
 * B == 0 or Q == 0 is a successful no-op (src/msda_triton/ops.py:186-187).
 */
MSDA_API int msda_forward(const void* value, const int64_t* spatial_shapes, const int64_t* level_start_index,
                 const void* sampling_locations, const void* attention_weights, void* output,
                 int64_t batch, int64_t num_values, int64_t num_queries, int32_t num_heads,
                 int32_t head_dim, int32_t num_levels, int32_t num_points, int32_t dtype,
                 void* stream);

/*
 * Forward with the layer's prologue fused in (no counterpart in the
 * reference op; it replaces the prologue of the reference's Deformable-DETR
 * layer, labs/solutions/lab00.py:199-208, followed by msda_forward): instead
 * of sampling locations and attention weights it takes
 *   reference_points  (B, Q, 2)          normalised (x, y) per query,
 *   sampling_offsets  (B, Q, M, L, K, 2) in pixels of each level,
 *   attention_logits  (B, Q, M, L, K),
 * and samples point (l, k) of head m at reference + offset / (W_l, H_l) with
 * weight softmax over the head's L*K logits -- the same maths as
 * msda_forward on the materialised locations and weights, without writing
 * or reading them. All in `dtype`.
 */
MSDA_API int msda_forward_fused(const void* value, const int64_t* spatial_shapes,
                                const int64_t* level_start_index, const void* reference_points,
                                const void* sampling_offsets, const void* attention_logits,
                                void* output, int64_t batch, int64_t num_values,
                                int64_t num_queries, int32_t num_heads, int32_t head_dim,
                                int32_t num_levels, int32_t num_points, int32_t dtype,
                                void* stream);

/*
 * Backward of msda_forward_fused: grad_value (B,S,M,D), the gradient of the
 * sampling offsets (B,Q,M,L,K,2) and of the attention logits (B,Q,M,L,K)
 * (through the softmax), in `dtype`. The reference points' gradient is the
 * offsets' gradient times (W_l, H_l), summed over (m, l, k); the caller forms
 * it. Workspace and flags as msda_backward (same workspace size).
 */
MSDA_API int msda_backward_fused(const void* value, const int64_t* spatial_shapes,
                                 const int64_t* level_start_index, const void* reference_points,
                                 const void* sampling_offsets, const void* attention_logits,
                                 const void* grad_output, void* grad_value,
                                 void* grad_sampling_offsets, void* grad_attention_logits,
                                 void* workspace, size_t workspace_bytes, int64_t batch,
                                 int64_t num_values, int64_t num_queries, int32_t num_heads,
                                 int32_t head_dim, int32_t num_levels, int32_t num_points,
                                 int32_t dtype, uint32_t flags, void* stream);

/*
 * Bytes of workspace msda_backward needs for these sizes and flags (0 when
 * the chosen algorithm uses none). Replaces the allocation of the fp32
 * grad_value buffer at src/msda_triton/ops.py:76-77.
 */
MSDA_API size_t msda_backward_workspace_size(int64_t batch, int64_t num_values, int64_t num_queries,
                                             int32_t num_heads, int32_t head_dim, int32_t num_levels,
                                             int32_t num_points, int32_t dtype, uint32_t flags);

/*
 * Backward: writes grad_value (B,S,M,D), grad_sampling_locations
 * (B,Q,M,L,K,2) and grad_attention_weights (B,Q,M,L,K), all in `dtype`.
 * grad_value need not be zeroed by the caller: the call initialises it.
 * Replaces _MSDAFunction.backward's zero-fill, kernel launch and downcast
 * (src/msda_triton/ops.py:76-92; kernel src/msda_triton/kernels.py:166-291).
 * grad_value is accumulated with atomics: without MSDA_BWD_DETERMINISTIC
 * results are not bitwise deterministic from run to run (as in the
 * reference, ops.py:135-138).
 */
MSDA_API int msda_backward(const void* value, const int64_t* spatial_shapes, const int64_t* level_start_index,
                  const void* sampling_locations, const void* attention_weights,
                  const void* grad_output, void* grad_value, void* grad_sampling_locations,
                  void* grad_attention_weights, void* workspace, size_t workspace_bytes,
                  int64_t batch, int64_t num_values, int64_t num_queries, int32_t num_heads,
                  int32_t head_dim, int32_t num_levels, int32_t num_points, int32_t dtype,
                  uint32_t flags, void* stream);

/*
 * Backward for callers that cannot allocate device memory (no counterpart in
 * the reference, which always allocates its fp32 buffer with torch).
 *
 * A caller that plans all device memory ahead of time and may not call
 * cudaMalloc while it runs (a TensorRT-style plugin's enqueue, which must
 * not allocate outside its planned buffers; an embedder without a device
 * allocator of its own) cannot hand msda_backward the fp32
 * workspace it needs for fp32 accumulation of fp16/bf16 gradients. This entry
 * point computes the same three gradients as msda_backward with
 * MSDA_BWD_FP32_ACCUM | MSDA_BWD_FORCE_SCATTER, taking that workspace from a
 * static device array of MSDA_NOALLOC_SCRATCH_BYTES inside the library. It
 * calls no cudaMalloc/cudaFree and no allocating library routine; the caller
 * still passes every input and output buffer.
 *
 * Limits and caveats:
 * - B*S*M*D*4 bytes (the fp32 accumulation buffer) must fit in
 *   MSDA_NOALLOC_SCRATCH_BYTES (16 MiB, i.e. 4M grad_value elements) for
 *   fp16/bf16; larger sizes fail with MSDA_ERR_INVALID_ARGUMENT. fp32 inputs
 *   accumulate directly in grad_value and use no scratch.
 * - Every GPU that loads the library holds the 16 MiB array until exit.
 * - The array's device address belongs to a CUDA context: the first call in
 *   each context (the device's primary context, or one the caller created
 *   and made current) looks it up (cudaGetSymbolAddress, with that context
 *   current) and keeps it per context handle; make that first call before
 *   any stream capture, and again after cudaDeviceReset. The stream must
 *   belong to the current device. Sizes are checked as msda_backward checks
 *   them before the scratch limit is.
 * - All calls on a device share the one array (each call zeroes what it
 *   uses): calls that overlap on the GPU -- on different streams, or from
 *   different threads -- race and corrupt each other's gradients. Serialise
 *   them on one stream.
 */
#define MSDA_NOALLOC_SCRATCH_BYTES (16u << 20)
MSDA_API int msda_backward_noalloc(const void* value, const int64_t* spatial_shapes,
                                   const int64_t* level_start_index, const void* sampling_locations,
                                   const void* attention_weights, const void* grad_output,
                                   void* grad_value, void* grad_sampling_locations,
                                   void* grad_attention_weights, int64_t batch, int64_t num_values,
                                   int64_t num_queries, int32_t num_heads, int32_t head_dim,
                                   int32_t num_levels, int32_t num_points, int32_t dtype,
                                   void* stream);

/*
 * Sibling gathers (no counterpart in the reference, which names them as the
 * operators its recipe transfers to, docs/course/08-exercises.md:39): the
 * same channel-vector bilinear gathers and scatters, for grid_sample and
 * ROI-Align. Channels-last (NHWC) layouts, all in `dtype` unless stated:
 *   input        (N, H, W, C)
 *   grid         (N, out_h, out_w, 2)   normalised (x, y) in [-1, 1]
 *   output       (N, out_h, out_w, C)   grid_sample
 *   rois         (num_rois, 5) fp32     (batch index, x1, y1, x2, y2)
 *   output       (num_rois, pooled_height, pooled_width, C)   roi_align
 * Backward flags: MSDA_BWD_FP32_ACCUM (fp32 workspace + downcast for
 * fp16/bf16), MSDA_BWD_DETERMINISTIC (64-bit fixed-point accumulation,
 * bitwise reproducible), MSDA_BWD_GRAD_INPUT_NCHW (grad_input written
 * (N, C, H, W)); the workspace size depends on them.
 * grad_input need not be zeroed by the caller.
 */

/* Layout conversion for the NHWC kernels: dst[n][c][r] = src[n][r][c] for
 * (N, R, C) -> (N, C, R) -- NCHW -> NHWC with (R, C) = (C, H*W), and back
 * with (R, C) = (H*W, C). */
MSDA_API int msda_transpose(const void* src, void* dst, int64_t N, int64_t R, int64_t C, int32_t dtype,
                            void* stream);

/* torch.nn.functional.grid_sample(input, grid, mode, padding_mode,
 * align_corners) on NHWC data; mode 0 = "bilinear", 1 = "nearest"
 * ("bicubic" is not supported: MSDA_ERR_UNSUPPORTED); padding_mode
 * 0 = "zeros", 1 = "border", 2 = "reflection". */
MSDA_API int msda_grid_sample_forward(const void* input, const void* grid, void* output, int64_t N,
                                      int64_t H, int64_t W, int64_t C, int64_t out_h, int64_t out_w,
                                      int32_t mode, int32_t padding_mode, int32_t align_corners,
                                      int32_t dtype, void* stream);
MSDA_API size_t msda_grid_sample_backward_workspace_size(int64_t N, int64_t H, int64_t W, int64_t C,
                                                         int64_t out_h, int64_t out_w, int32_t dtype,
                                                         uint32_t flags);
/* grad_input (N, H, W, C), or (N, C, H, W) with MSDA_BWD_GRAD_INPUT_NCHW,
 * and grad_grid (N, out_h, out_w, 2). */
MSDA_API int msda_grid_sample_backward(const void* input, const void* grid, const void* grad_output,
                                       void* grad_input, void* grad_grid, void* workspace,
                                       size_t workspace_bytes, int64_t N, int64_t H, int64_t W,
                                       int64_t C, int64_t out_h, int64_t out_w, int32_t mode,
                                       int32_t padding_mode, int32_t align_corners, int32_t dtype,
                                       uint32_t flags, void* stream);

/* torchvision.ops.roi_align(input, rois, (pooled_height, pooled_width),
 * spatial_scale, sampling_ratio, aligned) on NHWC data. An ROI whose batch
 * index is outside [0, N) yields zeros. sampling_ratio > 1024 fails with
 * MSDA_ERR_UNSUPPORTED; with sampling_ratio <= 0 (adaptive: ceil(bin size)
 * samples per side, as torchvision) a bin walks at most 1024 samples per
 * side, so boxes whose bins span more than 1024 pixels (or non-finite boxes)
 * are sampled more coarsely than torchvision would. */
MSDA_API int msda_roi_align_forward(const void* input, const float* rois, void* output, int64_t N,
                                    int64_t H, int64_t W, int64_t C, int64_t num_rois,
                                    int32_t pooled_height, int32_t pooled_width, float spatial_scale,
                                    int32_t sampling_ratio, int32_t aligned, int32_t dtype,
                                    void* stream);
MSDA_API size_t msda_roi_align_backward_workspace_size(int64_t N, int64_t H, int64_t W, int64_t C,
                                                       int32_t dtype, uint32_t flags);
/* grad_input (N, H, W, C), or (N, C, H, W) with MSDA_BWD_GRAD_INPUT_NCHW;
 * the boxes get no gradient (as in torchvision). */
MSDA_API int msda_roi_align_backward(const float* rois, const void* grad_output, void* grad_input,
                                     void* workspace, size_t workspace_bytes, int64_t N, int64_t H,
                                     int64_t W, int64_t C, int64_t num_rois, int32_t pooled_height,
                                     int32_t pooled_width, float spatial_scale, int32_t sampling_ratio,
                                     int32_t aligned, int32_t dtype, uint32_t flags, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MSDA_B200_H_ */
