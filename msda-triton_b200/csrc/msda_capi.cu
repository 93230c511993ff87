// C ABI entry points (declared in include/msda_b200.h): argument checks,
// kernel-shape selection, zero-fill / downcast orchestration.
#include <cstdarg>
#include <cstdio>
#include <string>

#include "msda_b200.h"
#include "msda_abi.cuh"
#include "msda_launch.cuh"

namespace {

using namespace msda::abi;

thread_local std::string g_last_error;

// Largest pixel-index range the kernels address with 32-bit level arithmetic.
constexpr int64_t kMaxS = int64_t(1) << 30;

struct Shape {
  int64_t B, S, Q;
  int32_t M, D, L, K;
};

int check_shape(const Shape& s, int32_t dtype) {
  if (elem_size(dtype) == 0) return fail(MSDA_ERR_UNSUPPORTED, "unsupported dtype code %d (0=f32, 1=f16, 2=bf16)", dtype);
  if (s.B < 0 || s.Q < 0) return fail(MSDA_ERR_INVALID_ARGUMENT, "batch (%lld) and num_queries (%lld) must be >= 0", (long long)s.B, (long long)s.Q);
  if (s.S < 1 || s.S > kMaxS) return fail(MSDA_ERR_INVALID_ARGUMENT, "num_values S=%lld must be in [1, 2^30]", (long long)s.S);
  if (s.M < 1 || s.D < 1 || s.K < 1) return fail(MSDA_ERR_INVALID_ARGUMENT, "num_heads (%d), head_dim (%d) and num_points (%d) must be >= 1", s.M, s.D, s.K);
  if (s.L < 1 || s.L > msda::kMaxLevels) return fail(MSDA_ERR_UNSUPPORTED, "num_levels=%d outside [1, %d]", s.L, msda::kMaxLevels);
  if ((int64_t)s.L * s.K > 4096) return fail(MSDA_ERR_UNSUPPORTED, "num_levels*num_points=%lld exceeds 4096", (long long)s.L * s.K);
  // The kernels address a (batch item, head) slice of value / grad_value with
  // 32-bit offsets: S*M*D elements per batch item must stay below 2^31.
  if (s.S * (int64_t)s.M * s.D >= (int64_t(1) << 31))
    return fail(MSDA_ERR_UNSUPPORTED, "num_values*num_heads*head_dim=%lld per batch item exceeds 2^31 - 1",
                (long long)(s.S * (int64_t)s.M * s.D));
  // Grid (ceil(Q / 8), M, B): y and z are limited to 65535.
  if (s.B > 65535 || s.M > 65535)
    return fail(MSDA_ERR_UNSUPPORTED, "batch (%lld) and num_heads (%d) must be <= 65535", (long long)s.B, s.M);
  return MSDA_OK;
}

// Whether the one-query-per-warp grid (ceil(Q / 8), M, B) is at most
// kShortGridWaves waves of 4 CTAs per SM (a decoder's few hundred queries);
// longer grids take the multi-query launch shapes.
bool short_grid(const Shape& s) {
  const int64_t ctas = (s.Q + msda::kWarpsPerCta - 1) / msda::kWarpsPerCta * s.M * s.B;
  return ctas <= (int64_t)msda::kShortGridWaves * 4 * sm_count();
}

int kshift_of(int32_t K) {
  if ((K & (K - 1)) != 0) return -1;
  int s = 0;
  while ((1 << s) < K) ++s;
  return s;
}

// Sampling points per value row (per head) up to which fp32 accumulation
// uses the hit-counted scatter; denser sampling hits almost every row more
// than once, and the plain fp32 scatter is cheaper.
constexpr double kCountedMaxPointsPerRow = 2.0;

// Sampling points per value row (per head) above which the scatter merges a
// warp's same-row contributions before reducing them.
constexpr double kMergeMinPointsPerRow = 2.0;

// Every flag bit msda_backward / msda_backward_fused understand.
constexpr uint32_t kKnownBwdFlags = MSDA_BWD_FP32_ACCUM | MSDA_BWD_FORCE_SCATTER | MSDA_BWD_FORCE_COUNTED |
                                    MSDA_BWD_DETERMINISTIC;

enum class Algo { kScatterNative, kScatterF32, kCounted, kScatterFixed, kCountedFixed, kCountedExact };

Algo choose_algo(const Shape& s, int32_t dtype, uint32_t flags) {
  const bool fp32_ws = (flags & MSDA_BWD_FP32_ACCUM) && dtype != MSDA_DTYPE_F32;
  const bool fp32_semantics = (flags & MSDA_BWD_FP32_ACCUM) || dtype == MSDA_DTYPE_F32;
  const double density = (double)s.Q * s.L * s.K / (double)s.S;
  if (flags & MSDA_BWD_DETERMINISTIC) {
    // Hit-counted: exact integer-valued fp32 rows for fp16 / bf16, 64-bit
    // fixed point for fp32 values; the scatter: 64-bit fixed point.
    const Algo counted = dtype == MSDA_DTYPE_F32 ? Algo::kCountedFixed : Algo::kCountedExact;
    if (flags & MSDA_BWD_FORCE_SCATTER) return Algo::kScatterFixed;
    if (flags & MSDA_BWD_FORCE_COUNTED) return counted;
    return density <= kCountedMaxPointsPerRow ? counted : Algo::kScatterFixed;
  }
  const Algo scatter = fp32_ws ? Algo::kScatterF32 : Algo::kScatterNative;
  if (flags & MSDA_BWD_FORCE_SCATTER) return scatter;
  if (flags & MSDA_BWD_FORCE_COUNTED) return Algo::kCounted;
  if (!fp32_semantics) return scatter;
  if (density <= kCountedMaxPointsPerRow) return Algo::kCounted;
  return scatter;
}


// Deterministic (fixed-point) algorithms: the workspace starts with the
// absmax header (2 words, padded).
constexpr size_t kFixedHeaderBytes = 256;

// Workspace of the hit-counted scatter: [absmax header (fixed point only)]
// per-row hit counts (exact rows: (count, bound) pairs), then one
// accumulator row per grad_value row -- fp32 (fp16/bf16 only; fp32 values
// accumulate in grad_value itself) or 64-bit fixed point (every dtype).
size_t counted_ws_bytes(const Shape& s, int32_t dtype, bool fixed, bool exact, size_t* counts_offset,
                        size_t* acc_offset) {
  const size_t rows = (size_t)s.B * s.S * s.M;
  const size_t head = fixed ? kFixedHeaderBytes : 0;
  const size_t counts = align256(rows * sizeof(unsigned) * (exact ? 2 : 1));
  *counts_offset = head;
  *acc_offset = head + counts;
  if (fixed || exact) return head + counts + rows * (size_t)s.D * sizeof(long long);
  if (dtype == MSDA_DTYPE_F32) return counts;
  return counts + rows * (size_t)s.D * sizeof(float);
}

}  // namespace

namespace msda {

// Lets other translation units of the library (msda_noalloc.cu) report a
// failure through msda_last_error(). Not exported.
void set_last_error(const char* msg) { g_last_error = msg ? msg : ""; }

// The size checks of msda_backward, for entry points that size their own
// buffers before calling it (msda_noalloc.cu). Not exported.
int check_backward_shape(int64_t B, int64_t S, int64_t Q, int32_t M, int32_t D, int32_t L, int32_t K,
                         int32_t dtype) {
  return check_shape(Shape{B, S, Q, M, D, L, K}, dtype);
}

}  // namespace msda

extern "C" {

const char* msda_version(void) { return "msda_b200 0.1.0 sm_100a"; }

const char* msda_last_error(void) { return g_last_error.c_str(); }

// The forward behind msda_forward and msda_forward_fused. Fused: `loc` holds
// sampling offsets in level pixels, `attn` attention logits, `ref` the
// reference points.
static int forward_impl(const char* fn, const void* value, const int64_t* spatial_shapes,
                        const int64_t* level_start_index, const void* ref, const void* loc,
                        const void* attn, void* output, bool fused, const Shape& s, int32_t dtype,
                        void* stream) {
  const void* sampling_locations = loc;
  const void* attention_weights = attn;
  if (int rc = check_shape(s, dtype)) return rc;
  if (s.B == 0 || s.Q == 0) return succeed();
  if (!value || !spatial_shapes || !level_start_index || !sampling_locations || !attention_weights ||
      !output || (fused && !ref))
    return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: null pointer argument", fn);
  const int es = elem_size(dtype);
  if (!aligned(sampling_locations, 2 * es) || !aligned(value, es) || !aligned(output, es) ||
      !aligned(attention_weights, es) || !aligned(spatial_shapes, 8) || !aligned(level_start_index, 8) ||
      (fused && !aligned(ref, 2 * es)))
    return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: misaligned buffer (sampling_locations / offsets and reference points need %d-byte alignment)", fn, 2 * es);
  msda::Cfg cfg;
  if (int rc = choose_cfg(s.D, es, aligned(value, 16) && aligned(output, 16), &cfg)) return rc;
  if (fused && cfg.vec != 16 / es)
    return fail(MSDA_ERR_UNSUPPORTED, "%s: the fused prologue needs 16-byte aligned buffers and head_dim a multiple of %d", fn, 16 / es);
  cfg.short_grid = short_grid(s);

  msda::OpParams p{};
  p.value = value;
  p.shapes = spatial_shapes;
  p.starts = level_start_index;
  p.loc = sampling_locations;
  p.attn = attention_weights;
  p.ref = ref;
  p.fused = fused ? 1 : 0;
  p.out = output;
  p.B = s.B; p.S = s.S; p.Q = s.Q;
  p.M = s.M; p.D = s.D; p.L = s.L; p.K = s.K;
  p.kshift = kshift_of(s.K);
  p.BQM = s.B * s.Q * s.M;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e;
  switch (dtype) {
    case MSDA_DTYPE_F32: e = msda::launch_forward<float>(p, cfg, st); break;
    case MSDA_DTYPE_F16: e = msda::launch_forward<__half>(p, cfg, st); break;
    default: e = msda::launch_forward<__nv_bfloat16>(p, cfg, st); break;
  }
  if (e != cudaSuccess) return cuda_fail(e, "forward launch");
  return succeed();
}

int msda_forward(const void* value, const int64_t* spatial_shapes, const int64_t* level_start_index,
                 const void* sampling_locations, const void* attention_weights, void* output,
                 int64_t batch, int64_t num_values, int64_t num_queries, int32_t num_heads,
                 int32_t head_dim, int32_t num_levels, int32_t num_points, int32_t dtype,
                 void* stream) {
  const Shape s{batch, num_values, num_queries, num_heads, head_dim, num_levels, num_points};
  return forward_impl("msda_forward", value, spatial_shapes, level_start_index, nullptr,
                      sampling_locations, attention_weights, output, false, s, dtype, stream);
}

int msda_forward_fused(const void* value, const int64_t* spatial_shapes,
                       const int64_t* level_start_index, const void* reference_points,
                       const void* sampling_offsets, const void* attention_logits, void* output,
                       int64_t batch, int64_t num_values, int64_t num_queries, int32_t num_heads,
                       int32_t head_dim, int32_t num_levels, int32_t num_points, int32_t dtype,
                       void* stream) {
  const Shape s{batch, num_values, num_queries, num_heads, head_dim, num_levels, num_points};
  return forward_impl("msda_forward_fused", value, spatial_shapes, level_start_index,
                      reference_points, sampling_offsets, attention_logits, output, true, s, dtype,
                      stream);
}

size_t msda_backward_workspace_size(int64_t batch, int64_t num_values, int64_t num_queries,
                                    int32_t num_heads, int32_t head_dim, int32_t num_levels,
                                    int32_t num_points, int32_t dtype, uint32_t flags) {
  const Shape s{batch, num_values, num_queries, num_heads, head_dim, num_levels, num_points};
  const int es = elem_size(dtype);
  if (es == 0 || batch <= 0 || num_queries <= 0 || num_values <= 0 || num_heads <= 0 ||
      head_dim <= 0 || num_levels <= 0 || num_points <= 0)
    return 0;
  if (flags & ~kKnownBwdFlags) return 0;
  const Algo a = choose_algo(s, dtype, flags);
  if (a == Algo::kCounted || a == Algo::kCountedFixed || a == Algo::kCountedExact) {
    size_t coff, aoff;
    return counted_ws_bytes(s, dtype, a == Algo::kCountedFixed, a == Algo::kCountedExact, &coff, &aoff);
  }
  const size_t elems = (size_t)batch * (size_t)num_values * (size_t)num_heads * (size_t)head_dim;
  if (a == Algo::kScatterFixed) return kFixedHeaderBytes + elems * sizeof(long long);
  if (a != Algo::kScatterF32) return 0;
  return elems * sizeof(float);
}

// The backward behind msda_backward and msda_backward_fused (fused: offsets
// and logits in, their gradients out).
static int backward_impl(const char* fn, const void* value, const int64_t* spatial_shapes,
                         const int64_t* level_start_index, const void* ref,
                         const void* sampling_locations, const void* attention_weights,
                         const void* grad_output, void* grad_value, void* grad_sampling_locations,
                         void* grad_attention_weights, void* workspace, size_t workspace_bytes,
                         bool fused, const Shape& s, int32_t dtype, uint32_t flags, void* stream) {
  if (int rc = check_shape(s, dtype)) return rc;
  if (flags & MSDA_BWD_GRAD_INPUT_NCHW)
    return fail(MSDA_ERR_UNSUPPORTED, "%s: MSDA_BWD_GRAD_INPUT_NCHW is a flag of the sibling gathers", fn);
  if (flags & ~kKnownBwdFlags)
    return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: unknown flag bits 0x%x", fn, (unsigned)(flags & ~kKnownBwdFlags));
  if (s.B == 0) return succeed();
  const int es = elem_size(dtype);
  const size_t gv_bytes = (size_t)s.B * s.S * s.M * s.D * es;
  if (!grad_value) return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: null grad_value", fn);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (s.Q == 0) {
    cudaError_t e = cudaMemsetAsync(grad_value, 0, gv_bytes, st);
    if (e != cudaSuccess) return cuda_fail(e, "msda_backward zero-fill");
    return succeed();
  }
  if (!value || !spatial_shapes || !level_start_index || !sampling_locations || !attention_weights ||
      !grad_output || !grad_sampling_locations || !grad_attention_weights || (fused && !ref))
    return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: null pointer argument", fn);
  if (!aligned(sampling_locations, 2 * es) || !aligned(grad_sampling_locations, 2 * es) ||
      !aligned(value, es) || !aligned(grad_value, es) || !aligned(grad_output, es) ||
      !aligned(attention_weights, es) || !aligned(grad_attention_weights, es) ||
      !aligned(spatial_shapes, 8) || !aligned(level_start_index, 8) || (fused && !aligned(ref, 2 * es)))
    return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: misaligned buffer (locations / offsets and reference points need %d-byte alignment)", fn, 2 * es);

  const Algo algo = choose_algo(s, dtype, flags);
  const bool fixed = algo == Algo::kScatterFixed || algo == Algo::kCountedFixed;
  const bool fp32_ws = algo == Algo::kScatterF32;
  const bool exact = algo == Algo::kCountedExact;
  const bool counted = algo == Algo::kCounted || algo == Algo::kCountedFixed || exact;
  const bool ws_target = fp32_ws || algo == Algo::kScatterFixed;  // reductions into the workspace
  const size_t ws_need = msda_backward_workspace_size(s.B, s.S, s.Q, s.M, s.D, s.L, s.K, dtype, flags);
  if (fp32_ws || counted || fixed) {
    if (!workspace || workspace_bytes < ws_need)
      return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: %s accumulation needs a workspace of %zu bytes (got %zu)", fn, (fixed || exact) ? "deterministic" : "fp32", ws_need, workspace_bytes);
    if (!aligned(workspace, 16))
      return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: workspace must be 16-byte aligned", fn);
  }
  unsigned* fixed_hdr = fixed ? static_cast<unsigned*>(workspace) : nullptr;
  void* target = algo == Algo::kScatterFixed ? static_cast<void*>(static_cast<char*>(workspace) + kFixedHeaderBytes)
                 : fp32_ws                 ? workspace
                                           : grad_value;
  msda::Cfg cfg;
  const bool vec_ok = aligned(value, 16) && aligned(grad_output, 16) &&
                      aligned(target, 16) &&
                      (!counted || aligned(grad_value, 16));
  if (int rc = choose_cfg(s.D, es, vec_ok, &cfg)) return rc;
  if (fused && cfg.vec != 16 / es)
    return fail(MSDA_ERR_UNSUPPORTED, "%s: the fused prologue needs 16-byte aligned buffers and head_dim a multiple of %d", fn, 16 / es);
  cfg.short_grid = short_grid(s);

  cudaError_t e;
  size_t counts_off = 0, acc_off = 0;
  const size_t rows = (size_t)s.B * s.S * s.M;
  if (counted) {
    counted_ws_bytes(s, dtype, fixed, exact, &counts_off, &acc_off);
    // Counts (and the absmax header before them, the row bounds after them),
    // zeroed by our kernel (padded to 16 bytes inside the 256-byte-aligned
    // count region) so the passes behind it can start under its tail.
    const size_t zbytes = ((exact ? acc_off : counts_off + rows * sizeof(unsigned)) + 15) / 16 * 16;
    e = msda::launch_zero(workspace, zbytes, sm_count(), st);
    if (e != cudaSuccess) return cuda_fail(e, "msda_backward hit-count zero-fill");
  }
  // The backward may overlap the tail of the kernel before it when that
  // kernel is ours (the hit count, the zero-fill kernel or the absmax pass;
  // not a memset).
  bool bwd_pdl = counted;
  bool zero_kernel = counted;
  if (!counted) {
    // The deterministic scatter zeroes the header with the accumulator.
    void* zdst = algo == Algo::kScatterFixed ? workspace : target;
    const size_t zbytes = ws_target ? ws_need : gv_bytes;
    if (zbytes % 16 == 0 && aligned(zdst, 16)) {
      e = msda::launch_zero(zdst, zbytes, sm_count(), st);
      bwd_pdl = zbytes >= 16;
      zero_kernel = bwd_pdl;
    } else {
      e = cudaMemsetAsync(zdst, 0, zbytes, st);
    }
    if (e != cudaSuccess) return cuda_fail(e, "msda_backward zero-fill");
  }
  if (fixed) {
    // Pass 0: max |attention weight| (or the logits' finiteness) and
    // max |grad_out| into the header.
    const int64_t n_attn = s.B * s.Q * s.M * s.L * s.K, n_g = s.B * s.Q * s.M * s.D;
    switch (dtype) {
      case MSDA_DTYPE_F32: e = msda::launch_absmax<float>(attention_weights, n_attn, fused, grad_output, n_g, fixed_hdr, sm_count(), zero_kernel, st); break;
      case MSDA_DTYPE_F16: e = msda::launch_absmax<__half>(attention_weights, n_attn, fused, grad_output, n_g, fixed_hdr, sm_count(), zero_kernel, st); break;
      default: e = msda::launch_absmax<__nv_bfloat16>(attention_weights, n_attn, fused, grad_output, n_g, fixed_hdr, sm_count(), zero_kernel, st); break;
    }
    if (e != cudaSuccess) return cuda_fail(e, "msda_backward absmax launch");
    if (!counted) bwd_pdl = true;  // behind the absmax pass
  }

  msda::OpParams p{};
  p.value = value;
  p.shapes = spatial_shapes;
  p.starts = level_start_index;
  p.loc = sampling_locations;
  p.attn = attention_weights;
  p.ref = ref;
  p.fused = fused ? 1 : 0;
  p.grad_out = grad_output;
  p.grad_value = counted ? grad_value : target;
  p.acc_words = (fixed || exact) ? 2 : 1;
  if (exact) p.rowmax = reinterpret_cast<unsigned*>(static_cast<char*>(workspace) + counts_off) + 1;
  p.fixed_hdr = fixed_hdr;
  p.fixed_log2n = ceil_log2(s.Q * s.K);
  p.grad_loc = grad_sampling_locations;
  p.grad_attn = grad_attention_weights;
  if (counted) {
    p.counts = reinterpret_cast<unsigned*>(static_cast<char*>(workspace) + counts_off);
    p.acc = (dtype == MSDA_DTYPE_F32 && !fixed) ? grad_value
                                                : static_cast<void*>(static_cast<char*>(workspace) + acc_off);
  }
  p.B = s.B; p.S = s.S; p.Q = s.Q;
  p.M = s.M; p.D = s.D; p.L = s.L; p.K = s.K;
  p.kshift = kshift_of(s.K);
  p.BQM = s.B * s.Q * s.M;
  if (counted) {
    switch (dtype) {
      // behind the zero-fill, or behind the absmax pass that follows it
      case MSDA_DTYPE_F32: e = msda::launch_count<float>(p, sm_count(), exact, true, st); break;
      case MSDA_DTYPE_F16: e = msda::launch_count<__half>(p, sm_count(), exact, true, st); break;
      default: e = msda::launch_count<__nv_bfloat16>(p, sm_count(), exact, true, st); break;
    }
    if (e != cudaSuccess) return cuda_fail(e, "msda_backward hit-count launch");
  }
  // Dense sampling (more points than value rows per head, e.g. an encoder's
  // queries at every pixel) makes the points of one query share rows: merge
  // them before the reductions. Sparse sampling rarely does.
  const bool merge = (double)s.Q * s.L * s.K > kMergeMinPointsPerRow * (double)s.S;
  const int mode = counted ? msda::kCounted : merge ? msda::kScatterMerge : msda::kScatter;
  const int acc = fixed   ? msda::kAccFixed
                  : exact ? msda::kAccExact
                  : (fp32_ws || dtype == MSDA_DTYPE_F32) ? msda::kAccF32
                                                         : msda::kAccNative;
  switch (dtype) {
    case MSDA_DTYPE_F32: e = msda::launch_backward<float>(p, cfg, mode, acc, bwd_pdl, st); break;
    case MSDA_DTYPE_F16: e = msda::launch_backward<__half>(p, cfg, mode, acc, bwd_pdl, st); break;
    default: e = msda::launch_backward<__nv_bfloat16>(p, cfg, mode, acc, bwd_pdl, st); break;
  }
  if (e != cudaSuccess) return cuda_fail(e, "msda_backward launch");
  if (counted) {
    const bool fvec = aligned(grad_value, 16);
    switch (dtype) {
      case MSDA_DTYPE_F32: e = msda::launch_finalize<float>(p, fvec, fixed, exact, sm_count(), st); break;
      case MSDA_DTYPE_F16: e = msda::launch_finalize<__half>(p, fvec, fixed, exact, sm_count(), st); break;
      default: e = msda::launch_finalize<__nv_bfloat16>(p, fvec, fixed, exact, sm_count(), st); break;
    }
    if (e != cudaSuccess) return cuda_fail(e, "msda_backward finalize launch");
  }
  if (algo == Algo::kScatterFixed) {
    const int64_t n = s.B * s.S * s.M * s.D;
    const bool cast_vec = aligned(grad_value, 16);
    const long long* src = static_cast<const long long*>(target);
    switch (dtype) {
      case MSDA_DTYPE_F32: e = msda::launch_cast_fixed<float>(src, static_cast<float*>(grad_value), n, cast_vec, fixed_hdr, p.fixed_log2n, sm_count(), st); break;
      case MSDA_DTYPE_F16: e = msda::launch_cast_fixed<__half>(src, static_cast<__half*>(grad_value), n, cast_vec, fixed_hdr, p.fixed_log2n, sm_count(), st); break;
      default: e = msda::launch_cast_fixed<__nv_bfloat16>(src, static_cast<__nv_bfloat16*>(grad_value), n, cast_vec, fixed_hdr, p.fixed_log2n, sm_count(), st); break;
    }
    if (e != cudaSuccess) return cuda_fail(e, "msda_backward fixed-point downcast launch");
  }
  if (fp32_ws) {
    const int64_t n = s.B * s.S * s.M * s.D;
    const bool cast_vec = aligned(grad_value, 16);
    if (dtype == MSDA_DTYPE_F16)
      e = msda::launch_cast<__half>(static_cast<const float*>(workspace), static_cast<__half*>(grad_value), n, cast_vec, sm_count(), st);
    else
      e = msda::launch_cast<__nv_bfloat16>(static_cast<const float*>(workspace), static_cast<__nv_bfloat16*>(grad_value), n, cast_vec, sm_count(), st);
    if (e != cudaSuccess) return cuda_fail(e, "msda_backward downcast launch");
  }
  return succeed();
}

int msda_backward(const void* value, const int64_t* spatial_shapes, const int64_t* level_start_index,
                  const void* sampling_locations, const void* attention_weights,
                  const void* grad_output, void* grad_value, void* grad_sampling_locations,
                  void* grad_attention_weights, void* workspace, size_t workspace_bytes,
                  int64_t batch, int64_t num_values, int64_t num_queries, int32_t num_heads,
                  int32_t head_dim, int32_t num_levels, int32_t num_points, int32_t dtype,
                  uint32_t flags, void* stream) {
  const Shape s{batch, num_values, num_queries, num_heads, head_dim, num_levels, num_points};
  return backward_impl("msda_backward", value, spatial_shapes, level_start_index, nullptr,
                       sampling_locations, attention_weights, grad_output, grad_value,
                       grad_sampling_locations, grad_attention_weights, workspace, workspace_bytes,
                       false, s, dtype, flags, stream);
}

int msda_backward_fused(const void* value, const int64_t* spatial_shapes,
                        const int64_t* level_start_index, const void* reference_points,
                        const void* sampling_offsets, const void* attention_logits,
                        const void* grad_output, void* grad_value, void* grad_sampling_offsets,
                        void* grad_attention_logits, void* workspace, size_t workspace_bytes,
                        int64_t batch, int64_t num_values, int64_t num_queries, int32_t num_heads,
                        int32_t head_dim, int32_t num_levels, int32_t num_points, int32_t dtype,
                        uint32_t flags, void* stream) {
  const Shape s{batch, num_values, num_queries, num_heads, head_dim, num_levels, num_points};
  return backward_impl("msda_backward_fused", value, spatial_shapes, level_start_index,
                       reference_points, sampling_offsets, attention_logits, grad_output, grad_value,
                       grad_sampling_offsets, grad_attention_logits, workspace, workspace_bytes, true,
                       s, dtype, flags, stream);
}

}  // extern "C"
