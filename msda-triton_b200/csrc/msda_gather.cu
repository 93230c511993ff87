// C ABI of the sibling gathers (declared in include/msda_b200.h):
// grid_sample and ROI-Align forward / backward on NHWC data.
#include <algorithm>

#include "msda_abi.cuh"
#include "msda_gather.cuh"

namespace {

using namespace msda::abi;
using msda::GatherParams;

// Largest H*W the kernels address with 32-bit pixel arithmetic.
constexpr int64_t kMaxPixels = int64_t(1) << 30;

// (LPR, CPL) lane layouts the kernels are built for (see choose_cfg).
#define MSDA_GATHER_SHAPES(X) \
  X(1, 1) X(2, 1) X(4, 1) X(8, 1) X(16, 1) X(32, 1) X(32, 2) X(32, 4)

int64_t gather_ctas(int64_t rows, const msda::Cfg& c) {
  const int64_t rows_per_cta = (int64_t)msda::kGatherWarps * (32 / c.lpr);
  return (rows + rows_per_cta - 1) / rows_per_cta;
}

// One-dimensional grid over the output rows; its size is checked against
// gridDim.x's limit by `grid_fits` before any launch.
dim3 gather_grid(const GatherParams& p, const msda::Cfg& c) { return dim3((unsigned)gather_ctas(p.R * p.Q, c)); }

int grid_fits(const char* fn, int64_t rows, const msda::Cfg& c) {
  if (gather_ctas(rows, c) > 0x7fffffff) return fail(MSDA_ERR_UNSUPPORTED, "%s: too many output rows for one grid", fn);
  return MSDA_OK;
}

template <typename T, int VEC>
cudaError_t gs_fwd(const GatherParams& p, const msda::Cfg& c, cudaStream_t st) {
#define X(LPR_, CPL_)                                                                              \
  if (c.lpr == LPR_ && c.cpl == CPL_) {                                                            \
    msda::gs_fwd_kernel<T, VEC, LPR_, CPL_><<<gather_grid(p, c), msda::kGatherWarps * 32, 0, st>>>(p); \
    return cudaGetLastError();                                                                     \
  }
  MSDA_GATHER_SHAPES(X)
#undef X
  return cudaErrorInvalidConfiguration;
}

template <typename T, typename A, int VEC>
cudaError_t gs_bwd(const GatherParams& p, const msda::Cfg& c, bool pdl, cudaStream_t st) {
#define X(LPR_, CPL_)                                                                                   \
  if (c.lpr == LPR_ && c.cpl == CPL_)                                                                   \
    return msda::launch_ex(msda::gs_bwd_kernel<T, A, VEC, LPR_, CPL_>, gather_grid(p, c),                \
                           dim3(msda::kGatherWarps * 32), 0, st, pdl, p);
  MSDA_GATHER_SHAPES(X)
#undef X
  return cudaErrorInvalidConfiguration;
}

template <typename T, int VEC>
cudaError_t roi_fwd(const GatherParams& p, const msda::Cfg& c, cudaStream_t st) {
#define X(LPR_, CPL_)                                                                               \
  if (c.lpr == LPR_ && c.cpl == CPL_) {                                                             \
    msda::roi_fwd_kernel<T, VEC, LPR_, CPL_><<<gather_grid(p, c), msda::kGatherWarps * 32, 0, st>>>(p); \
    return cudaGetLastError();                                                                      \
  }
  MSDA_GATHER_SHAPES(X)
#undef X
  return cudaErrorInvalidConfiguration;
}

template <typename T, typename A, int VEC>
cudaError_t roi_bwd(const GatherParams& p, const msda::Cfg& c, bool pdl, cudaStream_t st) {
#define X(LPR_, CPL_)                                                                                    \
  if (c.lpr == LPR_ && c.cpl == CPL_)                                                                    \
    return msda::launch_ex(msda::roi_bwd_kernel<T, A, VEC, LPR_, CPL_>, gather_grid(p, c),                \
                           dim3(msda::kGatherWarps * 32), 0, st, pdl, p);
  MSDA_GATHER_SHAPES(X)
#undef X
  return cudaErrorInvalidConfiguration;
}

// Accumulator of a backward scatter.
enum class Acc { kNative, kF32, kFixed };

template <typename T>
cudaError_t launch_fwd(bool roi, const GatherParams& p, const msda::Cfg& c, cudaStream_t st) {
  constexpr int V16 = 16 / (int)sizeof(T);
  if (c.vec == V16) return roi ? roi_fwd<T, V16>(p, c, st) : gs_fwd<T, V16>(p, c, st);
  return roi ? roi_fwd<T, 1>(p, c, st) : gs_fwd<T, 1>(p, c, st);
}

template <typename T>
cudaError_t launch_bwd(bool roi, const GatherParams& p, const msda::Cfg& c, Acc acc, bool pdl, cudaStream_t st) {
  constexpr int V16 = 16 / (int)sizeof(T);
  if (roi) {
    if (acc == Acc::kFixed)
      return c.vec == V16 ? roi_bwd<T, long long, V16>(p, c, pdl, st) : roi_bwd<T, long long, 1>(p, c, pdl, st);
    if (acc == Acc::kF32 || sizeof(T) == 4)
      return c.vec == V16 ? roi_bwd<T, float, V16>(p, c, pdl, st) : roi_bwd<T, float, 1>(p, c, pdl, st);
    return c.vec == V16 ? roi_bwd<T, T, V16>(p, c, pdl, st) : roi_bwd<T, T, 1>(p, c, pdl, st);
  }
  if (acc == Acc::kFixed)
    return c.vec == V16 ? gs_bwd<T, long long, V16>(p, c, pdl, st) : gs_bwd<T, long long, 1>(p, c, pdl, st);
  if (acc == Acc::kF32 || sizeof(T) == 4)
    return c.vec == V16 ? gs_bwd<T, float, V16>(p, c, pdl, st) : gs_bwd<T, float, 1>(p, c, pdl, st);
  return c.vec == V16 ? gs_bwd<T, T, V16>(p, c, pdl, st) : gs_bwd<T, T, 1>(p, c, pdl, st);
}

struct Dims {
  int64_t N, H, W, C;  // input (N, H, W, C)
  int64_t R, Q;        // output items and rows per item
};

int check_dims(const char* fn, const Dims& d, int32_t dtype) {
  if (elem_size(dtype) == 0) return fail(MSDA_ERR_UNSUPPORTED, "%s: unsupported dtype code %d (0=f32, 1=f16, 2=bf16)", fn, dtype);
  if (d.N < 0 || d.R < 0 || d.Q < 0) return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: negative size", fn);
  if (d.H < 1 || d.W < 1 || d.H * d.W > kMaxPixels)
    return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: input height*width must be in [1, 2^30] (got %lld x %lld)", fn, (long long)d.H, (long long)d.W);
  if (d.C < 1) return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: channels must be >= 1", fn);
  if (d.R * d.Q > (int64_t(1) << 36)) return fail(MSDA_ERR_UNSUPPORTED, "%s: too many output rows", fn);
  return MSDA_OK;
}

// Grid of the tiled transposes for (N, R, C) -> (N, C, R): (column tiles,
// row tiles, N), with the row tiles on gridDim.x (`r_in_x`) when they exceed
// gridDim.y's 65535. False when the sizes do not fit one grid.
bool transpose_grid(int64_t N, int64_t R, int64_t C, dim3* grid, int* r_in_x) {
  constexpr int TL = msda::kTransposeTile;
  const int64_t tc = (C + TL - 1) / TL, tr = (R + TL - 1) / TL;
  *r_in_x = tr > 65535 ? 1 : 0;
  const int64_t gx = *r_in_x ? tr : tc, gy = *r_in_x ? tc : tr;
  if (gx > 0x7fffffff || gy > 65535 || N > 65535) return false;
  *grid = dim3((unsigned)gx, (unsigned)gy, (unsigned)N);
  return true;
}

// The 4-element-vector kernels apply: R and C multiples of 4, a batch slice
// below 2^31 elements, both buffers aligned to 4 elements of their type.
bool transpose_vec4(int64_t R, int64_t C, const void* src, int src_es, const void* dst, int dst_es) {
  return R % 4 == 0 && C % 4 == 0 && R * C < (int64_t(1) << 31) && aligned(src, 4 * src_es) &&
         aligned(dst, 4 * dst_es);
}

// Accumulator (NHWC, type S) -> grad_input (NCHW, data type D).
template <typename S, typename D>
cudaError_t launch_convert_transpose(const S* src, D* dst, int64_t N, int64_t R, int64_t C, const unsigned* hdr,
                                     int clog2n, cudaStream_t st) {
  dim3 grid;
  int r_in_x;
  transpose_grid(N, R, C, &grid, &r_in_x);  // checked before the first launch of the call
  if (transpose_vec4(R, C, src, sizeof(S), dst, sizeof(D)))
    return msda::launch_ex(msda::convert_transpose_kernel<S, D, true>, grid, dim3(256), 0, st, true, src, dst, R, C,
                           r_in_x, hdr, clog2n);
  return msda::launch_ex(msda::convert_transpose_kernel<S, D, false>, grid, dim3(256), 0, st, true, src, dst, R, C,
                         r_in_x, hdr, clog2n);
}

template <typename D>
cudaError_t launch_grad_nchw(int acc_kind, const void* ws, void* grad_input, int64_t N, int64_t R, int64_t C,
                             const unsigned* hdr, int clog2n, cudaStream_t st) {
  D* dst = static_cast<D*>(grad_input);
  switch (acc_kind) {
    case 2: return launch_convert_transpose(static_cast<const long long*>(ws), dst, N, R, C, hdr, clog2n, st);
    case 1: return launch_convert_transpose(static_cast<const float*>(ws), dst, N, R, C, hdr, clog2n, st);
    default: return launch_convert_transpose(static_cast<const D*>(ws), dst, N, R, C, hdr, clog2n, st);
  }
}

enum class Op { kGridSample, kRoiAlign };

size_t workspace_bytes_for(const Dims& d, int32_t dtype, uint32_t flags) {
  const size_t elems = (size_t)d.N * d.H * d.W * d.C;
  if (flags & MSDA_BWD_DETERMINISTIC) return 256 + elems * sizeof(long long);
  if ((flags & MSDA_BWD_FP32_ACCUM) && dtype != MSDA_DTYPE_F32) return elems * sizeof(float);
  if (flags & MSDA_BWD_GRAD_INPUT_NCHW) return elems * elem_size(dtype);
  return 0;
}

// Zero the scatter target, fill the absmax header (fixed point), run the
// backward kernel, and round the accumulator into grad_input.
int backward(const char* fn, Op op, GatherParams& p, const Dims& d, void* grad_input, void* workspace,
             size_t ws_bytes, int32_t dtype, uint32_t flags, cudaStream_t st) {
  const bool fixed = (flags & MSDA_BWD_DETERMINISTIC) != 0;
  const bool f32_ws = !fixed && (flags & MSDA_BWD_FP32_ACCUM) && dtype != MSDA_DTYPE_F32;
  const bool nchw = (flags & MSDA_BWD_GRAD_INPUT_NCHW) != 0;  // workspace + converting transpose
  const int es = elem_size(dtype);
  const size_t need = workspace_bytes_for(d, dtype, flags);
  const size_t gi_bytes = (size_t)d.N * d.H * d.W * d.C * es;
  if (need) {
    if (!workspace || ws_bytes < need)
      return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: needs a workspace of %zu bytes (got %zu)", fn, need, ws_bytes);
    if (!aligned(workspace, 16)) return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: workspace must be 16-byte aligned", fn);
  }
  void* target = fixed ? static_cast<void*>(static_cast<char*>(workspace) + 256)
                 : (f32_ws || nchw) ? workspace
                                    : grad_input;
  void* zdst = fixed ? workspace : target;
  const size_t zbytes = need ? need : gi_bytes;
  msda::Cfg cfg;
  if (nchw) {  // every check before the first launch
    dim3 g;
    int r_in_x;
    if (!transpose_grid(d.N, d.H * d.W, d.C, &g, &r_in_x))
      return fail(MSDA_ERR_UNSUPPORTED, "%s: the NCHW input gradient needs N <= 65535 and C <= %d", fn,
                  65535 * msda::kTransposeTile);
  }
  if (d.R * d.Q > 0) {
    const bool vec_ok = aligned(p.input ? p.input : p.grad_out, 16) && aligned(p.grad_out, 16) && aligned(target, 16);
    if (int rc = choose_cfg((int32_t)d.C, es, vec_ok, &cfg)) return rc;
    if (int rc = grid_fits(fn, d.R * d.Q, cfg)) return rc;
  }
  cudaError_t e;
  bool pdl = false;
  if (zbytes % 16 == 0 && aligned(zdst, 16)) {
    e = msda::launch_zero(zdst, zbytes, sm_count(), st);
    pdl = zbytes >= 16;
  } else {
    e = cudaMemsetAsync(zdst, 0, zbytes, st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "zero-fill");
  // Nothing to scatter and no accumulator to round: grad_input is the zeros.
  if (d.R * d.Q == 0 && !need) return succeed();
  p.grad_in = target;
  if (fixed) {
    p.fixed_hdr = static_cast<const unsigned*>(workspace);
    // Bound on the terms of one input pixel's sum, each at most max|grad_out|
    // (interpolation weights <= 1): grid_sample, the output pixels of its
    // image; ROI-Align, every output bin (a bin's sampling weights average
    // to 1, so its contributions to one pixel sum to at most max|grad_out|).
    p.fixed_log2n = ceil_log2(std::max<int64_t>(op == Op::kRoiAlign ? d.R * d.Q : d.Q, 1));
    const int64_t ng = d.R * d.Q * d.C;
    unsigned* hdr = static_cast<unsigned*>(workspace);
    switch (dtype) {
      case MSDA_DTYPE_F32: e = msda::launch_absmax<float>(nullptr, 0, true, p.grad_out, ng, hdr, sm_count(), pdl, st); break;
      case MSDA_DTYPE_F16: e = msda::launch_absmax<__half>(nullptr, 0, true, p.grad_out, ng, hdr, sm_count(), pdl, st); break;
      default: e = msda::launch_absmax<__nv_bfloat16>(nullptr, 0, true, p.grad_out, ng, hdr, sm_count(), pdl, st); break;
    }
    if (e != cudaSuccess) return cuda_fail(e, "absmax launch");
    pdl = true;
  }
  if (d.R * d.Q > 0) {
    const Acc acc = fixed ? Acc::kFixed : (f32_ws || dtype == MSDA_DTYPE_F32) ? Acc::kF32 : Acc::kNative;
    const bool roi = op == Op::kRoiAlign;
    switch (dtype) {
      case MSDA_DTYPE_F32: e = launch_bwd<float>(roi, p, cfg, acc, pdl, st); break;
      case MSDA_DTYPE_F16: e = launch_bwd<__half>(roi, p, cfg, acc, pdl, st); break;
      default: e = launch_bwd<__nv_bfloat16>(roi, p, cfg, acc, pdl, st); break;
    }
    if (e != cudaSuccess) return cuda_fail(e, "backward launch");
  }
  const int64_t n = d.N * d.H * d.W * d.C;
  const bool cast_vec = aligned(grad_input, 16) && aligned(target, 16);
  if (nchw) {
    const int kind = fixed ? 2 : f32_ws ? 1 : 0;  // accumulator: fixed point, fp32, data type
    const int64_t hw = d.H * d.W;
    switch (dtype) {
      case MSDA_DTYPE_F32: e = launch_grad_nchw<float>(kind, target, grad_input, d.N, hw, d.C, p.fixed_hdr, p.fixed_log2n, st); break;
      case MSDA_DTYPE_F16: e = launch_grad_nchw<__half>(kind, target, grad_input, d.N, hw, d.C, p.fixed_hdr, p.fixed_log2n, st); break;
      default: e = launch_grad_nchw<__nv_bfloat16>(kind, target, grad_input, d.N, hw, d.C, p.fixed_hdr, p.fixed_log2n, st); break;
    }
    if (e != cudaSuccess) return cuda_fail(e, "NCHW input gradient launch");
  } else if (fixed) {
    const long long* src = static_cast<const long long*>(target);
    switch (dtype) {
      case MSDA_DTYPE_F32: e = msda::launch_cast_fixed<float>(src, static_cast<float*>(grad_input), n, cast_vec, p.fixed_hdr, p.fixed_log2n, sm_count(), st); break;
      case MSDA_DTYPE_F16: e = msda::launch_cast_fixed<__half>(src, static_cast<__half*>(grad_input), n, cast_vec, p.fixed_hdr, p.fixed_log2n, sm_count(), st); break;
      default: e = msda::launch_cast_fixed<__nv_bfloat16>(src, static_cast<__nv_bfloat16*>(grad_input), n, cast_vec, p.fixed_hdr, p.fixed_log2n, sm_count(), st); break;
    }
    if (e != cudaSuccess) return cuda_fail(e, "fixed-point downcast launch");
  } else if (f32_ws) {
    const float* src = static_cast<const float*>(target);
    e = dtype == MSDA_DTYPE_F16
            ? msda::launch_cast<__half>(src, static_cast<__half*>(grad_input), n, cast_vec, sm_count(), st)
            : msda::launch_cast<__nv_bfloat16>(src, static_cast<__nv_bfloat16*>(grad_input), n, cast_vec, sm_count(), st);
    if (e != cudaSuccess) return cuda_fail(e, "downcast launch");
  }
  return succeed();
}

int forward(const char* fn, Op op, GatherParams& p, const Dims& d, int32_t dtype, cudaStream_t st) {
  if (d.R * d.Q == 0) return succeed();
  const int es = elem_size(dtype);
  msda::Cfg cfg;
  if (int rc = choose_cfg((int32_t)d.C, es, aligned(p.input, 16) && aligned(p.out, 16), &cfg)) return rc;
  if (int rc = grid_fits(fn, d.R * d.Q, cfg)) return rc;
  cudaError_t e;
  const bool roi = op == Op::kRoiAlign;
  switch (dtype) {
    case MSDA_DTYPE_F32: e = launch_fwd<float>(roi, p, cfg, st); break;
    case MSDA_DTYPE_F16: e = launch_fwd<__half>(roi, p, cfg, st); break;
    default: e = launch_fwd<__nv_bfloat16>(roi, p, cfg, st); break;
  }
  if (e != cudaSuccess) return cuda_fail(e, "forward launch");
  return succeed();
}

}  // namespace

extern "C" {

int msda_transpose(const void* src, void* dst, int64_t N, int64_t R, int64_t C, int32_t dtype,
                   void* stream) {
  const char* fn = "msda_transpose";
  const int es = elem_size(dtype);
  if (es == 0) return fail(MSDA_ERR_UNSUPPORTED, "%s: unsupported dtype code %d", fn, dtype);
  if (N < 0 || R < 0 || C < 0) return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: negative size", fn);
  if (N == 0 || R == 0 || C == 0) return succeed();
  if (!src || !dst) return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: null pointer argument", fn);
  if (!aligned(src, es) || !aligned(dst, es)) return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: misaligned buffer", fn);
  dim3 grid;
  int r_in_x;
  if (!transpose_grid(N, R, C, &grid, &r_in_x))
    return fail(MSDA_ERR_UNSUPPORTED, "%s: sizes too large (N <= 65535, min(R, C) <= %d)", fn,
                65535 * msda::kTransposeTile);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (transpose_vec4(R, C, src, es, dst, es)) {
    if (es == 4)
      msda::transpose4_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(src), static_cast<float*>(dst),
                                                          (int)R, (int)C, r_in_x);
    else
      msda::transpose4_kernel<unsigned short><<<grid, 256, 0, st>>>(
          static_cast<const unsigned short*>(src), static_cast<unsigned short*>(dst), (int)R, (int)C, r_in_x);
  } else if (es == 4) {
    msda::transpose_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(src), static_cast<float*>(dst), R, C,
                                                        r_in_x);
  } else {
    msda::transpose_kernel<unsigned short><<<grid, 256, 0, st>>>(static_cast<const unsigned short*>(src),
                                                               static_cast<unsigned short*>(dst), R, C, r_in_x);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "transpose launch");
  return succeed();
}

int msda_grid_sample_forward(const void* input, const void* grid, void* output, int64_t N, int64_t H,
                             int64_t W, int64_t C, int64_t out_h, int64_t out_w, int32_t mode,
                             int32_t padding_mode, int32_t align_corners, int32_t dtype, void* stream) {
  const char* fn = "msda_grid_sample_forward";
  const Dims d{N, H, W, C, N, out_h * out_w};
  if (out_h < 0 || out_w < 0) return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: negative output size", fn);
  if (int rc = check_dims(fn, d, dtype)) return rc;
  if (padding_mode < 0 || padding_mode > 2)
    return fail(MSDA_ERR_UNSUPPORTED, "%s: padding_mode %d not supported (0 = zeros, 1 = border, 2 = reflection)", fn, padding_mode);
  if (mode != 0 && mode != 1)
    return fail(MSDA_ERR_UNSUPPORTED, "%s: mode %d not supported (0 = bilinear, 1 = nearest)", fn, mode);
  if (d.R * d.Q == 0) return succeed();
  const int es = elem_size(dtype);
  if (!input || !grid || !output) return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: null pointer argument", fn);
  if (!aligned(input, es) || !aligned(output, es) || !aligned(grid, 2 * es))
    return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: misaligned buffer (grid needs %d-byte alignment)", fn, 2 * es);
  GatherParams p{};
  p.input = input;
  p.coords = grid;
  p.out = output;
  p.N = N; p.R = N; p.Q = d.Q;
  p.H = (int)H; p.W = (int)W; p.C = (int)C;
  p.padding = padding_mode;
  p.nearest = mode == 1;
  p.align = align_corners != 0;
  return forward(fn, Op::kGridSample, p, d, dtype, reinterpret_cast<cudaStream_t>(stream));
}

size_t msda_grid_sample_backward_workspace_size(int64_t N, int64_t H, int64_t W, int64_t C, int64_t out_h,
                                                int64_t out_w, int32_t dtype, uint32_t flags) {
  if (elem_size(dtype) == 0 || N < 0 || H < 1 || W < 1 || C < 1 || out_h < 0 || out_w < 0) return 0;
  return workspace_bytes_for(Dims{N, H, W, C, N, out_h * out_w}, dtype, flags);
}

int msda_grid_sample_backward(const void* input, const void* grid, const void* grad_output, void* grad_input,
                              void* grad_grid, void* workspace, size_t workspace_bytes, int64_t N, int64_t H,
                              int64_t W, int64_t C, int64_t out_h, int64_t out_w, int32_t mode,
                              int32_t padding_mode, int32_t align_corners, int32_t dtype, uint32_t flags,
                              void* stream) {
  const char* fn = "msda_grid_sample_backward";
  const Dims d{N, H, W, C, N, out_h * out_w};
  if (out_h < 0 || out_w < 0) return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: negative output size", fn);
  if (int rc = check_dims(fn, d, dtype)) return rc;
  if (padding_mode < 0 || padding_mode > 2)
    return fail(MSDA_ERR_UNSUPPORTED, "%s: padding_mode %d not supported (0 = zeros, 1 = border, 2 = reflection)", fn, padding_mode);
  if (mode != 0 && mode != 1)
    return fail(MSDA_ERR_UNSUPPORTED, "%s: mode %d not supported (0 = bilinear, 1 = nearest)", fn, mode);
  if (N == 0) return succeed();
  const int es = elem_size(dtype);
  if (!grad_input || (d.Q > 0 && (!input || !grid || !grad_output || !grad_grid)))
    return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: null pointer argument", fn);
  if (!aligned(grad_input, es) || (d.Q > 0 && (!aligned(input, es) || !aligned(grad_output, es) ||
                                               !aligned(grid, 2 * es) || !aligned(grad_grid, 2 * es))))
    return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: misaligned buffer (grid and grad_grid need %d-byte alignment)", fn, 2 * es);
  GatherParams p{};
  p.input = input;
  p.coords = grid;
  p.grad_out = grad_output;
  p.grad_grid = grad_grid;
  p.N = N; p.R = N; p.Q = d.Q;
  p.H = (int)H; p.W = (int)W; p.C = (int)C;
  p.padding = padding_mode;
  p.nearest = mode == 1;
  p.align = align_corners != 0;
  return backward(fn, Op::kGridSample, p, d, grad_input, workspace, workspace_bytes, dtype, flags,
                  reinterpret_cast<cudaStream_t>(stream));
}

static int roi_checks(const char* fn, const Dims& d, int32_t ph, int32_t pw, int32_t sampling_ratio,
                      int32_t dtype) {
  if (ph < 1 || pw < 1) return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: output size must be >= 1", fn);
  // The kernels walk at most kRoiMaxGrid samples per bin side; a larger
  // explicit ratio would be clamped and differ from torchvision.
  if (sampling_ratio > msda::kRoiMaxGrid)
    return fail(MSDA_ERR_UNSUPPORTED, "%s: sampling_ratio=%d exceeds %d", fn, sampling_ratio,
                msda::kRoiMaxGrid);
  return check_dims(fn, d, dtype);
}

int msda_roi_align_forward(const void* input, const float* rois, void* output, int64_t N, int64_t H,
                           int64_t W, int64_t C, int64_t num_rois, int32_t pooled_height,
                           int32_t pooled_width, float spatial_scale, int32_t sampling_ratio,
                           int32_t aligned_, int32_t dtype, void* stream) {
  const char* fn = "msda_roi_align_forward";
  const Dims d{N, H, W, C, num_rois, (int64_t)pooled_height * pooled_width};
  if (int rc = roi_checks(fn, d, pooled_height, pooled_width, sampling_ratio, dtype)) return rc;
  if (num_rois == 0) return succeed();
  const int es = elem_size(dtype);
  if (!input || !rois || !output) return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: null pointer argument", fn);
  if (!aligned(input, es) || !aligned(output, es) || !aligned(rois, 4))
    return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: misaligned buffer", fn);
  GatherParams p{};
  p.input = input;
  p.coords = rois;
  p.out = output;
  p.N = N; p.R = num_rois; p.Q = d.Q;
  p.H = (int)H; p.W = (int)W; p.C = (int)C;
  p.PH = pooled_height; p.PW = pooled_width;
  p.spatial_scale = spatial_scale;
  p.sampling_ratio = sampling_ratio;
  p.aligned = aligned_ != 0;
  return forward(fn, Op::kRoiAlign, p, d, dtype, reinterpret_cast<cudaStream_t>(stream));
}

size_t msda_roi_align_backward_workspace_size(int64_t N, int64_t H, int64_t W, int64_t C, int32_t dtype,
                                              uint32_t flags) {
  if (elem_size(dtype) == 0 || N < 0 || H < 1 || W < 1 || C < 1) return 0;
  return workspace_bytes_for(Dims{N, H, W, C, 0, 0}, dtype, flags);
}

int msda_roi_align_backward(const float* rois, const void* grad_output, void* grad_input, void* workspace,
                            size_t workspace_bytes, int64_t N, int64_t H, int64_t W, int64_t C,
                            int64_t num_rois, int32_t pooled_height, int32_t pooled_width,
                            float spatial_scale, int32_t sampling_ratio, int32_t aligned_, int32_t dtype,
                            uint32_t flags, void* stream) {
  const char* fn = "msda_roi_align_backward";
  const Dims d{N, H, W, C, num_rois, (int64_t)pooled_height * pooled_width};
  if (int rc = roi_checks(fn, d, pooled_height, pooled_width, sampling_ratio, dtype)) return rc;
  if (N == 0) return succeed();
  const int es = elem_size(dtype);
  if (!grad_input || (num_rois > 0 && (!rois || !grad_output)))
    return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: null pointer argument", fn);
  if (!aligned(grad_input, es) || (num_rois > 0 && (!aligned(grad_output, es) || !aligned(rois, 4))))
    return fail(MSDA_ERR_INVALID_ARGUMENT, "%s: misaligned buffer", fn);
  GatherParams p{};
  p.coords = rois;
  p.grad_out = grad_output;
  p.N = N; p.R = num_rois; p.Q = d.Q;
  p.H = (int)H; p.W = (int)W; p.C = (int)C;
  p.PH = pooled_height; p.PW = pooled_width;
  p.spatial_scale = spatial_scale;
  p.sampling_ratio = sampling_ratio;
  p.aligned = aligned_ != 0;
  return backward(fn, Op::kRoiAlign, p, d, grad_input, workspace, workspace_bytes, dtype, flags,
                  reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
