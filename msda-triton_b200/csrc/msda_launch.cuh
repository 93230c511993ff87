// Host-side launch helpers: pick a (VEC, LPR, CPL) instantiation for the
// head dim and dtype, and launch it on the caller's stream.
#pragma once

#include "msda_kernels.cuh"

namespace msda {

// VEC: elements per lane load (16 bytes, or 1 for the scalar path).
// LPR: lanes per corner row (power of two <= 32); CPL: chunks per lane.
struct Cfg {
  int vec;
  int lpr;
  int cpl;
  bool short_grid;  // the query-block grid is at most kShortGridWaves waves
};

// Forward grids of at most this many waves (at 4 CTAs per SM) use the
// register-richer forward variant.
constexpr int kShortGridWaves = 4;

// Launch `kernel` on `st`; with `pdl` the launch may overlap the tail of the
// kernel before it in the stream (programmatic stream serialization): the
// kernel must call pdl_wait() before it reads anything that kernel writes.
// Only for a kernel whose predecessor in the stream is one of ours.
template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                      bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

constexpr int kWarpsPerCta = 8;

template <typename T>
cudaError_t launch_forward(const OpParams& p, const Cfg& c, cudaStream_t st);

// Accumulator of the grad_value reductions.
enum AccKind : int {
  kAccNative = 0,  // the value dtype (packed f16x2 / bf16x2 `red`)
  kAccF32 = 1,     // fp32
  kAccFixed = 2,   // 64-bit fixed point (deterministic; needs p.fixed_hdr)
  kAccExact = 3,   // fp16 / bf16, hit-counted: fp32 rows of exact integer-valued sums (deterministic; needs p.rowmax)
};

// Backward over sampling points: grad_loc / grad_attn, plus the grad_value
// handling `mode` (ScatterMode): kScatter (kScatterMerge: after merging a
// warp's same-row contributions; vector path only) adds into p.grad_value
// (accumulator `acc`: fp32 for fp32 values whatever `acc` says, unless
// kAccFixed); kCounted stores one-hit rows and reduces multi-hit rows into
// p.acc (fp32, or fixed point with kAccFixed; needs the counts).
// `pdl`: the kernel before this one in the stream is our zero-fill, hit
// count or absmax pass (the backward waits for it only before its first
// count read / reduction).
template <typename T>
cudaError_t launch_backward(const OpParams& p, const Cfg& c, int mode, int acc, bool pdl,
                            cudaStream_t st);
// Hit-counted scatter passes 1 (count hits, zero the accumulators that will
// be reduced into) and 3 (zeros / downcast). p.counts must be zeroed before
// launch_count.
// `exact`: the kAccExact counting (every level, row bounds into p.rowmax,
// which must be zeroed too).
// `pdl`: the kernel before it is ours (the zero-fill of the counts or the
// absmax pass): the count pass loads and resolves its points under that
// kernel's tail and waits before its first count or accumulator write.
template <typename T>
cudaError_t launch_count(const OpParams& p, int num_sms, bool exact, bool pdl, cudaStream_t st);
template <typename T>
cudaError_t launch_finalize(const OpParams& p, bool vec_ok, bool fixed, bool exact, int num_sms, cudaStream_t st);
// Deterministic grad_value: the absmax header (pass 0; `pdl` when the kernel
// before it is our zero-fill) and the fixed-point -> dtype pass of the
// deterministic scatter.
template <typename T>
cudaError_t launch_absmax(const void* attn, int64_t n_attn, bool logits, const void* grad_out,
                          int64_t n_g, unsigned* hdr, int num_sms, bool pdl, cudaStream_t st);
template <typename T>
cudaError_t launch_cast_fixed(const long long* src, T* dst, int64_t n, bool vec_ok,
                              const unsigned* hdr, int clog2n, int num_sms, cudaStream_t st);

template <typename T>
cudaError_t launch_cast(const float* src, T* dst, int64_t n, bool vec_ok, int num_sms, cudaStream_t st);
// Zero `bytes` (a multiple of 16, 16-byte aligned) with L2 evict_last stores.
cudaError_t launch_zero(void* dst, size_t bytes, int num_sms, cudaStream_t st);

// ---------------------------------------------------------------------------
// Template dispatch (included by the per-dtype translation units only).
// ---------------------------------------------------------------------------
#ifdef MSDA_LAUNCH_IMPL

#define MSDA_FOR_EACH_SHAPE(X) \
  X(1, 1, 2)                   \
  X(2, 1, 2)                   \
  X(4, 1, 2)                   \
  X(8, 1, 2)                   \
  X(16, 1, 2)                  \
  X(32, 1, 2)                  \
  X(32, 2, 1)                  \
  X(32, 4, 1)

// Grid of the query-block kernels: (ceil(Q / kWarpsPerCta), M, B).
inline dim3 query_block_grid(const OpParams& p) {
  return dim3((unsigned)((p.Q + kWarpsPerCta - 1) / kWarpsPerCta), (unsigned)p.M, (unsigned)p.B);
}

// Forward launch shapes. Grids of at most kShortGridWaves waves (a decoder's
// few hundred queries per head) keep one query per warp in 8-warp CTAs with
// the register-rich budget (3 CTAs / SM) and NB points per group in flight.
// Longer grids (an encoder's query at every pixel) take 4-warp CTAs whose
// warps serve 2 queries at once over kLongRounds rounds of consecutive
// queries, one point per lane group per step (measured on B200: encoder
// forward 405 -> 332 us, Mask2Former 201 -> 139 us; the decoder is fastest
// with the short shape).
constexpr int kLongWarps = 4;
constexpr int kLongRounds = 4;

template <typename T, int VEC, int LPR, int CPL, int NB, bool FUSED>
static cudaError_t fwd_launch(const OpParams& p, bool short_grid, cudaStream_t st) {
  const dim3 grid_short = query_block_grid(p);
  if (short_grid) {
    if constexpr (VEC > 1)
      msda_fwd_kernel<T, VEC, LPR, CPL, kWarpsPerCta, NB, 3, FUSED><<<grid_short, kWarpsPerCta * 32, 0, st>>>(p);
    else
      msda_fwd_kernel<T, VEC, LPR, CPL, kWarpsPerCta, NB, 0, FUSED><<<grid_short, kWarpsPerCta * 32, 0, st>>>(p);
    return cudaGetLastError();
  }
  constexpr int QW = (FUSED || LPR == 32) ? 1 : 2;
  constexpr int NBL = FUSED ? NB : 1;
  constexpr int per_cta = kLongWarps * QW * kLongRounds;
  const dim3 grid((unsigned)((p.Q + per_cta - 1) / per_cta), (unsigned)p.M, (unsigned)p.B);
  // When the warp's queries have at most 32 points between them, each lane
  // resolves one point per round and the lane groups fetch it by shuffle
  // (measured: encoder forward 351 -> 299 us, Mask2Former 150 -> 129 us).
  if constexpr (!FUSED) {
    if (QW * p.L * p.K <= 32) {
      msda_fwd_kernel<T, VEC, LPR, CPL, kLongWarps, 1, 0, false, QW, kLongRounds, true>
          <<<grid, kLongWarps * 32, 0, st>>>(p);
      return cudaGetLastError();
    }
  }
  msda_fwd_kernel<T, VEC, LPR, CPL, kLongWarps, NBL, 0, FUSED, QW, kLongRounds><<<grid, kLongWarps * 32, 0, st>>>(p);
  return cudaGetLastError();
}

template <typename T, int VEC, bool FUSED = false>
static cudaError_t fwd_by_shape(const OpParams& p, const Cfg& c, cudaStream_t st) {
#define MSDA_FWD_CASE(LPR_, CPL_, NB_) \
  if (c.lpr == LPR_ && c.cpl == CPL_) return fwd_launch<T, VEC, LPR_, CPL_, NB_, FUSED>(p, c.short_grid, st);
  MSDA_FOR_EACH_SHAPE(MSDA_FWD_CASE)
#undef MSDA_FWD_CASE
  return cudaErrorInvalidConfiguration;
}

// Backward launch shapes. The hit-counted mode (sparse sampling), the fused
// prologue and short grids keep one query per warp in 8-warp CTAs. Long
// grids of the scatter modes on the 16-byte vector path take the forward's
// long shape -- 4-warp CTAs, 2 queries per warp, kLongRounds rounds of
// consecutive queries (measured on B200: encoder fp32-accumulation backward
// 1005 -> 853 us, Mask2Former 465 -> 333 us).
template <typename T, typename A, int VEC, int LPR, int CPL, int MODE, bool FUSED>
static cudaError_t bwd_launch(const OpParams& p, bool short_grid, bool pdl, cudaStream_t st) {
  constexpr bool kLongOk = !FUSED && MODE != kCounted && VEC * sizeof(T) == 16 && LPR <= 16;
  if constexpr (kLongOk) {
    if (!short_grid) {
      constexpr int per_cta = kLongWarps * 2 * kLongRounds;
      const dim3 grid((unsigned)((p.Q + per_cta - 1) / per_cta), (unsigned)p.M, (unsigned)p.B);
      // Points shared by lane when the warp's 2 queries have at most 32
      // (encoder fp32 backward 851 -> 836 us, native 828 -> 800 us).
      if (2 * p.L * p.K <= 32)
        return launch_ex(msda_bwd_kernel<T, A, VEC, LPR, CPL, kLongWarps, 1, MODE, false, 2, kLongRounds, true>,
                         grid, dim3(kLongWarps * 32), 0, st, pdl, p);
      return launch_ex(msda_bwd_kernel<T, A, VEC, LPR, CPL, kLongWarps, 1, MODE, false, 2, kLongRounds>, grid,
                       dim3(kLongWarps * 32), 0, st, pdl, p);
    }
  }
  // One point per group in flight (NB = 1): the backward's per-point state
  // (gradients, weights, scatter operands) makes NB = 2 cost occupancy.
  return launch_ex(msda_bwd_kernel<T, A, VEC, LPR, CPL, kWarpsPerCta, 1, MODE, FUSED>, query_block_grid(p),
                   dim3(kWarpsPerCta * 32), 0, st, pdl, p);
}

template <typename T, typename A, int VEC, int MODE, bool FUSED = false>
static cudaError_t bwd_by_shape(const OpParams& p, const Cfg& c, bool pdl, cudaStream_t st) {
#define MSDA_BWD_CASE(LPR_, CPL_, NB_) \
  if (c.lpr == LPR_ && c.cpl == CPL_) return bwd_launch<T, A, VEC, LPR_, CPL_, MODE, FUSED>(p, c.short_grid, pdl, st);
  MSDA_FOR_EACH_SHAPE(MSDA_BWD_CASE)
#undef MSDA_BWD_CASE
  return cudaErrorInvalidConfiguration;
}

template <typename T>
cudaError_t launch_forward(const OpParams& p, const Cfg& c, cudaStream_t st) {
  constexpr int V16 = 16 / (int)sizeof(T);
  if (p.fused) return c.vec == V16 ? fwd_by_shape<T, V16, true>(p, c, st) : cudaErrorNotSupported;
  if (c.vec == V16) return fwd_by_shape<T, V16>(p, c, st);
  if (c.vec == 1) return fwd_by_shape<T, 1>(p, c, st);
  return cudaErrorInvalidConfiguration;
}

template <typename T>
cudaError_t launch_backward(const OpParams& p, const Cfg& c, int mode, int acc, bool pdl,
                            cudaStream_t st) {
  constexpr int V16 = 16 / (int)sizeof(T);
  const bool fp32_scatter = acc == kAccF32;
  if (acc == kAccExact) {
    if constexpr (sizeof(T) == 2) {
      if (mode != kCounted) return cudaErrorNotSupported;
      if (p.fused)
        return c.vec == V16 ? bwd_by_shape<T, ExactF32, V16, kCounted, true>(p, c, pdl, st) : cudaErrorNotSupported;
      if (c.vec == V16) return bwd_by_shape<T, ExactF32, V16, kCounted>(p, c, pdl, st);
      if (c.vec == 1) return bwd_by_shape<T, ExactF32, 1, kCounted>(p, c, pdl, st);
      return cudaErrorInvalidConfiguration;
    }
    return cudaErrorNotSupported;
  }
  if (acc == kAccFixed) {
    using F = long long;
    if (mode == kNoScatter) return cudaErrorNotSupported;
    if (p.fused) {  // vector path only
      if (c.vec != V16) return cudaErrorNotSupported;
      if (mode == kCounted) return bwd_by_shape<T, F, V16, kCounted, true>(p, c, pdl, st);
      return mode == kScatterMerge ? bwd_by_shape<T, F, V16, kScatterMerge, true>(p, c, pdl, st)
                                   : bwd_by_shape<T, F, V16, kScatter, true>(p, c, pdl, st);
    }
    if (c.vec == V16) {
      if (mode == kCounted) return bwd_by_shape<T, F, V16, kCounted>(p, c, pdl, st);
      return mode == kScatterMerge ? bwd_by_shape<T, F, V16, kScatterMerge>(p, c, pdl, st)
                                   : bwd_by_shape<T, F, V16, kScatter>(p, c, pdl, st);
    }
    if (c.vec == 1)
      return mode == kCounted ? bwd_by_shape<T, F, 1, kCounted>(p, c, pdl, st)
                              : bwd_by_shape<T, F, 1, kScatter>(p, c, pdl, st);
    return cudaErrorInvalidConfiguration;
  }
  if (p.fused) {  // vector path only
    if (c.vec != V16 || mode == kNoScatter) return cudaErrorNotSupported;
    if (mode == kCounted) return bwd_by_shape<T, T, V16, kCounted, true>(p, c, pdl, st);
    if (fp32_scatter || sizeof(T) == 4)
      return mode == kScatterMerge ? bwd_by_shape<T, float, V16, kScatterMerge, true>(p, c, pdl, st)
                                   : bwd_by_shape<T, float, V16, kScatter, true>(p, c, pdl, st);
    return mode == kScatterMerge ? bwd_by_shape<T, T, V16, kScatterMerge, true>(p, c, pdl, st)
                                 : bwd_by_shape<T, T, V16, kScatter, true>(p, c, pdl, st);
  }
  if (mode == kNoScatter) return cudaErrorNotSupported;
  if (mode == kCounted) {
    if (c.vec == V16) return bwd_by_shape<T, T, V16, kCounted>(p, c, pdl, st);
    if (c.vec == 1) return bwd_by_shape<T, T, 1, kCounted>(p, c, pdl, st);
  } else if (fp32_scatter || sizeof(T) == 4) {
    if (c.vec == V16 && mode == kScatterMerge) return bwd_by_shape<T, float, V16, kScatterMerge>(p, c, pdl, st);
    if (c.vec == V16) return bwd_by_shape<T, float, V16, kScatter>(p, c, pdl, st);
    if (c.vec == 1) return bwd_by_shape<T, float, 1, kScatter>(p, c, pdl, st);
  } else {
    if (c.vec == V16 && mode == kScatterMerge) return bwd_by_shape<T, T, V16, kScatterMerge>(p, c, pdl, st);
    if (c.vec == V16) return bwd_by_shape<T, T, V16, kScatter>(p, c, pdl, st);
    if (c.vec == 1) return bwd_by_shape<T, T, 1, kScatter>(p, c, pdl, st);
  }
  return cudaErrorInvalidConfiguration;
}

template <typename T>
cudaError_t launch_count(const OpParams& p, int num_sms, bool exact, bool pdl, cudaStream_t st) {
  const int64_t n = p.BQM * p.L * p.K;
  const int64_t point_blocks = (n + 255) / 256;
  // The dense rows are not known on the host (the level table is on the
  // device; one warp per dense pixel row, grid-stride): the blocks that the
  // point blocks leave free in one wave, at least one per SM.
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, msda_count_kernel<T>, 256, 0) != cudaSuccess)
    per_sm = 4;
  const int64_t dense_blocks = std::max<int64_t>(num_sms, (int64_t)per_sm * num_sms - point_blocks);
  if (point_blocks + dense_blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
  const dim3 grid((unsigned)(point_blocks + dense_blocks));
  const unsigned pb = (unsigned)point_blocks;
  if (exact) {
    if constexpr (sizeof(T) == 2) {
      if (p.fused) return launch_ex(msda_count_kernel<T, true, true>, grid, dim3(256), 0, st, pdl, p, pb);
      return launch_ex(msda_count_kernel<T, false, true>, grid, dim3(256), 0, st, pdl, p, pb);
    }
    return cudaErrorNotSupported;
  }
  if (p.fused) return launch_ex(msda_count_kernel<T, true>, grid, dim3(256), 0, st, pdl, p, pb);
  return launch_ex(msda_count_kernel<T>, grid, dim3(256), 0, st, pdl, p, pb);
}

template <typename T>
cudaError_t launch_finalize(const OpParams& p, bool vec_ok, bool fixed, bool exact, int num_sms, cudaStream_t st) {
  constexpr int V16 = 16 / (int)sizeof(T);
  const int64_t rows = p.B * p.S * p.M;
  const int vec = (vec_ok && p.D % V16 == 0 && p.D % 4 == 0) ? V16 : 1;
  const int64_t n = (rows + 3) / 4 * (p.D / vec);
  // One thread per 4 rows x VEC elements (a one-wave grid-stride variant
  // measured slower behind the backward's programmatic launch).
  (void)num_sms;
  const int64_t blocks = (n + 255) / 256;
  // The backward runs right before: overlap its tail (the finalize waits).
  const dim3 grid((unsigned)std::max<int64_t>(blocks, 1));
  if (fixed) {
    if (vec == V16) return launch_ex(msda_finalize_kernel<T, V16, true>, grid, dim3(256), 0, st, true, p);
    return launch_ex(msda_finalize_kernel<T, 1, true>, grid, dim3(256), 0, st, true, p);
  }
  if (exact) {
    if constexpr (sizeof(T) == 2) {
      if (vec == V16) return launch_ex(msda_finalize_kernel<T, V16, false, true>, grid, dim3(256), 0, st, true, p);
      return launch_ex(msda_finalize_kernel<T, 1, false, true>, grid, dim3(256), 0, st, true, p);
    }
    return cudaErrorNotSupported;
  }
  if (vec == V16) return launch_ex(msda_finalize_kernel<T, V16>, grid, dim3(256), 0, st, true, p);
  return launch_ex(msda_finalize_kernel<T, 1>, grid, dim3(256), 0, st, true, p);
}

template <typename T>
cudaError_t launch_absmax(const void* attn, int64_t n_attn, bool logits, const void* grad_out,
                          int64_t n_g, unsigned* hdr, int num_sms, bool pdl, cudaStream_t st) {
  constexpr int V16 = 16 / (int)sizeof(T);
  const int64_t longest = std::max(n_attn, n_g) / V16 + 1;
  const int64_t blocks = std::min<int64_t>((int64_t)num_sms * 4, (longest + 255) / 256);
  return launch_ex(msda_absmax_kernel<T>, dim3((unsigned)std::max<int64_t>(blocks, 1)), dim3(256), 0,
                   st, pdl, static_cast<const T*>(attn), n_attn, logits ? 1 : 0,
                   static_cast<const T*>(grad_out), n_g, hdr);
}

template <typename T>
cudaError_t launch_cast_fixed(const long long* src, T* dst, int64_t n, bool vec_ok,
                              const unsigned* hdr, int clog2n, int num_sms, cudaStream_t st) {
  constexpr int V16 = 16 / (int)sizeof(T);
  const int64_t max_blocks = (int64_t)num_sms * 8;
  // The backward runs right before: overlap its tail (the pass waits).
  if (vec_ok && n % V16 == 0) {
    const int64_t nvec = n / V16;
    const int64_t blocks = std::min<int64_t>(max_blocks, (nvec + 255) / 256);
    return launch_ex(msda_cast_fixed_kernel<T, V16>, dim3((unsigned)std::max<int64_t>(blocks, 1)),
                     dim3(256), 0, st, true, src, dst, nvec, hdr, clog2n);
  }
  const int64_t blocks = std::min<int64_t>(max_blocks, (n + 255) / 256);
  return launch_ex(msda_cast_fixed_kernel<T, 1>, dim3((unsigned)std::max<int64_t>(blocks, 1)), dim3(256),
                   0, st, true, src, dst, n, hdr, clog2n);
}

template <typename T>
cudaError_t launch_cast(const float* src, T* dst, int64_t n, bool vec_ok, int num_sms, cudaStream_t st) {
  constexpr int V16 = 16 / (int)sizeof(T);
  const int64_t max_blocks = (int64_t)num_sms * 8;
  // The backward runs right before: overlap its tail (the cast waits).
  if (vec_ok && n % V16 == 0) {
    const int64_t nvec = n / V16;
    const int64_t blocks = std::min<int64_t>(max_blocks, (nvec + 255) / 256);
    return launch_ex(msda_cast_kernel<T, V16>, dim3((unsigned)std::max<int64_t>(blocks, 1)), dim3(256),
                     0, st, true, src, dst, nvec);
  }
  const int64_t blocks = std::min<int64_t>(max_blocks, (n + 255) / 256);
  return launch_ex(msda_cast_kernel<T, 1>, dim3((unsigned)std::max<int64_t>(blocks, 1)), dim3(256), 0,
                   st, true, src, dst, n);
}

#endif  // MSDA_LAUNCH_IMPL

#ifdef MSDA_LAUNCH_ZERO_IMPL
cudaError_t launch_zero(void* dst, size_t bytes, int num_sms, cudaStream_t st) {
  const int64_t n16 = (int64_t)(bytes / 16);
  if (n16 == 0) return cudaSuccess;
  const int64_t blocks = std::min<int64_t>((int64_t)num_sms * 8, (n16 + 255) / 256);
  msda_zero_kernel<0><<<(unsigned)std::max<int64_t>(blocks, 1), 256, 0, st>>>(dst, n16);
  return cudaGetLastError();
}
#endif  // MSDA_LAUNCH_ZERO_IMPL

#ifdef MSDA_LAUNCH_IMPL
#define MSDA_INSTANTIATE(T)                                                                       \
  template cudaError_t launch_forward<T>(const OpParams&, const Cfg&, cudaStream_t);              \
  template cudaError_t launch_backward<T>(const OpParams&, const Cfg&, int, int, bool, cudaStream_t); \
  template cudaError_t launch_count<T>(const OpParams&, int, bool, bool, cudaStream_t);             \
  template cudaError_t launch_finalize<T>(const OpParams&, bool, bool, bool, int, cudaStream_t);  \
  template cudaError_t launch_absmax<T>(const void*, int64_t, bool, const void*, int64_t, unsigned*, int, bool, cudaStream_t); \
  template cudaError_t launch_cast_fixed<T>(const long long*, T*, int64_t, bool, const unsigned*, int, int, cudaStream_t); \
  template cudaError_t launch_cast<T>(const float*, T*, int64_t, bool, int, cudaStream_t);

#endif  // MSDA_LAUNCH_IMPL

}  // namespace msda
