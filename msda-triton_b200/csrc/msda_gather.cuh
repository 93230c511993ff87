// Sibling gathers on the MSDA kernel skeleton: grid_sample (bilinear) and
// ROI-Align, forward and backward, channels-last.
//
// Both operators have MSDA's anatomy -- data-dependent bilinear gathers of
// channel rows forward, atomic scatters backward -- so they reuse its
// building blocks: a lane group of LPR lanes owns one output row (an output
// pixel, an ROI bin) and covers its C channels with 16-byte vectors (VEC
// elements, CPL chunks per lane), every corner gather is LPR x 16 B of
// consecutive bytes, parameters are read once per group, accumulation is in
// fp32 registers, and the backward scatter takes the MSDA accumulators: fp32
// (interleaved quads for 16-bit data), native packed 16-bit, or the
// deterministic 64-bit fixed point of msda_common.cuh. A CTA is 8 warps of
// 32 / LPR groups each.
//
// Semantics follow the public operators they replace:
// * grid_sample: torch.nn.functional.grid_sample(mode "bilinear" or
//   "nearest", padding_mode "zeros", "border" or "reflection",
//   align_corners) on NHWC data; the source coordinate is
//   ((g + 1) * size - 1) / 2 (align_corners=False) or (g + 1) / 2 * (size - 1)
//   (True); "border" clips it to [0, size - 1] and zeroes the grid gradient
//   where it clips; "reflection" first reflects it about the borders (at
//   -0.5 and size - 0.5, or at 0 and size - 1 with align_corners; the grid
//   gradient flips sign on reflected segments), then clips; "zeros"
//   samples 0 outside. "nearest" reads the pixel at the coordinate rounded
//   half to even; its grid gradient is zero.
// * ROI-Align: torchvision.ops.roi_align (Mask R-CNN's RoIAlign): each
//   output bin averages a grid of sampling points (sampling_ratio per bin
//   side, or ceil(roi size / bins) when sampling_ratio <= 0); a point more
//   than one pixel outside the map contributes 0, otherwise it is clamped
//   to the map and interpolated bilinearly; `aligned` shifts boxes by -0.5
//   pixel. No gradient flows to the boxes. (One bound torchvision has not:
//   at most 1024 sampling points per bin side.)
#pragma once

#include "msda_common.cuh"

namespace msda {

constexpr int kGatherWarps = 8;

struct GatherParams {
  const void* input;   // (N, H*W, C)
  const void* coords;  // grid_sample: grid (N, Q, 2); roi_align: rois (K, 5) fp32
  void* out;           // (N or K, Q, C)
  const void* grad_out;
  void* grad_in;       // scatter target (N, H*W, C): value dtype, fp32 or 64-bit fixed point
  void* grad_grid;     // grid_sample: (N, Q, 2)
  int64_t N;           // batch items of the input
  int64_t R, Q;        // output items (grid_sample: N; roi_align: ROIs), output rows per item
  int H, W, C;
  // grid_sample
  int padding;         // 0 "zeros", 1 "border", 2 "reflection"
  int nearest;         // mode == "nearest" (else bilinear)
  int align;           // align_corners
  // roi_align
  int PH, PW;          // output bins (Q = PH * PW)
  float spatial_scale;
  int sampling_ratio;
  int aligned;
  // deterministic accumulation
  const unsigned* fixed_hdr;
  int fixed_log2n;
};

// ---------------------------------------------------------------------------
// grid_sample: one output pixel -> a Bilinear on the (single-level) input
// ---------------------------------------------------------------------------
struct GridPoint {
  Bilinear bl;
  float dx, dy;  // d(pixel coordinate) / d(grid coordinate); 0 where a border clips
};

// Clip to [0, size - 1]; the gradient through a clipped coordinate is 0.
__device__ __forceinline__ float gs_clip(float x, int size, float& d) {
  const float hi = (float)(size - 1);
  if (x <= 0.f) {
    d = 0.f;
    return 0.f;
  }
  if (x >= hi) {
    d = 0.f;
    return hi;
  }
  return x;
}

// Reflect about the borders at twice_lo / 2 and twice_hi / 2 (a coordinate
// past one border comes back from it); d flips sign on reflected segments.
__device__ __forceinline__ float gs_reflect(float x, int twice_lo, int twice_hi, float& d) {
  if (twice_lo == twice_hi) {
    d = 0.f;
    return 0.f;
  }
  const float lo = (float)twice_lo * 0.5f, span = (float)(twice_hi - twice_lo) * 0.5f;
  x -= lo;
  if (x < 0.f) {
    d = -d;
    x = -x;
  }
  const float extra = fmodf(x, span);
  const int flips = (int)floorf(x / span);
  if (flips % 2 == 0) return extra + lo;
  d = -d;
  return span - extra + lo;
}

// torch's source-index computation: unnormalise, then clip ("border") or
// reflect and clip ("reflection"). d = d(coordinate) / d(grid value).
__device__ __forceinline__ float gs_source(float g, int size, int align, int padding, float& d) {
  float x;
  if (align) {
    x = ((g + 1.f) * 0.5f) * (float)(size - 1);
    d = 0.5f * (float)(size - 1);
  } else {
    x = ((g + 1.f) * (float)size - 1.f) * 0.5f;
    d = 0.5f * (float)size;
  }
  if (padding == 2) {
    // A NaN coordinate stays NaN (the bilinear / nearest resolution sends it
    // outside: it samples nothing); |x| <= 1e9 keeps the reflection's flip
    // count within int range (span >= 1 pixel whenever size > 1).
    if (!(x == x)) return x;
    x = fminf(fmaxf(x, -1.0e9f), 1.0e9f);
    x = align ? gs_reflect(x, 0, 2 * (size - 1), d) : gs_reflect(x, -1, 2 * size - 1, d);
    x = gs_clip(x, size, d);
  } else if (padding == 1) {
    x = gs_clip(x, size, d);
  }
  return x;
}

template <typename T>
__device__ __forceinline__ GridPoint grid_point(const GatherParams& p, int64_t row) {
  const float2 g = load_pair(reinterpret_cast<const T*>(p.coords) + 2 * row);
  GridPoint r;
  const float x = gs_source(g.x, p.W, p.align, p.padding, r.dx);
  const float y = gs_source(g.y, p.H, p.align, p.padding, r.dy);
  if (p.nearest) {
    // The pixel at the coordinate rounded half to even, as one corner of
    // weight 1 (the clamp keeps the integer conversion defined for NaN /
    // huge coordinates, all of which land outside).
    const float xr = rintf(fminf(fmaxf(x, -2.0f), (float)p.W + 1.0f));
    const float yr = rintf(fminf(fmaxf(y, -2.0f), (float)p.H + 1.0f));
    const int xi = (int)xr, yi = (int)yr;
    r.bl = empty_slot();
    r.bl.valid = ((unsigned)xi < (unsigned)p.W && (unsigned)yi < (unsigned)p.H) ? 1u : 0u;
    r.bl.pix[0] = r.bl.valid ? yi * p.W + xi : 0;
    r.bl.w[0] = 1.f;
    r.dx = r.dy = 0.f;  // piecewise constant in the grid
    return r;
  }
  LevelInfo L;
  L.H = p.H;
  L.W = p.W;
  L.start = 0;
  L.fH = (float)p.H;
  L.fW = (float)p.W;
  L.dense = 0;
  r.bl = resolve_px(x, y, L);
  return r;
}

// ---------------------------------------------------------------------------
// ROI-Align: one sampling point of one bin -> 4 weighted pixels
// (torchvision's bilinear_interpolate; clamped corners may coincide).
// ---------------------------------------------------------------------------
constexpr int kRoiMaxGrid = 1024;

struct RoiBin {
  int n;             // batch item of the ROI
  float y0, x0;      // bin origin: roi start + bin index * bin size
  float bh, bw;      // bin size
  int gh, gw;        // sampling grid of the bin
  float count;       // max(gh * gw, 1)
};

__device__ __forceinline__ RoiBin roi_bin(const GatherParams& p, int64_t row) {
  const int64_t k = row / p.Q;
  const int q = (int)(row - k * p.Q);
  const int ph = q / p.PW, pw = q - ph * p.PW;
  const float* r = reinterpret_cast<const float*>(p.coords) + 5 * k;
  const float off = p.aligned ? 0.5f : 0.f;
  const float x1 = r[1] * p.spatial_scale - off, y1 = r[2] * p.spatial_scale - off;
  const float x2 = r[3] * p.spatial_scale - off, y2 = r[4] * p.spatial_scale - off;
  float rw = x2 - x1, rh = y2 - y1;
  if (!p.aligned) {
    rw = fmaxf(rw, 1.f);
    rh = fmaxf(rh, 1.f);
  }
  const float bh = rh / (float)p.PH, bw = rw / (float)p.PW;
  RoiBin b;
  b.n = (int)r[0];
  b.gh = p.sampling_ratio > 0 ? p.sampling_ratio : (int)ceilf(rh / (float)p.PH);
  b.gw = p.sampling_ratio > 0 ? p.sampling_ratio : (int)ceilf(rw / (float)p.PW);
  // At most kRoiMaxGrid samples per bin side: a non-finite or absurdly large
  // box (bins wider than kRoiMaxGrid pixels with sampling_ratio <= 0) must
  // not turn into an unbounded loop.
  b.gh = min(max(b.gh, 0), kRoiMaxGrid);
  b.gw = min(max(b.gw, 0), kRoiMaxGrid);
  b.count = (float)max(b.gh * b.gw, 1);
  b.y0 = y1 + (float)ph * bh;
  b.x0 = x1 + (float)pw * bw;
  b.bh = bh;
  b.bw = bw;
  return b;
}

// Sample (iy, ix) of a bin: y = y1 + ph * bin_h + (iy + 0.5) * bin_h / gh.
__device__ __forceinline__ Bilinear roi_point(const GatherParams& p, const RoiBin& b, int iy, int ix) {
  float y = b.y0 + ((float)iy + 0.5f) * b.bh / (float)b.gh;
  float x = b.x0 + ((float)ix + 0.5f) * b.bw / (float)b.gw;
  Bilinear r;
  r.lx = r.ly = 0.f;
  if (y < -1.f || y > (float)p.H || x < -1.f || x > (float)p.W || !(y == y) || !(x == x)) {
    r.valid = 0u;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      r.pix[c] = 0;
      r.w[c] = 0.f;
    }
    return r;
  }
  if (y <= 0.f) y = 0.f;
  if (x <= 0.f) x = 0.f;
  int ylo = (int)y, xlo = (int)x, yhi, xhi;
  if (ylo >= p.H - 1) {
    yhi = ylo = p.H - 1;
    y = (float)ylo;
  } else {
    yhi = ylo + 1;
  }
  if (xlo >= p.W - 1) {
    xhi = xlo = p.W - 1;
    x = (float)xlo;
  } else {
    xhi = xlo + 1;
  }
  const float ly = y - (float)ylo, lx = x - (float)xlo, hy = 1.f - ly, hx = 1.f - lx;
  r.pix[0] = ylo * p.W + xlo;
  r.pix[1] = ylo * p.W + xhi;
  r.pix[2] = yhi * p.W + xlo;
  r.pix[3] = yhi * p.W + xhi;
  r.w[0] = hy * hx;
  r.w[1] = hy * lx;
  r.w[2] = ly * hx;
  r.w[3] = ly * lx;
  r.valid = 0xfu;
  return r;
}

// Output row handled by this lane group; rows past `rows` are idle groups.
template <int LPR>
__device__ __forceinline__ int64_t gather_row() {
  constexpr int G = 32 / LPR;
  const int lane = threadIdx.x & 31;
  return ((int64_t)blockIdx.x * kGatherWarps + (threadIdx.x >> 5)) * G + lane / LPR;
}

// Accumulates w * row[ch..] of the 4 corners of `bl` (rows of `vb`, C
// elements apart) into acc.
template <typename T, int VEC, int LPR, int CPL>
__device__ __forceinline__ void gather_corners(const T* vb, int C, int sub, const Bilinear& bl, float scale,
                                               float (&acc)[CPL][VEC]) {
  using Raw = typename Pack<T, VEC>::Raw;
  Raw raw[4][CPL];
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      const int ch = (j * LPR + sub) * VEC;
      Raw r{};
      if (((bl.valid >> c) & 1u) && ch < C) r = load_raw<T, VEC>(vb + (int64_t)bl.pix[c] * C + ch);
      raw[c][j] = r;
    }
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const float wc = bl.w[c] * scale;
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      float v[VEC];
      unpack_raw<T, VEC>(raw[c][j], v);
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc[j][e] = fmaf(wc, v[e], acc[j][e]);
    }
  }
}

template <typename T, int VEC, int LPR, int CPL>
__device__ __forceinline__ void store_row(T* dst, int C, int sub, const float (&acc)[CPL][VEC]) {
#pragma unroll
  for (int j = 0; j < CPL; ++j) {
    const int ch = (j * LPR + sub) * VEC;
    if (ch < C) store_vec<T, VEC>(dst + ch, acc[j]);
  }
}

// ---------------------------------------------------------------------------
// The backward scatter of one output row's gradient g (this lane's channels)
// into input rows, for every accumulator type. Holds g in the orders the
// reductions want: natural (VEC consecutive channels per chunk), interleaved
// quads (fp32 reductions of 16-bit data: two neighbouring lanes fill a
// 32-byte sector) and interleaved scalars (8-byte fixed-point reductions:
// four lanes fill a sector).
// ---------------------------------------------------------------------------
template <typename T, typename A, int VEC, int LPR, int CPL>
struct RowScatter {
  static constexpr bool FIXED = IsFixed<A>::value;
  static constexpr bool QUADS = sizeof(T) == 2 && VEC == 8 && !FIXED && sizeof(A) == 4;
  float g[CPL][VEC];
  float gq[QUADS ? CPL : 1][2][4];
  float gi[FIXED ? CPL : 1][FIXED ? VEC : 1];
  int sub, C;
  uint64_t pol;
  FixedScale fx;

  __device__ __forceinline__ void load(const T* gp, bool live, int sub_, int C_) {
    sub = sub_;
    C = C_;
    pol = policy_evict_last();
    fx = FixedScale{1.0, 1.f, 1.f, true};
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      const int ch = (j * LPR + sub) * VEC;
      if (live && ch < C) {
        load_vec<T, VEC>(gp + ch, g[j]);
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) g[j][e] = 0.f;
      }
    }
    if constexpr (QUADS) {
#pragma unroll
      for (int j = 0; j < CPL; ++j)
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const int cq = j * LPR * VEC + (k * LPR + sub) * 4;
          if (live && cq < C) {
            load_vec<T, 4>(gp + cq, gq[j][k]);
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) gq[j][k][e] = 0.f;
          }
        }
    }
    if constexpr (FIXED) {
#pragma unroll
      for (int j = 0; j < CPL; ++j)
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
          const int ci = j * LPR * VEC + k * LPR + sub;
          gi[j][k] = (live && ci < C) ? to_f32(gp[ci]) : 0.f;
        }
    }
  }

  // After the producer of the accumulator's header (pdl_wait) has finished.
  __device__ __forceinline__ void set_scale(const unsigned* hdr, int clog2n) {
    if constexpr (FIXED) fx = fixed_scale(hdr, clog2n);
  }

  // row[...] += wc * g
  __device__ __forceinline__ void add(A* row, float wc) const {
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      if constexpr (FIXED) {
        long long* r = reinterpret_cast<long long*>(row);
        if (fx.ok) {
          const double wd = (double)wc * fx.scale;
#pragma unroll
          for (int k = 0; k < VEC; ++k) {
            const int ci = j * LPR * VEC + k * LPR + sub;
            if (ci < C) red_fixed(r + ci, wd, (double)gi[j][k], pol);
          }
        } else {
#pragma unroll
          for (int k = 0; k < VEC; ++k) {
            const int ci = j * LPR * VEC + k * LPR + sub;
            if (ci < C) atomicAdd(reinterpret_cast<float*>(r + ci), wc * gi[j][k]);
          }
        }
      } else if constexpr (QUADS) {
        float* r = reinterpret_cast<float*>(row);
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const int cq = j * LPR * VEC + (k * LPR + sub) * 4;
          if (cq < C)
            red_add_f32x4_hint(r + cq, wc * gq[j][k][0], wc * gq[j][k][1], wc * gq[j][k][2], wc * gq[j][k][3],
                               pol);
        }
      } else {
        const int ch = (j * LPR + sub) * VEC;
        if (ch < C) {
          float contrib[VEC];
#pragma unroll
          for (int e = 0; e < VEC; ++e) contrib[e] = wc * g[j][e];
          red_add_vec_hint<A, VEC>(row + ch, contrib, pol);
        }
      }
    }
  }
};

// ---------------------------------------------------------------------------
// grid_sample forward / backward
// ---------------------------------------------------------------------------
template <typename T, int VEC, int LPR, int CPL>
__global__ void __launch_bounds__(kGatherWarps * 32) gs_fwd_kernel(const GatherParams p) {
  const int64_t row = gather_row<LPR>();
  if (row >= p.R * p.Q) return;  // whole lane groups; no shuffles follow
  const int sub = (threadIdx.x & 31) % LPR;
  const int64_t n = row / p.Q;
  const GridPoint pt = grid_point<T>(p, row);
  float acc[CPL][VEC];
#pragma unroll
  for (int j = 0; j < CPL; ++j)
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[j][e] = 0.f;
  gather_corners<T, VEC, LPR, CPL>(reinterpret_cast<const T*>(p.input) + n * p.H * p.W * p.C, p.C, sub,
                                   pt.bl, 1.f, acc);
  store_row<T, VEC, LPR, CPL>(reinterpret_cast<T*>(p.out) + row * p.C, p.C, sub, acc);
}

// grad_grid: the bilinear derivative dotted with grad_out over the channels
// (reduced across the group's lanes); grad_input: w_c * grad_out scattered
// into the 4 corner rows.
template <typename T, typename A, int VEC, int LPR, int CPL>
__global__ void __launch_bounds__(kGatherWarps * 32) gs_bwd_kernel(const GatherParams p) {
  using Raw = typename Pack<T, VEC>::Raw;
  pdl_trigger();
  const int64_t row_raw = gather_row<LPR>();
  const bool live = row_raw < p.R * p.Q;  // idle groups stay for the shuffles
  const int64_t row = live ? row_raw : 0;
  const int sub = (threadIdx.x & 31) % LPR;
  const int64_t n = row / p.Q;
  const int C = p.C;
  const int64_t img = n * p.H * p.W * C;
  GridPoint pt = grid_point<T>(p, row);
  if (!live) pt.bl = empty_slot();
  RowScatter<T, A, VEC, LPR, CPL> sc;
  sc.load(reinterpret_cast<const T*>(p.grad_out) + row * C, live, sub, C);
  const T* vb = reinterpret_cast<const T*>(p.input) + img;
  Raw raw[4][CPL];
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      const int ch = (j * LPR + sub) * VEC;
      Raw r{};
      if (((pt.bl.valid >> c) & 1u) && ch < C) r = load_raw<T, VEC>(vb + (int64_t)pt.bl.pix[c] * C + ch);
      raw[c][j] = r;
    }
  float P[4] = {0.f, 0.f, 0.f, 0.f};  // P_c = sum_d g_d * v_c,d
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      float v[VEC];
      unpack_raw<T, VEC>(raw[c][j], v);
#pragma unroll
      for (int e = 0; e < VEC; ++e) P[c] = fmaf(sc.g[j][e], v[e], P[c]);
    }
  const float lx = pt.bl.lx, ly = pt.bl.ly;
  float gx = (1.f - ly) * (P[1] - P[0]);
  gx = fmaf(ly, P[3] - P[2], gx);
  float gy = (1.f - lx) * (P[2] - P[0]);
  gy = fmaf(lx, P[3] - P[1], gy);
#pragma unroll
  for (int off = 1; off < LPR; off <<= 1) {
    gx += __shfl_xor_sync(kFullMask, gx, off);
    gy += __shfl_xor_sync(kFullMask, gy, off);
  }
  if (live && sub == 0) store_pair(reinterpret_cast<T*>(p.grad_grid) + 2 * row, gx * pt.dx, gy * pt.dy);
  pdl_wait();  // the zero-fill (and absmax header) of the scatter target
  sc.set_scale(p.fixed_hdr, p.fixed_log2n);
  A* gb = reinterpret_cast<A*>(p.grad_in) + img;
#pragma unroll
  for (int c = 0; c < 4; ++c)
    if ((pt.bl.valid >> c) & 1u) sc.add(gb + (int64_t)pt.bl.pix[c] * C, pt.bl.w[c]);
}

// ---------------------------------------------------------------------------
// ROI-Align forward / backward
// ---------------------------------------------------------------------------
template <typename T, int VEC, int LPR, int CPL>
__global__ void __launch_bounds__(kGatherWarps * 32) roi_fwd_kernel(const GatherParams p) {
  const int64_t row = gather_row<LPR>();
  if (row >= p.R * p.Q) return;  // whole lane groups; no shuffles follow
  const int sub = (threadIdx.x & 31) % LPR;
  const RoiBin b = roi_bin(p, row);
  float acc[CPL][VEC];
#pragma unroll
  for (int j = 0; j < CPL; ++j)
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[j][e] = 0.f;
  if (b.n >= 0 && b.n < p.N) {  // an ROI naming a missing batch item samples nothing
    const T* vb = reinterpret_cast<const T*>(p.input) + (int64_t)b.n * p.H * p.W * p.C;
    for (int iy = 0; iy < b.gh; ++iy)
      for (int ix = 0; ix < b.gw; ++ix)
        gather_corners<T, VEC, LPR, CPL>(vb, p.C, sub, roi_point(p, b, iy, ix), 1.f, acc);
  }
#pragma unroll
  for (int j = 0; j < CPL; ++j)
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[j][e] /= b.count;
  store_row<T, VEC, LPR, CPL>(reinterpret_cast<T*>(p.out) + row * p.C, p.C, sub, acc);
}

template <typename T, typename A, int VEC, int LPR, int CPL>
__global__ void __launch_bounds__(kGatherWarps * 32) roi_bwd_kernel(const GatherParams p) {
  pdl_trigger();
  const int64_t row = gather_row<LPR>();
  if (row >= p.R * p.Q) return;  // whole lane groups; no shuffles follow
  const int sub = (threadIdx.x & 31) % LPR;
  const RoiBin b = roi_bin(p, row);
  RowScatter<T, A, VEC, LPR, CPL> sc;
  sc.load(reinterpret_cast<const T*>(p.grad_out) + row * p.C, true, sub, p.C);
  pdl_wait();  // the zero-fill (and absmax header) of the scatter target
  sc.set_scale(p.fixed_hdr, p.fixed_log2n);
  if (b.n < 0 || b.n >= p.N) return;
  A* gb = reinterpret_cast<A*>(p.grad_in) + (int64_t)b.n * p.H * p.W * p.C;
  for (int iy = 0; iy < b.gh; ++iy)
    for (int ix = 0; ix < b.gw; ++ix) {
      const Bilinear bl = roi_point(p, b, iy, ix);
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if ((bl.valid >> c) & 1u) sc.add(gb + (int64_t)bl.pix[c] * p.C, bl.w[c] / b.count);
    }
}

// ---------------------------------------------------------------------------
// Layout conversion on either side of the channels-last kernels:
// dst[n][c][r] = src[n][r][c] for (N, R, C) -> (N, C, R) (NCHW <-> NHWC with
// R or C = H*W). A 64 x 64 tile goes through shared memory (a row pitch of
// an odd number of 4-byte words keeps the column reads conflict-free), so
// both the loads and the stores are coalesced along the contiguous axis of
// their tensor. The grid is (column tiles, row tiles, N), or (row tiles,
// column tiles, N) with `r_in_x` when the row tiles exceed gridDim.y's limit.
// ---------------------------------------------------------------------------
constexpr int kTransposeTile = 64;

template <typename T>
__global__ void __launch_bounds__(256) transpose_kernel(const T* __restrict__ src, T* __restrict__ dst,
                                                        int64_t R, int64_t C, int r_in_x) {
  constexpr int TL = kTransposeTile;
  __shared__ T tile[TL][TL + 4 / sizeof(T)];
  const int64_t n = blockIdx.z;
  const int64_t r0 = (int64_t)(r_in_x ? blockIdx.x : blockIdx.y) * TL;
  const int64_t c0 = (int64_t)(r_in_x ? blockIdx.y : blockIdx.x) * TL;
  const T* s = src + n * R * C;
  T* d = dst + n * R * C;
  const int tx = threadIdx.x & (TL - 1), ty = threadIdx.x / TL;  // 64 x 4 threads
#pragma unroll
  for (int k = 0; k < TL; k += 4) {
    const int64_t r = r0 + ty + k, c = c0 + tx;
    if (r < R && c < C) tile[ty + k][tx] = s[r * C + c];
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < TL; k += 4) {
    const int64_t c = c0 + ty + k, r = r0 + tx;
    if (c < C && r < R) d[c * R + r] = tile[tx][ty + k];
  }
}

// Vector variant (R and C multiples of 4, 4-element aligned buffers, a batch
// slice below 2^31 elements): every global access moves 4 elements (8 bytes
// for 16-bit types, 16 for fp32), 16 lanes cover one 64-element tile row on
// either side, and offsets are 32-bit.
template <typename T>
__global__ void __launch_bounds__(256) transpose4_kernel(const T* __restrict__ src, T* __restrict__ dst,
                                                         int R, int C, int r_in_x) {
  constexpr int TL = kTransposeTile;
  using V4 = typename RawVec<4 * sizeof(T)>::type;  // 4 elements
  __shared__ T tile[TL][TL + 1];
  const int64_t n = blockIdx.z;
  const int r0 = (r_in_x ? blockIdx.x : blockIdx.y) * TL, c0 = (r_in_x ? blockIdx.y : blockIdx.x) * TL;
  const T* s = src + n * (int64_t)R * C;
  T* d = dst + n * (int64_t)R * C;
  const int lo = threadIdx.x & 15, hi = threadIdx.x >> 4;  // 16 x 16 threads
#pragma unroll
  for (int k = 0; k < TL; k += 16) {
    const int r = r0 + hi + k, c = c0 + 4 * lo;
    if (r < R && c < C) {
      union { V4 v; T e[4]; } u;
      u.v = __ldcs(reinterpret_cast<const V4*>(s + r * C + c));
#pragma unroll
      for (int e = 0; e < 4; ++e) tile[hi + k][4 * lo + e] = u.e[e];
    }
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < TL; k += 16) {
    const int c = c0 + hi + k, r = r0 + 4 * lo;
    if (c < C && r < R) {
      union { V4 v; T e[4]; } u;
#pragma unroll
      for (int e = 0; e < 4; ++e) u.e[e] = tile[4 * lo + e][hi + k];
      *reinterpret_cast<V4*>(d + c * R + r) = u.v;
    }
  }
}

// Converting transpose, the last pass of a gather backward that writes an
// NCHW input gradient: the NHWC accumulator (S = fp32, 64-bit fixed point
// scaled by the header, or the data type) of shape (N, R = H*W, C) becomes
// dst (N, C, R) in the data type D, each element rounded once. The tiling
// of transpose4_kernel (V4: 4-element accesses, R and C multiples of 4,
// a batch slice below 2^31 elements) or transpose_kernel (any size), with
// the conversion to fp32 on the way into shared memory.
template <typename S, typename D, bool V4>
__global__ void __launch_bounds__(256) convert_transpose_kernel(const S* __restrict__ src, D* __restrict__ dst,
                                                                int64_t R, int64_t C, int r_in_x,
                                                                const unsigned* hdr, int clog2n) {
  constexpr int TL = kTransposeTile;
  __shared__ float tile[TL][TL + 1];
  pdl_wait();  // the accumulator rows (and the fixed-point header) come from the backward
  FixedScale fx{};
  if constexpr (IsFixed<S>::value) fx = fixed_scale(hdr, clog2n);
  const int64_t n = blockIdx.z;
  const int64_t r0 = (int64_t)(r_in_x ? blockIdx.x : blockIdx.y) * TL;
  const int64_t c0 = (int64_t)(r_in_x ? blockIdx.y : blockIdx.x) * TL;
  const S* s = src + n * R * C;
  D* d = dst + n * R * C;
  auto cvt = [&](S v) -> float {
    if constexpr (IsFixed<S>::value) return fixed_to_f32(v, fx);
    else return to_f32(v);
  };
  if constexpr (V4) {
    const int lo = threadIdx.x & 15, hi = threadIdx.x >> 4;  // 16 x 16 threads
    const int Ri = (int)R, Ci = (int)C;
#pragma unroll
    for (int k = 0; k < TL; k += 16) {
      const int r = (int)r0 + hi + k, c = (int)c0 + 4 * lo;
      if (r < Ri && c < Ci) {
        const S* p = s + r * Ci + c;
        float v[4];
        if constexpr (sizeof(S) == 8) {
          const longlong2 a = __ldcs(reinterpret_cast<const longlong2*>(p));
          const longlong2 b = __ldcs(reinterpret_cast<const longlong2*>(p) + 1);
          v[0] = cvt(a.x); v[1] = cvt(a.y); v[2] = cvt(b.x); v[3] = cvt(b.y);
        } else if constexpr (sizeof(S) == 4) {
          const float4 a = __ldcs(reinterpret_cast<const float4*>(p));
          v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        } else {
          union { uint2 u; S e[4]; } a;
          a.u = __ldcs(reinterpret_cast<const uint2*>(p));
#pragma unroll
          for (int e = 0; e < 4; ++e) v[e] = cvt(a.e[e]);
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) tile[hi + k][4 * lo + e] = v[e];
      }
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < TL; k += 16) {
      const int c = (int)c0 + hi + k, r = (int)r0 + 4 * lo;
      if (c < Ci && r < Ri) {
        float v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = tile[4 * lo + e][hi + k];
        store_vec<D, 4>(d + c * Ri + r, v);
      }
    }
  } else {
    const int tx = threadIdx.x & (TL - 1), ty = threadIdx.x / TL;  // 64 x 4 threads
#pragma unroll
    for (int k = 0; k < TL; k += 4) {
      const int64_t r = r0 + ty + k, c = c0 + tx;
      if (r < R && c < C) tile[ty + k][tx] = cvt(__ldcs(s + r * C + c));
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < TL; k += 4) {
      const int64_t c = c0 + ty + k, r = r0 + tx;
      if (c < C && r < R) d[c * R + r] = from_f32<D>(tile[tx][ty + k]);
    }
  }
}

}  // namespace msda
