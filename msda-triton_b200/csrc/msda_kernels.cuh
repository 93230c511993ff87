// MSDA forward / backward kernels for sm_100a.
//
// Work decomposition (one warp per (b, q, m), lanes over D):
//   * A warp owns one (batch, query, head) triple -- the unit the reference's
//     Triton programs tile over (src/msda_triton/kernels.py:83-96).
//   * Its 32 lanes split into G = 32 / LPR groups of LPR lanes. A group owns
//     one sampling point (l, k) at a time; its LPR lanes cover the D channels
//     of each bilinear corner row with VEC-element (16-byte) vector loads, so
//     one corner gather is LPR x 16 B of consecutive bytes.
//   * The groups walk the L*K sampling points of the triple in steps of G,
//     NB points per step with all 4*NB corner loads issued before any of them
//     is consumed (memory-level parallelism for a latency-bound gather).
//   * Forward: each group accumulates its points in fp32 registers; the G
//     partial rows are then summed across groups with xor-shuffles and group 0
//     stores the output row.
//   * Backward: the same gather recomputes the corners; grad_attn and
//     grad_loc are dot products over D, reduced inside the group with
//     xor-shuffles; grad_value is scattered with 16-byte vector `red.global`
//     adds, either in fp32 (into an fp32 accumulation buffer) or natively in
//     the value dtype (packed f16x2 / bf16x2).
#pragma once

#include "msda_common.cuh"

namespace msda {

struct OpParams {
  const void* value;
  const int64_t* shapes;
  const int64_t* starts;
  const void* loc;
  const void* attn;
  void* out;
  const void* grad_out;
  void* grad_value;   // scatter target of the backward (value dtype or fp32)
  void* grad_loc;
  void* grad_attn;
  int64_t B, S, Q;
  int M, D, L, K;
  int kshift;  // log2(K) when K is a power of two, else -1
  int64_t BQM;  // B * Q * M
};

__device__ __forceinline__ int level_of(int s, int K, int kshift) {
  return kshift >= 0 ? (s >> kshift) : (s / K);
}

// ---------------------------------------------------------------------------
// Forward: out[b,q,m,:] = sum_{l,k} a * sum_c w_c * value[b, pix_c, m, :]
// (src/msda_triton/kernels.py:100-163)
// ---------------------------------------------------------------------------
template <typename T, int VEC, int LPR, int CPL, int WARPS, int NB>
__global__ void __launch_bounds__(WARPS * 32) msda_fwd_kernel(const OpParams p) {
  __shared__ LevelInfo lv[kMaxLevels];
  load_levels(p.shapes, p.starts, p.L, p.S, lv);

  constexpr int G = 32 / LPR;
  using Raw = typename Pack<T, VEC>::Raw;
  const int lane = threadIdx.x & 31;
  const int64_t qm = (int64_t)blockIdx.x * WARPS + (threadIdx.x >> 5);
  if (qm >= p.BQM) return;
  const int grp = lane / LPR, sub = lane % LPR;
  const int64_t b = qm / (p.Q * p.M);
  const int m = (int)(qm % p.M);
  const int D = p.D;
  const int64_t rs = (int64_t)p.M * D;
  const T* vb = reinterpret_cast<const T*>(p.value) + (b * p.S * p.M + m) * D;
  const int LK = p.L * p.K;
  const T* lp = reinterpret_cast<const T*>(p.loc) + qm * (2 * LK);
  const T* ap = reinterpret_cast<const T*>(p.attn) + qm * LK;

  float acc[CPL][VEC];
#pragma unroll
  for (int j = 0; j < CPL; ++j)
#pragma unroll
    for (int v = 0; v < VEC; ++v) acc[j][v] = 0.f;

  for (int s0 = 0; s0 < LK; s0 += G * NB) {
    Bilinear bl[NB];
    float at[NB];
#pragma unroll
    for (int n = 0; n < NB; ++n) {
      const int s = s0 + n * G + grp;
      if (s < LK) {
        const float2 xy = load_pair(lp + 2 * s);
        at[n] = to_f32(ap[s]);
        bl[n] = resolve(xy.x, xy.y, lv[level_of(s, p.K, p.kshift)]);
      } else {
        at[n] = 0.f;
        bl[n] = empty_slot();
      }
    }
    Raw raw[NB][4][CPL];
#pragma unroll
    for (int n = 0; n < NB; ++n)
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int j = 0; j < CPL; ++j) {
          const int ch = (j * LPR + sub) * VEC;
          Raw r{};
          if (((bl[n].valid >> c) & 1u) && ch < D) r = load_raw<T, VEC>(vb + bl[n].pix[c] * rs + ch);
          raw[n][c][j] = r;
        }
#pragma unroll
    for (int n = 0; n < NB; ++n)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float wc = at[n] * bl[n].w[c];
#pragma unroll
        for (int j = 0; j < CPL; ++j) {
          float v[VEC];
          unpack_raw<T, VEC>(raw[n][c][j], v);
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc[j][e] = fmaf(wc, v[e], acc[j][e]);
        }
      }
  }

#pragma unroll
  for (int off = LPR; off < 32; off <<= 1)
#pragma unroll
    for (int j = 0; j < CPL; ++j)
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc[j][e] += __shfl_xor_sync(kFullMask, acc[j][e], off);

  if (grp == 0) {
    T* op = reinterpret_cast<T*>(p.out) + qm * D;
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      const int ch = (j * LPR + sub) * VEC;
      if (ch < D) store_vec<T, VEC>(op + ch, acc[j]);
    }
  }
}

// ---------------------------------------------------------------------------
// Backward (src/msda_triton/kernels.py:205-291):
//   grad_attn[s]    = sum_d g_d * sampled_d
//   grad_loc[s].x   = a * W * sum_d g_d * ((v01-v00)(1-ly) + (v11-v10) ly)
//   grad_loc[s].y   = a * H * sum_d g_d * ((v10-v00)(1-lx) + (v11-v01) lx)
//   grad_value[c]  += a * w_c * g          (SCATTER; A = accumulator type)
// ---------------------------------------------------------------------------
template <typename T, typename A, int VEC, int LPR, int CPL, int WARPS, int NB, bool SCATTER>
__global__ void __launch_bounds__(WARPS * 32) msda_bwd_kernel(const OpParams p) {
  __shared__ LevelInfo lv[kMaxLevels];
  load_levels(p.shapes, p.starts, p.L, p.S, lv);

  constexpr int G = 32 / LPR;
  using Raw = typename Pack<T, VEC>::Raw;
  const int lane = threadIdx.x & 31;
  const int64_t qm = (int64_t)blockIdx.x * WARPS + (threadIdx.x >> 5);
  if (qm >= p.BQM) return;
  const int grp = lane / LPR, sub = lane % LPR;
  const int64_t b = qm / (p.Q * p.M);
  const int m = (int)(qm % p.M);
  const int D = p.D;
  const int64_t rs = (int64_t)p.M * D;
  const int64_t head_base = (b * p.S * p.M + m) * D;
  const T* vb = reinterpret_cast<const T*>(p.value) + head_base;
  A* gvb = reinterpret_cast<A*>(p.grad_value) + head_base;
  const int LK = p.L * p.K;
  const T* lp = reinterpret_cast<const T*>(p.loc) + qm * (2 * LK);
  const T* ap = reinterpret_cast<const T*>(p.attn) + qm * LK;
  T* glp = reinterpret_cast<T*>(p.grad_loc) + qm * (2 * LK);
  T* gap = reinterpret_cast<T*>(p.grad_attn) + qm * LK;

  float g[CPL][VEC];
  {
    const T* gp = reinterpret_cast<const T*>(p.grad_out) + qm * D;
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      const int ch = (j * LPR + sub) * VEC;
      if (ch < D) {
        load_vec<T, VEC>(gp + ch, g[j]);
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) g[j][e] = 0.f;
      }
    }
  }

  for (int s0 = 0; s0 < LK; s0 += G * NB) {
    Bilinear bl[NB];
    float at[NB];
    float fw[NB], fh[NB];
#pragma unroll
    for (int n = 0; n < NB; ++n) {
      const int s = s0 + n * G + grp;
      if (s < LK) {
        const float2 xy = load_pair(lp + 2 * s);
        at[n] = to_f32(ap[s]);
        const LevelInfo& L = lv[level_of(s, p.K, p.kshift)];
        bl[n] = resolve(xy.x, xy.y, L);
        fw[n] = L.fW;
        fh[n] = L.fH;
      } else {
        at[n] = 0.f;
        fw[n] = fh[n] = 0.f;
        bl[n] = empty_slot();
      }
    }
    Raw raw[NB][4][CPL];
#pragma unroll
    for (int n = 0; n < NB; ++n)
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int j = 0; j < CPL; ++j) {
          const int ch = (j * LPR + sub) * VEC;
          Raw r{};
          if (((bl[n].valid >> c) & 1u) && ch < D) r = load_raw<T, VEC>(vb + bl[n].pix[c] * rs + ch);
          raw[n][c][j] = r;
        }

#pragma unroll
    for (int n = 0; n < NB; ++n) {
      const float lx = bl[n].lx, ly = bl[n].ly;
      float ga = 0.f, gx = 0.f, gy = 0.f;
#pragma unroll
      for (int j = 0; j < CPL; ++j) {
        float v00[VEC], v01[VEC], v10[VEC], v11[VEC];
        unpack_raw<T, VEC>(raw[n][0][j], v00);
        unpack_raw<T, VEC>(raw[n][1][j], v01);
        unpack_raw<T, VEC>(raw[n][2][j], v10);
        unpack_raw<T, VEC>(raw[n][3][j], v11);
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          const float gd = g[j][e];
          const float smp = bl[n].w[0] * v00[e] + bl[n].w[1] * v01[e] + bl[n].w[2] * v10[e] +
                            bl[n].w[3] * v11[e];
          const float dx = (v01[e] - v00[e]) * (1.f - ly) + (v11[e] - v10[e]) * ly;
          const float dy = (v10[e] - v00[e]) * (1.f - lx) + (v11[e] - v01[e]) * lx;
          ga = fmaf(gd, smp, ga);
          gx = fmaf(gd, dx, gx);
          gy = fmaf(gd, dy, gy);
        }
      }
#pragma unroll
      for (int off = 1; off < LPR; off <<= 1) {
        ga += __shfl_xor_sync(kFullMask, ga, off);
        gx += __shfl_xor_sync(kFullMask, gx, off);
        gy += __shfl_xor_sync(kFullMask, gy, off);
      }
      const int s = s0 + n * G + grp;
      if (s < LK) {
        if (sub == 0) {
          store_pair(glp + 2 * s, at[n] * fw[n] * gx, at[n] * fh[n] * gy);
          gap[s] = from_f32<T>(ga);
        }
        if constexpr (SCATTER) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            if ((bl[n].valid >> c) & 1u) {
              const float wc = at[n] * bl[n].w[c];
#pragma unroll
              for (int j = 0; j < CPL; ++j) {
                const int ch = (j * LPR + sub) * VEC;
                if (ch < D) {
                  float contrib[VEC];
#pragma unroll
                  for (int e = 0; e < VEC; ++e) contrib[e] = wc * g[j][e];
                  red_add_vec<A, VEC>(gvb + bl[n].pix[c] * rs + ch, contrib);
                }
              }
            }
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// grad_value by pixel-chunk ownership (no atomics in global memory, no
// workspace, no zero-fill, no downcast pass).
//
// CTA (chunk c, head-slice bm = b*M + m) owns grad_value[b, p0:p1, m, :]
// (p0 = c*P) as an fp32 tile in shared memory. For every level overlapping
// [p0, p1) it scans that head's Q*K sampling points of the level, keeps the
// points with at least one bilinear corner inside the chunk in a shared queue,
// then adds a * w_c * grad_out[b, q, m, :] into the tile with shared-memory
// atomics (lanes over D: one warp instruction per corner row, conflict-free).
// Finally the tile is written out once, densely, in the value dtype -- every
// grad_value element is written exactly once by exactly one CTA.
//
// When a chunk collects many points per query, the (b, :, m, :) slice of
// grad_out is staged in shared memory once instead of being gathered from L2
// per point.
// ---------------------------------------------------------------------------
struct OwnerHit {
  int q;
  int rel00;     // pixel of corner 0 minus p0
  unsigned mask; // bit c: corner c lies inside [p0, p1)
  int W;
  float coef[4]; // a * w_c
};

constexpr int kOwnerThreads = 256;
constexpr int kOwnerQueue = 512;   // hits per scan batch (one per thread slot, two slots per thread)
constexpr int kOwnerBatch = 512;   // sampling points scanned per batch
constexpr int kOwnerHitsPerWarp = 4;

template <typename T, int CH, int OVEC>
__global__ void __launch_bounds__(kOwnerThreads) msda_bwd_value_owner_kernel(const OpParams p, int P,
                                                                           int stage_limit) {
  extern __shared__ float4 owner_smem[];
  float* acc = reinterpret_cast<float*>(owner_smem);                 // P * D floats
  OwnerHit* queue = reinterpret_cast<OwnerHit*>(acc + (size_t)P * p.D);  // kOwnerQueue
  T* gstage = reinterpret_cast<T*>(queue + kOwnerQueue);             // Q * D (optional)
  __shared__ LevelInfo lv[kMaxLevels];
  __shared__ int qcount;
  __shared__ int staged;
  load_levels(p.shapes, p.starts, p.L, p.S, lv);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int NW = kOwnerThreads / 32;
  const int D = p.D;
  const int64_t p0 = (int64_t)blockIdx.x * P;
  const int64_t p1 = min(p0 + P, p.S);
  const int npix = (int)(p1 - p0);
  const int bm = blockIdx.y;
  const int64_t b = bm / p.M;
  const int m = bm % p.M;
  const int LK = p.L * p.K;
  const int64_t QK = p.Q * (int64_t)p.K;

  for (int i = tid; i < npix * D; i += kOwnerThreads) acc[i] = 0.f;
  if (tid == 0) {
    qcount = 0;
    staged = 0;
  }
  __syncthreads();

  const T* gout = reinterpret_cast<const T*>(p.grad_out);
  const T* locp = reinterpret_cast<const T*>(p.loc);
  const T* attp = reinterpret_cast<const T*>(p.attn);

  for (int l = 0; l < p.L; ++l) {
    const LevelInfo L = lv[l];
    if (L.W == 0 || L.start >= p1 || (int64_t)L.start + (int64_t)L.H * L.W <= p0) continue;
    for (int64_t base = 0; base < QK; base += kOwnerBatch) {
      // ---- scan: queue the points with a corner inside the chunk ----------
      for (int j = tid; j < kOwnerBatch; j += kOwnerThreads) {
        const int64_t i = base + j;
        if (i >= QK) break;
        const int64_t q = p.kshift >= 0 ? (i >> p.kshift) : (i / p.K);
        const int k = (int)(i - q * p.K);
        const int64_t qm = (b * p.Q + q) * p.M + m;
        const int64_t sidx = qm * LK + l * p.K + k;
        const float2 xy = load_pair(locp + 2 * sidx);
        const Bilinear bl = resolve(xy.x, xy.y, L);
        unsigned mask = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (((bl.valid >> c) & 1u) && bl.pix[c] >= p0 && bl.pix[c] < p1) mask |= 1u << c;
        if (mask) {
          const float a = to_f32(attp[sidx]);
          const int slot = atomicAdd(&qcount, 1);
          OwnerHit h;
          h.q = (int)q;
          h.rel00 = (int)(bl.pix[0] - p0);
          h.mask = mask;
          h.W = L.W;
#pragma unroll
          for (int c = 0; c < 4; ++c) h.coef[c] = a * bl.w[c];
          queue[slot] = h;
        }
      }
      __syncthreads();
      const int n = qcount;
      // ---- stage grad_out[b, :, m, :] once if this chunk is busy ----------
      if (!staged && stage_limit > 0 && n * 4 >= p.Q) {
        const int64_t rows = p.Q;
        for (int64_t e = tid; e < rows * D; e += kOwnerThreads) {
          const int64_t q = e / D;
          const int d = (int)(e - q * D);
          gstage[e] = gout[((b * p.Q + q) * p.M + m) * D + d];
        }
        __syncthreads();
        if (tid == 0) staged = 1;
      }
      const bool use_stage = staged || (stage_limit > 0 && n * 4 >= p.Q);
      // ---- accumulate: lanes over D, kOwnerHitsPerWarp points in flight ---
      for (int h0 = warp * kOwnerHitsPerWarp; h0 < n; h0 += NW * kOwnerHitsPerWarp) {
        float gv[kOwnerHitsPerWarp][CH];
#pragma unroll
        for (int u = 0; u < kOwnerHitsPerWarp; ++u) {
          const int h = h0 + u;
          const int q = h < n ? queue[h].q : 0;
#pragma unroll
          for (int c = 0; c < CH; ++c) {
            const int d = lane + 32 * c;
            float v = 0.f;
            if (h < n && d < D) {
              v = use_stage ? to_f32(gstage[(int64_t)q * D + d])
                            : to_f32(__ldg(gout + ((b * p.Q + q) * p.M + m) * D + d));
            }
            gv[u][c] = v;
          }
        }
#pragma unroll
        for (int u = 0; u < kOwnerHitsPerWarp; ++u) {
          const int h = h0 + u;
          if (h >= n) break;
          const OwnerHit hit = queue[h];
          const int rel[4] = {hit.rel00, hit.rel00 + 1, hit.rel00 + hit.W, hit.rel00 + hit.W + 1};
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            if (!((hit.mask >> c) & 1u)) continue;
            float* row = acc + (size_t)rel[c] * D;
#pragma unroll
            for (int cc = 0; cc < CH; ++cc) {
              const int d = lane + 32 * cc;
              if (d < D) atomicAdd(row + d, hit.coef[c] * gv[u][cc]);
            }
          }
        }
      }
      __syncthreads();
      if (tid == 0) qcount = 0;
      __syncthreads();
    }
  }

  // ---- write the tile once (dense, value dtype) ---------------------------
  T* gvout = reinterpret_cast<T*>(p.grad_value);
  const int64_t rs = (int64_t)p.M * D;
  const int64_t head0 = ((b * p.S + p0) * p.M + m) * D;
  const int nvec = npix * D / OVEC;
  for (int e = tid; e < nvec; e += kOwnerThreads) {
    const int flat = e * OVEC;
    const int r = flat / D;
    const int d = flat - r * D;
    float v[OVEC];
#pragma unroll
    for (int k = 0; k < OVEC; ++k) v[k] = acc[flat + k];
    store_vec<T, OVEC>(gvout + head0 + r * rs + d, v);
  }
}

// fp32 accumulation buffer -> value dtype (the downcast of src/msda_triton/ops.py:91-92).
template <typename T, int VEC>
__global__ void __launch_bounds__(256) msda_cast_kernel(const float* __restrict__ src, T* __restrict__ dst,
                                                       int64_t nvec) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec;
       i += (int64_t)gridDim.x * blockDim.x) {
    float v[VEC];
    if constexpr (VEC % 4 == 0) {
#pragma unroll
      for (int k = 0; k < VEC; k += 4) {
        const float4 f = __ldcs(reinterpret_cast<const float4*>(src + i * VEC + k));
        v[k] = f.x;
        v[k + 1] = f.y;
        v[k + 2] = f.z;
        v[k + 3] = f.w;
      }
    } else {
#pragma unroll
      for (int k = 0; k < VEC; ++k) v[k] = __ldcs(src + i * VEC + k);
    }
    store_vec<T, VEC>(dst + i * VEC, v);
  }
}

}  // namespace msda
