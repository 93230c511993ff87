// MSDA forward / backward kernels for sm_100a.
//
// Work decomposition (one warp per (b, q, m), lanes over D):
//   * A CTA owns a block of consecutive queries of one (batch, head) slice --
//     the reference's query-block tiling (src/msda_triton/kernels.py:83-96) --
//     and each of its warps one (batch, query, head) triple.
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
  unsigned* counts;   // counted scatter: bilinear hits per (b, pixel, m) row
  void* acc;          // counted scatter: accumulator rows of the multi-hit rows
  // Exact counted scatter: per-row bound of |a| * max|grad_out row|, packed
  // with the count -- (count, bound) word pairs, p.rowmax = p.counts + 1 --
  // so one 8-byte load reads both.
  unsigned* rowmax;
  int acc_words;      // 32-bit words per accumulator element: 1 (fp32), 2 (64-bit fixed point)
  // Deterministic grad_value (64-bit fixed point): the absmax header and
  // ceil(log2(Q*K)), the bound on contributions per row.
  const unsigned* fixed_hdr;
  int fixed_log2n;
  // Fused prologue (fused != 0): `loc` holds sampling offsets in level
  // pixels, `attn` attention logits (softmaxed over a query-head's L*K
  // points), `ref` reference points (B, Q, 2); the sampling location of a
  // point is ref + offset / (W_l, H_l).
  const void* ref;
  int fused;
  int64_t B, S, Q;
  int M, D, L, K;
  int kshift;  // log2(K) when K is a power of two, else -1
  int64_t BQM;  // B * Q * M
};

__device__ __forceinline__ int level_of(int s, int K, int kshift) {
  return kshift >= 0 ? (s >> kshift) : (s / K);
}

// Query-block tiling (src/msda_triton/kernels.py:83-96): a CTA owns WARPS
// consecutive queries of one (batch, head) slice, one warp per query, so the
// overlapping corner rows of neighbouring queries are re-read from L1. Grid:
// x = query block, y = head, z = batch (no integer division in the mapping).
__device__ __forceinline__ bool query_block_of(const OpParams& p, int warps, int64_t& b, int& m,
                                               int64_t& q) {
  q = (int64_t)blockIdx.x * warps + (threadIdx.x >> 5);
  m = (int)blockIdx.y;
  b = (int64_t)blockIdx.z;
  return q < p.Q;
}

// Sums the partial rows of the GQ lane groups that share a query (GQ = 32 /
// LPR when the warp serves one query) and stores the output row when `live`.
template <typename T, int VEC, int LPR, int CPL, int GQ = 32 / LPR>
__device__ __forceinline__ void fwd_store_row(T* op, int D, int lane, float (&acc)[CPL][VEC],
                                              bool live = true) {
  const int gq = (lane / LPR) % GQ, sub = lane % LPR;
  if constexpr (CPL == 1 && GQ > 1 && VEC >= 2) {
    // Reduce-scatter across the GQ groups: each xor stage halves the values a
    // lane keeps (it keeps the half its partner sends it the other of), so
    // log2(VEC) stages cost VEC-1 shuffles instead of VEC*log2(GQ); once a
    // lane holds one value the remaining stages are plain xor-sums.
    constexpr int STAGES = __builtin_ctz(GQ);
    int base = 0;
#pragma unroll
    for (int st = 0; st < STAGES; ++st) {
      const int off = LPR << st;
      const int n = VEC >> st;  // live values before this stage (compile time after unrolling)
      if (n > 1) {
        const bool upper = (lane & off) != 0;
        const int half = n / 2;
#pragma unroll
        for (int i = 0; i < half; ++i) {
          const float send = upper ? acc[0][i] : acc[0][half + i];
          const float keep = upper ? acc[0][half + i] : acc[0][i];
          acc[0][i] = keep + __shfl_xor_sync(kFullMask, send, off);
        }
        if (upper) base += half;
      } else {
        acc[0][0] += __shfl_xor_sync(kFullMask, acc[0][0], off);
      }
    }
    constexpr int NF = (VEC >> STAGES) > 0 ? (VEC >> STAGES) : 1;  // values left per lane
    constexpr int HALVINGS = __builtin_ctz(VEC) < STAGES ? __builtin_ctz(VEC) : STAGES;
    // Lanes that only replicated a value in the plain xor stages skip the store.
    const int rep_mask = ((GQ - 1) << __builtin_ctz(LPR)) & ~(((1 << HALVINGS) - 1) << __builtin_ctz(LPR));
    const int ch = sub * VEC + base;
    if (live && (lane & rep_mask) == 0 && sub * VEC < D) {
      float outv[NF];
#pragma unroll
      for (int i = 0; i < NF; ++i) outv[i] = acc[0][i];
      store_vec<T, NF>(op + ch, outv);
    }
  } else {
#pragma unroll
    for (int off = LPR; off < LPR * GQ; off <<= 1)
#pragma unroll
      for (int j = 0; j < CPL; ++j)
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[j][e] += __shfl_xor_sync(kFullMask, acc[j][e], off);
    if (live && gq == 0) {
#pragma unroll
      for (int j = 0; j < CPL; ++j) {
        const int ch = (j * LPR + sub) * VEC;
        if (ch < D) store_vec<T, VEC>(op + ch, acc[j]);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Forward: out[b,q,m,:] = sum_{l,k} a * sum_c w_c * value[b, pix_c, m, :]
// (src/msda_triton/kernels.py:100-163)
// ---------------------------------------------------------------------------
// MINB: minimum resident CTAs per SM the forward is compiled for (0 leaves
// the register budget to the compiler). A grid of a few waves runs faster
// with fewer, register-richer warps per SM (MINB = 3); a long grid needs the
// occupancy of the compiler's default.
// QW: queries a warp serves at once -- its G = 32 / LPR lane groups split
// into QW sets of GQ = G / QW groups, each set walking one query's L*K
// points GQ*NB at a time (QW = 2 packs the 12 points of a 3-level, 4-point
// head into 4 groups x 3 steps with no idle slot, where one query per warp
// leaves 4 of 16 slots empty).
// QPW: rounds per warp; a CTA covers WARPS*QW*QPW consecutive queries of one
// (batch, head) slice, so neighbouring queries' shared corner rows are
// re-read from L1 and the level table is loaded once per CTA.
// FUSED: the layer's prologue runs here (OpParams::ref / fused; QW = 1).
// SHARE (needs QW * L * K <= 32, checked on the host): lane i resolves point
// i of the warp's QW queries once per round (coalesced parameter loads), and
// each step fetches its point's corner rows, fractions, weight and validity
// from that lane by shuffle instead of the group's lanes each resolving it.
template <typename T, int VEC, int LPR, int CPL, int WARPS, int NB, int MINB, bool FUSED = false,
          int QW = 1, int QPW = 1, bool SHARE = false>
__global__ void __launch_bounds__(WARPS * 32, MINB) msda_fwd_kernel(const OpParams p) {
  static_assert(!FUSED || QW == 1, "the fused prologue's softmax spans the warp");
  static_assert(!SHARE || !FUSED, "SHARE: no fused prologue");
  constexpr int G = 32 / LPR;
  static_assert(QW >= 1 && G % QW == 0, "QW must divide the lane groups");
  constexpr int GQ = G / QW;
  __shared__ LevelInfo lv[kMaxLevels];
  load_levels(p.shapes, p.starts, p.L, p.S, lv);

  using Raw = typename Pack<T, VEC>::Raw;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int grp = lane / LPR, sub = lane % LPR;
  const int qsub = grp / GQ, gq = grp % GQ;
  const int m = (int)blockIdx.y;
  const int64_t b = (int64_t)blockIdx.z;
  const int D = p.D;
  const int rs = p.M * D;  // row stride; pix * rs < S*M*D < 2^31 (checked on the host)
  const T* vb = reinterpret_cast<const T*>(p.value) + (b * p.S * p.M + m) * D;
  const int LK = p.L * p.K;
  // With several rounds and one step covering a query's points, a lane's NB
  // point slots sit on the same levels for every query: keep those levels in
  // registers (a single round reads them from shared memory, off the
  // dependent chain of its first loads).
  const bool one_step = QPW > 1 && LK <= GQ * NB;
  LevelInfo lvn[QPW > 1 ? NB : 1];
  if constexpr (QPW > 1) {
#pragma unroll
    for (int n = 0; n < NB; ++n) {
      const int s = n * GQ + gq;
      lvn[n] = lv[s < LK ? level_of(s, p.K, p.kshift) : 0];
    }
  }

  // Packed-pair accumulators (f32x2 FMA) on the vector path, scalars otherwise.
  constexpr bool kPairs = VEC >= 2 && VEC % 2 == 0;
  constexpr int NP = kPairs ? VEC / 2 : 1;
  for (int round = 0; round < QPW; ++round) {
    const int64_t q = (((int64_t)blockIdx.x * QPW + round) * WARPS + warp) * QW + qsub;
    const bool live = q < p.Q;
    if (!__any_sync(kFullMask, live)) break;  // warp-uniform: past the last query
    const int64_t qm = (b * p.Q + (live ? q : 0)) * p.M + m;
    const T* lp = reinterpret_cast<const T*>(p.loc) + qm * (2 * LK);
    const T* ap = reinterpret_cast<const T*>(p.attn) + qm * LK;
    // Fused prologue: this query's reference point and its head's softmax.
    float2 refp = make_float2(0.f, 0.f);
    float smx = 0.f, sinv = 1.f;
    if constexpr (FUSED) {
      refp = load_pair(reinterpret_cast<const T*>(p.ref) + 2 * (b * p.Q + q));
      warp_softmax_stats(ap, LK, lane, smx, sinv);
    }
    uint64_t acc2[CPL][NP];
    float acc[CPL][VEC];
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
#pragma unroll
      for (int v = 0; v < NP; ++v) acc2[j][v] = 0ull;
#pragma unroll
      for (int v = 0; v < VEC; ++v) acc[j][v] = 0.f;
    }
    // SHARE: this lane's own point (query my_q of the warp, point my_s).
    int sh_p00 = 0, sh_p10 = 0;
    unsigned sh_valid = 0u;
    float sh_lx = 0.f, sh_ly = 0.f, sh_at = 0.f;
    if constexpr (SHARE) {
      const int my_q = lane / LK, my_s = lane - my_q * LK;
      const int64_t q_mine = q - qsub + my_q;  // the warp's first query + my_q
      if (my_q < QW && q_mine < p.Q) {
        const int64_t qm_mine = (b * p.Q + q_mine) * p.M + m;
        const T* lpm = reinterpret_cast<const T*>(p.loc) + qm_mine * (2 * LK);
        const float2 xy = load_pair(lpm + 2 * my_s);
        sh_at = to_f32(reinterpret_cast<const T*>(p.attn)[qm_mine * LK + my_s]);
        const Bilinear bm = resolve(xy.x, xy.y, lv[level_of(my_s, p.K, p.kshift)]);
        sh_p00 = bm.pix[0];
        sh_p10 = bm.pix[2];
        sh_lx = bm.lx;
        sh_ly = bm.ly;
        sh_valid = bm.valid;
      }
    }

    for (int s0 = 0; s0 < LK; s0 += GQ * NB) {
      Bilinear bl[NB];
      float at[NB];
      if constexpr (SHARE) {
#pragma unroll
        for (int n = 0; n < NB; ++n) {
          const int s = s0 + n * GQ + gq;
          const int src = qsub * LK + (s < LK ? s : 0);
          const int p00 = __shfl_sync(kFullMask, sh_p00, src), p10 = __shfl_sync(kFullMask, sh_p10, src);
          const float lx = __shfl_sync(kFullMask, sh_lx, src), ly = __shfl_sync(kFullMask, sh_ly, src);
          const float a = __shfl_sync(kFullMask, sh_at, src);
          const unsigned v = __shfl_sync(kFullMask, sh_valid, src);
          bl[n].pix[0] = p00;
          bl[n].pix[1] = p00 + 1;
          bl[n].pix[2] = p10;
          bl[n].pix[3] = p10 + 1;
          bl[n].lx = lx;
          bl[n].ly = ly;
          bl[n].w[0] = (1.0f - lx) * (1.0f - ly);
          bl[n].w[1] = lx * (1.0f - ly);
          bl[n].w[2] = (1.0f - lx) * ly;
          bl[n].w[3] = lx * ly;
          const bool ok = live && s < LK;
          bl[n].valid = ok ? v : 0u;
          at[n] = ok ? a : 0.f;
        }
      } else {
#pragma unroll
        for (int n = 0; n < NB; ++n) {
          const int s = s0 + n * GQ + gq;
          if (live && s < LK) {
            const float2 xy = load_pair(lp + 2 * s);
            const float a = to_f32(ap[s]);
            const LevelInfo& L = one_step ? lvn[QPW > 1 ? n : 0] : lv[level_of(s, p.K, p.kshift)];
            if constexpr (FUSED) {
              at[n] = expf(a - smx) * sinv;
              bl[n] = resolve_fused(refp, xy, L);
            } else {
              at[n] = a;
              bl[n] = resolve(xy.x, xy.y, L);
            }
          } else {
            at[n] = 0.f;
            bl[n] = empty_slot();
          }
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
          if constexpr (kPairs) {
            const uint64_t w2 = f2_pack(wc, wc);
#pragma unroll
            for (int j = 0; j < CPL; ++j) {
              uint64_t v2[NP];
              raw_to_f2<T, VEC>(raw[n][c][j], v2);
#pragma unroll
              for (int e = 0; e < NP; ++e) acc2[j][e] = f2_fma(w2, v2[e], acc2[j][e]);
            }
          } else {
#pragma unroll
            for (int j = 0; j < CPL; ++j) {
              float v[VEC];
              unpack_raw<T, VEC>(raw[n][c][j], v);
#pragma unroll
              for (int e = 0; e < VEC; ++e) acc[j][e] = fmaf(wc, v[e], acc[j][e]);
            }
          }
        }
    }
    if constexpr (kPairs) {
#pragma unroll
      for (int j = 0; j < CPL; ++j)
#pragma unroll
        for (int e = 0; e < NP; ++e) f2_unpack(acc2[j][e], acc[j][2 * e], acc[j][2 * e + 1]);
    }
    fwd_store_row<T, VEC, LPR, CPL, GQ>(reinterpret_cast<T*>(p.out) + qm * D, D, lane, acc, live);
  }
}

// ---------------------------------------------------------------------------
// Backward (src/msda_triton/kernels.py:205-291):
//   grad_attn[s]    = sum_d g_d * sampled_d
//   grad_loc[s].x   = a * W * sum_d g_d * ((v01-v00)(1-ly) + (v11-v10) ly)
//   grad_loc[s].y   = a * H * sum_d g_d * ((v10-v00)(1-lx) + (v11-v01) lx)
//   grad_value[c]  += a * w_c * g          (SCATTER; A = accumulator type)
// ---------------------------------------------------------------------------
// grad_value handling of msda_bwd_kernel.
enum ScatterMode : int {
  kNoScatter = 0,  // gradients of the sampling parameters only
  kScatter = 1,    // vector `red` into p.grad_value (type A), zero-filled beforehand
  kCounted = 2,    // hit-counted: one-hit rows stored, multi-hit rows reduced in fp32
  kScatterMerge = 3,  // kScatter with same-row contributions of a warp merged first
};

// Hit-counted scatter: flag in a row's hit count marking a row of a dense
// level (accumulated in fp32 whatever its count).
constexpr unsigned kDenseRow = 0x80000000u;

// Fused prologue: points per query-head whose attention-weight gradients the
// backward keeps in fp32 shared memory for the softmax backward (beyond that
// they take a round trip through the logits' gradient buffer).
constexpr int kFusedMaxLK = 128;

// Minimum resident CTAs per SM the backward is compiled for (register cap).
// The hit-counted mode measured faster at 3 (80 registers), the plain
// scatter modes at 4 (64 registers).
#ifndef MSDA_BWD_MIN_BLOCKS
#define MSDA_BWD_MIN_BLOCKS 4
#endif
#ifndef MSDA_BWD_COUNTED_MIN_BLOCKS
#define MSDA_BWD_COUNTED_MIN_BLOCKS 3
#endif
// The caps above count CTAs of kBwdCapWarps warps; smaller CTAs scale the
// count so the per-thread register budget stays the same.
constexpr int kBwdCapWarps = 8;

// QW / QPW as in the forward: a warp serves QW queries at once (GQ = G / QW
// lane groups each) over QPW rounds of consecutive queries; the same-row
// merge then matches (row, query) keys, since only one query's corners share
// a grad_out vector. FUSED and the hit-counted mode take QW = QPW = 1.
// SHARE as in the forward: lane i resolves point i of the warp's queries once
// per round and the lane groups fetch it by shuffle (QW * L * K <= 32).
template <typename T, typename A, int VEC, int LPR, int CPL, int WARPS, int NB, int MODE, bool FUSED = false,
          int QW = 1, int QPW = 1, bool SHARE = false>
__global__ void __launch_bounds__(WARPS * 32, (MODE == kCounted ? MSDA_BWD_COUNTED_MIN_BLOCKS : MSDA_BWD_MIN_BLOCKS) *
                                                  kBwdCapWarps / WARPS)
    msda_bwd_kernel(const OpParams p) {
  constexpr bool SCATTER = MODE != kNoScatter;
  // A = long long: deterministic grad_value in 64-bit fixed point (see
  // fixed_scale); the scatter target (kScatter*) or the multi-hit rows
  // (kCounted) hold fixed-point elements.
  constexpr bool FIXED = IsFixed<A>::value;
  // A = ExactF32: deterministic fp16 / bf16 in the hit-counted mode -- rows
  // with three or more hits receive integer-valued contributions on the
  // row's scale (exact_scale) in their fp32 accumulator rows.
  constexpr bool EXACT = IsExact<A>::value;
  static_assert(!EXACT || (MODE == kCounted && sizeof(T) == 2), "exact rows: hit-counted fp16 / bf16");
  pdl_trigger();
  __shared__ LevelInfo lv[kMaxLevels];
  __shared__ float fused_ga[FUSED ? WARPS : 1][FUSED ? kFusedMaxLK : 1];  // fused: dL/da per point

  constexpr int G = 32 / LPR;
  static_assert((QW == 1 || QW == 2) && G % QW == 0, "QW: 1 or 2 queries per warp");
  static_assert(QW == 1 || (!FUSED && MODE != kCounted), "one query per warp for FUSED / kCounted");
  static_assert(!SHARE || (!FUSED && NB == 1), "SHARE: one point per group, no fused prologue");
  constexpr int GQ = G / QW;
  using Raw = typename Pack<T, VEC>::Raw;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int m = (int)blockIdx.y;
  const int64_t b = (int64_t)blockIdx.z;
  const int grp = lane / LPR, sub = lane % LPR;
  const int qsub = grp / GQ, gq_ = grp % GQ;
  const int D = p.D;
  const int rs = p.M * D;  // row stride; pix * rs < S*M*D < 2^31 (checked on the host)
  const int64_t head_base = (b * p.S * p.M + m) * D;
  const T* vb = reinterpret_cast<const T*>(p.value) + head_base;
  A* gvb = reinterpret_cast<A*>(p.grad_value) + head_base;
  T* gvt = reinterpret_cast<T*>(p.grad_value) + head_base;  // kCounted: one-hit rows
  float* accb = reinterpret_cast<float*>(p.acc) + head_base;  // kCounted, fp32 rows
  long long* faccb = reinterpret_cast<long long*>(p.acc) + head_base;  // kCounted, fixed point
  const unsigned* cnb = p.counts + (b * p.S * p.M + m);  // kCounted: row pix at cnb[pix * M]
  // EXACT: (count, bound) of row pix at cpb[pix * M]
  const uint2* cpb = reinterpret_cast<const uint2*>(p.counts) + (b * p.S * p.M + m);
  const int LK = p.L * p.K;
  // Scatter: keep the reduction target in L2, let the gathered value rows go first.
  uint64_t pol_keep = 0, pol_stream = 0;
  if constexpr (SCATTER) {
    pol_keep = policy_evict_last();
    pol_stream = policy_evict_first();
  }
  FixedScale fx{1.0, 1.f, 1.f, true};

  for (int round = 0; round < QPW; ++round) {
    const int64_t q = (((int64_t)blockIdx.x * QPW + round) * WARPS + warp) * QW + qsub;
    const bool live = q < p.Q;
    const int64_t qm = (b * p.Q + (live ? q : 0)) * p.M + m;
    const T* lp = reinterpret_cast<const T*>(p.loc) + qm * (2 * LK);
    const T* ap = reinterpret_cast<const T*>(p.attn) + qm * LK;
    T* glp = reinterpret_cast<T*>(p.grad_loc) + qm * (2 * LK);
    T* gap = reinterpret_cast<T*>(p.grad_attn) + qm * LK;

    // Dot products of 16-bit data by mixed-precision FMA on the raw words
    // (fewer instructions; measured faster where the backward is throughput
    // bound, slower in the latency-bound hit-counted mode, which keeps the
    // packed f32x2 FMAs).
    constexpr bool MIXED = sizeof(T) == 2 && VEC == 8 && MODE != kCounted;
    float g[CPL][VEC];
    Raw graw[MIXED ? CPL : 1];
    {
      const T* gp = reinterpret_cast<const T*>(p.grad_out) + qm * D;
#pragma unroll
      for (int j = 0; j < CPL; ++j) {
        const int ch = (j * LPR + sub) * VEC;
        Raw r{};
        if (live && ch < D) r = load_raw<T, VEC>(gp + ch);
        unpack_raw<T, VEC>(r, g[j]);
        if constexpr (MIXED) graw[j] = r;
      }
    }
    // grad_out as packed fp32 pairs (VEC even).
    uint64_t g2[CPL][VEC / 2 > 0 ? VEC / 2 : 1];
#pragma unroll
    for (int j = 0; j < CPL; ++j)
#pragma unroll
      for (int e = 0; e < VEC / 2; ++e) g2[j][e] = f2_pack(g[j][2 * e], g[j][2 * e + 1]);
    // fp32 reductions of 16-bit data: a lane's 8 channels are 32 bytes of
    // fp32, and two `red.v4` per lane would put the lanes of one instruction
    // in different 32-byte sectors. Reduce channel quads interleaved instead:
    // in reduction k (0, 1) lane `sub` adds channels (k*LPR + sub)*4 .. +3, so
    // neighbouring lanes fill one sector per instruction. gq holds grad_out in
    // that order.
    constexpr bool QUADS = sizeof(T) == 2 && VEC == 8 && !FIXED &&
                           (MODE == kCounted || (MODE != kNoScatter && sizeof(A) == 4));
    // Same-row merging (see the scatter below): one corner item per lane needs
    // the 4 corners of a group to fit in its LPR lanes, one point per group.
    // It pays where a query's points share rows (dense, local sampling such as
    // an encoder's) and costs where they do not, so the host selects it.
    constexpr bool COMBINE = MODE == kScatterMerge && LPR >= 4 && NB == 1;
    // Fixed-point reductions are scalar 8-byte `red`s; in reduction k lane
    // `sub` adds channel j*LPR*VEC + k*LPR + sub, so the LPR lanes of a group
    // fill consecutive 8-byte words. gi holds grad_out in that order.
    float gi[FIXED ? CPL : 1][FIXED ? VEC : 1];
    if constexpr (FIXED) {
      const T* gp = reinterpret_cast<const T*>(p.grad_out) + qm * D;
#pragma unroll
      for (int j = 0; j < CPL; ++j)
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
          const int ch = j * LPR * VEC + k * LPR + sub;
          gi[j][k] = (live && ch < D) ? to_f32(gp[ch]) : 0.f;
        }
    }
    float gq[QUADS ? CPL : 1][2][4];
    if constexpr (QUADS) {
      const T* gp = reinterpret_cast<const T*>(p.grad_out) + qm * D;
#pragma unroll
      for (int j = 0; j < CPL; ++j)
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const int ch = j * LPR * VEC + (k * LPR + sub) * 4;
          if (live && ch < D) {
            load_vec<T, 4>(gp + ch, gq[j][k]);
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) gq[j][k][e] = 0.f;
          }
        }
    }

    // The first NB points' (x, y, a) are in flight while the level table loads;
    // every iteration then loads the next one's while its gathers are in flight.
    float2 pxy[NB];
    float pat[NB];
    // SHARE: this lane's own point (query my_q of the warp, point my_s).
    const int my_q = SHARE ? lane / LK : 0, my_s = SHARE ? lane - my_q * LK : 0;
    const bool my_live = SHARE && my_q < QW && q - qsub + my_q < p.Q;
#pragma unroll
    for (int n = 0; n < NB; ++n) {
      const int s = n * GQ + gq_;
      pxy[n] = make_float2(0.f, 0.f);
      pat[n] = 0.f;
      if constexpr (SHARE) {
        if (my_live) {
          const int64_t qm_mine = (b * p.Q + (q - qsub + my_q)) * p.M + m;
          pxy[n] = load_pair(reinterpret_cast<const T*>(p.loc) + qm_mine * (2 * LK) + 2 * my_s);
          pat[n] = to_f32(reinterpret_cast<const T*>(p.attn)[qm_mine * LK + my_s]);
        }
      } else if (live && s < LK) {
        pxy[n] = load_pair(lp + 2 * s);
        pat[n] = to_f32(ap[s]);
      }
    }
    if (round == 0) load_levels(p.shapes, p.starts, p.L, p.S, lv, p.Q, p.K);  // syncs the block
    if (!__any_sync(kFullMask, live)) break;  // warp-uniform: past the last query
    int sh_p00 = 0, sh_p10 = 0;
    unsigned sh_valid = 0u;
    float sh_lx = 0.f, sh_ly = 0.f;
    if constexpr (SHARE) {
      if (my_live) {
        const Bilinear bm = resolve(pxy[0].x, pxy[0].y, lv[level_of(my_s, p.K, p.kshift)]);
        sh_p00 = bm.pix[0];
        sh_p10 = bm.pix[2];
        sh_lx = bm.lx;
        sh_ly = bm.ly;
        sh_valid = bm.valid;
      }
    }
    // Fused prologue: this query's reference point and its head's softmax;
    // sdot accumulates sum_s a_s * dL/da_s for the softmax backward.
    float2 refp = make_float2(0.f, 0.f);
    float smx = 0.f, sinv = 1.f, sdot = 0.f;
    if constexpr (FUSED) {
      refp = load_pair(reinterpret_cast<const T*>(p.ref) + 2 * (b * p.Q + q));
      warp_softmax_stats(ap, LK, lane, smx, sinv);
    }

    for (int s0 = 0; s0 < LK; s0 += GQ * NB) {
      Bilinear bl[NB];
      float at[NB];
      float fw[NB], fh[NB];
      bool dense[NB];
      if constexpr (SHARE) {
        const int s = s0 + gq_;
        const bool ok = live && s < LK;
        const int src = qsub * LK + (s < LK ? s : 0);
        const int p00 = __shfl_sync(kFullMask, sh_p00, src), p10 = __shfl_sync(kFullMask, sh_p10, src);
        const float lx = __shfl_sync(kFullMask, sh_lx, src), ly = __shfl_sync(kFullMask, sh_ly, src);
        const float a = __shfl_sync(kFullMask, pat[0], src);
        const unsigned v = __shfl_sync(kFullMask, sh_valid, src);
        bl[0].pix[0] = p00;
        bl[0].pix[1] = p00 + 1;
        bl[0].pix[2] = p10;
        bl[0].pix[3] = p10 + 1;
        bl[0].lx = lx;
        bl[0].ly = ly;
        bl[0].w[0] = (1.0f - lx) * (1.0f - ly);
        bl[0].w[1] = lx * (1.0f - ly);
        bl[0].w[2] = (1.0f - lx) * ly;
        bl[0].w[3] = lx * ly;
        bl[0].valid = ok ? v : 0u;
        at[0] = ok ? a : 0.f;
        const LevelInfo& L = lv[level_of(ok ? s : 0, p.K, p.kshift)];
        fw[0] = ok ? L.fW : 0.f;
        fh[0] = ok ? L.fH : 0.f;
        dense[0] = ok && L.dense;
      } else {
#pragma unroll
        for (int n = 0; n < NB; ++n) {
          const int s = s0 + n * GQ + gq_;
          if (live && s < LK) {
            const float2 xy = pxy[n];  // loaded one iteration ahead
            const LevelInfo& L = lv[level_of(s, p.K, p.kshift)];
            if constexpr (FUSED) {
              at[n] = expf(pat[n] - smx) * sinv;
              bl[n] = resolve_fused(refp, xy, L);
            } else {
              at[n] = pat[n];
              bl[n] = resolve(xy.x, xy.y, L);
            }
            fw[n] = L.fW;
            fh[n] = L.fH;
            dense[n] = L.dense;
          } else {
            at[n] = 0.f;
            fw[n] = fh[n] = 0.f;
            bl[n] = empty_slot();
            dense[n] = false;
          }
        }
      }
      Raw raw[NB][4][CPL];
      unsigned hits[NB][4];
      unsigned rmx[EXACT ? NB : 1][4];  // EXACT: the rows' bounds
#pragma unroll
      for (int n = 0; n < NB; ++n)
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int j = 0; j < CPL; ++j) {
            const int ch = (j * LPR + sub) * VEC;
            Raw r{};
            if (((bl[n].valid >> c) & 1u) && ch < D) {
              if constexpr (SCATTER && VEC * sizeof(T) == 16) {
                const uint4 u = ldg16_hint(vb + bl[n].pix[c] * rs + ch, pol_stream);
                r = *reinterpret_cast<const Raw*>(&u);
              } else {
                r = load_raw<T, VEC>(vb + bl[n].pix[c] * rs + ch);
              }
            }
            raw[n][c][j] = r;
          }

      // The next iteration's (x, y, a), in flight with this iteration's gathers.
#pragma unroll
      for (int n = 0; n < NB; ++n) {
        const int sn = s0 + GQ * NB + n * GQ + gq_;
        if (!SHARE && live && sn < LK) {
          pxy[n] = load_pair(lp + 2 * sn);
          pat[n] = to_f32(ap[sn]);
        }
      }
      // The value gathers above need nothing from the kernel before this one
      // (the zero-fill or the hit count); the counts and the reduction target do.
      if constexpr (SCATTER) pdl_wait();
      if constexpr (FIXED) {
        if (round == 0 && s0 == 0) fx = fixed_scale(p.fixed_hdr, p.fixed_log2n);  // written by the absmax pass
      }
#pragma unroll
      for (int n = 0; n < NB; ++n)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          hits[n][c] = 0u;
          if constexpr (EXACT) rmx[n][c] = 0u;
          // Dense-level rows are always reduced in fp32: no count to read.
          // Counts and bounds come from the kernel before this one, which may
          // still run when this kernel starts (programmatic dependent
          // launch): ordinary (L2) loads, never the read-only `__ldg` path,
          // whose loads the compiler treats as invariant and may issue before
          // pdl_wait().
          if constexpr (MODE == kCounted && !COMBINE)
            if ((bl[n].valid >> c) & 1u) {
              // (EXACT reads them too: the scale needs the count below the flag)
              if constexpr (EXACT) {
                const uint2 cb = __ldcg(cpb + (int64_t)bl[n].pix[c] * p.M);
                hits[n][c] = cb.x;
                rmx[n][c] = cb.y;
              } else {
                hits[n][c] = dense[n] ? kDenseRow : __ldcg(cnb + (int64_t)bl[n].pix[c] * p.M);
              }
            }
        }
#pragma unroll
      for (int n = 0; n < NB; ++n) {
        // Per-corner dot products over this lane's channels,
        // P_c = sum_d g_d * v_c,d; the three gradients are linear in them:
        //   ga = sum_c w_c P_c
        //   gx = (1 - ly)(P01 - P00) + ly (P11 - P10)
        //   gy = (1 - lx)(P10 - P00) + lx (P11 - P01)
        float P[4];
        if constexpr (MIXED) {
          // Two fp32 accumulators per corner (low / high halves of each word).
          float pl[4] = {0.f, 0.f, 0.f, 0.f}, ph[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int j = 0; j < CPL; ++j) {
            const unsigned* gw = reinterpret_cast<const unsigned*>(&graw[j]);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const unsigned* vw = reinterpret_cast<const unsigned*>(&raw[n][c][j]);
#pragma unroll
              for (int e = 0; e < VEC / 2; ++e) {
                pl[c] = fma_lo16(gw[e], vw[e], pl[c], (const T*)nullptr);
                ph[c] = fma_hi16(gw[e], vw[e], ph[c], (const T*)nullptr);
              }
            }
          }
#pragma unroll
          for (int c = 0; c < 4; ++c) P[c] = pl[c] + ph[c];
        } else if constexpr (VEC % 2 == 0) {
          uint64_t acc2[4];
#pragma unroll
          for (int c = 0; c < 4; ++c) acc2[c] = 0ull;
#pragma unroll
          for (int j = 0; j < CPL; ++j)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              uint64_t v2[VEC / 2];
              raw_to_f2<T, VEC>(raw[n][c][j], v2);
#pragma unroll
              for (int e = 0; e < VEC / 2; ++e) acc2[c] = f2_fma(g2[j][e], v2[e], acc2[c]);
            }
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            float lo, hi;
            f2_unpack(acc2[c], lo, hi);
            P[c] = lo + hi;
          }
        } else {
#pragma unroll
          for (int c = 0; c < 4; ++c) P[c] = 0.f;
#pragma unroll
          for (int j = 0; j < CPL; ++j)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              float v[VEC];
              unpack_raw<T, VEC>(raw[n][c][j], v);
#pragma unroll
              for (int e = 0; e < VEC; ++e) P[c] = fmaf(g[j][e], v[e], P[c]);
            }
        }
        const float lx = bl[n].lx, ly = bl[n].ly;
        float ga = bl[n].w[0] * P[0];
        ga = fmaf(bl[n].w[1], P[1], ga);
        ga = fmaf(bl[n].w[2], P[2], ga);
        ga = fmaf(bl[n].w[3], P[3], ga);
        float gx = (1.f - ly) * (P[1] - P[0]);
        gx = fmaf(ly, P[3] - P[2], gx);
        float gy = (1.f - lx) * (P[2] - P[0]);
        gy = fmaf(lx, P[3] - P[1], gy);
#pragma unroll
        for (int off = 1; off < LPR; off <<= 1) {
          ga += __shfl_xor_sync(kFullMask, ga, off);
          gx += __shfl_xor_sync(kFullMask, gx, off);
          gy += __shfl_xor_sync(kFullMask, gy, off);
        }
        const int s = s0 + n * GQ + gq_;
        if (live && s < LK && sub == 0) {
          if constexpr (FUSED) {
            // d/d offset = d/d pixel coordinate; dL/da kept (fp32 in shared
            // memory when it fits) for the softmax pass.
            store_pair(glp + 2 * s, at[n] * gx, at[n] * gy);
            sdot = fmaf(at[n], ga, sdot);
            if (LK <= kFusedMaxLK)
              fused_ga[threadIdx.x >> 5][s] = ga;
            else
              gap[s] = from_f32<T>(ga);
          } else {
            store_pair(glp + 2 * s, at[n] * fw[n] * gx, at[n] * fh[n] * gy);
            gap[s] = from_f32<T>(ga);
          }
        }
        if constexpr (SCATTER) {
          // Writes this lane's channels of a * w * grad_out into row `pix`
          // (weight wc; `hits` is the row's count in the counted mode).
          auto scatter_row = [&](int pix, float wc, unsigned hits, unsigned rmax) {
            // EXACT (rows of 64-bit words; fp32 rows in their first half): a
            // row with 2 .. kExactMaxHits hits gets each contribution fl(wc g)
            // as an integer-valued float on the row's scale, a row with
            // more hits wc g * 2^F rounded to a 64-bit integer (wide); nothing
            // when the bound is zero (every contribution is zero), plain fp32
            // when the scale falls back.
            bool exact_row = false, wide = false;
            ExactScale xs{1.f, 1.f, 1.f, 1.f};
            double wd = 0.0;
            if constexpr (EXACT) {
              if (hits > 1u) {  // a dense-level row (flagged) whatever its count
                if (rmax == 0u) return;
                const unsigned nh = hits & ~kDenseRow;
                if (nh > kExactMaxHits) {
                  double inv;
                  wide = wide_scale(rmax, nh, wd, inv);
                  wd *= (double)wc;  // exact: a power-of-two scale
                } else {
                  exact_row = exact_scale(rmax, nh, xs);
                }
              }
            }
            // exact rows: one FMA rounds the exact product wc 2^F g to an
            // integer (wc 2^F is exact); a weight that 2^F would push past
            // 2^100 (its grad_out row is tiny) is split as (wc 2^F1)(g 2^F2)
            const float wx = wc * xs.s1 * xs.s2;
            const bool split = !(fabsf(wx) < 0x1p100f);
            const float wa = split ? wc * xs.s1 : wx, gb = split ? xs.s2 : 1.f;
            auto term = [&](float gv) {
              return exact_row ? fmaf(wa, split ? gv * gb : gv, kExactMagic) - kExactMagic : __fmul_rn(wc, gv);
            };
#pragma unroll
            for (int j = 0; j < CPL; ++j) {
              const int ch = (j * LPR + sub) * VEC;
              if constexpr (FIXED) {
                // Fixed-point reduction in interleaved channels (see gi). In
                // the counted mode a one-hit row is stored and a two-hit row
                // reduced in fp32 (below): fp32 addition is commutative, so
                // 0 + a + b == 0 + b + a bitwise and two terms need no fixed
                // point; three or more (and dense-level rows) do.
                if (MODE != kCounted || hits > 2u) {
                  long long* row = (MODE == kCounted ? faccb : reinterpret_cast<long long*>(gvb)) + pix * rs;
                  if (fx.ok) {
                    const double wd = (double)wc * fx.scale;  // exact
#pragma unroll
                    for (int k = 0; k < VEC; ++k) {
                      const int ci = j * LPR * VEC + k * LPR + sub;
                      if (ci < D) red_fixed(row + ci, wd, (double)gi[j][k], pol_keep);
                    }
                  } else {  // fp32 fallback into the low words
#pragma unroll
                    for (int k = 0; k < VEC; ++k) {
                      const int ci = j * LPR * VEC + k * LPR + sub;
                      if (ci < D) atomicAdd(reinterpret_cast<float*>(row + ci), wc * gi[j][k]);
                    }
                  }
                  continue;
                }
              }
              if constexpr (QUADS) {
                // fp32 reduction in interleaved quads (see gq); a counted
                // one-hit row is stored in the natural layout.
                if (MODE != kCounted || hits != 1u) {
                  if constexpr (EXACT) {
                    if (wide) {  // a lane's 4 channels fill one 32-byte sector
#pragma unroll
                      for (int k = 0; k < 2; ++k) {
                        const int cq = j * LPR * VEC + (k * LPR + sub) * 4;
                        if (cq < D)
#pragma unroll
                          for (int e = 0; e < 4; ++e)
                            red_fixed(faccb + pix * rs + cq + e, wd, (double)gq[j][k][e], pol_keep);
                      }
                      continue;
                    }
                  }
                  float* row = MODE != kCounted ? reinterpret_cast<float*>(gvb) + pix * rs
                               : EXACT          ? reinterpret_cast<float*>(faccb + pix * rs)
                                                : accb + pix * rs;
#pragma unroll
                  for (int k = 0; k < 2; ++k) {
                    const int cq = j * LPR * VEC + (k * LPR + sub) * 4;
                    if (cq < D)
                      red_add_f32x4_hint(row + cq, term(gq[j][k][0]), term(gq[j][k][1]), term(gq[j][k][2]),
                                         term(gq[j][k][3]), pol_keep);
                  }
                  continue;
                }
              }
              if (ch < D) {
                float contrib[VEC];
                if constexpr (VEC % 2 == 0) {
                  const uint64_t wc2 = f2_pack(wc, wc);
#pragma unroll
                  for (int e = 0; e < VEC / 2; ++e)
                    f2_unpack(f2_mul(wc2, g2[j][e]), contrib[2 * e], contrib[2 * e + 1]);
                } else {
#pragma unroll
                  for (int e = 0; e < VEC; ++e) contrib[e] = wc * g[j][e];
                }
                if constexpr (EXACT) {
                  if (exact_row) {
#pragma unroll
                    for (int e = 0; e < VEC; ++e) contrib[e] = term(g[j][e]);
                  }
                }
                if constexpr (MODE == kCounted) {
                  // A row with one hit gets its only contribution stored
                  // (rounded once, as fp32 accumulation would); rows with
                  // more hits accumulate in fp32.
                  if (hits == 1u) {
                    store_vec<T, VEC>(gvt + pix * rs + ch, contrib);
                  } else if constexpr (EXACT) {
                    if (wide) {
#pragma unroll
                      for (int e = 0; e < VEC; ++e) red_fixed(faccb + pix * rs + ch + e, wd, (double)g[j][e], pol_keep);
                    } else {
                      red_add_vec_hint<float, VEC>(reinterpret_cast<float*>(faccb + pix * rs) + ch, contrib, pol_keep);
                    }
                  } else if constexpr (!FIXED)
                    red_add_vec_hint<float, VEC>(accb + pix * rs + ch, contrib, pol_keep);
                  else  // two hits: fp32 in the first half of the 64-bit row
                    red_add_vec_hint<float, VEC>(reinterpret_cast<float*>(faccb + pix * rs) + ch, contrib,
                                                 pol_keep);
                } else if constexpr (!FIXED) {
                  red_add_vec_hint<A, VEC>(gvb + pix * rs + ch, contrib, pol_keep);
                }
              }
            }
          };
          if constexpr (COMBINE) {
            // Same-row merging. Every contribution of this query is a multiple
            // of the same grad_out vector, so corners of the warp's points that
            // land on one row need one write of (sum of their weights) *
            // grad_out. Lane `sub` < 4 of a group holds corner `sub` of the
            // group's point as an item (row, weight); lanes with equal rows
            // find each other with a match, the lowest one leads and owns the
            // summed weight (added in lane order: deterministic).
            const int cs = sub & 3;
            const unsigned vbit = (bl[n].valid >> cs) & 1u;
            const bool have = live && s < LK && sub < 4 && vbit != 0u;
            const int pix_s = cs == 0 ? bl[n].pix[0] : cs == 1 ? bl[n].pix[1] : cs == 2 ? bl[n].pix[2] : bl[n].pix[3];
            const float w_s = cs == 0 ? bl[n].w[0] : cs == 1 ? bl[n].w[1] : cs == 2 ? bl[n].w[2] : bl[n].w[3];
            // rows are >= 0 (pix * QW + query stays below 2^31: S <= 2^30, QW <= 2);
            // empty items never match
            const int key = have ? pix_s * QW + qsub : -1 - lane;
            const float wt = have ? at[n] * w_s : 0.f;
            const unsigned same = __match_any_sync(kFullMask, key);
            float wsum = wt;
            if (__any_sync(kFullMask, __popc(same) > 1)) {
              wsum = 0.f;
              unsigned rest = same;
              const int rounds = __reduce_max_sync(kFullMask, (unsigned)__popc(same));
              for (int r = 0; r < rounds; ++r) {
                const int src = rest ? __ffs(rest) - 1 : lane;
                const float v = __shfl_sync(kFullMask, wt, src);
                if (rest) {
                  wsum += v;
                  rest &= rest - 1;
                }
              }
            }
            const int lead = have && __ffs(same) - 1 == lane;
            unsigned hits_me = 0u;
            if constexpr (MODE == kCounted)
              if (lead) hits_me = dense[n] ? kDenseRow : __ldcg(cnb + (int64_t)(key / QW) * p.M);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const int src = grp * LPR + c;
              const int lead_c = __shfl_sync(kFullMask, lead, src);
              const int pix_c = __shfl_sync(kFullMask, key, src);
              const float w_c = __shfl_sync(kFullMask, wsum, src);
              unsigned hits_c = 0u;
              if constexpr (MODE == kCounted) hits_c = __shfl_sync(kFullMask, hits_me, src);
              if (lead_c) scatter_row(pix_c / QW, w_c, hits_c, 0u);
            }
          } else if (live && s < LK) {
#pragma unroll
            for (int c = 0; c < 4; ++c)
              if ((bl[n].valid >> c) & 1u)
                scatter_row(bl[n].pix[c], at[n] * bl[n].w[c], hits[n][c], EXACT ? rmx[EXACT ? n : 0][c] : 0u);
          }
        }
      }
    }
    if constexpr (FUSED) {
      // Softmax backward over the query-head's L*K points:
      //   dL/dlogit_s = a_s * (dL/da_s - sum_t a_t * dL/da_t),
      // dL/da_s as written above by this warp's lanes.
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sdot += __shfl_xor_sync(kFullMask, sdot, off);
      __syncwarp();
      for (int s = lane; s < LK; s += 32) {
        const float a = expf(to_f32(ap[s]) - smx) * sinv;
        const float ga = LK <= kFusedMaxLK ? fused_ga[threadIdx.x >> 5][s] : to_f32(gap[s]);
        gap[s] = from_f32<T>(a * (ga - sdot));
      }
    }
  }  // rounds
}

// ---------------------------------------------------------------------------
// Hit-counted scatter, pass 1 (one kernel, two roles).
//
// Point blocks: one thread per sampling point of a sparse level counts the
// bilinear hits of its corner rows (b, pixel, m); the hit that raises a
// row's count from 1 to 2 zero-fills that row's fp32 accumulator, so exactly
// the multi-hit rows are zeroed, once. The four corner atomics are issued
// before any zeroing waits on their results. Points of dense levels do
// nothing here.
//
// Dense blocks (the last blocks of the grid): flag every row of the dense
// levels with kDenseRow and zero its fp32 accumulator. The backward reduces
// into flagged rows without reading their counts, the finalize rounds them.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void zero_row(float* a, int D) {
  if ((D & 3) == 0 && (reinterpret_cast<uintptr_t>(a) & 15) == 0) {
    for (int d = 0; d < D; d += 4) *reinterpret_cast<float4*>(a + d) = make_float4(0.f, 0.f, 0.f, 0.f);
  } else {
    for (int d = 0; d < D; ++d) a[d] = 0.f;
  }
}

// r-th pixel (0-based) of the concatenated dense levels -> pixel index in S.
__device__ __forceinline__ int64_t dense_pixel(const LevelInfo* lv, int L, int64_t r) {
  for (int l = 0; l < L; ++l) {
    if (!lv[l].dense) continue;
    const int64_t n = (int64_t)lv[l].H * lv[l].W;
    if (r < n) return lv[l].start + r;
    r -= n;
  }
  return 0;  // unreachable for r < dense pixels per batch
}

// One warp per dense pixel row (the M*D accumulator elements of all heads of
// one pixel): flag its M counts and zero its accumulator.
__device__ __forceinline__ void count_dense_rows(const OpParams& p, const LevelInfo* lv, int64_t warp,
                                                 int64_t nwarps, int cstride) {
  int64_t per_batch = 0;
  for (int l = 0; l < p.L; ++l)
    if (lv[l].dense) per_batch += (int64_t)lv[l].H * lv[l].W;
  if (per_batch == 0) return;
  const int lane = threadIdx.x & 31;
  const int64_t row_floats = (int64_t)p.M * p.D * p.acc_words;  // 32-bit words
  const bool vec = row_floats % 4 == 0 && (reinterpret_cast<uintptr_t>(p.acc) & 15) == 0;
  for (int64_t px = warp; px < p.B * per_batch; px += nwarps) {
    const int64_t b = px / per_batch;
    const int64_t pix = dense_pixel(lv, p.L, px - b * per_batch);
    const int64_t row0 = (b * p.S + pix) * p.M;  // first (b, pix, m) row
    for (int m = lane; m < p.M; m += 32) atomicOr(p.counts + (row0 + m) * cstride, kDenseRow);
    float* a = reinterpret_cast<float*>(p.acc) + row0 * p.D * p.acc_words;
    if (vec) {
      for (int64_t k = lane; k < row_floats / 4; k += 32)
        reinterpret_cast<float4*>(a)[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    } else {
      for (int64_t k = lane; k < row_floats; k += 32) a[k] = 0.f;
    }
  }
}

// Query-heads a block of 256 points can touch (256 / (L*K) + 2).
constexpr int kCountMaxQm = 258;

// EXACT (deterministic fp16 / bf16): the dense levels are counted too, with
// fire-and-forget `red.add`s below the dense blocks' flag (the exact scale
// needs every row's count), and each valid corner raises its row's bound
// p.rowmax to the bits of |a| * max|grad_out[qm, :]| (|a| <= 1 for the fused
// softmax weights) with a `red.max`; the point blocks compute max|grad_out|
// of their query-heads first.
template <typename T, bool FUSED = false, bool EXACT = false>
__global__ void __launch_bounds__(256) msda_count_kernel(const OpParams p, unsigned point_blocks) {
  pdl_trigger();
  __shared__ LevelInfo lv[kMaxLevels];
  __shared__ unsigned s_gmax[EXACT ? kCountMaxQm : 1];
  const int LK = p.L * p.K;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const bool point = blockIdx.x < point_blocks && i < p.BQM * LK;
  float2 xy = make_float2(0.f, 0.f);
  if (point) xy = load_pair(reinterpret_cast<const T*>(p.loc) + 2 * i);  // in flight across the sync
  float amag = 1.f;
  int64_t qm0 = 0;
  int nq = 0;
  // EXACT: max |grad_out| (NaN kept) of the block's query-heads, whose rows
  // are consecutive (nq * D elements from row qm0); the first kCountPreload
  // 16-byte vectors of each thread are in flight across the level-table sync.
  constexpr int V = 16 / (int)sizeof(T);
  constexpr int kCountPreload = 2;
  const T* g = reinterpret_cast<const T*>(p.grad_out);
  int64_t ne = 0;
  bool gvec = false;
  float pmx[EXACT ? kCountPreload : 1];
  int pq[EXACT ? kCountPreload : 1];
  if constexpr (EXACT) {
    if (!FUSED && point) amag = fabsf(to_f32(reinterpret_cast<const T*>(p.attn)[i]));
    const int64_t first = (int64_t)blockIdx.x * blockDim.x;
    const int64_t last = min(first + (int64_t)blockDim.x, p.BQM * LK) - 1;
    qm0 = first / LK;
    nq = first <= last ? (int)(last / LK - qm0 + 1) : 0;
    for (int k = threadIdx.x; k < nq; k += blockDim.x) s_gmax[k] = 0u;
    g += qm0 * p.D;
    ne = (int64_t)nq * p.D;
    gvec = (reinterpret_cast<uintptr_t>(g) & 15) == 0 && p.D % V == 0;
#pragma unroll
    for (int k = 0; k < kCountPreload; ++k) {
      const int64_t e = ((int64_t)k * blockDim.x + threadIdx.x) * V;
      pq[k] = -1;
      pmx[k] = 0.f;
      if (gvec && e < ne) {
        float v[V];
        load_vec<T, V>(g + e, v);
#pragma unroll
        for (int q = 0; q < V; ++q) pmx[k] = max_abs_nan(pmx[k], v[q]);
        pq[k] = (int)(e / p.D);
      }
    }
  }
  load_levels(p.shapes, p.starts, p.L, p.S, lv, p.Q, p.K);  // syncs the block
  if constexpr (EXACT) {
    // A row's D / V vectors sit in consecutive lanes when D / V is a power of
    // two up to 32 (the warp's vectors start at a multiple of 32 * V): their
    // maxima combine by shuffles and one lane writes the row's entry.
    const int vr = p.D / V;
    const bool lanes = gvec && vr <= 32 && (vr & (vr - 1)) == 0;
#pragma unroll
    for (int k = 0; k < kCountPreload; ++k) {
      if (lanes) {
        float mx = pmx[k];
        for (int off = 1; off < vr; off <<= 1) mx = max_abs_nan(mx, __shfl_xor_sync(kFullMask, mx, off));
        if (pq[k] >= 0 && (threadIdx.x & (vr - 1)) == 0) s_gmax[pq[k]] = __float_as_uint(mx) & 0x7fffffffu;
      } else if (pq[k] >= 0) {
        atomicMax(s_gmax + pq[k], __float_as_uint(pmx[k]) & 0x7fffffffu);
      }
    }
    if (gvec) {
      for (int64_t e = ((int64_t)kCountPreload * blockDim.x + threadIdx.x) * V; e < ne;
           e += (int64_t)blockDim.x * V) {
        float v[V];
        load_vec<T, V>(g + e, v);
        float mx = 0.f;
#pragma unroll
        for (int q = 0; q < V; ++q) mx = max_abs_nan(mx, v[q]);
        atomicMax(s_gmax + e / p.D, __float_as_uint(mx) & 0x7fffffffu);
      }
    } else {
      for (int64_t e = threadIdx.x; e < ne; e += blockDim.x)
        atomicMax(s_gmax + e / p.D, __float_as_uint(max_abs_nan(0.f, to_f32(g[e]))) & 0x7fffffffu);
    }
    __syncthreads();
  }
  // Counts (and the absmax header) are zeroed by the kernel before this one:
  // everything above ran under its tail; nothing below may precede it.
  pdl_wait();
  if (blockIdx.x >= point_blocks) {
    const int wpb = blockDim.x >> 5;
    count_dense_rows(p, lv, (int64_t)(blockIdx.x - point_blocks) * wpb + (threadIdx.x >> 5),
                     (int64_t)(gridDim.x - point_blocks) * wpb, EXACT ? 2 : 1);
    return;
  }
  if (!point) return;
  int64_t qm, b;
  int s, m;
  if (p.BQM * LK <= 0xffffffffll) {  // 32-bit index arithmetic
    const unsigned u = (unsigned)i, qmu = u / (unsigned)LK;
    s = (int)(u - qmu * (unsigned)LK);
    qm = qmu;
    b = qmu / (unsigned)(p.Q * p.M);
    m = (int)(qmu % (unsigned)p.M);
  } else {
    qm = i / LK;
    s = (int)(i - qm * LK);
    b = qm / (p.Q * p.M);
    m = (int)(qm % p.M);
  }
  const LevelInfo& L = lv[level_of(s, p.K, p.kshift)];
  if (!EXACT && L.dense) return;
  Bilinear bl;
  if constexpr (FUSED) {  // offsets around the query's reference point
    const int64_t bq = qm / p.M;  // b * Q + q
    bl = resolve_fused(load_pair(reinterpret_cast<const T*>(p.ref) + 2 * bq), xy, L);
  } else {
    bl = resolve(xy.x, xy.y, L);
  }
  unsigned old[4];
  int64_t row[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    old[c] = 0u;
    row[c] = (b * p.S + bl.pix[c]) * p.M + m;
    if ((bl.valid >> c) & 1u) {
      if (EXACT && L.dense)  // counted below the flag; the dense blocks zero the row
        asm volatile("red.global.add.u32 [%0], 1;" ::"l"(p.counts + 2 * row[c]) : "memory");
      else
        old[c] = atomicAdd(p.counts + (EXACT ? 2 : 1) * row[c], 1u);
    }
  }
  if constexpr (EXACT) {
    // |a| * gmax: non-negative float bits order as unsigned, NaN / Inf above
    // every finite bound
    const unsigned bound = __float_as_uint(amag * __uint_as_float(s_gmax[qm - qm0])) & 0x7fffffffu;
#pragma unroll
    for (int c = 0; c < 4; ++c)
      if ((bl.valid >> c) & 1u)
        asm volatile("red.global.max.u32 [%0], %1;" ::"l"(p.rowmax + 2 * row[c]), "r"(bound) : "memory");
  }
  // old == 1 only on unflagged rows: a flagged (dense) row is zeroed by the
  // dense blocks. EXACT: the second hit zeroes the fp32 half of the 64-bit
  // row, the hit that makes the row busy (old == kExactMaxHits) all of it.
  if (L.dense) return;
#pragma unroll
  for (int c = 0; c < 4; ++c)
    if ((bl.valid >> c) & 1u) {
      float* a = reinterpret_cast<float*>(p.acc) + row[c] * p.D * p.acc_words;
      if (old[c] == 1u) zero_row(a, EXACT ? p.D : p.D * p.acc_words);
      if (EXACT && old[c] == kExactMaxHits) zero_row(a, p.D * p.acc_words);
    }
}

// Hit-counted scatter, pass 3: rows nothing hit become zeros; multi-hit and
// dense-level rows (count > 1, or the kDenseRow flag) are rounded from their
// accumulator -- fp32, or 64-bit fixed point (FIXED) -- (skipped when
// grad_value itself is the fp32 accumulator); one-hit rows were already
// stored by the backward.
// One thread per 4 consecutive rows x VEC elements (one 16-byte count load).
// EXACT: the accumulator rows are 64-bit; rows with 2 .. kExactMaxHits hits
// hold integer-valued fp32 sums on the row's scale 2^F (exact_scale) in their
// first half and are multiplied by 2^-F (exact), busier rows a 64-bit
// integer sum (wide_scale), before the one rounding to the value dtype.
template <typename T, int VEC, bool FIXED = false, bool EXACT = false>
__global__ void __launch_bounds__(256, EXACT ? 6 : 8) msda_finalize_kernel(const OpParams p) {
  const int D = p.D;
  const int per_row = D / VEC;
  const int64_t rows = p.B * p.S * p.M;
  const int64_t quads = (rows + 3) / 4;
  const bool in_place = !FIXED && reinterpret_cast<const void*>(p.acc) == p.grad_value;
  const bool quad_loads = (reinterpret_cast<uintptr_t>(p.counts) & 15) == 0;
  pdl_wait();  // counts and accumulator rows come from the count pass and the backward
  // (ordinary loads, never the read-only `__ldg` path: the compiler treats
  // those as invariant and may issue them before the wait)
  FixedScale fx{1.0, 1.f, 1.f, true};
  if constexpr (FIXED) fx = fixed_scale(p.fixed_hdr, p.fixed_log2n);
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < quads * per_row;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t quad = t / per_row;  // rows 4*quad .. 4*quad+3
    const int chunk = (int)(t - quad * per_row);
    unsigned cnt[4], rmq[4];
    if (quad * 4 + 3 < rows && quad_loads) {
      if constexpr (EXACT) {  // (count, bound) pairs
        const uint4 a4 = __ldcg(reinterpret_cast<const uint4*>(p.counts) + 2 * quad);
        const uint4 b4 = __ldcg(reinterpret_cast<const uint4*>(p.counts) + 2 * quad + 1);
        cnt[0] = a4.x; rmq[0] = a4.y; cnt[1] = a4.z; rmq[1] = a4.w;
        cnt[2] = b4.x; rmq[2] = b4.y; cnt[3] = b4.z; rmq[3] = b4.w;
      } else {
        const uint4 c4 = __ldcg(reinterpret_cast<const uint4*>(p.counts) + quad);
        cnt[0] = c4.x; cnt[1] = c4.y; cnt[2] = c4.z; cnt[3] = c4.w;
      }
    } else {
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int64_t row = quad * 4 + r;
        cnt[r] = row < rows ? __ldcg(p.counts + (EXACT ? 2 : 1) * row) : 1u;
        if constexpr (EXACT) rmq[r] = row < rows ? __ldcg(p.rowmax + 2 * row) : 0u;
      }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      if (cnt[r] == 1u || (cnt[r] > 1u && in_place)) continue;
      const int64_t e = (quad * 4 + r) * D + chunk * VEC;
      float v[VEC];
      if (cnt[r] == 0u) {
#pragma unroll
        for (int k = 0; k < VEC; ++k) v[k] = 0.f;
      } else if constexpr (EXACT) {
        // 64-bit rows: busy rows hold a 64-bit integer sum, the others an
        // fp32 sum in the row's first half, integer-valued on the row's scale
        // (plain fp32 when the scale falls back)
        const long long* a = reinterpret_cast<const long long*>(p.acc) + e;
        const float* f = reinterpret_cast<const float*>(a - chunk * VEC) + chunk * VEC;
        const unsigned rm = rmq[r];
        const unsigned nh = cnt[r] & ~kDenseRow;
        double sc, inv;
        if (nh > kExactMaxHits && wide_scale(rm, nh, sc, inv)) {
          if constexpr (VEC % 2 == 0) {
#pragma unroll
            for (int k = 0; k < VEC; k += 2) {
              const longlong2 w = __ldcs(reinterpret_cast<const longlong2*>(a + k));
              v[k] = (float)((double)w.x * inv);
              v[k + 1] = (float)((double)w.y * inv);
            }
          } else {
#pragma unroll
            for (int k = 0; k < VEC; ++k) v[k] = (float)((double)__ldcs(a + k) * inv);
          }
        } else {
          if constexpr (VEC % 4 == 0) {
#pragma unroll
            for (int k = 0; k < VEC; k += 4) {
              const float4 w = __ldcs(reinterpret_cast<const float4*>(f + k));
              v[k] = w.x;
              v[k + 1] = w.y;
              v[k + 2] = w.z;
              v[k + 3] = w.w;
            }
          } else {
#pragma unroll
            for (int k = 0; k < VEC; ++k) v[k] = __ldcs(f + k);
          }
          ExactScale xs;
          if (nh <= kExactMaxHits && exact_scale(rm, nh, xs)) {
#pragma unroll
            for (int k = 0; k < VEC; ++k) v[k] = v[k] * xs.inv2 * xs.inv1;  // exact, but for denormal results
          }
        }
      } else if constexpr (FIXED) {
        const long long* a = reinterpret_cast<const long long*>(p.acc) + e;
        if (cnt[r] == 2u) {  // two hits: an fp32 row at the start of the 64-bit row
          const float* f = reinterpret_cast<const float*>(a - chunk * VEC) + chunk * VEC;
#pragma unroll
          for (int k = 0; k < VEC; ++k) v[k] = __ldcs(f + k);
        } else if constexpr (VEC % 2 == 0) {
#pragma unroll
          for (int k = 0; k < VEC; k += 2) {
            const longlong2 f = __ldcs(reinterpret_cast<const longlong2*>(a + k));
            v[k] = fixed_to_f32(f.x, fx);
            v[k + 1] = fixed_to_f32(f.y, fx);
          }
        } else {
#pragma unroll
          for (int k = 0; k < VEC; ++k) v[k] = fixed_to_f32(__ldcs(a + k), fx);
        }
      } else if constexpr (VEC % 4 == 0) {
#pragma unroll
        for (int k = 0; k < VEC; k += 4) {
          const float4 f = __ldcs(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.acc) + e + k));
          v[k] = f.x;
          v[k + 1] = f.y;
          v[k + 2] = f.z;
          v[k + 3] = f.w;
        }
      } else {
#pragma unroll
        for (int k = 0; k < VEC; ++k) v[k] = __ldcs(reinterpret_cast<const float*>(p.acc) + e + k);
      }
      store_vec<T, VEC>(reinterpret_cast<T*>(p.grad_value) + e, v);
    }
  }
}

// Zero-fill of the scatter target (grad_value or the fp32 workspace) with
// evict_last stores, so the lines the reductions hit next are already in L2.
template <int kUnused = 0>  // a template, so the header can define it in every unit
__global__ void __launch_bounds__(256) msda_zero_kernel(void* __restrict__ dst, int64_t n16) {
  pdl_trigger();
  const uint64_t pol = policy_evict_last();
  char* d = reinterpret_cast<char*>(dst);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16;
       i += (int64_t)gridDim.x * blockDim.x)
    st_zero16_hint(d + i * 16, pol);
}

// fp32 accumulation buffer -> value dtype (the downcast of src/msda_triton/ops.py:91-92).
template <typename T, int VEC>
__global__ void __launch_bounds__(256) msda_cast_kernel(const float* __restrict__ src, T* __restrict__ dst,
                                                       int64_t nvec) {
  pdl_wait();  // the fp32 rows come from the backward
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

// ---------------------------------------------------------------------------
// Deterministic grad_value, pass 0: the header fixed_scale reads --
// hdr[0] = max |attention weight| (with `logits`, the weights are a softmax,
// at most 1: 1.0 unless a logit is non-finite), hdr[1] = max |grad_out|, as
// fp32 bit patterns of magnitudes (NaN and Inf sort above every finite
// value). The header is zeroed by the kernel before this one.
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ unsigned abs_bits(T x) {
  return __float_as_uint(to_f32(x)) & 0x7fffffffu;
}

// max |x| bits over p[0, n), this thread's grid-stride share: 16-byte vectors,
// four in flight per thread, when p is 16-byte aligned.
template <typename T>
__device__ __forceinline__ unsigned absmax_share(const T* __restrict__ p, int64_t n) {
  constexpr int V = 16 / (int)sizeof(T);
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  unsigned m = 0u;
  int64_t done = 0;
  if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
    const int64_t nv = n / V;
    const uint4* pv = reinterpret_cast<const uint4*>(p);
    for (int64_t i = tid; i < nv; i += 4 * stride) {
      uint4 r[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) r[u] = i + u * stride < nv ? __ldcs(pv + i + u * stride) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const T* e = reinterpret_cast<const T*>(&r[u]);
#pragma unroll
        for (int k = 0; k < V; ++k) m = max(m, abs_bits(e[k]));
      }
    }
    done = nv * V;
  }
  for (int64_t i = done + tid; i < n; i += stride) m = max(m, abs_bits(p[i]));
  return m;
}

template <typename T>
__global__ void __launch_bounds__(256) msda_absmax_kernel(const T* __restrict__ attn, int64_t n_attn,
                                                          int logits, const T* __restrict__ g,
                                                          int64_t n_g, unsigned* hdr) {
  pdl_trigger();
  unsigned ma = __reduce_max_sync(kFullMask, absmax_share(attn, n_attn));
  const unsigned mg = __reduce_max_sync(kFullMask, absmax_share(g, n_g));
  if (logits) ma = ma >= 0x7f800000u ? ma : 0x3f800000u;  // softmax weights: |a| <= 1
  pdl_wait();  // the header is zeroed by the kernel before this one
  if ((threadIdx.x & 31) == 0) {
    atomicMax(hdr, ma);
    atomicMax(hdr + 1, mg);
  }
}

// Deterministic scatter, last pass: 64-bit fixed-point accumulator -> value
// dtype (or fp32), each element rounded once.
template <typename T, int VEC>
__global__ void __launch_bounds__(256) msda_cast_fixed_kernel(const long long* __restrict__ src,
                                                             T* __restrict__ dst, int64_t nvec,
                                                             const unsigned* hdr, int clog2n) {
  pdl_wait();  // the accumulator rows come from the backward
  const FixedScale fx = fixed_scale(hdr, clog2n);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec;
       i += (int64_t)gridDim.x * blockDim.x) {
    float v[VEC];
    if constexpr (VEC % 2 == 0) {
#pragma unroll
      for (int k = 0; k < VEC; k += 2) {
        const longlong2 f = __ldcs(reinterpret_cast<const longlong2*>(src + i * VEC + k));
        v[k] = fixed_to_f32(f.x, fx);
        v[k + 1] = fixed_to_f32(f.y, fx);
      }
    } else {
#pragma unroll
      for (int k = 0; k < VEC; ++k) v[k] = fixed_to_f32(__ldcs(src + i * VEC + k), fx);
    }
    store_vec<T, VEC>(dst + i * VEC, v);
  }
}

}  // namespace msda
