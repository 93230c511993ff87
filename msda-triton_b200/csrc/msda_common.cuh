// Device helpers shared by the MSDA forward and backward kernels (sm_100a).
//
// Layouts (all contiguous, row-major, as in the reference operator
// src/msda_triton/ops.py:96-199 and src/msda_triton/kernels.py:67-82):
//   value              (B, S, M, D)          one "pixel row" = M*D elements
//   spatial_shapes     (L, 2)  int64         (H_l, W_l)
//   level_start_index  (L,)    int64         offset of level l along S
//   sampling_locations (B, Q, M, L, K, 2)    normalised (x, y)
//   attention_weights  (B, Q, M, L, K)
//   output             (B, Q, M, D)          viewed as (B, Q, M*D) by the host
//
// Bilinear convention (src/msda_triton/kernels.py:29-35, tests/reference_impls.py:29-31):
//   x_im = x * W_l - 0.5, y_im = y * H_l - 0.5, zero padding outside the level,
// i.e. grid_sample(align_corners=False, padding_mode="zeros").
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace msda {

constexpr int kMaxLevels = 16;
constexpr unsigned kFullMask = 0xffffffffu;

// ---------------------------------------------------------------------------
// Scalar conversions
// ---------------------------------------------------------------------------
__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// ---------------------------------------------------------------------------
// Vector loads / stores of VEC elements (VEC * sizeof(T) in {2, 4, 8, 16} bytes,
// pointer aligned to that size), widened to / narrowed from fp32.
// ---------------------------------------------------------------------------
template <int BYTES> struct RawVec;
template <> struct RawVec<16> { using type = uint4; };
template <> struct RawVec<8> { using type = uint2; };
template <> struct RawVec<4> { using type = unsigned int; };
template <> struct RawVec<2> { using type = unsigned short; };

template <typename T, int VEC>
struct Pack {
  using Raw = typename RawVec<VEC * (int)sizeof(T)>::type;
  union {
    Raw raw;
    T e[VEC];
  };
};

// Read-only (non-coherent) load; the tensors read this way are never written
// by the same kernel.
template <typename T, int VEC>
__device__ __forceinline__ void load_vec(const T* __restrict__ p, float (&v)[VEC]) {
  Pack<T, VEC> pk;
  pk.raw = __ldg(reinterpret_cast<const typename Pack<T, VEC>::Raw*>(p));
#pragma unroll
  for (int i = 0; i < VEC; ++i) v[i] = to_f32(pk.e[i]);
}

// Raw load kept packed (to issue many loads before converting).
template <typename T, int VEC>
__device__ __forceinline__ typename Pack<T, VEC>::Raw load_raw(const T* __restrict__ p) {
  return __ldg(reinterpret_cast<const typename Pack<T, VEC>::Raw*>(p));
}

template <typename T, int VEC>
__device__ __forceinline__ void unpack_raw(typename Pack<T, VEC>::Raw r, float (&v)[VEC]) {
  Pack<T, VEC> pk;
  pk.raw = r;
#pragma unroll
  for (int i = 0; i < VEC; ++i) v[i] = to_f32(pk.e[i]);
}

template <typename T, int VEC>
__device__ __forceinline__ void store_vec(T* p, const float (&v)[VEC]) {
  Pack<T, VEC> pk;
#pragma unroll
  for (int i = 0; i < VEC; ++i) pk.e[i] = from_f32<T>(v[i]);
  *reinterpret_cast<typename Pack<T, VEC>::Raw*>(p) = pk.raw;
}

// max(m, |x|) that keeps a NaN (fmaxf would drop it).
__device__ __forceinline__ float max_abs_nan(float m, float x) {
  const float ax = fabsf(x);
  return (ax > m || ax != ax) ? ax : m;
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch. A kernel launched with programmatic stream
// serialization may start while the kernel before it still runs; pdl_wait()
// blocks until that kernel has completed and its writes are visible (it
// returns at once for a kernel launched without the attribute).
// pdl_trigger() lets the kernel after this one be scheduled as soon as
// every CTA of this grid has issued it (it still waits in pdl_wait()).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// Packed fp32 pairs for sm_100's f32x2 FMA (two fp32 lanes per 64-bit register).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t r, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// Mixed-precision FMA (sm_100): c + a*b for the low or high 16-bit halves
// of two words, a and b both bf16 (or both fp16), accumulated in fp32. The
// product of two 16-bit floats is exact in fp32, so this equals converting
// both to fp32 first.
__device__ __forceinline__ float fma_lo16(unsigned a, unsigned b, float c, const __nv_bfloat16*) {
  float d;
  asm("{\n\t.reg .b16 al, ah, bl, bh;\n\tmov.b32 {al, ah}, %1;\n\tmov.b32 {bl, bh}, %2;\n\t"
      "fma.rn.f32.bf16 %0, al, bl, %3;\n\t}" : "=f"(d) : "r"(a), "r"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float fma_hi16(unsigned a, unsigned b, float c, const __nv_bfloat16*) {
  float d;
  asm("{\n\t.reg .b16 al, ah, bl, bh;\n\tmov.b32 {al, ah}, %1;\n\tmov.b32 {bl, bh}, %2;\n\t"
      "fma.rn.f32.bf16 %0, ah, bh, %3;\n\t}" : "=f"(d) : "r"(a), "r"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float fma_lo16(unsigned a, unsigned b, float c, const __half*) {
  float d;
  asm("{\n\t.reg .b16 al, ah, bl, bh;\n\tmov.b32 {al, ah}, %1;\n\tmov.b32 {bl, bh}, %2;\n\t"
      "fma.rn.f32.f16 %0, al, bl, %3;\n\t}" : "=f"(d) : "r"(a), "r"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float fma_hi16(unsigned a, unsigned b, float c, const __half*) {
  float d;
  asm("{\n\t.reg .b16 al, ah, bl, bh;\n\tmov.b32 {al, ah}, %1;\n\tmov.b32 {bl, bh}, %2;\n\t"
      "fma.rn.f32.f16 %0, ah, bh, %3;\n\t}" : "=f"(d) : "r"(a), "r"(b), "f"(c));
  return d;
}

// A 32-bit word holding two 16-bit values -> packed fp32 pair.
__device__ __forceinline__ uint64_t word_to_f2(unsigned w, const __nv_bfloat16*) {
  uint64_t r;  // bf16 is the upper half of fp32: shift / mask, no conversion
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(w << 16), "r"(w & 0xffff0000u));
  return r;
}
__device__ __forceinline__ uint64_t word_to_f2(unsigned w, const __half*) {
  __half2 h;
  *reinterpret_cast<unsigned*>(&h) = w;
  const float2 f = __half22float2(h);
  return f2_pack(f.x, f.y);
}
// VEC elements of a Raw vector -> VEC/2 packed pairs (VEC even).
template <typename T, int VEC>
__device__ __forceinline__ void raw_to_f2(typename Pack<T, VEC>::Raw r, uint64_t (&out)[VEC / 2]) {
  const unsigned* w = reinterpret_cast<const unsigned*>(&r);
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int i = 0; i < VEC / 2; ++i) {
      uint64_t x;
      asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "r"(w[2 * i]), "r"(w[2 * i + 1]));
      out[i] = x;
    }
  } else {
#pragma unroll
    for (int i = 0; i < VEC / 2; ++i) out[i] = word_to_f2(w[i], (const T*)nullptr);
  }
}

// Two consecutive elements (a sampling location's (x, y) pair).
__device__ __forceinline__ float2 load_pair(const float* p) {
  return __ldg(reinterpret_cast<const float2*>(p));
}
__device__ __forceinline__ float2 load_pair(const __half* p) {
  return __half22float2(__ldg(reinterpret_cast<const __half2*>(p)));
}
__device__ __forceinline__ float2 load_pair(const __nv_bfloat16* p) {
  return __bfloat1622float2(__ldg(reinterpret_cast<const __nv_bfloat162*>(p)));
}

__device__ __forceinline__ void store_pair(float* p, float a, float b) {
  *reinterpret_cast<float2*>(p) = make_float2(a, b);
}
__device__ __forceinline__ void store_pair(__half* p, float a, float b) {
  *reinterpret_cast<__half2*>(p) = __floats2half2_rn(a, b);
}
__device__ __forceinline__ void store_pair(__nv_bfloat16* p, float a, float b) {
  *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a, b);
}

// ---------------------------------------------------------------------------
// Vector reductions into global memory (relaxed, gpu scope). sm_90+ supports
// the 16-byte vector forms of `red.global.add` for f32 and packed f16x2/bf16x2.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void red_add_f32x4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

__device__ __forceinline__ unsigned pack2(__half lo, __half hi) {
  return (unsigned)__half_as_ushort(lo) | ((unsigned)__half_as_ushort(hi) << 16);
}
__device__ __forceinline__ unsigned pack2(__nv_bfloat16 lo, __nv_bfloat16 hi) {
  return (unsigned)__bfloat16_as_ushort(lo) | ((unsigned)__bfloat16_as_ushort(hi) << 16);
}

__device__ __forceinline__ void red_add_x8(__half* p, const float (&v)[8]) {
  unsigned w0 = pack2(__float2half_rn(v[0]), __float2half_rn(v[1]));
  unsigned w1 = pack2(__float2half_rn(v[2]), __float2half_rn(v[3]));
  unsigned w2 = pack2(__float2half_rn(v[4]), __float2half_rn(v[5]));
  unsigned w3 = pack2(__float2half_rn(v[6]), __float2half_rn(v[7]));
  asm volatile("red.global.add.noftz.v4.f16x2 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(w0), "r"(w1),
               "r"(w2), "r"(w3)
               : "memory");
}
__device__ __forceinline__ void red_add_x8(__nv_bfloat16* p, const float (&v)[8]) {
  unsigned w0 = pack2(__float2bfloat16_rn(v[0]), __float2bfloat16_rn(v[1]));
  unsigned w1 = pack2(__float2bfloat16_rn(v[2]), __float2bfloat16_rn(v[3]));
  unsigned w2 = pack2(__float2bfloat16_rn(v[4]), __float2bfloat16_rn(v[5]));
  unsigned w3 = pack2(__float2bfloat16_rn(v[6]), __float2bfloat16_rn(v[7]));
  asm volatile("red.global.add.noftz.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(w0),
               "r"(w1), "r"(w2), "r"(w3)
               : "memory");
}

// ---------------------------------------------------------------------------
// L2 cache policies for the scatter backward: the rows it reduces into are
// zero-filled and reduced with evict_last, the value rows it gathers meanwhile
// with evict_first, so the gathers do not push the reduction targets out.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void red_add_f32x4_hint(float* p, float a, float b, float c, float d,
                                                   uint64_t pol) {
  asm volatile("red.global.add.L2::cache_hint.v4.f32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(p), "f"(a),
               "f"(b), "f"(c), "f"(d), "l"(pol)
               : "memory");
}
__device__ __forceinline__ void st_zero16_hint(void* p, uint64_t pol) {
  asm volatile("st.global.L2::cache_hint.v4.u32 [%0], {%1, %1, %1, %1}, %2;" ::"l"(p), "r"(0u),
               "l"(pol)
               : "memory");
}
__device__ __forceinline__ void red_add_scalar(float* p, float v) { atomicAdd(p, v); }
__device__ __forceinline__ void red_add_scalar(__half* p, float v) {
  atomicAdd(p, __float2half_rn(v));
}
__device__ __forceinline__ void red_add_scalar(__nv_bfloat16* p, float v) {
  atomicAdd(p, __float2bfloat16_rn(v));
}

__device__ __forceinline__ void red_add_x8_hint(__half* p, const float (&v)[8], uint64_t pol) {
  unsigned w0 = pack2(__float2half_rn(v[0]), __float2half_rn(v[1]));
  unsigned w1 = pack2(__float2half_rn(v[2]), __float2half_rn(v[3]));
  unsigned w2 = pack2(__float2half_rn(v[4]), __float2half_rn(v[5]));
  unsigned w3 = pack2(__float2half_rn(v[6]), __float2half_rn(v[7]));
  asm volatile("red.global.add.noftz.L2::cache_hint.v4.f16x2 [%0], {%1, %2, %3, %4}, %5;" ::"l"(p),
               "r"(w0), "r"(w1), "r"(w2), "r"(w3), "l"(pol)
               : "memory");
}
__device__ __forceinline__ void red_add_x8_hint(__nv_bfloat16* p, const float (&v)[8], uint64_t pol) {
  unsigned w0 = pack2(__float2bfloat16_rn(v[0]), __float2bfloat16_rn(v[1]));
  unsigned w1 = pack2(__float2bfloat16_rn(v[2]), __float2bfloat16_rn(v[3]));
  unsigned w2 = pack2(__float2bfloat16_rn(v[4]), __float2bfloat16_rn(v[5]));
  unsigned w3 = pack2(__float2bfloat16_rn(v[6]), __float2bfloat16_rn(v[7]));
  asm volatile("red.global.add.noftz.L2::cache_hint.v4.bf16x2 [%0], {%1, %2, %3, %4}, %5;" ::"l"(p),
               "r"(w0), "r"(w1), "r"(w2), "r"(w3), "l"(pol)
               : "memory");
}

// As red_add_vec, with the L2 policy `pol` on the 16-byte forms.
template <typename A, int VEC>
__device__ __forceinline__ void red_add_vec_hint(A* p, const float (&v)[VEC], uint64_t pol) {
  if constexpr (sizeof(A) == 4 && VEC % 4 == 0) {
#pragma unroll
    for (int i = 0; i < VEC; i += 4)
      red_add_f32x4_hint(reinterpret_cast<float*>(p) + i, v[i], v[i + 1], v[i + 2], v[i + 3], pol);
  } else if constexpr (sizeof(A) == 2 && VEC == 8) {
    red_add_x8_hint(p, v, pol);
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) red_add_scalar(p + i, v[i]);
  }
}

// ---------------------------------------------------------------------------
// Deterministic grad_value: 64-bit fixed-point accumulation.
//
// Every contribution c = a * w_c * g_d is rounded once to an integer multiple
// of 2^-F and added with an integer `red.global.add.u64`. Integer addition is
// associative, so the sum -- and the value rounded from it -- does not depend
// on the order in which the reductions land: the result is a function of the
// inputs alone (bitwise reproducible across runs, grids and streams).
//
// The scale 2^F comes from a 2-word header the backward's absmax pass fills:
// hdr[0] = bit pattern of max|attention weight| (1.0 for the fused prologue's
// softmax weights), hdr[1] = that of max|grad_out| (an atomicMax over |x|
// bit patterns, which order like the magnitudes). With |a| < 2^ea,
// |g| < 2^eg, |w_c| <= 1 and at most n = Q*K contributions per row (a row
// belongs to one level; each point of it adds at most one corner there),
//   F = 49 - ceil(log2 n) - ea - eg
// bounds every scaled contribution by 2^(49 - ceil(log2 n)) and every row
// sum by 2^49.
//
// Rounding without a float-to-integer conversion: the weight a * w_c is
// widened to fp64 and scaled by 2^F once per corner (exact in fp64's range),
// and each element is one
//   t = fma(a * w_c * 2^F, g, 1.5 * 2^52)
// -- the exact product rounded once to an integer v (fp64's ulp is 1 on
// [2^52, 2^53), and |product| < 2^51 keeps t there), read back as
// v = bits(t) - bits(1.5 * 2^52). The rounding error of one contribution is
// at most 2^-(F+1): relative to the largest possible contribution,
// 2^-(50 - ceil(log2 n)), i.e. below 2^-33 for n <= 2^17 -- finer than one
// fp32 add (2^-24), and of the exact product rather than an fp32-rounded
// one. A row sum is rounded once to fp32 and scaled by 2^-F as two fp32
// powers of two (exact unless the result is below fp32's normal range; an F
// beyond 252, i.e. max|a| * max|g| < 2^-203, leaves only underflowing
// results).
//
// Inputs with a non-finite maximum (or an attention weight so large that a
// merged fp32 weight could overflow) set `ok` false: the scatter then adds
// fp32 contributions to the low word of each 64-bit element with ordinary
// float atomics, which puts Inf / NaN where fp32 accumulation would (and is
// not order-independent -- there is no finite value to keep).
// ---------------------------------------------------------------------------
// Accumulator type tag: A = long long selects the fixed-point scatter.
template <typename A>
struct IsFixed {
  static constexpr bool value = false;
};
template <>
struct IsFixed<long long> {
  static constexpr bool value = true;
};

// Deterministic grad_value of fp16 / bf16 data in the hit-counted algorithm:
// the accumulator rows stay fp32, and every contribution to a row with three
// or more hits is made an integer-valued float (exact_scale), so the row's
// partial sums are exact integers below 2^24 and do not depend on the order
// the reductions land in.
struct ExactF32 {
  float v;
};
template <typename A>
struct IsExact {
  static constexpr bool value = false;
};
template <>
struct IsExact<ExactF32> {
  static constexpr bool value = true;
};

// 2^k as a float, k in [-126, 127].
__device__ __forceinline__ float pow2f(int k) { return __int_as_float((k + 127) << 23); }

// Rounds x (|x| < 2^22) to an integer-valued float: the FMA with 1.5 * 2^23
// leaves round(x) in the low mantissa bits, the subtraction is exact.
constexpr float kExactMagic = 12582912.0f;  // 1.5 * 2^23

// Scale 2^F of an exact row: n >= 2 hits whose products |a w_c g| are below
// the bound rowmax (the bits of max |a| * max|grad_out row| over the row's
// points) < 2^E. Each contribution fl(a w_c g) * 2^F is below 2^(E + F) =
// 2^(24 - max(ceil(log2 n), 2)) <= 2^22 before rounding, so every partial sum
// of the n rounded terms is an integer of magnitude <= 2^24: exact in fp32
// (and never a denormal, which fp32 `red` would flush). F lies in [-126, 147]
// and is applied as 2^F1 on the weight before the product
// (F1 = max(F - 64, 0): the products of tiny rows stay normal floats) and
// 2^F2 on the product. Returns false for the fp32 fallback: a non-finite
// bound, one so large that F < -126, or rowmax == 0 (then every contribution
// is zero).
struct ExactScale {
  float s1, s2;      // 2^F1, 2^F2
  float inv1, inv2;  // 2^-F1, 2^-F2
};

__device__ __forceinline__ bool exact_scale(unsigned rowmax, unsigned n, ExactScale& xs) {
  const int E = max((int)(rowmax >> 23), 1) - 126;  // rowmax < 2^E (denormals: 2^-125)
  const int l2n = max(32 - __clz(n - 1u), 2);       // ceil(log2 n), at least 2
  const int F = 24 - E - l2n;
  const bool ok = rowmax - 1u < 0x7f7fffffu && F >= -126;
  const int F2 = ok ? min(F, 64) : 0, F1 = ok ? F - F2 : 0;
  xs.s1 = pow2f(F1);
  xs.s2 = pow2f(F2);
  xs.inv1 = pow2f(-F1);
  xs.inv2 = pow2f(-F2);
  return ok;
}

// Rows of the exact hit-counted algorithm with more hits than this use
// 64-bit integers instead (wide_scale): the integer-valued fp32 grid is
// 2^(ceil(log2 hits) - 24) of the row's bound, at most 2^-19 of it up to here.
constexpr unsigned kExactMaxHits = 32;

// Scale 2^F of a 64-bit exact row (more than kExactMaxHits hits, bound
// rowmax < 2^E): contributions a w_c g (exact in fp64) times 2^F stay below
// 2^51 (rounded to an integer by one fp64 FMA) and n of them below 2^62.
// Returns false (fp32 fallback) for a zero or non-finite bound.
__device__ __forceinline__ bool wide_scale(unsigned rowmax, unsigned n, double& scale, double& inv) {
  const int E = max((int)(rowmax >> 23), 1) - 126;
  const int l2n = 32 - __clz(n - 1u);
  const int F = min(51 - E, 62 - E - l2n);  // in [-98, 176]
  scale = __longlong_as_double((long long)(1023 + F) << 52);
  inv = __longlong_as_double((long long)(1023 - F) << 52);
  return rowmax - 1u < 0x7f7fffffu;
}

constexpr double kFixedMagic = 6755399441055744.0;  // 1.5 * 2^52
constexpr long long kFixedMagicBits = 0x4338000000000000ll;

struct FixedScale {
  double scale;      // 2^F
  float inv1, inv2;  // 2^-F = inv1 * inv2
  bool ok;           // false: fp32 fallback (non-finite or overflowing inputs)
};

__device__ __forceinline__ FixedScale fixed_scale(const unsigned* __restrict__ hdr, int clog2n) {
  const unsigned ua = __ldcg(hdr), ug = __ldcg(hdr + 1);
  FixedScale fx;
  fx.ok = ua < 0x7f800000u && ug < 0x7f800000u;
  int F = 0;
  if (fx.ok && ua != 0u && ug != 0u) {
    // |x| < 2^(E - 126) for biased exponent E (denormals: below 2^-125).
    const int ea = max((int)(ua >> 23), 1) - 126;
    const int eg = max((int)(ug >> 23), 1) - 126;
    if (ea + clog2n > 127) fx.ok = false;  // a merged fp32 weight sum could overflow
    F = 49 - clog2n - ea - eg;             // in [-247, 300]: a normal fp64 power of two
  }
  if (!fx.ok) F = 0;
  fx.scale = __longlong_as_double((long long)(1023 + F) << 52);
  const int F1 = min(max(F, -126), 126), F2 = min(max(F - F1, -126), 126);
  fx.inv1 = __int_as_float((127 - F1) << 23);
  fx.inv2 = __int_as_float((127 - F2) << 23);
  return fx;
}

// Adds round(wd * gd) to a 64-bit element (wd = the corner weight
// a * w_c * 2^F in fp64, gd = g); zero contributions are skipped.
__device__ __forceinline__ void red_fixed(long long* p, double wd, double gd, uint64_t pol) {
  const long long v = __double_as_longlong(fma(wd, gd, kFixedMagic)) - kFixedMagicBits;
  if (v != 0)
    asm volatile("red.global.add.L2::cache_hint.u64 [%0], %1, %2;" ::"l"(p), "l"(v), "l"(pol) : "memory");
}

// A 64-bit accumulator element -> float (or the fallback's fp32 low word).
__device__ __forceinline__ float fixed_to_f32(long long v, const FixedScale& fx) {
  if (!fx.ok) return __int_as_float((int)(unsigned)(unsigned long long)v);
  return __ll2float_rn(v) * fx.inv1 * fx.inv2;
}

// Read-only 16-byte load with an L2 policy (value rows in the scatter backward).
__device__ __forceinline__ uint4 ldg16_hint(const void* p, uint64_t pol) {
  uint4 v;
  asm volatile("ld.global.nc.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(pol));
  return v;
}

// Adds VEC values (one lane's channel chunk) into an accumulator row of type A.
// A = float with VEC % 4 == 0 uses v4.f32; A = half type with VEC == 8 uses the
// packed 16-byte form; everything else falls back to scalar atomics.
template <typename A, int VEC>
__device__ __forceinline__ void red_add_vec(A* p, const float (&v)[VEC]) {
  if constexpr (sizeof(A) == 4 && VEC % 4 == 0) {
#pragma unroll
    for (int i = 0; i < VEC; i += 4) red_add_f32x4(reinterpret_cast<float*>(p) + i, v[i], v[i + 1], v[i + 2], v[i + 3]);
  } else if constexpr (sizeof(A) == 2 && VEC == 8) {
    red_add_x8(p, v);
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) red_add_scalar(p + i, v[i]);
  }
}

// ---------------------------------------------------------------------------
// Level table, staged in shared memory at CTA start (the spatial_shapes and
// level_start_index tensors live on the device; reading them in-kernel avoids
// a device->host sync and keeps the launch graph-capturable).
//
// A level whose (H, W, start) is inconsistent with S (non-positive size, or
// start + H*W outside [0, S]) is marked empty: every corner on it is treated as
// out of bounds, so a malformed shapes tensor can never index outside value.
// ---------------------------------------------------------------------------
struct LevelInfo {
  int H;
  int W;
  int start;
  float fH;
  float fW;
  int dense;  // hit-counted backward: the level's rows are accumulated in fp32 without counting
};

// A level is "dense" for the hit-counted backward when its Q*K sampling
// points per head put at least kDenseHitsPerRow bilinear corners on each of
// its H*W rows on average: most of its rows are then hit more than once, so
// counting them buys nothing and their same-row counters are the hottest.
constexpr int kDenseHitsPerRow = 2;

__device__ __forceinline__ void load_levels(const int64_t* __restrict__ shapes,
                                            const int64_t* __restrict__ starts, int L, int64_t S,
                                            LevelInfo* lv, int64_t Q = 0, int K = 0) {
  if ((int)threadIdx.x < L) {
    const int l = threadIdx.x;
    int64_t H = shapes[2 * l], W = shapes[2 * l + 1], st = starts[l];
    bool ok = H > 0 && W > 0 && st >= 0 && H <= S && W <= S && st <= S && H * W <= S - st;
    LevelInfo info;
    info.H = ok ? (int)H : 0;
    info.W = ok ? (int)W : 0;
    info.start = ok ? (int)st : 0;
    info.fH = (float)info.H;
    info.fW = (float)info.W;
    info.dense = ok && 4 * Q * K >= (int64_t)kDenseHitsPerRow * H * W;
    lv[l] = info;
  }
  __syncthreads();
}

// One sampling point resolved to its four bilinear corners:
//   corner 0 = (y0, x0), 1 = (y0, x0+1), 2 = (y0+1, x0), 3 = (y0+1, x0+1)
// (the v00, v01, v10, v11 order of src/msda_triton/kernels.py:130-149).
struct Bilinear {
  int pix[4];    // pixel index along S (only meaningful where valid)
  float w[4];    // bilinear weights (1-lx)(1-ly), lx(1-ly), (1-lx)ly, lx*ly
  float lx, ly;  // fractional offsets inside the cell
  unsigned valid;  // bit c set iff corner c lies inside the level
};

// An empty sampling slot (past the last point of the warp's triple): no
// corner is valid and every weight is zero, so it contributes nothing.
__device__ __forceinline__ Bilinear empty_slot() {
  Bilinear r;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    r.pix[c] = 0;
    r.w[c] = 0.f;
  }
  r.lx = r.ly = 0.f;
  r.valid = 0u;
  return r;
}

// x is clamped to [-2, W+1] before the integer conversion (a NaN or huge
// location then lands fully outside the level instead of overflowing the
// int cast); inside that range the clamp is the identity, so every in-bounds
// result equals the unclamped formula of src/msda_triton/kernels.py:112-128.
// resolve_px takes pixel coordinates x = loc_x * W - 0.5 (or, for the fused
// prologue, ref_x * W + offset_x - 0.5: the same point without forming loc).
__device__ __forceinline__ Bilinear resolve_px(float x, float y, const LevelInfo& L) {
  Bilinear r;
  x = fminf(fmaxf(x, -2.0f), L.fW + 1.0f);
  y = fminf(fmaxf(y, -2.0f), L.fH + 1.0f);
  const float x0f = floorf(x), y0f = floorf(y);
  const float lx = x - x0f, ly = y - y0f;
  const int x0 = (int)x0f, y0 = (int)y0f;
  const bool vx0 = (unsigned)x0 < (unsigned)L.W;
  const bool vx1 = (unsigned)(x0 + 1) < (unsigned)L.W;
  const bool vy0 = (unsigned)y0 < (unsigned)L.H;
  const bool vy1 = (unsigned)(y0 + 1) < (unsigned)L.H;
  r.valid = (unsigned)(vy0 && vx0) | ((unsigned)(vy0 && vx1) << 1) | ((unsigned)(vy1 && vx0) << 2) |
            ((unsigned)(vy1 && vx1) << 3);
  const int p00 = L.start + y0 * L.W + x0;
  r.pix[0] = p00;
  r.pix[1] = p00 + 1;
  r.pix[2] = p00 + L.W;
  r.pix[3] = p00 + L.W + 1;
  r.lx = lx;
  r.ly = ly;
  r.w[0] = (1.0f - lx) * (1.0f - ly);
  r.w[1] = lx * (1.0f - ly);
  r.w[2] = (1.0f - lx) * ly;
  r.w[3] = lx * ly;
  return r;
}

__device__ __forceinline__ Bilinear resolve(float locx, float locy, const LevelInfo& L) {
  return resolve_px(fmaf(locx, L.fW, -0.5f), fmaf(locy, L.fH, -0.5f), L);
}

// Fused prologue: the pixel coordinates of reference point + offset (offsets
// in level pixels, Deformable-DETR style) on level L.
__device__ __forceinline__ Bilinear resolve_fused(float2 ref, float2 off, const LevelInfo& L) {
  return resolve_px(fmaf(ref.x, L.fW, off.x - 0.5f), fmaf(ref.y, L.fH, off.y - 0.5f), L);
}

// Softmax statistics of n logits spread over a warp (lane i holds
// p[i], p[i + 32], ...): the maximum and 1 / sum(exp(v - max)), reduced with
// shuffles (every lane returns the same pair).
template <typename T>
__device__ __forceinline__ void warp_softmax_stats(const T* __restrict__ p, int n, int lane, float& mx,
                                                   float& inv_sum) {
  float m = -3.402823466e38f, sum = 0.f;
  for (int i = lane; i < n; i += 32) {  // online: rescale the running sum when the max grows
    const float v = to_f32(p[i]);
    if (v > m) {
      sum = sum * expf(m - v) + 1.f;
      m = v;
    } else {
      sum += expf(v - m);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
    const float s2 = __shfl_xor_sync(0xffffffffu, sum, off);
    const float mm = fmaxf(m, m2);
    sum = sum * expf(m - mm) + s2 * expf(m2 - mm);
    m = mm;
  }
  mx = m;
  inv_sum = 1.f / sum;
}

}  // namespace msda
