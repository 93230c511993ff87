// Host-side helpers shared by the C ABI translation units: error reporting
// through msda_last_error(), dtype sizes, alignment tests and the lane-layout
// choice of the channel-vector kernels.
#pragma once

#include <cstdarg>
#include <cstdint>
#include <cstdio>

#include "msda_b200.h"
#include "msda_launch.cuh"

namespace msda {

// Sets the thread-local message msda_last_error() returns (msda_capi.cu).
void set_last_error(const char* msg);

namespace abi {

inline int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  set_last_error(buf);
  return code;
}

inline int succeed() {
  set_last_error("");
  return MSDA_OK;
}

inline int cuda_fail(cudaError_t e, const char* what) {
  return fail(MSDA_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

inline int elem_size(int32_t dtype) {
  switch (dtype) {
    case MSDA_DTYPE_F32: return 4;
    case MSDA_DTYPE_F16: return 2;
    case MSDA_DTYPE_BF16: return 2;
    default: return 0;
  }
}

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

inline int next_pow2(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// ceil(log2(n)) for n >= 1.
inline int ceil_log2(int64_t n) {
  int r = 0;
  while (r < 62 && ((int64_t)1 << r) < n) ++r;
  return r;
}

inline int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

// Picks the lane layout for a channel count D (a head dim, or the channels
// of a feature map): 16-byte vectors when `vec_ptrs_aligned` (every buffer
// read or written in D-chunks is 16-byte aligned) and D is a multiple of the
// vector, else scalars; LPR lanes per row, CPL chunks per lane.
inline int choose_cfg(int32_t D, int es, bool vec_ptrs_aligned, Cfg* c) {
  const int v16 = 16 / es;
  c->short_grid = false;
  c->vec = ((D % v16) == 0 && vec_ptrs_aligned) ? v16 : 1;
  const int nc = D / c->vec;
  c->lpr = next_pow2(nc < 32 ? nc : 32);
  c->cpl = (nc + c->lpr - 1) / c->lpr;
  if (c->cpl == 3) c->cpl = 4;
  if (c->cpl > 4)
    return fail(MSDA_ERR_UNSUPPORTED, "head_dim=%d too large for the %s path (max %d)", D,
                c->vec > 1 ? "vector" : "scalar", 128 * c->vec);
  return MSDA_OK;
}

}  // namespace abi
}  // namespace msda
