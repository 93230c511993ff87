// Backward entry point for callers that cannot allocate device memory.
//
// Some callers have no way to obtain a scratch buffer at the moment they run
// the backward: a runtime that plans every device buffer ahead of time and
// forbids cudaMalloc on its execution path (a TensorRT-style plugin's enqueue,
// for instance), or an embedder with no device allocator of its own. msda_backward needs an fp32 workspace from its caller
// whenever it accumulates fp16/bf16 gradients in fp32 with the scatter
// kernel; msda_backward_noalloc runs that same kernel sequence with the
// workspace taken from a fixed-size array compiled into the library.
//
// The array is a file-scope `__device__` variable: every GPU that loads the
// library holds MSDA_NOALLOC_SCRATCH_BYTES of device memory for it until the
// process exits. In host code its name is only a host-side stand-in, never a
// device address. A module variable's address belongs to one CUDA context,
// so the address is looked up with cudaGetSymbolAddress by the first call
// made in each context (the device's primary context, or a context the
// caller created and made current), with that context current, and kept per
// context handle. A context destroyed and re-created (cudaDeviceReset) may
// come back under the same handle: call msda_backward_noalloc again only
// after the reset has finished, before any stream capture.
#include <cuda.h>

#include <cstdio>
#include <mutex>

#include "msda_b200.h"

namespace msda {
void set_last_error(const char* msg);
int check_backward_shape(int64_t B, int64_t S, int64_t Q, int32_t M, int32_t D, int32_t L, int32_t K,
                         int32_t dtype);
}

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[MSDA_NOALLOC_SCRATCH_BYTES];

// (context, scratch address) pairs: one per CUDA context the entry point ran in.
constexpr int kMaxContexts = 64;
std::mutex g_scratch_mu;
CUcontext g_scratch_ctx[kMaxContexts] = {};
void* g_scratch_ptr[kMaxContexts] = {};
int g_scratch_n = 0;

using CtxGetCurrent = CUresult (*)(CUcontext*);

// The current context's handle, through the driver entry point the runtime
// hands out (the library links the runtime statically and not libcuda).
cudaError_t current_context(CUcontext* ctx) {
  static CtxGetCurrent fn = nullptr;
  if (fn == nullptr) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q);
    if (e != cudaSuccess) return e;
    if (q != cudaDriverEntryPointSuccess || f == nullptr) return cudaErrorSymbolNotFound;
    fn = reinterpret_cast<CtxGetCurrent>(f);
  }
  *ctx = nullptr;
  return fn(ctx) == CUDA_SUCCESS ? cudaSuccess : cudaErrorDeviceUninitialized;
}

int report(int code, const char* msg) {
  msda::set_last_error(msg);
  return code;
}

}  // namespace

extern "C" int msda_backward_noalloc(const void* value, const int64_t* spatial_shapes,
                                     const int64_t* level_start_index, const void* sampling_locations,
                                     const void* attention_weights, const void* grad_output,
                                     void* grad_value, void* grad_sampling_locations,
                                     void* grad_attention_weights, int64_t batch,
                                     int64_t num_values, int64_t num_queries, int32_t num_heads,
                                     int32_t head_dim, int32_t num_levels, int32_t num_points,
                                     int32_t dtype, void* stream) {
  const uint32_t flags = MSDA_BWD_FP32_ACCUM | MSDA_BWD_FORCE_SCATTER;
  // msda_backward's own size checks first, so unsupported sizes fail as
  // they would there instead of as a scratch overflow.
  if (int rc = msda::check_backward_shape(batch, num_values, num_queries, num_heads, head_dim, num_levels,
                                          num_points, dtype))
    return rc;
  const size_t need = msda_backward_workspace_size(batch, num_values, num_queries, num_heads,
                                                   head_dim, num_levels, num_points, dtype, flags);
  char msg[256];
  if (need > (size_t)MSDA_NOALLOC_SCRATCH_BYTES) {
    snprintf(msg, sizeof(msg),
             "msda_backward_noalloc: these sizes need %zu bytes of fp32 scratch, more than the "
             "%u-byte static scratch (MSDA_NOALLOC_SCRATCH_BYTES); call msda_backward with a "
             "caller-provided workspace instead",
             need, (unsigned)MSDA_NOALLOC_SCRATCH_BYTES);
    return report(MSDA_ERR_INVALID_ARGUMENT, msg);
  }
  void* scratch = nullptr;
  if (need > 0) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess && stream != nullptr) {
      // The scratch address belongs to the current device: the stream must too.
      int sdev = -1;
      e = cudaStreamGetDevice(reinterpret_cast<cudaStream_t>(stream), &sdev);
      if (e == cudaSuccess && sdev != dev) {
        snprintf(msg, sizeof(msg),
                 "msda_backward_noalloc: the stream belongs to device %d but device %d is "
                 "current; make the stream's device current first", sdev, dev);
        return report(MSDA_ERR_INVALID_ARGUMENT, msg);
      }
    }
    CUcontext ctx = nullptr;
    if (e == cudaSuccess) e = current_context(&ctx);
    if (e == cudaSuccess) {
      std::lock_guard<std::mutex> lock(g_scratch_mu);
      for (int i = 0; i < g_scratch_n && ctx != nullptr && scratch == nullptr; ++i)
        if (g_scratch_ctx[i] == ctx) scratch = g_scratch_ptr[i];
      if (scratch == nullptr) {
        // First call in this context (with none current yet, the lookup
        // binds the device's primary context, whose handle is read after it).
        void* ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e == cudaSuccess && ctx == nullptr) e = current_context(&ctx);
        if (e == cudaSuccess) {
          scratch = ptr;
          if (ctx != nullptr && g_scratch_n < kMaxContexts) {
            g_scratch_ctx[g_scratch_n] = ctx;
            g_scratch_ptr[g_scratch_n++] = ptr;
          }
        }
      }
    }
    if (e != cudaSuccess) {
      snprintf(msg, sizeof(msg), "msda_backward_noalloc: static scratch unavailable: %s (%s)",
               cudaGetErrorName(e), cudaGetErrorString(e));
      return report(MSDA_ERR_CUDA, msg);
    }
  }
  // msda_backward zeroes the part of the scratch this call uses (an
  // asynchronous memset, no allocation) before the scatter, so nothing an
  // earlier call left there reaches this call's result.
  return msda_backward(value, spatial_shapes, level_start_index, sampling_locations,
                       attention_weights, grad_output, grad_value, grad_sampling_locations,
                       grad_attention_weights, scratch, need > 0 ? need : 0, batch, num_values,
                       num_queries, num_heads, head_dim, num_levels, num_points, dtype, flags,
                       stream);
}
