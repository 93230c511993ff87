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
// device address; the address is looked up with cudaGetSymbolAddress once per
// device, with that device current, by the first call made on that device.
#include <cstdio>
#include <mutex>

#include "msda_b200.h"

namespace msda {
void set_last_error(const char* msg);
}

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[MSDA_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_dev[kMaxDevices] = {};

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
    if (e == cudaSuccess && (dev < 0 || dev >= kMaxDevices)) e = cudaErrorInvalidDevice;
    if (e == cudaSuccess) {
      std::lock_guard<std::mutex> lock(g_scratch_mu);
      if (g_scratch_dev[dev] == nullptr) {
        void* ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e == cudaSuccess) g_scratch_dev[dev] = ptr;
      }
      scratch = g_scratch_dev[dev];
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
