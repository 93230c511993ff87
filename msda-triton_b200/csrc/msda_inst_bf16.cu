// Kernel instantiations for value dtype __nv_bfloat16 (one translation unit per
// dtype so the build compiles them in parallel).
#include <algorithm>
#define MSDA_LAUNCH_IMPL
#include "msda_launch.cuh"

namespace msda {
MSDA_INSTANTIATE(__nv_bfloat16)
}  // namespace msda
