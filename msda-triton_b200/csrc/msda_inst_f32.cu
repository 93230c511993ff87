// Kernel instantiations for value dtype float (one translation unit per
// dtype so the build compiles them in parallel).
#include <algorithm>
#define MSDA_LAUNCH_IMPL
#define MSDA_LAUNCH_ZERO_IMPL
#include "msda_launch.cuh"

namespace msda {
MSDA_INSTANTIATE(float)
}  // namespace msda
