// Kernel instantiations for value dtype __half (one translation unit per
// dtype so the build compiles them in parallel).
#include <algorithm>
#define MSDA_LAUNCH_IMPL
#include "msda_launch.cuh"

namespace msda {
MSDA_INSTANTIATE(__half)
}  // namespace msda
