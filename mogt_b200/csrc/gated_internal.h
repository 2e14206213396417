// Internal launchers shared between the gated-scan translation units.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>
#include <cstdlib>

namespace mogt {
namespace gated {

int launch_fwd_seq(const float* q, const float* k, const float* v, const float* f, float* o,
                   const float* S0, float* S_final, float* decay_final, int BH, int T, int dk,
                   int dv, cudaStream_t s);


}  // namespace gated
}  // namespace mogt
