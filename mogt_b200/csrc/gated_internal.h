// Internal launchers shared between the gated-scan translation units.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <cstdlib>

namespace mogt {
namespace gated {

int launch_fwd_seq(const float* q, const float* k, const float* v, const float* f, float* o,
                   const float* S0, float* S_final, float* decay_final, int BH, int T, int dk,
                   int dv, cudaStream_t s);

// Warp-specialised tensor-core forward (gated_fwd_ws.cu): `params` points to
// a ws::Params, `maps` to the q, k, v tensor maps; one CTA per stripe.
int launch_fwd_ws(const CUtensorMap* maps, const void* params, bool out_f32, unsigned grid,
                  cudaStream_t s);

}  // namespace gated
}  // namespace mogt
