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

int launch_fwd_ws(const void* q, const void* k, const void* v, const float* f, void* o,
                  const float* S0, float* S_final, float* decay_final, void* chunk_states, int BH,
                  int T, bool out_f32, void* workspace, size_t workspace_bytes, cudaStream_t s);
size_t fwd_ws_workspace_bytes(int64_t BH, int64_t T);

}  // namespace gated
}  // namespace mogt
