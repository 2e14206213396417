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

// Chunk-parallel bf16 forward (gated_fwd_chunked.cu): segment-local chunk
// states, segment carries, then every chunk's outputs independently.
size_t chunked_fwd_workspace_bytes(int64_t BH, int64_t T);
// The segment carry of the chunk-parallel forward on its own: state[g] =
// state entering segment g from a zero start, over [BH][nseg][4096]
// aggregates and log2 decays (layout-agnostic per element).
int launch_seg_carry(const float* agg, const float* lam, float* state, int64_t BH, int nseg,
                     cudaStream_t s);
int launch_chunked_fwd(const void* q, const void* k, const void* v, const float* f, void* o,
                       const float* S0, float* S_final, float* decay_final, void* chunk_states,
                       int64_t BH, int64_t T, int out_dtype, void* workspace,
                       size_t workspace_bytes, cudaStream_t s, bool resume);


}  // namespace gated
}  // namespace mogt
