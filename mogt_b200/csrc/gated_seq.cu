// Headed gated scan, exact fp32 path (fp32 q/k/v): one CTA (8 warps) per
// (batch, head) steps the recurrence in time exactly as the reference does,
//     S_t = f_t S_{t-1} + (1 - f_t) (k_t v_t^T),   o_t = S_t^T q_t,
// with the products rounded separately (affine_scan.py:48-51 computes
// bmm(f I, S) + V_t, and V_t = (1-f) (k v^T) is formed before the scan).
// Lane l of warp w owns state rows i = l + 32*ri and columns j = w + 8*cj.
#include "common.cuh"
#include "gated_internal.h"

namespace mogt {
namespace gated {

template <int RI, int CJ>
__global__ void __launch_bounds__(256)
    gated_fwd_seq(const float* __restrict__ q, const float* __restrict__ k,
                  const float* __restrict__ v, const float* __restrict__ f, float* __restrict__ o,
                  const float* __restrict__ S0, float* __restrict__ S_final,
                  float* __restrict__ decay_final, int T, int dk, int dv) {
  const int bh = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float S[RI][CJ];
#pragma unroll
  for (int ri = 0; ri < RI; ++ri)
#pragma unroll
    for (int cj = 0; cj < CJ; ++cj) {
      const int i = lane + 32 * ri, j = warp + 8 * cj;
      S[ri][cj] = (S0 && i < dk && j < dv) ? S0[((size_t)bh * dk + i) * dv + j] : 0.f;
    }
  float dec = 1.f;
  const float* qb = q + (size_t)bh * T * dk;
  const float* kb = k + (size_t)bh * T * dk;
  const float* vb = v + (size_t)bh * T * dv;
  const float* fb = f + (size_t)bh * T;
  float* ob = o ? o + (size_t)bh * T * dv : nullptr;
  for (int t = 0; t < T; ++t) {
    const float fv = __ldg(fb + t), w = 1.f - fv;
    dec *= fv;
    float qi[RI], ki[RI], vj[CJ];
#pragma unroll
    for (int ri = 0; ri < RI; ++ri) {
      const int i = lane + 32 * ri;
      qi[ri] = i < dk ? __ldg(qb + (size_t)t * dk + i) : 0.f;
      ki[ri] = i < dk ? __ldg(kb + (size_t)t * dk + i) : 0.f;
    }
#pragma unroll
    for (int cj = 0; cj < CJ; ++cj) {
      const int j = warp + 8 * cj;
      vj[cj] = j < dv ? __ldg(vb + (size_t)t * dv + j) : 0.f;
    }
#pragma unroll
    for (int cj = 0; cj < CJ; ++cj) {
      float part = 0.f;
#pragma unroll
      for (int ri = 0; ri < RI; ++ri) {
        // reference arithmetic: bmm(f I, S) + (1-f) * (k v^T), each product rounded
        S[ri][cj] = __fadd_rn(__fmul_rn(fv, S[ri][cj]), __fmul_rn(w, __fmul_rn(ki[ri], vj[cj])));
        part = fmaf(S[ri][cj], qi[ri], part);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
      const int j = warp + 8 * cj;
      if (ob && lane == 0 && j < dv) ob[(size_t)t * dv + j] = part;
    }
  }
  if (S_final) {
#pragma unroll
    for (int ri = 0; ri < RI; ++ri)
#pragma unroll
      for (int cj = 0; cj < CJ; ++cj) {
        const int i = lane + 32 * ri, j = warp + 8 * cj;
        if (i < dk && j < dv) S_final[((size_t)bh * dk + i) * dv + j] = S[ri][cj];
      }
  }
  if (decay_final && threadIdx.x == 0) decay_final[bh] = dec;
}

}  // namespace gated
}  // namespace mogt

int mogt::gated::launch_fwd_seq(const float* q, const float* k, const float* v, const float* f,
                                float* o, const float* S0, float* S_final, float* decay_final,
                                int BH, int T, int dk, int dv, cudaStream_t s) {
  if (dk > 128 || dv > 128) return MOGT_ERR_UNSUPPORTED;
  if (dk <= 32 && dv <= 32)
    gated_fwd_seq<1, 4><<<BH, 256, 0, s>>>(q, k, v, f, o, S0, S_final, decay_final, T, dk, dv);
  else if (dk <= 64 && dv <= 64)
    gated_fwd_seq<2, 8><<<BH, 256, 0, s>>>(q, k, v, f, o, S0, S_final, decay_final, T, dk, dv);
  else
    gated_fwd_seq<4, 16><<<BH, 256, 0, s>>>(q, k, v, f, o, S0, S_final, decay_final, T, dk, dv);
  return mogt_host::launch_status();
}
