// Headed gated scan, backward.
//
// Forward:  S_t = f_t S_{t-1} + (1 - f_t) k_t v_t^T,  o_t = S_t^T q_t,  L = sum <o_t, do_t>.
// Adjoint:  G_t = dL/dS_t = q_t do_t^T + f_{t+1} G_{t+1}         (reverse scan)
//   dq_t = S_t do_t,   dk_t = (1-f_t) G_t v_t,   dv_t = (1-f_t) G_t^T k_t,
//   df_t = <G_t, S_{t-1}> - k_t^T G_t v_t,   dS_0 (initial state) = f_0 G_0.
// This is the chain rule through the reference's backward (affine_scan.py:
// 65-124: Sigma_t = g_t + U_{t+1}^T Sigma_{t+1}, dU_t = Sigma_t H_{t-1}^T) with
// U_t = f_t I, V_t = (1-f_t) k_t v_t^T and g_t = q_t do_t^T.  df_t is formed
// directly from <G_t, S_{t-1}>: the shortcut through a reverse cumulative sum
// of q.dq - k.dk loses all precision on long sequences.
//
// fp32 path (this file): one CTA per (batch, head), exact sequential sweeps.
//   sweep 1 (forward in time): S_t, dq_t; the state entering every 64-step
//           chunk is saved in the workspace;
//   sweep 2 (backward in time, chunk by chunk): the chunk's states are
//           recomputed from its saved entry state into the workspace, then
//           the adjoint steps back through the chunk.
// Layout: warp w owns state rows i = w + 8*ri, lane l owns columns
// j = l + 32*cj, so row reductions (dq, dk) are warp shuffles and column
// reductions (dv) and the full contraction (df) go through shared memory.
#include "common.cuh"
#include "gated_internal.h"

namespace mogt {
namespace gated {

constexpr int BWD_CHUNK = 64;

template <int RI, int CJ>
__global__ void __launch_bounds__(256)
    gated_bwd_seq(const float* __restrict__ q, const float* __restrict__ k,
                  const float* __restrict__ v, const float* __restrict__ f,
                  const float* __restrict__ dout, const float* __restrict__ S0,
                  float* __restrict__ dq, float* __restrict__ dk, float* __restrict__ dv,
                  float* __restrict__ df, float* __restrict__ dS0, float* __restrict__ ws_chunk,
                  float* __restrict__ ws_step, int T, int dk_, int dv_) {
  const int bh = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = (T + BWD_CHUNK - 1) / BWD_CHUNK;
  const int DD = dk_ * dv_;
  __shared__ float red_dv[2][8][128];
  __shared__ float red_df[2][8];
  const float* qb = q + (size_t)bh * T * dk_;
  const float* kb = k + (size_t)bh * T * dk_;
  const float* vb = v + (size_t)bh * T * dv_;
  const float* db = dout + (size_t)bh * T * dv_;
  const float* fb = f + (size_t)bh * T;
  float* wchunk = ws_chunk + (size_t)bh * nch * DD;
  float* wstep = ws_step + (size_t)bh * BWD_CHUNK * DD;

  auto row = [&](int ri) { return warp + 8 * ri; };
  auto col = [&](int cj) { return lane + 32 * cj; };
  auto store_state = [&](float* dst, const float (&S)[RI][CJ]) {
#pragma unroll
    for (int ri = 0; ri < RI; ++ri)
#pragma unroll
      for (int cj = 0; cj < CJ; ++cj)
        if (row(ri) < dk_ && col(cj) < dv_) dst[row(ri) * dv_ + col(cj)] = S[ri][cj];
  };
  auto load_state = [&](float (&S)[RI][CJ], const float* src) {
#pragma unroll
    for (int ri = 0; ri < RI; ++ri)
#pragma unroll
      for (int cj = 0; cj < CJ; ++cj)
        S[ri][cj] = (row(ri) < dk_ && col(cj) < dv_) ? src[row(ri) * dv_ + col(cj)] : 0.f;
  };
  // one step of the forward recurrence, with the reference's rounding
  auto fwd_step = [&](float (&S)[RI][CJ], int t) {
    const float fv = __ldg(fb + t), w = 1.f - fv;
    float ki[RI], vj[CJ];
#pragma unroll
    for (int ri = 0; ri < RI; ++ri) ki[ri] = row(ri) < dk_ ? __ldg(kb + (size_t)t * dk_ + row(ri)) : 0.f;
#pragma unroll
    for (int cj = 0; cj < CJ; ++cj) vj[cj] = col(cj) < dv_ ? __ldg(vb + (size_t)t * dv_ + col(cj)) : 0.f;
#pragma unroll
    for (int ri = 0; ri < RI; ++ri)
#pragma unroll
      for (int cj = 0; cj < CJ; ++cj)
        S[ri][cj] = __fadd_rn(__fmul_rn(fv, S[ri][cj]), __fmul_rn(w, __fmul_rn(ki[ri], vj[cj])));
  };

  // ---- sweep 1: states forward, dq_t = S_t do_t ----
  float S[RI][CJ];
  if (S0) load_state(S, S0 + (size_t)bh * DD);
  else {
#pragma unroll
    for (int ri = 0; ri < RI; ++ri)
#pragma unroll
      for (int cj = 0; cj < CJ; ++cj) S[ri][cj] = 0.f;
  }
  for (int t = 0; t < T; ++t) {
    if (t % BWD_CHUNK == 0) store_state(wchunk + (size_t)(t / BWD_CHUNK) * DD, S);
    fwd_step(S, t);
    float dj[CJ];
#pragma unroll
    for (int cj = 0; cj < CJ; ++cj) dj[cj] = col(cj) < dv_ ? __ldg(db + (size_t)t * dv_ + col(cj)) : 0.f;
#pragma unroll
    for (int ri = 0; ri < RI; ++ri) {
      float part = 0.f;
#pragma unroll
      for (int cj = 0; cj < CJ; ++cj) part = fmaf(S[ri][cj], dj[cj], part);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
      if (lane == 0 && row(ri) < dk_) dq[((size_t)bh * T + t) * dk_ + row(ri)] = part;
    }
  }

  // ---- sweep 2: adjoint backward in time ----
  float G[RI][CJ];
#pragma unroll
  for (int ri = 0; ri < RI; ++ri)
#pragma unroll
    for (int cj = 0; cj < CJ; ++cj) G[ri][cj] = 0.f;
  int par = 0;
  for (int c = nch - 1; c >= 0; --c) {
    const int t0 = c * BWD_CHUNK, t1 = min(T, t0 + BWD_CHUNK);
    float X[RI][CJ];
    load_state(X, wchunk + (size_t)c * DD);
    for (int t = t0; t < t1; ++t) {
      fwd_step(X, t);
      store_state(wstep + (size_t)(t - t0) * DD, X);
    }
    for (int t = t1 - 1; t >= t0; --t) {
      const float fv = __ldg(fb + t), w = 1.f - fv;
      float qi[RI], ki[RI], vj[CJ], dj[CJ];
#pragma unroll
      for (int ri = 0; ri < RI; ++ri) {
        qi[ri] = row(ri) < dk_ ? __ldg(qb + (size_t)t * dk_ + row(ri)) : 0.f;
        ki[ri] = row(ri) < dk_ ? __ldg(kb + (size_t)t * dk_ + row(ri)) : 0.f;
      }
#pragma unroll
      for (int cj = 0; cj < CJ; ++cj) {
        vj[cj] = col(cj) < dv_ ? __ldg(vb + (size_t)t * dv_ + col(cj)) : 0.f;
        dj[cj] = col(cj) < dv_ ? __ldg(db + (size_t)t * dv_ + col(cj)) : 0.f;
      }
      // state before step t (each thread reads back only its own elements)
      float Sp[RI][CJ];
      if (t > t0) load_state(Sp, wstep + (size_t)(t - 1 - t0) * DD);
      else load_state(Sp, wchunk + (size_t)c * DD);
      float dfp = 0.f, kdk = 0.f;
      float dvp[CJ];
#pragma unroll
      for (int cj = 0; cj < CJ; ++cj) dvp[cj] = 0.f;
#pragma unroll
      for (int ri = 0; ri < RI; ++ri) {
        float dkr = 0.f;
#pragma unroll
        for (int cj = 0; cj < CJ; ++cj) {
          G[ri][cj] = fmaf(qi[ri], dj[cj], G[ri][cj]);
          dkr = fmaf(G[ri][cj], vj[cj], dkr);
          dvp[cj] = fmaf(G[ri][cj], ki[ri], dvp[cj]);
          dfp = fmaf(G[ri][cj], Sp[ri][cj], dfp);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) dkr += __shfl_xor_sync(0xffffffffu, dkr, o);
        kdk = fmaf(ki[ri], dkr, kdk);  // identical in every lane of the warp
        if (lane == 0 && row(ri) < dk_) dk[((size_t)bh * T + t) * dk_ + row(ri)] = w * dkr;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) dfp += __shfl_xor_sync(0xffffffffu, dfp, o);
#pragma unroll
      for (int cj = 0; cj < CJ; ++cj)
        if (col(cj) < dv_) red_dv[par][warp][col(cj)] = dvp[cj];
      if (lane == 0) red_df[par][warp] = dfp - kdk;
      __syncthreads();
      for (int j = threadIdx.x; j < dv_; j += blockDim.x) {
        float s = 0.f;
#pragma unroll
        for (int ww = 0; ww < 8; ++ww) s += red_dv[par][ww][j];
        dv[((size_t)bh * T + t) * dv_ + j] = w * s;
      }
      if (threadIdx.x == 0) {
        float s = 0.f;
#pragma unroll
        for (int ww = 0; ww < 8; ++ww) s += red_df[par][ww];
        df[(size_t)bh * T + t] = s;
      }
      par ^= 1;
      // carry f_t G_t into step t-1
#pragma unroll
      for (int ri = 0; ri < RI; ++ri)
#pragma unroll
        for (int cj = 0; cj < CJ; ++cj) G[ri][cj] *= fv;
    }
  }
  if (dS0) store_state(dS0 + (size_t)bh * DD, G);
}

template <int RI, int CJ>
int launch_bwd_seq_t(const float* q, const float* k, const float* v, const float* f, const float* dout,
                     const float* S0, float* dq, float* dk, float* dv, float* df, float* dS0,
                     float* ws, int BH, int T, int dk_, int dv_, cudaStream_t s) {
  const size_t nch = (size_t)(T + BWD_CHUNK - 1) / BWD_CHUNK;
  float* ws_chunk = ws;
  float* ws_step = ws + (size_t)BH * nch * dk_ * dv_;
  gated_bwd_seq<RI, CJ><<<BH, 256, 0, s>>>(q, k, v, f, dout, S0, dq, dk, dv, df, dS0, ws_chunk,
                                           ws_step, T, dk_, dv_);
  return mogt_host::launch_status();
}

size_t bwd_tc_workspace_bytes(int64_t BH, int64_t T);
int launch_bwd_tc(const void* q, const void* k, const void* v, const float* f, const void* d_o,
                  const void* chunk_states, void* dq, void* dk, void* dv, float* df, float* dS0,
                  int BH, int T, void* workspace, size_t workspace_bytes, cudaStream_t s);

size_t bwd_seq_workspace_bytes(int64_t BH, int64_t T, int64_t dk, int64_t dv) {
  const size_t nch = (size_t)(T + BWD_CHUNK - 1) / BWD_CHUNK;
  return (size_t)BH * (nch + BWD_CHUNK) * dk * dv * sizeof(float);
}

}  // namespace gated
}  // namespace mogt

using namespace mogt;
using namespace mogt::gated;

extern "C" {

size_t mogt_gated_scan_bwd_workspace_bytes(int64_t BH, int64_t T, int64_t dk, int64_t dv,
                                           int in_dtype) {
  if (BH <= 0 || T <= 0 || dk <= 0 || dv <= 0) return 0;
  if (in_dtype == MOGT_DTYPE_F32) return bwd_seq_workspace_bytes(BH, T, dk, dv);
  if (in_dtype == MOGT_DTYPE_BF16 && dk == 64 && dv == 64) return bwd_tc_workspace_bytes(BH, T);
  return 0;
}

int mogt_gated_scan_bwd(const void* q, const void* k, const void* v, const float* f,
                        const void* d_o, const float* S0, const void* chunk_states, void* dq,
                        void* dk, void* dv, float* df, float* dS0, int64_t BH, int64_t T, int64_t dk_, int64_t dv_, int in_dtype,
                        void* workspace, size_t workspace_bytes, void* stream) {
  if (BH <= 0 || T < 0 || dk_ <= 0 || dv_ <= 0) return MOGT_ERR_SHAPE;
  if (T == 0) return MOGT_OK;
  if (!q || !k || !v || !f || !d_o || !dq || !dk || !dv || !df) return MOGT_ERR_ARG;
  if (BH >= ((int64_t)1 << 31) || T >= ((int64_t)1 << 31)) return MOGT_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (in_dtype == MOGT_DTYPE_BF16) {
    if (dk_ != 64 || dv_ != 64) return MOGT_ERR_UNSUPPORTED;
    if (!chunk_states) return MOGT_ERR_ARG;
    const void* ptrs[8] = {q, k, v, d_o, chunk_states, dq, dk, dv};
    for (const void* p : ptrs)
      if ((reinterpret_cast<uintptr_t>(p) & 15u) != 0) return MOGT_ERR_ALIGN;
    return launch_bwd_tc(q, k, v, f, d_o, chunk_states, dq, dk, dv, df, dS0, (int)BH, (int)T,
                         workspace, workspace_bytes, s);
  }
  if (in_dtype != MOGT_DTYPE_F32) return MOGT_ERR_DTYPE;
  if (chunk_states) return MOGT_ERR_ARG;
  if (dk_ > 128 || dv_ > 128) return MOGT_ERR_UNSUPPORTED;
  if (!workspace || workspace_bytes < bwd_seq_workspace_bytes(BH, T, dk_, dv_)) return MOGT_ERR_WORKSPACE;
  const float *qf = static_cast<const float*>(q), *kf = static_cast<const float*>(k),
              *vf = static_cast<const float*>(v), *df_o = static_cast<const float*>(d_o);
  float *gq = static_cast<float*>(dq), *gk = static_cast<float*>(dk), *gv = static_cast<float*>(dv);
  float* ws = static_cast<float*>(workspace);
  const int B = (int)BH, Ti = (int)T, a = (int)dk_, b = (int)dv_;
  if (dk_ <= 32 && dv_ <= 32)
    return launch_bwd_seq_t<4, 1>(qf, kf, vf, f, df_o, S0, gq, gk, gv, df, dS0, ws, B, Ti, a, b, s);
  if (dk_ <= 64 && dv_ <= 64)
    return launch_bwd_seq_t<8, 2>(qf, kf, vf, f, df_o, S0, gq, gk, gv, df, dS0, ws, B, Ti, a, b, s);
  return launch_bwd_seq_t<16, 4>(qf, kf, vf, f, df_o, S0, gq, gk, gv, df, dS0, ws, B, Ti, a, b, s);
}

}  // extern "C"
