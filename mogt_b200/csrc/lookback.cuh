// Windowed decoupled look-back for chains whose carry combines as
//     S = A * S_prev + S_agg          (scalar decay A, 64x64 fp32 state)
// which is the gated scan's carry in both directions.
//
// The units of one chain are  unit(s) = base + s * stride,  s = 0, 1, ...
// Unit s publishes an aggregate (A_agg, S_agg) and later an inclusive state
// (a_inc, S_inc).  To get the state entering unit s_self, warp 0 polls the
// flags of up to 32 predecessors at once, finds the nearest inclusive one,
// and all threads then accumulate the aggregates in between with pipelined
// L2 loads.  States use the producer's fragment-native layout: thread `tid`
// of the NTH participating threads owns floats [tid*4*NF, (tid+1)*4*NF) of
// every 4096-float state, so NF * 4 * NTH == 4096.
#pragma once

#include "common.cuh"

namespace mogt {

struct LookbackBufs {
  const uint32_t* flags;
  const float* a_agg;
  const float* a_inc;
  const float* st_agg;
  const float* st_inc;
  WsHeader* hdr;
};

// scl: 32 floats of shared memory; ctl: 4 words of shared memory.
// Called by the NTH threads of a warp-aligned group, `tid` = index in the
// group, synchronised by named barrier `bar_id` (0 with NTH = blockDim.x is
// the CTA barrier).
template <int NF, int NTH = 256>
__device__ __forceinline__ void lookback_scalar_state(float (&acc)[NF][4], float& a_in,
                                                      const LookbackBufs& lb, int s_self,
                                                      uint32_t base, uint32_t stride,
                                                      uint32_t epoch, uint32_t unit_id, float* scl,
                                                      volatile uint32_t* ctl, int tid = -1,
                                                      int bar_id = 0) {
  static_assert(NF * 4 * NTH == 4096, "state layout");
  if (tid < 0) tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
#pragma unroll
  for (int n = 0; n < NF; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;
  const uint32_t want = epoch & 0x3FFFFFFFu;
  float run = 1.f;
  int sp = s_self - 1;
  for (;;) {
    if (warp == 0) {
      const int s_l = sp - lane;
      const bool valid = s_l >= 0;
      const uint32_t m = base + (uint32_t)(valid ? s_l : 0) * stride;
      const int nvalid = sp + 1 < 32 ? sp + 1 : 32;
      int n = 0;
      bool end = false;
      for (uint32_t it = 0;; ++it) {
        uint32_t st = kFlagNone;
        if (valid) {
          const uint32_t v = ld_acquire_u32(lb.flags + m);
          st = ((v >> 2) == want) ? (v & 3u) : kFlagNone;
        }
        const uint32_t incm = __ballot_sync(0xffffffffu, valid && st == kFlagInc);
        const uint32_t nrm = __ballot_sync(0xffffffffu, valid && st == kFlagNone);
        const int fi = incm ? __ffs(incm) - 1 : 32;
        const int fn = nrm ? __ffs(nrm) - 1 : 32;
        if (fi < fn) {
          n = fi + 1;
          end = true;
          break;
        }
        if (fn > 0) {
          n = fn < nvalid ? fn : nvalid;
          break;
        }
        if (it >= kSpinLimit) {
          if (lane == 0) record_error(lb.hdr, MOGT_ERR_TIMEOUT, unit_id);
          n = 1;
          end = true;
          break;
        }
        if (it > 16) __nanosleep(it > 1024 ? 256 : 32);
      }
      float A = 1.f;
      if (lane < n) A = (end && lane == n - 1) ? __ldcg(lb.a_inc + m) : __ldcg(lb.a_agg + m);
      float incl = A;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl *= y;
      }
      float excl = __shfl_up_sync(0xffffffffu, incl, 1);
      if (lane == 0) excl = 1.f;
      if (lane < n) scl[lane] = run * excl;
      const float tot = __shfl_sync(0xffffffffu, incl, n - 1);
      if (lane == 0) {
        ctl[0] = (uint32_t)n;
        ctl[1] = end ? 1u : 0u;
        ctl[2] = __float_as_uint(run * tot);
      }
    }
    group_sync(bar_id, NTH);
    const int n = (int)ctl[0];
    const bool end = ctl[1] != 0;
    const float run_next = __uint_as_float(ctl[2]);
#pragma unroll 4
    for (int l = 0; l < n; ++l) {
      const uint32_t m = base + (uint32_t)(sp - l) * stride;
      const bool inc = end && l == n - 1;
      const float4* src = reinterpret_cast<const float4*>((inc ? lb.st_inc : lb.st_agg) +
                                                          (size_t)m * 4096 + (size_t)tid * (4 * NF));
      const float s = scl[l];
#pragma unroll
      for (int q = 0; q < NF; ++q) {
        const float4 v = __ldcg(src + q);
        acc[q][0] = fmaf(s, v.x, acc[q][0]);
        acc[q][1] = fmaf(s, v.y, acc[q][1]);
        acc[q][2] = fmaf(s, v.z, acc[q][2]);
        acc[q][3] = fmaf(s, v.w, acc[q][3]);
      }
    }
    if (end) {
      a_in = run_next;
      break;
    }
    run = run_next;
    sp -= n;
    group_sync(bar_id, NTH);
  }
}

}  // namespace mogt
